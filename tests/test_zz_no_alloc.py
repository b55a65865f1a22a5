"""AnnB200BitmapRowsStatic: filter-bitmap expansion without device allocation.

Callers that cannot allocate device memory on their request path (a worker
serving from a budget reserved at start-up, or one that cannot take the
device synchronisation of cudaMalloc / cudaFree between requests) use this
entry point instead of AnnB200BitmapRows; its scratch is a fixed array in
device memory. This file checks, through the C ABI, that two calls in a row
return exactly the rows the allocating entry point returns, that the second
call does not depend on what the first left in the shared scratch, and that
bitmaps beyond the array's limit are refused. It sits last in collection
order and passes both alone in a fresh process and after the other tests.
"""
import ctypes

import numpy as np
import pytest

from pgvector_b200 import synth

pytestmark = pytest.mark.gpu


def to_dev(a, cuda):
    import torch
    return torch.from_numpy(np.ascontiguousarray(a).view(np.int32)).to(cuda)


def static_rows(words, nbits, cuda):
    import torch
    import pgvector_b200 as pb
    lib = pb.load()
    rows = torch.full((max(nbits, 1),), -1, dtype=torch.int32, device=cuda)
    n = ctypes.c_uint64()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    status = lib.AnnB200BitmapRowsStatic(ctypes.c_void_p(words.data_ptr()), nbits, ctypes.c_void_p(rows.data_ptr()),
                                         ctypes.byref(n), stream)
    assert status == 0, lib.AnnB200LastError()
    return rows[:n.value].cpu().numpy().view(np.uint32)


def test_two_calls_match_the_allocating_entry_point(cuda):
    import pgvector_b200 as pb
    # a large dense bitmap first, then a smaller sparse one: the second call
    # must not pick up block offsets or the count the first left behind
    for nbits, sel, seed in ((20 * 32768 * 32 + 77, 0.7, 51), (100003, 0.1, 52)):
        words, expected = synth.bitmap(nbits, sel, seed=seed)
        dw = to_dev(words, cuda)
        allocating = pb.bitmap_rows(dw, nbits).cpu().numpy().view(np.uint32)
        got = static_rows(dw, nbits, cuda)
        assert np.array_equal(allocating, expected)
        assert np.array_equal(got, allocating)


def test_bitmaps_beyond_the_limit_are_refused(cuda):
    import torch
    import pgvector_b200 as pb
    lib = pb.load()
    dummy = torch.zeros((4,), dtype=torch.int32, device=cuda)
    n = ctypes.c_uint64(123)
    status = lib.AnnB200BitmapRowsStatic(ctypes.c_void_p(dummy.data_ptr()), (1 << 31) + 1,
                                         ctypes.c_void_p(dummy.data_ptr()), ctypes.byref(n), None)
    assert status == pb.INVALID
    assert n.value == 0
    assert b'limit' in lib.AnnB200LastError()
