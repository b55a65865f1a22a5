"""The C ABI library without a GPU: it loads, exports every symbol
include/*.h declares, fills the backend vtable as the worker expects, and the
host-side validation and fault-injection paths need no device."""
import ctypes
import os
import re
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INCLUDE = os.path.join(ROOT, 'include')

import pgvector_b200 as pb
from pgvector_b200 import _abi
from pgvector_b200._lib import SIGNATURES


def declared_functions():
    names = set()
    for f in os.listdir(INCLUDE):
        text = open(os.path.join(INCLUDE, f)).read()
        text = re.sub(r'/\*.*?\*/', '', text, flags=re.S)
        for m in re.finditer(r'\b(AnnB200\w+)\s*\(', text):
            names.add(m.group(1))
    return names


def test_library_exports_every_declared_symbol():
    lib = pb.load()
    names = declared_functions()
    assert {'AnnB200Backend', 'AnnB200Search', 'AnnB200ShardCreate', 'AnnB200MergeTopk'} <= names
    for name in names:
        assert hasattr(lib, name), name
    assert names <= set(SIGNATURES), names - set(SIGNATURES)
    out = subprocess.run(['nm', '-D', '--defined-only', pb._lib.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r' T (AnnB200\w+)', out))
    assert names <= exported


def test_library_is_sm100a_and_not_linked_to_oracle():
    out = subprocess.run(['ldd', pb._lib.LIB_PATH], capture_output=True, text=True).stdout
    assert 'oracle' not in out and 'annref' not in out


def test_backend_vtable_matches_worker_layout():
    b = pb.backend()
    assert b.name == b'b200'
    assert b.metrics == 7 and b.filters == 7
    assert b.exact == 1 and b.max_k == 0xffffffff
    assert b.algorithm == b'flat' and b.storage == b'fp32'
    assert b.device_jobs and b.lost
    assert not b.load_index and not b.search_index and not b.scan_preferred
    assert b.search_typed
    # positional layout: the reference's 17 slots, pointers after the 8
    # scalar fields, then the typed search slot
    assert ctypes.sizeof(_abi.AnnBackend) == 8 * 3 + 4 * 2 + 4 + 4 * 2 + 8 * 9 + 4 + 8


def test_gathered_job_struct_layout():
    # AnnCandidate {u32 id; f64 distance} is 16 bytes; AnnGatheredJob 48
    assert ctypes.sizeof(_abi.AnnCandidate) == 16
    assert ctypes.sizeof(_abi.AnnGatheredJob) == 48


def test_invalid_gathered_jobs_rejected_on_host():
    q = np.zeros(2, np.float32)
    v = np.ones((3, 2), np.float32)
    # (a non-finite row value is found on the device: tests/test_parity_gpu.py)
    res = pb.search_gathered([
        (q, v, 1, 3),                                  # metric beyond 2
        (np.array([np.nan, 0], np.float32), v, 1, 0),  # non-finite query
        (q, np.array([[np.inf, 0]], np.float32), 0, 0),  # k = 0 with a non-finite row
        (q, v, 1, 2),                                  # zero query under cosine
        (q, v, 0, 0),                                  # k = 0: no results, OK
        (q, np.zeros((0, 2), np.float32), 5, 0),       # no rows: OK
    ])
    assert [s for s, _ in res] == [1, 1, 1, 1, 0, 0]
    assert all(not r for _, r in res)


def test_device_count_without_gpu():
    import torch
    if torch.cuda.is_available():
        pytest.skip('a GPU is visible')
    assert pb.device_count() == 0


LOST_SCRIPT = r'''
import os, sys, ctypes
import numpy as np
sys.path.insert(0, %r)
import pgvector_b200 as pb
res = pb.search_gathered([(np.ones(2, np.float32), np.ones((4, 2), np.float32), 1, 0)])
lost = ctypes.CFUNCTYPE(ctypes.c_char_p)(pb.backend().lost)()
print(res[0][0], lost.decode())
'''


def test_simulated_device_loss_reported_without_a_gpu():
    # the mock-GPU style injection (ann/server/mockgpu.c:148-200): the
    # worker would exit 70 on this lost() reason
    env = dict(os.environ, ANN_B200_LOST_AFTER='0')
    out = subprocess.run([sys.executable, '-c', LOST_SCRIPT % ROOT], capture_output=True, text=True, env=env,
                         timeout=300)
    assert out.returncode == 0, out.stderr
    status, reason = out.stdout.strip().split(' ', 1)
    assert int(status) == pb.BACKEND_ERROR
    assert 'GPU context lost (simulated' in reason


def test_quantized_index_arguments_checked_on_host():
    # AnnB200IndexCreateQuant / AnnB200RescoreRows refuse bad arguments
    # before touching a device
    lib = pb.load()
    out = ctypes.c_void_p()
    codes = np.zeros((4, 16), np.uint8)
    scales = np.zeros((4, 1), np.uint8)
    rs = np.ones(4, np.float32)
    v = np.zeros((4, 16), np.float32)
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    rows = (ctypes.c_uint64 * 2)(3, 2)
    cases = [
        (0, 0, 4, pb.NVFP4, P(codes), P(scales), P(rs), P(v), 0, None),      # dims 0
        (0, 16, 4, pb.BIT, P(codes), P(scales), P(rs), P(v), 0, None),       # not a copy format
        (0, 16, 4, pb.NVFP4, P(codes), None, P(rs), P(v), 0, None),          # NVFP4 without block scales
        (0, 16, 4, pb.E4M3, P(codes), None, P(rs), None, 0, None),           # no FP32 rows
        (0, 16, 4, pb.E4M3, P(codes), None, P(rs), P(v), 2, rows),           # shards cover 5 rows, not 4
    ]
    for i, c in enumerate(cases):
        st = lib.AnnB200IndexCreateQuant(*c[:8], c[8], c[9], 256, 100, ctypes.byref(out))
        assert st == pb.INVALID and not out.value, i
    assert lib.AnnB200RescoreRows(None, 0, 4, None, 8, None, None, None) == 0   # nothing to do
    assert lib.AnnB200RescoreRows(None, 2, 4, None, 8, None, None, None) == pb.INVALID


def test_typed_jobs_checked_on_host():
    # AnnB200SearchTyped refuses bad jobs before touching a device
    q = np.ones((2, 4), np.float32)
    rows = np.ones((3, 4), np.float32)
    bad_q = q.copy()
    bad_q[1, 2] = np.nan
    e4 = np.zeros((3, 16), np.uint8)
    e4_nan = e4.copy()
    e4_nan[2, 1] = 0xff
    half_inf = np.full((3, 4), 0x7c00, np.uint16)
    cases = [
        dict(dtype=pb.F32, metric=3, dims=4, k=1, queries=q, codes=rows),                 # Hamming on floats
        dict(dtype=pb.BIT, metric=0, dims=32, k=1, queries=np.zeros((1, 4), np.uint8),
             codes=np.zeros((3, 4), np.uint8)),                                            # bits without Hamming
        dict(dtype=pb.F32, metric=0, dims=4, k=1, queries=bad_q, codes=rows),             # non-finite query
        dict(dtype=pb.F32, metric=2, dims=4, k=1, queries=np.zeros((1, 4), np.float32), codes=rows),
        dict(dtype=pb.E4M3, metric=1, dims=4, k=1, queries=q, codes=e4),                  # no row scales
        dict(dtype=pb.E4M3, metric=1, dims=4, k=1, queries=q, codes=e4_nan, row_scales=np.ones(3, np.float32)),
        dict(dtype=pb.F16, metric=0, dims=4, k=1, queries=q, codes=half_inf),             # infinite halves
        dict(dtype=pb.NVFP4, metric=0, dims=4, k=1, queries=q, codes=np.zeros((3, 8), np.uint8),
             row_scales=np.ones(3, np.float32)),                                           # no block scales
        dict(dtype=9, metric=0, dims=4, k=1, queries=q, codes=rows),
    ]
    got = pb.search_typed(cases)
    assert [s for s, _ in got] == [pb.INVALID] * len(cases)
    # nothing to do: OK without a device
    got = pb.search_typed([dict(dtype=pb.F32, metric=0, dims=4, k=0, queries=q, codes=rows),
                           dict(dtype=pb.F32, metric=0, dims=4, k=3, queries=q, codes=rows[:0])])
    assert got == [(0, [[], []]), (0, [[], []])]
