"""The CPU oracle, pinned against the reference before it is trusted.

Pins: golden vectors made by the reference's own builder quantizers and its
compiled AnnGatheredExact / AnnIndexTreeMerge (tests/golden/make_golden.py),
the live reference library when this machine has it (oracle/_ref), and the
known answers of the reference's worker tests (boundary ties, the metric
oracle of test_worker.py:60-87, tie handling of test_worker.py:89-95).
"""
import math
import os

import numpy as np
import pytest

import oracle
from pgvector_b200 import synth

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), 'golden')


def golden(name):
    return np.load(os.path.join(GOLDEN, name))


# ---------------------------------------------------------------- decoders

def test_e4m3_decode_matches_format_definition():
    # exponent bits 6..3 (bias 7), mantissa 2..0, subnormals at exponent 0
    # (ann/builder/build_cuvs_index.py:296-301); 0x7f is NaN, bit 7 the sign
    L = oracle.lib()
    assert L.orc_e4m3(0x00) == 0.0
    assert L.orc_e4m3(0x01) == 2.0 ** -9
    assert L.orc_e4m3(0x07) == 7 * 2.0 ** -9
    assert L.orc_e4m3(0x08) == 2.0 ** -6
    assert L.orc_e4m3(0x38) == 1.0
    assert L.orc_e4m3(0x7e) == 448.0
    assert L.orc_e4m3(0xb8) == -1.0
    assert math.isnan(L.orc_e4m3(0x7f))
    values = [L.orc_e4m3(c) for c in range(127)]
    assert all(a < b for a, b in zip(values, values[1:]))


def test_e2m1_decode():
    L = oracle.lib()
    assert [L.orc_e2m1(n) for n in range(8)] == [0, 0.5, 1, 1.5, 2, 3, 4, 6]
    assert [L.orc_e2m1(n | 8) for n in range(1, 8)] == [-0.5, -1, -1.5, -2, -3, -4, -6]


def test_half_roundtrip_matches_numpy():
    rng = np.random.default_rng(3)
    x = np.concatenate([rng.standard_normal(2000).astype(np.float32) * 10.0 ** rng.integers(-9, 5, 2000),
                        np.array([0, -0.0, 65504, 1e-8, 6e-8, 70000, -3e-5], dtype=np.float32)])
    h = oracle.float_to_half(x)
    assert np.array_equal(h, x.astype(np.float16).view(np.uint16))
    assert np.array_equal(oracle.half_to_float(h), h.view(np.float16).astype(np.float32))


# ---------------------------------------------------------------- quantizers vs the reference builder

@pytest.mark.parametrize('i', range(4))
def test_quantizers_match_reference_builder(i):
    g = golden('quant.npz')
    v = g['v%d' % i]
    codes, scale = oracle.quantize_fp8(v)
    assert np.array_equal(codes, g['fp8_codes%d' % i])
    assert np.array_equal(scale, g['fp8_scale%d' % i])
    packed, sc, row = oracle.quantize_nvfp4(v)
    assert np.array_equal(packed, g['nvfp4_packed%d' % i])
    assert np.array_equal(sc, g['nvfp4_scales%d' % i])
    assert np.array_equal(row, g['nvfp4_row%d' % i])


# ---------------------------------------------------------------- search vs the reference worker

def _gathered_jobs():
    g = golden('gathered.npz')
    for n in range(int(g['count'][0])):
        k, metric, status = (int(x) for x in g['meta%d' % n])
        yield g['q%d' % n], g['v%d' % n], k, metric, status, g['ids%d' % n], g['dist%d' % n]


def test_window_search_matches_reference_golden():
    for q, v, k, metric, status, ids, dist in _gathered_jobs():
        d, i, c, s = oracle.search(oracle.F32, q.shape[0], v, q[None, :], k, metric, window=True)
        assert s[0] == status
        assert c[0] == len(ids)
        assert np.array_equal(i[0, :c[0]], ids)
        assert np.array_equal(d[0, :c[0]], dist)   # bit for bit


@pytest.mark.skipif(not oracle.ref_available(), reason='reference library not built on this machine')
def test_window_search_matches_live_reference():
    rng = np.random.default_rng(11)
    for trial in range(40):
        dims = int(rng.choice([3, 16, 96]))
        rows = int(rng.integers(1, 700))
        metric = trial % 3
        k = int(rng.choice([1, 10, 100, 400]))
        v = np.round(rng.uniform(-2, 2, (rows, dims)), 2).astype(np.float32)
        q = np.round(rng.uniform(-2, 2, dims), 2).astype(np.float32)
        status, res = oracle.ref_gathered_exact(q, v, k, metric)
        d, i, c, s = oracle.search(oracle.F32, dims, v, q[None, :], k, metric, window=True)
        assert s[0] == status
        assert [r[0] for r in res] == list(i[0, :c[0]])
        assert [r[1] for r in res] == list(d[0, :c[0]])


def test_boundary_ties_are_retained():
    # known answer of the reference server test (test_server.py:189-195)
    v = np.array([[1, 0], [0, 1], [-1, 0], [0, -1], [3, 3]], dtype=np.float32)
    d, i, c, s = oracle.search(oracle.F32, 2, v, np.zeros((1, 2), np.float32), 1, 0, window=True)
    assert sorted(i[0, :c[0]]) == [0, 1, 2, 3]


def test_metric_oracle_with_filters():
    # the independent Python oracle of the reference's test_worker.py:60-87,
    # restated: ties ordered by id, cosine skips zero-norm rows
    import random
    rng = random.Random(42)
    vectors = np.array([[rng.randint(-5, 5) for _ in range(7)] for _ in range(80)], dtype=np.float32)
    queries = np.array([[rng.randint(1, 5) for _ in range(7)] for _ in range(5)], dtype=np.float32)
    filters = [sorted(rng.sample(range(80), n)) for n in [0, 1, 8, 25, 80]]
    for metric in range(3):
        for k in [0, 1, 7, 100]:
            for query, ids in zip(queries, filters):
                expected = []
                for j in ids:
                    vec = vectors[j]
                    dot = float(sum(float(a) * float(b) for a, b in zip(vec, query)))
                    if metric == 0:
                        dist = math.sqrt(sum((float(a) - float(b)) ** 2 for a, b in zip(vec, query)))
                    elif metric == 1:
                        dist = -dot
                    else:
                        norm = float(sum(float(a) ** 2 for a in vec)) * float(sum(float(b) ** 2 for b in query))
                        if not norm:
                            continue
                        dist = 1 - max(-1, min(1, dot / math.sqrt(norm)))
                    expected.append((j, dist))
                expected.sort(key=lambda x: (x[1], x[0]))
                d, i, c, s = oracle.search(oracle.F32, 7, vectors, query[None, :], k, metric,
                                           ids=np.array(ids, dtype=np.uint32) if ids else np.zeros(0, np.uint32))
                assert s[0] == 0
                assert list(i[0, :c[0]]) == [e[0] for e in expected[:k]]
                for got, want in zip(d[0, :c[0]], expected[:k]):
                    assert abs(got - want[1]) < 1e-12


def test_shared_none_empty_and_ties():
    # test_worker.py:89-95 restated: ties by id, empty filter, zero-query cosine invalid
    v = np.array([[1, 0], [-1, 0], [0, 0]], dtype=np.float32)
    d, i, c, s = oracle.search(oracle.F32, 2, v, np.zeros((1, 2), np.float32), 4, 0)
    assert list(zip(i[0, :c[0]], d[0, :c[0]])) == [(2, 0), (0, 1), (1, 1)]
    d, i, c, s = oracle.search(oracle.F32, 2, v, np.zeros((1, 2), np.float32), 4, 0, ids=np.zeros(0, np.uint32))
    assert c[0] == 0
    d, i, c, s = oracle.search(oracle.F32, 2, v, np.zeros((1, 2), np.float32), 2, 2)
    assert s[0] == 1
    d, i, c, s = oracle.search(oracle.F32, 2, v, np.array([[1, 0]], np.float32), 9, 2)
    assert c[0] == 2   # the zero row is skipped under cosine


def test_invalid_inputs():
    v = np.array([[np.nan, 0]], dtype=np.float32)
    d, i, c, s = oracle.search(oracle.F32, 2, v, np.zeros((1, 2), np.float32), 1, 0, window=True)
    assert s[0] == 1
    d, i, c, s = oracle.search(oracle.F32, 2, np.zeros((2, 2), np.float32), np.array([[np.inf, 0]], np.float32), 1, 1)
    assert s[0] == 1


# ---------------------------------------------------------------- typed formats

def test_fp16_cosine_equals_reference_on_decoded_rows():
    rng = np.random.default_rng(5)
    x = rng.standard_normal((300, 24)).astype(np.float32)
    h = x.astype(np.float16)
    q = rng.standard_normal((4, 24)).astype(np.float32).astype(np.float16).astype(np.float32)
    d16, i16, c16, _ = oracle.search(oracle.F16, 24, h.view(np.uint16), q, 10, 2)
    d32, i32, c32, _ = oracle.search(oracle.F32, 24, h.astype(np.float32), q, 10, 2)
    assert np.array_equal(i16, i32) and np.array_equal(d16, d32)


def test_fp8_and_nvfp4_decode_then_search():
    rng = np.random.default_rng(6)
    x = rng.standard_normal((200, 40)).astype(np.float32)
    q = rng.standard_normal((3, 40)).astype(np.float32)
    codes, scale = oracle.quantize_fp8(x)
    dec = oracle.decode_rows(oracle.E4M3, 40, codes, row_scales=scale)
    # decoded values: e4m3 x row scale in FP32
    L = oracle.lib()
    assert dec[7, 3] == np.float32(L.orc_e4m3(int(codes[7, 3]))) * scale[7]
    a = oracle.search(oracle.E4M3, 40, codes, q, 5, 1, row_scales=scale)
    b = oracle.search(oracle.F32, 40, dec, q, 5, 1)
    assert np.array_equal(a[1], b[1]) and np.array_equal(a[0], b[0])
    packed, sc, row = oracle.quantize_nvfp4(x)
    dec4 = oracle.decode_rows(oracle.NVFP4, 40, packed, block_scales=sc, row_scales=row)
    a = oracle.search(oracle.NVFP4, 40, packed, q, 5, 0, block_scales=sc, row_scales=row)
    b = oracle.search(oracle.F32, 40, dec4, q, 5, 0)
    assert np.array_equal(a[1], b[1]) and np.array_equal(a[0], b[0])
    # quantization error is bounded (recall sanity of the format)
    assert np.abs(dec - x).max() <= np.abs(x).max(axis=1).max() / 448 * 32


def test_hamming_known_answers():
    rows = np.array([[0x00, 0x00], [0xff, 0x00], [0x0f, 0x01], [0x00, 0x80], [0xff, 0xff]], dtype=np.uint8)
    q = np.array([[0x00, 0x00]], dtype=np.uint8)
    d, i, c, s = oracle.search(oracle.BIT, 16, rows, q, 5, 3)
    assert list(i[0]) == [0, 3, 2, 1, 4]
    assert list(d[0]) == [0, 1, 5, 8, 16]
    # ties broken by row id
    rows = np.array([[1], [2], [4], [8]], dtype=np.uint8)
    d, i, c, s = oracle.search(oracle.BIT, 8, rows, np.zeros((1, 1), np.uint8), 2, 3)
    assert list(i[0]) == [0, 1] and list(d[0]) == [1, 1]


def test_ivf_list_gather():
    rng = np.random.default_rng(8)
    x = rng.standard_normal((100, 8)).astype(np.float32)
    offsets = np.array([0, 10, 40, 41, 100], dtype=np.uint64)
    row_ids = rng.permutation(1000)[:100].astype(np.int64)
    q = rng.standard_normal((2, 8)).astype(np.float32)
    probes = np.array([[1, 3], [0, 2]], dtype=np.uint32)
    d, i, c = oracle.search_lists(oracle.F32, 8, x, q, offsets, probes, 5, 0, row_ids=row_ids)
    for qi, pr in enumerate(probes):
        rows = np.concatenate([np.arange(offsets[p], offsets[p + 1]) for p in pr]).astype(np.int64)
        cand = sorted((math.sqrt(float(((x[r].astype(np.float64) - q[qi]) ** 2).sum())), row_ids[r]) for r in rows)
        assert list(i[qi, :c[qi]]) == [cid for _, cid in cand[:5]]


# ---------------------------------------------------------------- merge vs the reference's tree merge

def test_tree_merge_golden_equals_sorted_union():
    g = golden('merge.npz')
    for t in range(int(g['count'][0])):
        k = int(g['k%d' % t][0])
        lists = g['lists%d' % t]
        union = sorted((float(np.float32(d)), int(key)) for _, key, d in lists)
        merged = g['merged%d' % t]
        assert [int(key) for key, _ in merged] == [key for _, key in union[:k]]


@pytest.mark.parametrize('dims', [768, 37, 1024])
def test_torch_quantizers_match_the_oracle(dims):
    # the bench encodes full-size corpora on the GPU with the torch statement
    # of the builder's quantizers; on the CPU both must agree bit for bit
    import torch
    x = synth.mixture(3000, dims, 20, seed=90 + dims)
    x[5] = 0.0
    x[7, :5] = [448.0, -1e-9, 3e-7, -6.0, 0.25]
    codes, scale = oracle.quantize_fp8(x)
    tc, ts = synth.torch_quantize_fp8(torch.from_numpy(x))
    assert np.array_equal(tc.numpy(), codes) and np.array_equal(ts.numpy(), scale)
    packed, sc, row = oracle.quantize_nvfp4(x)
    tp, tsc, tr = synth.torch_quantize_nvfp4(torch.from_numpy(x))
    assert np.array_equal(tp.numpy(), packed) and np.array_equal(tsc.numpy(), sc) and np.array_equal(tr.numpy(), row)
