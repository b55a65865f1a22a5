"""GPU parity: libannb200 through its C ABI against the CPU oracle.

Bar: bit-exact. Result ids, counts and FP64 distances must equal the
oracle's exactly (the oracle itself equals the reference worker bit for bit,
tests/test_oracle.py), for every storage format, metric, candidate-set form
and selection mode, on both scan paths (tcgen05 tensor cores and CUDA cores).
"""
import numpy as np
import pytest

import oracle
from pgvector_b200 import synth

pytestmark = pytest.mark.gpu


def to_dev(a, cuda):
    import torch
    a = np.ascontiguousarray(a)
    if a.dtype == np.uint16:
        a = a.view(np.int16)
    if a.dtype == np.uint32:
        a = a.view(np.int32)
    return torch.from_numpy(a).to(cuda)


def gpu_search(cuda, dtype, dims, codes, queries, k, metric, ids=None, bs=None, rs=None, window=False,
               force_simt=False, cap=None, force_f16=False):
    import pgvector_b200 as pb
    shard = pb.Shard(dtype, dims, to_dev(codes, cuda), None if bs is None else to_dev(bs, cuda),
                     None if rs is None else to_dev(rs, cuda))
    d, i, c = shard.search(to_dev(queries, cuda), k, metric, rows=None if ids is None else to_dev(ids, cuda),
                           window=window, force_simt=force_simt, out_cap=cap, force_f16=force_f16)
    return d.cpu().numpy(), i.cpu().numpy(), c.cpu().numpy()


def assert_same(cuda, dtype, dims, codes, queries, k, metric, ids=None, bs=None, rs=None, window=False,
                force_simt=False, check=None, force_f16=False):
    """The device answers the whole batch; the oracle answers the queries
    `check` selects (all of them by default) and those must be equal."""
    n = codes.shape[0] if ids is None else len(ids)
    cap = max(n, 1) if window else max(k, 1)
    sel = np.arange(queries.shape[0]) if check is None else np.asarray(check)
    od, oi, oc, os_ = oracle.search(dtype, dims, codes, queries[sel], k, metric, ids=ids, block_scales=bs,
                                    row_scales=rs, window=window, cap=cap)
    assert (os_ == 0).all()
    gd, gi, gc = gpu_search(cuda, dtype, dims, codes, queries, k, metric, ids, bs, rs, window, force_simt, cap,
                            force_f16)
    gd, gi, gc = gd[sel], gi[sel], gc[sel]
    assert np.array_equal(gc, oc.astype(gc.dtype)), (gc[:8], oc[:8])
    for q in range(len(sel)):
        c = int(oc[q])
        assert np.array_equal(gi[q, :c], oi[q, :c]), (q, gi[q, :c][:10], oi[q, :c][:10])
        assert np.array_equal(gd[q, :c], od[q, :c]), (q, gd[q, :c][:10], od[q, :c][:10])
    return oc


# ---------------------------------------------------------------- fp32 (config 1 shape)

@pytest.mark.parametrize('metric', [0, 1, 2])
def test_f32_small_all_metrics(cuda, metric):
    x = synth.mixture(5000, 37, 20, seed=1)
    q = synth.mixture_queries(40, 37, 20, seed=1)
    assert_same(cuda, oracle.F32, 37, x, q, 10, metric)


def test_f32_config1_shape_sampled(cuda):
    # config 1: 100-centre mixture, d=128, k=10 (fewer queries to keep the oracle quick)
    x = synth.mixture(100000, 128, 100, seed=2)
    q = synth.mixture_queries(64, 128, 100, seed=2)
    assert_same(cuda, oracle.F32, 128, x, q, 10, 0)


def test_f32_row_list_and_window(cuda):
    x = synth.mixture(60000, 64, 50, seed=3)
    q = synth.mixture_queries(24, 64, 50, seed=3)
    _, ids = synth.bitmap(60000, 0.6, seed=3)
    assert_same(cuda, oracle.F32, 64, x, q, 25, 0, ids=ids)
    assert_same(cuda, oracle.F32, 64, x, q, 25, 0, ids=ids, window=True)
    assert_same(cuda, oracle.F32, 64, x, q, 25, 2, ids=ids, window=True)


# ---------------------------------------------------------------- fp16 / halfvec (config 2 shape)

@pytest.mark.parametrize('metric', [2, 0, 1])
def test_f16_tensor_path(cuda, metric):
    x = synth.mixture(40000, 768, 100, seed=4, normalize=True)
    h = synth.to_half_bits(x)
    q = synth.mixture_queries(300, 768, 100, seed=4, normalize=True).astype(np.float16).astype(np.float32)
    _, ids = synth.bitmap(40000, 0.9, seed=4)
    assert_same(cuda, oracle.F16, 768, h, q, 100, metric, ids=ids)


def test_f16_gathered_and_contiguous_scans(cuda):
    # batches of 256+ FP16 queries: contiguous rows read by TMA, row lists
    # gathered by the scan's own copy warps; rows not a multiple of the tile,
    # a padded last query tile
    x = synth.mixture(70001, 256, 200, seed=12, normalize=True)
    h = synth.to_half_bits(x)
    q = synth.mixture_queries(520, 256, 200, seed=12, normalize=True)
    _, ids = synth.bitmap(70001, 0.55, seed=13)
    assert_same(cuda, oracle.F16, 256, h, q, 64, 2)
    assert_same(cuda, oracle.F16, 256, h, q, 40, 1, ids=ids)
    assert_same(cuda, oracle.F16, 256, h, q[:256], 10, 0, window=True)
    assert_same(cuda, oracle.F16, 256, h, q[:300], 25, 0, ids=ids[::3], window=True)


def test_f16_simt_path_matches(cuda):
    x = synth.mixture(20000, 96, 30, seed=5, normalize=True)
    h = synth.to_half_bits(x)
    q = synth.mixture_queries(50, 96, 30, seed=5, normalize=True)
    assert_same(cuda, oracle.F16, 96, h, q, 20, 2, force_simt=True)
    assert_same(cuda, oracle.F16, 96, h, q, 20, 2)


def test_f16_fp32_queries_and_odd_dims(cuda):
    # FP32 queries over FP16 rows (query rounding covered by the bound), and
    # dims not a multiple of 64 (zero-filled K tail in the tensor scan)
    x = synth.mixture(35000, 200, 40, seed=6)
    h = synth.to_half_bits(x)
    q = synth.mixture_queries(40, 200, 40, seed=6)
    assert_same(cuda, oracle.F16, 200, h, q, 30, 0)
    x = synth.mixture(3000, 13, 10, seed=6)
    assert_same(cuda, oracle.F16, 13, synth.to_half_bits(x), synth.mixture_queries(20, 13, 10, seed=6), 5, 2)


# ---------------------------------------------------------------- FP8 / NVFP4 / bits

def test_fp8_inner_product(cuda):
    x = synth.mixture(36000, 256, 64, seed=7)
    codes, scale = oracle.quantize_fp8(x)
    q = synth.mixture_queries(32, 256, 64, seed=7)
    assert_same(cuda, oracle.E4M3, 256, codes, q, 50, 1, rs=scale)
    assert_same(cuda, oracle.E4M3, 256, codes, q, 50, 0, rs=scale)


def test_nvfp4_l2_and_cosine(cuda):
    x = synth.mixture(36000, 768, 64, seed=8)
    packed, sc, row = oracle.quantize_nvfp4(x)
    q = synth.mixture_queries(16, 768, 64, seed=8)
    assert_same(cuda, oracle.NVFP4, 768, packed, q, 100, 0, bs=sc, rs=row)
    assert_same(cuda, oracle.NVFP4, 768, packed, q, 10, 2, bs=sc, rs=row)


@pytest.mark.parametrize('dtype,dims', [(2, 1024), (2, 200), (3, 768), (3, 224)])
@pytest.mark.parametrize('simt', [False, True])
def test_quantized_tensor_and_simt_paths(cuda, dtype, dims, simt):
    # the tensor scan converts E4M3 / NVFP4 codes to FP16 on chip; dims that
    # end inside a 64-dimension k-block exercise the zero-filled tail and the
    # block scales past the row's last block
    x = synth.mixture(40000, dims, 128, seed=60 + dims)
    q = synth.mixture_queries(48, dims, 128, seed=60 + dims)
    if dtype == oracle.E4M3:
        codes, rs = oracle.quantize_fp8(x)
        bs = None
    else:
        codes, bs, rs = oracle.quantize_nvfp4(x)
    _, ids = synth.bitmap(40000, 0.3, seed=61)
    assert_same(cuda, dtype, dims, codes, q, 100, 1, bs=bs, rs=rs, force_simt=simt)
    assert_same(cuda, dtype, dims, codes, q, 50, 0, ids=ids, bs=bs, rs=rs, force_simt=simt)
    assert_same(cuda, dtype, dims, codes, q, 20, 2, ids=ids, bs=bs, rs=rs, window=True, force_simt=simt)


@pytest.mark.parametrize('dims', [1024, 200, 96, 64, 1000])
@pytest.mark.parametrize('f16', [False, True])
def test_e4m3_fp8_and_fp16_tensor_paths(cuda, dims, f16):
    # E4M3 rows on FP8 tensor cores (codes straight from TMA, queries as two
    # E4M3 terms with a power-of-two scale each) and through the on-chip FP16
    # conversion (ANNB200_FORCE_F16): both bit-exact with the oracle, for
    # every metric, whole shard, a row list (staged rows), window mode,
    # heavy ties and dims that end inside a 128-code k-block
    x = synth.mixture(36000, dims, 48, seed=90 + dims)
    q = synth.mixture_queries(64, dims, 48, seed=91 + dims)
    q[5] *= 1e-3                                        # a small query: its terms' scale is small too
    x[9000:9300] = x[77]                                # ties ordered by row id
    codes, rs = oracle.quantize_fp8(x)
    _, ids = synth.bitmap(36000, 0.4, seed=92)
    for metric in (1, 0, 2):
        assert_same(cuda, oracle.E4M3, dims, codes, q, 60, metric, rs=rs, force_f16=f16)
    assert_same(cuda, oracle.E4M3, dims, codes, q, 30, 1, ids=ids, rs=rs, force_f16=f16)
    assert_same(cuda, oracle.E4M3, dims, codes, q[:20], 10, 0, ids=ids[:5000], rs=rs, window=True, force_f16=f16)


@pytest.mark.parametrize('dims', [128, 200, 36, 37])
@pytest.mark.parametrize('simt', [False, True])
def test_f32_split_tensor_and_simt_paths(cuda, dims, simt):
    # FP32 rows whose pitch is a multiple of 16 bytes (dims % 4 == 0) score on
    # tensor cores as two BF16 halves (hi.hi + hi.lo + lo.hi) for L2 and inner
    # product; cosine, 37 dims and ANNB200_FORCE_SIMT use CUDA cores. Whole
    # shard, a row list (staged rows), window mode, and columns over many
    # binades with a few subnormal elements.
    x = synth.mixture(30000, dims, 64, seed=80 + dims)
    q = synth.mixture_queries(40, dims, 64, seed=80 + dims)
    x[:, ::5] *= np.float32(1e-5)
    x[::101, 1] = np.float32(2e-40)
    x[7000:7200] = x[55]                          # duplicates: ties ordered by row id
    _, ids = synth.bitmap(30000, 0.3, seed=81)
    for metric in (0, 1, 2):
        assert_same(cuda, oracle.F32, dims, x, q, 50, metric, force_simt=simt)
    assert_same(cuda, oracle.F32, dims, x, q, 20, 0, ids=ids, force_simt=simt)
    assert_same(cuda, oracle.F32, dims, x, q[:16], 10, 1, ids=ids[:3000], window=True, force_simt=simt)


def test_hamming_bit_exact_with_ties(cuda):
    rows, proto = synth.bit_rows(60000, 1024, 256, flip=0.05, seed=9)
    rng = np.random.default_rng(9)
    qs = proto[rng.integers(0, 256, 48)] ^ np.packbits(rng.random((48, 1024)) < 0.05, axis=1, bitorder='little')
    assert_same(cuda, oracle.BIT, 1024, rows, qs, 100, 3)
    assert_same(cuda, oracle.BIT, 1024, rows[:500], qs[:4], 7, 3)


@pytest.mark.parametrize('dims', [1024, 512, 128, 1000, 136])
@pytest.mark.parametrize('simt', [False, True])
def test_hamming_tensor_and_simt_paths(cuda, dims, simt):
    # rows whose byte pitch is a multiple of 16 (1024, 512, 128 bits) are
    # expanded to +-1 int8 and scored by kind::i8 MMAs (exact S32 dot
    # products); 1000 and 136 bits (125 and 17 bytes) stay on CUDA cores.
    # Whole shard, a row list (staged rows), window mode, duplicated rows
    # (ties ordered by row id) and a k past the shared-memory sort.
    rows, proto = synth.bit_rows(50000, dims, 64, flip=0.05, seed=dims)
    rows[7000:7300] = rows[123]
    rng = np.random.default_rng(dims)
    nb = rows.shape[1]
    qs = proto[rng.integers(0, 64, 40)] ^ np.packbits(rng.random((40, nb * 8)) < 0.05, axis=1,
                                                      bitorder='little')[:, :nb]
    if dims % 8:
        qs[:, -1] &= (1 << (dims % 8)) - 1       # the row's padding bits are zero, as the rows'
    qs[3] = rows[123]
    _, ids = synth.bitmap(50000, 0.3, seed=dims + 1)
    assert_same(cuda, oracle.BIT, dims, rows, qs, 100, 3, force_simt=simt)
    assert_same(cuda, oracle.BIT, dims, rows, qs, 20, 3, ids=ids, force_simt=simt)
    assert_same(cuda, oracle.BIT, dims, rows, qs[:16], 10, 3, ids=ids[:3000], window=True, force_simt=simt)
    assert_same(cuda, oracle.BIT, dims, rows, qs[:16], 5000, 3, force_simt=simt)


# ---------------------------------------------------------------- edge cases

def test_edge_k_values(cuda):
    x = synth.mixture(1000, 16, 5, seed=10)
    q = synth.mixture_queries(8, 16, 5, seed=10)
    assert_same(cuda, oracle.F32, 16, x, q, 1000, 0)       # k = n
    assert_same(cuda, oracle.F32, 16, x, q, 5000, 1)       # k > n
    assert_same(cuda, oracle.F32, 16, x, q, 1, 2)
    gd, gi, gc = gpu_search(cuda, oracle.F32, 16, x, q, 0, 0)
    assert (gc == 0).all()
    gd, gi, gc = gpu_search(cuda, oracle.F32, 16, x, q, 5, 0, ids=np.zeros(0, np.uint32))
    assert (gc == 0).all()


def test_heavy_ties_window(cuda):
    # test_server.py:213-219 shape: 3000 identical rows must all come back
    v = np.array([[1.0, 0.0]] * 3000 + [[5.0, 5.0]] * 100, dtype=np.float32)
    assert_same(cuda, oracle.F32, 2, v, np.zeros((1, 2), np.float32), 5, 0, window=True)


def test_overflow_regrowth_and_large_sort(cuda):
    # 20,000 equal rows inside a 60,000-row shard: the window keeps all of
    # them, more than the initial candidate capacity and the shared-memory sort
    x = synth.mixture(60000, 32, 10, seed=11)
    x[1000:21000] = x[5]
    q = x[5:6] + 0.001
    c = assert_same(cuda, oracle.F32, 32, x, q, 10, 0, window=True)
    assert c[0] >= 20000
    assert_same(cuda, oracle.F32, 32, x, q, 10, 0)


def test_invalid_row_list_rejected(cuda):
    import pgvector_b200 as pb
    x = synth.mixture(100, 8, 3, seed=12)
    with pytest.raises(pb.AnnB200Error) as e:
        gpu_search(cuda, oracle.F32, 8, x, x[:2], 3, 0, ids=np.array([5, 3, 9], np.uint32))
    assert e.value.status == pb.INVALID


# ---------------------------------------------------------------- merge, bitmap, backend

def test_merge_of_shards_equals_whole_search(cuda):
    import torch
    import pgvector_b200 as pb
    x = synth.mixture(80000, 64, 40, seed=13)
    q = synth.mixture_queries(32, 64, 40, seed=13)
    k = 50
    parts = np.array_split(np.arange(80000), 4)
    ds, is_, cs = [], [], []
    for p in parts:
        shard = pb.Shard(pb.F32, 64, to_dev(x[p[0]:p[-1] + 1], cuda), first_id=int(p[0]))
        d, i, c = shard.search(to_dev(q, cuda), k, 0)
        ds.append(d), is_.append(i), cs.append(c)
    md, mi, mc = pb.merge_topk(torch.stack(ds), torch.stack(is_), torch.stack(cs), k)
    od, oi, oc, _ = oracle.search(oracle.F32, 64, x, q, k, 0)
    assert np.array_equal(mi.cpu().numpy(), oi) and np.array_equal(md.cpu().numpy(), od)


def test_bitmap_rows(cuda):
    import pgvector_b200 as pb
    for n, sel in ((1, 1.0), (33, 0.5), (100003, 0.1), (3 * 32768 + 5, 0.7)):
        words, ids = synth.bitmap(n, sel, seed=n)
        got = pb.bitmap_rows(to_dev(words, cuda), n).cpu().numpy().view(np.uint32)
        assert np.array_equal(got, ids)


def test_backend_gathered_jobs_match_reference(cuda):
    import pgvector_b200 as pb
    rng = np.random.default_rng(11)
    jobs = []
    for r in range(12):
        dims = int(rng.choice([3, 16, 96]))
        rows = int(rng.integers(2048, 5000))
        v = np.round(rng.uniform(-2, 2, (rows, dims)), 2).astype(np.float32)
        qv = np.round(rng.uniform(-2, 2, dims), 2).astype(np.float32)
        jobs.append((qv, v, int(rng.choice([1, 10, 100, 400])), r % 3))
    got = pb.search_gathered(jobs)
    for (qv, v, k, metric), (status, res) in zip(jobs, got):
        d, i, c, s = oracle.search(oracle.F32, qv.shape[0], v, qv[None], k, metric, window=True)
        assert status == s[0] == 0
        assert [r[0] for r in res] == list(i[0, :c[0]])
        assert [r[1] for r in res] == list(d[0, :c[0]])
        if oracle.ref_available():
            rs, rres = oracle.ref_gathered_exact(qv, v, k, metric)
            assert rres == res and rs == status
    # boundary ties (test_server.py:189-195)
    st, res = pb.search_gathered([(np.zeros(2, np.float32),
                                   np.array([[1, 0], [0, 1], [-1, 0], [0, -1], [3, 3]], np.float32), 1, 0)])[0]
    assert st == 0 and sorted(r[0] for r in res) == [0, 1, 2, 3]
    jobs_done = pb.backend().device_jobs
    import ctypes
    assert ctypes.CFUNCTYPE(ctypes.c_uint64)(jobs_done)() >= 13
    # one call, one submission: valid jobs beside ones the device rejects (a
    # non-finite row value: ANN_INVALID, cpu.c:246-251) and ones the host
    # settles, each answered as the reference answers it
    bad = jobs[1][1].copy()
    bad[7, 0] = np.inf
    mixed = [jobs[0], (jobs[1][0], bad, 10, 1), jobs[2], (jobs[3][0], jobs[3][1], 0, 0),
             (np.zeros(jobs[4][0].shape, np.float32), jobs[4][1], 5, 2), jobs[5]]
    got = pb.search_gathered(mixed)
    assert [g[0] for g in got] == [0, 1, 0, 0, 1, 0]
    for j in (0, 2, 5):
        qv, v, k, metric = mixed[j]
        d, i, c, s = oracle.search(oracle.F32, qv.shape[0], v, qv[None], k, metric, window=True)
        assert [r[0] for r in got[j][1]] == list(i[0, :c[0]]) and [r[1] for r in got[j][1]] == list(d[0, :c[0]])
    # a batch of 64 jobs in one call equals the jobs one at a time
    many = [jobs[j % 12] for j in range(64)]
    assert pb.search_gathered(many) == [pb.search_gathered([j])[0] for j in many]


def test_backend_in_memory_index(cuda):
    import ctypes
    import pgvector_b200 as pb
    from pgvector_b200 import _abi
    b = pb.backend()
    rng = np.random.default_rng(42)
    vectors = np.array([[rng.integers(-5, 6) for _ in range(7)] for _ in range(80)], dtype=np.float32)
    index = _abi.AnnIndex()
    assert b.build(ctypes.byref(index), 1, 80, 7, vectors.ctypes.data_as(ctypes.POINTER(ctypes.c_float))) == 0
    query = np.array([1, 2, 3, 4, 5, 1, 2], dtype=np.float32)
    ids = np.array(sorted(rng.choice(80, 25, replace=False)), dtype=np.uint32)
    for metric in range(3):
        for k in (1, 7, 100):
            res = (_abi.AnnCandidate * 100)()
            n = ctypes.c_uint32()
            st = b.search(ctypes.byref(index), query.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), metric,
                          ids.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)), len(ids), k, res, ctypes.byref(n))
            d, i, c, s = oracle.search(oracle.F32, 7, vectors, query[None], k, metric, ids=ids)
            assert st == 0 and n.value == c[0]
            assert [res[j].id for j in range(n.value)] == list(i[0, :c[0]])
            assert [res[j].distance for j in range(n.value)] == list(d[0, :c[0]])
    b.destroy(ctypes.byref(index))


# ---------------------------------------------------------------- typed gathered jobs

def test_typed_gathered_jobs(cuda):
    # AnnB200SearchTyped: host rows in every storage format, a batch of
    # queries each, window results equal to the oracle's window search
    import pgvector_b200 as pb
    d = 96
    x = synth.mixture(3000, d, 30, seed=31)
    q = synth.mixture_queries(24, d, 30, seed=32)
    h = synth.to_half_bits(x)
    c8, r8 = oracle.quantize_fp8(x)
    c4, b4, r4 = oracle.quantize_nvfp4(x)
    bits, proto = synth.bit_rows(3000, 256, 16, flip=0.05, seed=33)
    qb = bits[np.random.default_rng(34).integers(0, 3000, 20)].copy()
    cases = [
        (oracle.F32, 0, x, q, None, None, 10, d),
        (oracle.F32, 2, x, q[:1], None, None, 7, d),            # one query (CUDA cores)
        (oracle.F16, 2, h, q, None, None, 100, d),              # halfvec cosine, a tensor-core batch
        (oracle.E4M3, 1, c8, q, None, r8, 50, d),
        (oracle.NVFP4, 0, c4, q[:5], b4, r4, 20, d),
        (oracle.BIT, 3, bits, qb, None, None, 30, 256),         # Hamming: ties kept in the window
    ]
    jobs = [dict(dtype=dt, metric=m, dims=dims, k=k, queries=qs, codes=codes, block_scales=bs, row_scales=rs)
            for dt, m, codes, qs, bs, rs, k, dims in cases]
    for run in range(2):                                        # the lane's buffers reused
        got = pb.search_typed(jobs)
        for (dt, m, codes, qs, bs, rs, k, dims), (status, res) in zip(cases, got):
            od, oi, oc, os_ = oracle.search(dt, dims, codes, qs, k, m, block_scales=bs, row_scales=rs,
                                            window=True, cap=codes.shape[0])
            assert status == 0 and (os_ == 0).all()
            for qi in range(qs.shape[0]):
                want = [(int(oi[qi, r]), float(od[qi, r])) for r in range(oc[qi])]
                assert res[qi] == want, (dt, m, qi, res[qi][:4], want[:4])
    # a window that outgrows cap, and the rows' duplicates under Hamming
    dup = np.repeat(bits[:10], 50, axis=0)
    st, res = pb.search_typed([dict(dtype=oracle.BIT, metric=3, dims=256, k=1, queries=bits[:1], codes=dup,
                                    cap=10)])[0]
    assert st == pb.INVALID and res == [[]]


def test_typed_gathered_jobs_odd_shapes(cuda):
    # row pitches the tensor-core scan cannot read (CUDA-core path), padded
    # FP8 rows, odd NVFP4 block counts, a k past the rows, and a query batch
    # split into several jobs
    import pgvector_b200 as pb
    rng = np.random.default_rng(51)
    cases = []
    for d in (37, 20, 72):
        x = synth.mixture(700, d, 9, seed=d)
        q = synth.mixture_queries(18, d, 9, seed=d + 1)
        cases.append((oracle.F16, 0, synth.to_half_bits(x), q, None, None, 12, d))
        c8, r8 = oracle.quantize_fp8(x)
        cases.append((oracle.E4M3, 2, c8, q, None, r8, 5, d))
        c4, b4, r4 = oracle.quantize_nvfp4(x)
        cases.append((oracle.NVFP4, 1, c4, q, b4, r4, 900, d))   # k past the 700 rows
    bits = np.packbits(rng.random((500, 1000)) < 0.5, axis=1, bitorder='little')
    cases.append((oracle.BIT, 3, bits, bits[rng.integers(0, 500, 17)], None, None, 8, 1000))
    jobs = [dict(dtype=dt, metric=m, dims=dims, k=k, queries=qs, codes=codes, block_scales=bs, row_scales=rs)
            for dt, m, codes, qs, bs, rs, k, dims in cases]
    got = pb.search_typed(jobs)
    for (dt, m, codes, qs, bs, rs, k, dims), (status, res) in zip(cases, got):
        od, oi, oc, os_ = oracle.search(dt, dims, codes, qs, k, m, block_scales=bs, row_scales=rs, window=True,
                                        cap=codes.shape[0])
        assert status == 0 and (os_ == 0).all()
        for qi in range(qs.shape[0]):
            assert res[qi] == [(int(oi[qi, r]), float(od[qi, r])) for r in range(oc[qi])], (dt, dims, qi)


# ---------------------------------------------------------------- the benchmark configurations' batch and k

def test_config3_batch_e4m3_ip_k500(cuda):
    # config 3 at its batch and k on fewer rows: FP8-E4M3 rows with row
    # scales, inner product, d=1024, 1,024 queries, k=500, whole shard and a
    # 90% row list (both past the 32,768 rows below which no sample is taken)
    # rows from a 64-centre mixture; the device answers all 1,024 queries
    # (four 256-query tiles), the oracle checks every 8th (32 in each tile)
    x = synth.mixture(40000, 1024, 64, seed=301)
    q = synth.mixture_queries(1024, 1024, 64, seed=302)
    codes, rs = oracle.quantize_fp8(x)
    assert_same(cuda, oracle.E4M3, 1024, codes, q, 500, 1, rs=rs, check=np.arange(3, 1024, 8))
    _, ids = synth.bitmap(40000, 0.9, seed=303)
    assert_same(cuda, oracle.E4M3, 1024, codes, q, 500, 1, ids=ids, rs=rs, check=np.arange(5, 1024, 8))


def test_config5_batch_hamming_1024_queries(cuda):
    # config 5 at its batch and k: 1,024-bit rows XOR-perturbed (5%) from
    # prototypes, 1,024 queries (four query tiles), k=100; integer distances
    # with many ties, ordered by row id
    rows, proto = synth.bit_rows(120000, 1024, 512, flip=0.05, seed=501)
    rng = np.random.default_rng(502)
    qs = proto[rng.integers(0, 512, 1024)] ^ np.packbits(rng.random((1024, 1024)) < 0.05, axis=1,
                                                         bitorder='little')
    assert_same(cuda, oracle.BIT, 1024, rows, qs, 100, 3)
