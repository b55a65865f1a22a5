"""GPU parity of the IVF list gather (AnnB200SearchLists) against the oracle.

The reference's IVFFlat scan visits each query's probed lists, scores every
entry and orders them (src/ivfscan.c:124-186); oracle.search_lists restates
it. Bar: bit-exact ids, counts and FP64 distances, ties ordered by global id,
for every vector storage format and metric.
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
    if a.dtype == np.uint64:
        a = a.view(np.int64)
    return torch.from_numpy(a).to(cuda)


def encode(dtype, x):
    if dtype == oracle.F32:
        return x, None, None
    if dtype == oracle.F16:
        return synth.to_half_bits(x), None, None
    if dtype == oracle.E4M3:
        codes, rs = oracle.quantize_fp8(x)
        return codes, None, rs
    codes, bs, rs = oracle.quantize_nvfp4(x)
    return codes, bs, rs


def gpu_lists(cuda, dtype, dims, codes, bs, rs, q, offsets, probes, k, metric, row_ids=None, status=None,
              force_simt=False):
    import pgvector_b200 as pb
    shard = pb.Shard(dtype, dims, to_dev(codes, cuda), None if bs is None else to_dev(bs, cuda),
                     None if rs is None else to_dev(rs, cuda))
    d, i, c = shard.search_lists(to_dev(q, cuda), k, metric, to_dev(offsets, cuda), to_dev(probes, cuda),
                                 row_ids=None if row_ids is None else to_dev(row_ids, cuda), status=status,
                                 force_simt=force_simt)
    return d.cpu().numpy(), i.cpu().numpy(), c.cpu().numpy()


def assert_lists_same(cuda, dtype, dims, codes, bs, rs, q, offsets, probes, k, metric, row_ids=None,
                      force_simt=False, check=None):
    """The device answers the whole batch; the oracle answers the queries
    `check` selects (all by default) and those must be equal."""
    sel = np.arange(q.shape[0]) if check is None else np.asarray(check)
    od, oi, oc = oracle.search_lists(dtype, dims, codes, q[sel], offsets, probes[sel], k, metric, row_ids=row_ids,
                                     block_scales=bs, row_scales=rs)
    gd, gi, gc = gpu_lists(cuda, dtype, dims, codes, bs, rs, q, offsets, probes, k, metric, row_ids,
                           force_simt=force_simt)
    gd, gi, gc = gd[sel], gi[sel], gc[sel]
    assert np.array_equal(gc, oc.astype(gc.dtype)), (gc[:8], oc[:8])
    for j in range(len(sel)):
        c = int(oc[j])
        assert np.array_equal(gi[j, :c], oi[j, :c]), (j, gi[j, :c][:10], oi[j, :c][:10])
        assert np.array_equal(gd[j, :c], od[j, :c]), (j, gd[j, :c][:10], od[j, :c][:10])
    return oc


@pytest.mark.parametrize('dtype,dims,metric', [(0, 37, 0), (0, 37, 1), (0, 37, 2), (1, 96, 2), (1, 96, 0),
                                               (1, 200, 1), (2, 96, 1), (2, 200, 0), (3, 96, 0), (3, 256, 0),
                                               (3, 512, 2)])
@pytest.mark.parametrize('simt', [False, True])
def test_list_gather_formats_and_metrics(cuda, dtype, dims, metric, simt):
    # tensor cores for FP16 / E4M3 rows and NVFP4 rows whose scale rows are
    # a multiple of 16 bytes (dims % 256 == 0); CUDA cores otherwise and
    # with ANNB200_FORCE_SIMT
    x, offsets, cent, row_ids = synth.ivf_corpus(30000, dims, 128, seed=10 + dtype)
    q = synth.mixture_queries(48, dims, 16, seed=11)
    q = cent[np.arange(48) % 128] + 0.1 * q.astype(np.float32)
    probes = synth.ivf_probes(q, cent, 8)
    codes, bs, rs = encode(dtype, x)
    assert_lists_same(cuda, dtype, dims, codes, bs, rs, q.astype(np.float32), offsets, probes, 20, metric, row_ids,
                      force_simt=simt)


@pytest.mark.parametrize('simt', [False, True])
def test_config4_shape_nvfp4_l2(cuda, simt):
    # config 4's format and probe pattern at a size the oracle finishes quickly:
    # NVFP4 d=768, Zipf(1.1) list sizes, nprobe 64, k 100
    x, offsets, cent, row_ids = synth.ivf_corpus(60000, 768, 1024, seed=20)
    q = cent[np.random.default_rng(21).integers(0, 1024, 32)] + 0.1 * synth.mixture_queries(32, 768, 8, seed=21)
    probes = synth.ivf_probes(q, cent, 64)
    codes, bs, rs = oracle.quantize_nvfp4(x)
    assert_lists_same(cuda, oracle.NVFP4, 768, codes, bs, rs, q.astype(np.float32), offsets, probes, 100, 0,
                      row_ids, force_simt=simt)


def test_config4_batch_4096_nvfp4_l2(cuda):
    # config 4 at its batch, nprobe and k: NVFP4 d=768, 4,096 queries (64-query
    # groups of the tensor list scan, many groups a list), Zipf(1.1) list
    # sizes, nprobe 64, k 100; queries near uniformly chosen centres; the
    # oracle checks every 8th query
    x, offsets, cent, row_ids = synth.ivf_corpus(80000, 768, 512, seed=401)
    rng = np.random.default_rng(402)
    q = cent[rng.integers(0, 512, 4096)] + 0.1 * rng.standard_normal((4096, 768)).astype(np.float32)
    probes = synth.ivf_probes(q, cent, 64)
    codes, bs, rs = oracle.quantize_nvfp4(x)
    assert_lists_same(cuda, oracle.NVFP4, 768, codes, bs, rs, q.astype(np.float32), offsets, probes, 100, 0,
                      row_ids, check=np.arange(1, 4096, 8))


@pytest.mark.parametrize('dtype', [0, 1])
def test_ties_order_by_global_id_across_lists(cuda, dtype):
    # the same vector stored in several lists under different global ids:
    # equal distances must come out in id order whatever the storage order
    rng = np.random.default_rng(30)
    base = rng.standard_normal((50, 16)).astype(np.float32)
    x = np.concatenate([base, base, base, base])          # 4 lists of 50 identical rows
    codes, bs, rs = encode(dtype, x)
    offsets = np.array([0, 50, 100, 150, 200], dtype=np.uint64)
    row_ids = rng.permutation(200).astype(np.int64) * 3 + 7
    q = base[:6] + 0.01
    probes = np.tile(np.array([3, 0, 2, 1], dtype=np.uint32), (6, 1))
    for metric in (0, 1, 2):
        assert_lists_same(cuda, dtype, 16, codes, bs, rs, q, offsets, probes, 30, metric, row_ids)
    # without row_ids the ids are the storage rows
    assert_lists_same(cuda, dtype, 16, codes, bs, rs, q, offsets, probes, 30, 0)


@pytest.mark.parametrize('dtype', [0, 1])
def test_small_and_empty_lists_and_large_k(cuda, dtype):
    # empty lists, lists shorter than k, and a k past the shared-memory sort
    # (more than 4,096 survivors: the large-sort path)
    x, offsets, cent, row_ids = synth.ivf_corpus(20000, 32, 64, zipf=1.6, seed=40)
    codes, bs, rs = encode(dtype, x)
    sizes = np.diff(offsets.astype(np.int64))
    offsets2 = offsets.copy()
    offsets2[1:] = np.cumsum(np.where(np.arange(64) % 7 == 0, 0, sizes))   # every 7th list empty
    n2 = int(offsets2[-1])
    q = cent[:40] + 0.05
    probes = synth.ivf_probes(q, cent, 5)
    oc = assert_lists_same(cuda, dtype, 32, codes[:n2], None, None, q, offsets2, probes, 50, 0, row_ids[:n2])
    assert (oc < 50).any()       # some queries probe fewer than k rows
    assert_lists_same(cuda, dtype, 32, codes, None, None, q, offsets, probes, 5000, 0, row_ids)


def test_bad_probes_are_invalid_queries(cuda):
    import torch
    import pgvector_b200 as pb
    x, offsets, cent, _ = synth.ivf_corpus(5000, 16, 32, seed=50)
    q = cent[:4] + 0.05
    probes = synth.ivf_probes(q, cent, 4)
    probes[1, 2] = probes[1, 0]      # a duplicate list
    probes[2, 3] = 32                # a list past nlists
    status = torch.zeros((4,), dtype=torch.int32, device=cuda)
    with pytest.raises(pb.AnnB200Error):
        gpu_lists(cuda, oracle.F32, 16, x, None, None, q, offsets, probes, 5, 0, status=status)
    assert status.cpu().numpy().tolist() == [0, 1, 1, 0]
    good = probes[[0, 3]]
    od, oi, oc = oracle.search_lists(oracle.F32, 16, x, q[[0, 3]], offsets, good, 5, 0)
    gd, gi, gc = gpu_lists(cuda, oracle.F32, 16, x, None, None, q[[0, 3]], offsets, good, 5, 0)
    assert np.array_equal(gi, oi) and np.array_equal(gd, od)


@pytest.mark.parametrize('dtype', [0, 1])
def test_padding_probes_and_list_shards(cuda, dtype):
    # lists sharded over two "ranks": each shard sees only its own lists, the
    # others padded with UINT32_MAX; merging both shards' results gives the
    # unsharded answer
    import torch
    import pgvector_b200 as pb
    x, offsets, cent, row_ids = synth.ivf_corpus(30000, 48, 96, seed=70)
    x, _, _ = encode(dtype, x)
    q = cent[np.arange(40) % 96] + 0.05
    probes = synth.ivf_probes(q, cent, 10)
    od, oi, oc = oracle.search_lists(dtype, 48, x, q, offsets, probes, 25, 0, row_ids=row_ids)
    parts = []
    for l0, l1 in ((0, 50), (50, 96)):
        lo, hi = int(offsets[l0]), int(offsets[l1])
        local = np.where((probes >= l0) & (probes < l1), probes - l0, 0xffffffff).astype(np.uint32)
        off = (offsets[l0:l1 + 1] - offsets[l0]).astype(np.uint64)
        parts.append(gpu_lists(cuda, dtype, 48, x[lo:hi], None, None, q, off, local, 25, 0, row_ids[lo:hi]))
    gd = torch.from_numpy(np.stack([p[0] for p in parts])).to(cuda)
    gi = torch.from_numpy(np.stack([p[1] for p in parts])).to(cuda)
    gc = torch.from_numpy(np.stack([p[2] for p in parts]).astype(np.int32)).to(cuda)
    md, mi, mc = pb.merge_topk(gd, gi, gc, 25)
    assert np.array_equal(mc.cpu().numpy(), oc.astype(np.int32))
    assert np.array_equal(mi.cpu().numpy(), oi) and np.array_equal(md.cpu().numpy(), od)


def oracle_probes(dtype, dims, centres, q, nprobe, metric):
    # the nprobe nearest centroids by (exact distance, list number), padding past the lists
    od, oi, oc, _ = oracle.search(dtype, dims, centres, q, nprobe, metric)
    want = np.full((q.shape[0], nprobe), 0xffffffff, dtype=np.uint32)
    for j in range(q.shape[0]):
        want[j, :oc[j]] = oi[j, :oc[j]]
    return want


@pytest.mark.parametrize('dtype', [0, 1])
@pytest.mark.parametrize('nq', [48, 8])
def test_coarse_probe_matches_oracle(cuda, dtype, nq):
    # the coarse probe (src/ivfscan.c:48-122) as an exact search of the
    # centroids: 48 queries take the tensor scan (FP32 centres as two BF16
    # halves, or FP16), 8 the CUDA-core scan; a duplicated centre makes an
    # exact tie at the boundary (the lower list number is kept)
    import pgvector_b200 as pb
    rng = np.random.default_rng(90 + dtype)
    cent = rng.standard_normal((3000, 64)).astype(np.float32)
    cent[100] = cent[7]
    q = (cent[rng.integers(0, 3000, nq)] + 0.3 * rng.standard_normal((nq, 64))).astype(np.float32)
    q[0] = cent[7] + np.float32(0.01)
    codes, _, _ = encode(dtype, cent)
    shard = pb.Shard(dtype, 64, to_dev(codes, cuda))
    qd = to_dev(q, cuda)
    for metric in (0, 1, 2):
        for nprobe in (1, 16, 64):
            got = shard.probe_lists(qd, nprobe, metric).cpu().numpy().view(np.uint32)
            assert np.array_equal(got, oracle_probes(dtype, 64, codes, q, nprobe, metric)), (metric, nprobe)
    few = pb.Shard(dtype, 64, to_dev(codes[:10], cuda))           # fewer lists than probes: padding
    got = few.probe_lists(qd, 16, 0).cpu().numpy().view(np.uint32)
    assert np.array_equal(got, oracle_probes(dtype, 64, codes[:10], q, 16, 0))
    assert (got[:, 10:] == 0xffffffff).all()


def test_probe_then_list_scan_end_to_end(cuda):
    # queries -> coarse probe on the FP32 centres -> list scan: equals the
    # oracle's list scan over the oracle's probes
    import pgvector_b200 as pb
    x, offsets, cent, row_ids = synth.ivf_corpus(40000, 96, 256, seed=95)
    q = (cent[np.random.default_rng(96).integers(0, 256, 40)] + 0.05).astype(np.float32)
    codes = synth.to_half_bits(x)
    centres = pb.Shard(pb.F32, 96, to_dev(cent.astype(np.float32), cuda))
    rows = pb.Shard(pb.F16, 96, to_dev(codes, cuda))
    qd = to_dev(q, cuda)
    probes = centres.probe_lists(qd, 12, 0)
    d, i, c = rows.search_lists(qd, 30, 0, to_dev(offsets, cuda), probes, row_ids=to_dev(row_ids, cuda))
    want = oracle_probes(0, 96, cent.astype(np.float32), q, 12, 0)
    assert np.array_equal(probes.cpu().numpy().view(np.uint32), want)
    od, oi, oc = oracle.search_lists(oracle.F16, 96, codes, q, offsets, want, 30, 0, row_ids=row_ids)
    assert np.array_equal(c.cpu().numpy(), oc.astype(np.int32))
    assert np.array_equal(i.cpu().numpy(), oi) and np.array_equal(d.cpu().numpy(), od)
