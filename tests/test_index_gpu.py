"""Loaded on-disk indexes: the b200 backend's load_index / search_index
against the reference worker's own cpu backend on the same directory.

Both backends are driven through the worker's backend vtable
(ann/server/backend.h:114-151) in one process: the reference's cpu backend
and index registry from oracle/_ref/libannref.so (compiled from the
reference sources), and AnnB200WorkerBackend() from
oracle/_ref/libannb200_worker.so (pgvector_b200/csrc/worker_index.c linked
against that registry and libannb200.so, as the worker's build links it).
Bar: every hit's key, FP32 distance (bit for bit) and ordinal, the counts,
routes and statuses equal the cpu backend's (ann/server/cpu.c:298-407).
"""
import ctypes
import os

import numpy as np
import pytest

import oracle
from pgvector_b200 import _abi, synth

pytestmark = pytest.mark.gpu

WORKER_SO = os.path.join(os.path.dirname(oracle.REF_SO), 'libannb200_worker.so')


@pytest.fixture(scope='module')
def backends(cuda):
    if not (os.path.exists(oracle.REF_SO) and os.path.exists(WORKER_SO)):
        pytest.skip('reference worker library not built (make -C oracle ref worker)')
    import pgvector_b200 as pb
    pb.load()
    ref = ctypes.CDLL(oracle.REF_SO, mode=ctypes.RTLD_GLOBAL)
    ref.AnnCpuBackend.restype = ctypes.POINTER(_abi.AnnBackend)
    worker = ctypes.CDLL(WORKER_SO, mode=ctypes.RTLD_GLOBAL)
    worker.AnnB200WorkerBackend.restype = ctypes.POINTER(_abi.AnnBackend)
    return ref.AnnCpuBackend().contents, worker.AnnB200WorkerBackend().contents


def load(backend, name, directory):
    return _abi.LOAD_INDEX(backend.load_index)(name.encode(), directory.encode())


class Jobs:
    """A batch of AnnIndexJob with the buffers they point at kept alive."""

    def __init__(self):
        self.specs = []

    def add(self, name, query, k, keys=None, ordinals=None, exclude=None, dims=None, bitsets=None):
        """keys / ordinals / bitsets: arrays shared by every job given the
        same object (the server's same-filter jobs share their arrays);
        bitsets: a list of per-shard uint32 words."""
        self.specs.append(dict(name=name, query=np.ascontiguousarray(query, dtype=np.float32), k=k, keys=keys,
                               ordinals=ordinals, exclude=exclude, dims=dims, bitsets=bitsets))
        return self

    def run(self, backend, rename=None):
        n = len(self.specs)
        jobs = (_abi.AnnIndexJob * n)()
        keep = []
        shared = {}

        def arr_of(obj, dtype):
            # one C array per Python object: jobs given the same array share its pointer
            if id(obj) not in shared:
                shared[id(obj)] = np.ascontiguousarray(obj, dtype=dtype)
                keep.append(obj)
            return shared[id(obj)]
        for job, s in zip(jobs, self.specs):
            name = s['name'] if rename is None else rename.get(s['name'], s['name'])
            job.name = name.encode()
            job.dimensions = s['dims'] if s['dims'] is not None else s['query'].shape[0]
            job.k = s['k']
            job.query = s['query'].ctypes.data_as(ctypes.POINTER(ctypes.c_float))
            res = (_abi.AnnIndexHit * max(s['k'], 1))()
            job.results = res
            keep += [s['query'], res]
            if s['keys'] is not None:
                arr = arr_of(s['keys'], np.int64)
                job.filter = arr.ctypes.data_as(ctypes.POINTER(ctypes.c_int64))
                job.nfilter = len(arr)
                job.filtered = 1
            if s['ordinals'] is not None:
                arr = arr_of(s['ordinals'], np.uint64)
                job.ordinals = arr.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))
                job.nfilter = len(arr)
                job.filtered = 1
            if s['bitsets'] is not None:
                if id(s['bitsets']) not in shared:
                    words = [np.ascontiguousarray(w, dtype=np.uint32) for w in s['bitsets']]
                    ptrs = (ctypes.c_void_p * len(words))(*[w.ctypes.data for w in words])
                    shared[id(s['bitsets'])] = ptrs
                    keep += [words, ptrs, s['bitsets']]
                job.bitsets = ctypes.cast(shared[id(s['bitsets'])], ctypes.c_void_p)
                job.filtered = 1
                if s['keys'] is None and s['ordinals'] is None:
                    job.nfilter = sum(int(np.unpackbits(np.ascontiguousarray(w, dtype=np.uint32).view(np.uint8)).sum())
                                      for w in s['bitsets'])
            if s['exclude'] is not None:
                arr = np.ascontiguousarray(s['exclude'], dtype=np.uint64)
                job.exclude = arr.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))
                job.nexclude = len(arr)
                keep.append(arr)
        _abi.SEARCH_INDEX(backend.search_index)(jobs, n)
        out = []
        for job in jobs:
            hits = [(job.results[i].key, np.float32(job.results[i].distance).view(np.uint32).item(),
                     job.results[i].ordinal) for i in range(job.nresults)]
            out.append((job.status, job.route, hits))
        del keep
        return out


def assert_same_as_cpu(backends, jobs, ref_name, ours_name):
    cpu, ours = backends
    want = jobs.run(cpu, rename={'IX': ref_name})
    got = jobs.run(ours, rename={'IX': ours_name})
    assert len(want) == len(got)
    for i, (w, g) in enumerate(zip(want, got)):
        assert g[0] == w[0], (i, 'status', g[0], w[0])
        assert g[1] == w[1], (i, 'route', g[1], w[1])
        assert g[2] == w[2], (i, g[2][:5], w[2][:5])
    return want


def test_unfiltered_batch_and_filters(backends, tmp_path):
    rng = np.random.default_rng(7)
    n, d = 30000, 96
    x = synth.mixture(n, d, 60, seed=7)
    keys = rng.choice(np.arange(-10 ** 9, 10 ** 9), n, replace=False)
    skeys, rows = synth.write_index_dir(str(tmp_path / 'ix'), keys, x, shards=3)
    cpu, ours = backends
    assert load(cpu, 'cpu_a', str(tmp_path / 'ix')) == 0
    assert load(ours, 'b200_a', str(tmp_path / 'ix')) == 0
    q = synth.mixture_queries(48, d, 60, seed=8)
    jobs = Jobs()
    for i in range(40):                       # one unfiltered batch (tensor-path size), mixed k
        jobs.add('IX', q[i], (10, 50, 100, 7)[i % 4])
    sel = np.sort(rng.choice(skeys, 3000, replace=False))
    missing = np.setdiff1d(rng.integers(-10 ** 9, 10 ** 9, 50), skeys)
    jobs.add('IX', q[40], 25, keys=np.sort(np.concatenate([sel, missing])))       # key filter, some unknown
    ords = np.sort(rng.choice(n, 500, replace=False))
    jobs.add('IX', q[41], 30, ordinals=ords)                                        # ordinals given
    jobs.add('IX', q[42], 30, ordinals=ords, exclude=ords[::3])                     # residual exclusions
    jobs.add('IX', q[43], 50, keys=sel[:20])                                        # k past the eligible rows
    jobs.add('IX', q[44], 10, keys=np.array([], dtype=np.int64))                    # empty filter
    jobs.add('IX', q[45], 0)                                                        # k = 0
    jobs.add('missing_index', q[46], 10)                                            # not loaded: ANN_STALE
    jobs.add('IX', q[47][:90], 10, dims=90)                                         # dimension mismatch
    want = assert_same_as_cpu(backends, jobs, 'cpu_a', 'b200_a')
    assert want[0][0] == 0 and len(want[0][2]) == 10
    assert want[-2][0] == 3            # ANN_STALE
    assert want[-1][0] == 1            # ANN_INVALID


def test_ties_and_duplicate_rows(backends, tmp_path):
    # identical rows under different keys: equal FP32 distances order by key
    rng = np.random.default_rng(9)
    base = rng.standard_normal((100, 24)).astype(np.float32)
    x = np.concatenate([base] * 30)
    keys = rng.permutation(len(x)) * 7 - 5000
    synth.write_index_dir(str(tmp_path / 'ties'), keys, x, shards=2)
    cpu, ours = backends
    assert load(cpu, 'cpu_t', str(tmp_path / 'ties')) == 0
    assert load(ours, 'b200_t', str(tmp_path / 'ties')) == 0
    jobs = Jobs()
    for i in range(20):
        jobs.add('IX', base[i] + 1e-3 * i, 45)
    jobs.add('IX', base[3], 61, ordinals=np.arange(0, len(x), 2))
    assert_same_as_cpu(backends, jobs, 'cpu_t', 'b200_t')


def test_odd_dimensions_and_single_query(backends, tmp_path):
    rng = np.random.default_rng(11)
    x = rng.standard_normal((5000, 37)).astype(np.float32) * 3
    keys = np.arange(5000) * 3 + 1
    synth.write_index_dir(str(tmp_path / 'odd'), keys, x, shards=1)
    cpu, ours = backends
    assert load(cpu, 'cpu_o', str(tmp_path / 'odd')) == 0
    assert load(ours, 'b200_o', str(tmp_path / 'odd')) == 0
    jobs = Jobs().add('IX', rng.standard_normal(37), 17)
    assert_same_as_cpu(backends, jobs, 'cpu_o', 'b200_o')


def test_rescore_rows_kernel(cuda):
    # AnnB200RescoreRows against the restated ExactDistance
    # (ann/server/cuvs.c:2930-2942), over the 16-byte and the scalar loads
    import torch
    import pgvector_b200 as pb
    lib = pb.load()
    rng = np.random.default_rng(13)
    for d, shift in ((64, 0), (64, 1), (37, 0), (3, 0)):
        nq, stride = 5, 40
        q = (rng.standard_normal((nq, d)) * 3).astype(np.float32)
        rows = (rng.standard_normal((nq, stride, d)) * 10 ** rng.uniform(-2, 2, (nq, stride, 1))).astype(np.float32)
        counts = np.array([40, 0, 17, 1, 39], dtype=np.uint32)
        qd = torch.from_numpy(q).to(cuda)
        flat = torch.zeros(nq * stride * d + shift, dtype=torch.float32, device=cuda)
        flat[shift:] = torch.from_numpy(rows.ravel()).to(cuda)
        cd = torch.from_numpy(counts.view(np.int32)).to(cuda)
        out = torch.full((nq, stride), -1.0, dtype=torch.float32, device=cuda)
        st = lib.AnnB200RescoreRows(ctypes.c_void_p(qd.data_ptr()), nq, d,
                                    ctypes.c_void_p(flat.data_ptr() + 4 * shift), stride,
                                    ctypes.c_void_p(cd.data_ptr()), ctypes.c_void_p(out.data_ptr()),
                                    ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
        assert st == 0
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        for i in range(nq):
            c = int(counts[i])
            want = oracle.exact_distance_f64(rows[i, :c], q[i])
            assert np.array_equal(got[i, :c].view(np.uint32), want.view(np.uint32)), (d, shift, i)
            assert np.all(got[i, c:] == -1.0)


def _eligible(skeys, spec):
    """A job's eligible ordinals as the worker resolves them (None: all)."""
    if spec.get('keys') is not None:
        pos = np.searchsorted(skeys, spec['keys'])
        ok = (pos < len(skeys)) & (skeys[np.minimum(pos, len(skeys) - 1)] == spec['keys'])
        elig = pos[ok].astype(np.uint64)
    elif spec.get('ordinals') is not None:
        elig = np.asarray(spec['ordinals'], dtype=np.uint64)
    else:
        return None
    if spec.get('exclude') is not None:
        elig = np.setdiff1d(elig, np.asarray(spec['exclude'], dtype=np.uint64))
    return elig


@pytest.mark.parametrize('kind,d', [('fp8', 96), ('nvfp4', 96), ('nvfp4', 72)])
def test_quantized_copy_route(backends, tmp_path, monkeypatch, kind, d):
    # an index served from its quantized copy: the reference's quantized scan
    # route (SearchGather, ann/server/cuvs.c:4585-4930) against its
    # restatement (oracle.quant_index_search), bit for bit, and its recall
    # against the cpu backend's exact answer
    rng = np.random.default_rng(21)
    n = 24000
    x = synth.mixture(n, d, 60, seed=21)
    keys = rng.choice(np.arange(-10 ** 9, 10 ** 9), n, replace=False)
    order = np.argsort(keys, kind='stable')
    if kind == 'fp8':
        codes, rs = oracle.quantize_fp8(x)
        quant, bs, dt = ('fp8', codes, rs), None, oracle.E4M3
    else:
        codes, bs, rs = oracle.quantize_nvfp4(x)
        quant, dt = ('nvfp4', codes, bs, rs), oracle.NVFP4
    directory = str(tmp_path / ('q_%s_%d' % (kind, d)))
    skeys, xs = synth.write_index_dir(directory, keys, x, shards=3, quant=quant)
    cs, rss, bss = codes[order], rs[order], None if bs is None else bs[order]
    bounds = [n * i // 3 for i in range(4)]
    cpu, ours = backends
    ref_name, our_name = 'cpu_q_%s_%d' % (kind, d), 'b200_q_%s_%d' % (kind, d)
    assert load(cpu, ref_name, directory) == 0
    monkeypatch.setenv('ANN_B200_INDEX_COPY', 'quant')
    # 8 MB of staged rows a chunk: the 32-query batch runs as two chunks
    # (27 queries on the tensor-core scan, then 5), the second one's rows
    # copied while the first is re-scored
    monkeypatch.setenv('ANN_B200_QUANT_STAGE_MB', '8')
    assert load(ours, our_name, directory) == 0
    q = synth.mixture_queries(48, d, 60, seed=22)
    jobs = Jobs()
    for i in range(32):                              # one tensor-path batch at k = 10
        jobs.add('IX', q[i], 10)
    for i in range(32, 40):                          # a small batch at k = 100
        jobs.add('IX', q[i], 100)
    sel = np.sort(rng.choice(skeys, 3000, replace=False))
    missing = np.setdiff1d(rng.integers(-10 ** 9, 10 ** 9, 50), skeys)
    jobs.add('IX', q[40], 25, keys=np.sort(np.concatenate([sel, missing])))
    ords = np.sort(rng.choice(n, 500, replace=False))
    jobs.add('IX', q[41], 30, ordinals=ords)
    jobs.add('IX', q[42], 30, ordinals=ords, exclude=ords[::3])
    jobs.add('IX', q[43], 50, keys=sel[:20])         # k past the eligible rows
    jobs.add('IX', q[44], 10, keys=np.array([], dtype=np.int64))
    jobs.add('IX', q[45], 0)
    jobs.add('IX', q[46], 300)                       # k + slack = 600 candidates a shard
    got = jobs.run(ours, rename={'IX': our_name})
    exact = jobs.run(cpu, rename={'IX': ref_name})
    found = total = 0
    for i, (spec, g, e) in enumerate(zip(jobs.specs, got, exact)):
        elig = _eligible(skeys, spec)
        want = oracle.quant_index_search(dt, xs, cs, spec['query'][None], spec['k'], bounds, ordinals=elig,
                                         block_scales=bss, row_scales=rss)[0]
        hits = [(int(skeys[o]), dist.view(np.uint32).item(), o) for o, dist in want]
        assert g[0] == 0, (i, 'status', g[0])
        assert g[1] == 2, (i, 'route', g[1])                        # ANN_ROUTE_EXACT
        assert g[2] == hits, (i, g[2][:4], hits[:4])
        found += len({h[0] for h in g[2]} & {h[0] for h in e[2]})
        total += len(e[2])
    recall = found / total
    print('%s d=%d recall against the exact FP32 answer: %.4f' % (kind, d, recall))
    assert recall >= 0.97


def test_quantized_index_and_typed_jobs_from_threads(cuda):
    # the worker calls from many lane threads at once: each thread stages
    # through its own buffers, searches of one shard take turns on its lock,
    # and every thread's answers equal the one-thread answers
    import threading
    import pgvector_b200 as pb
    lib = pb.load()
    n, d = 20000, 64
    x = synth.mixture(n, d, 40, seed=41)
    q = synth.mixture_queries(64, d, 40, seed=42)
    codes, bs, rs = oracle.quantize_nvfp4(x)
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    ix = ctypes.c_void_p()
    shard_rows = (ctypes.c_uint64 * 2)(12000, 8000)
    assert lib.AnnB200IndexCreateQuant(0, d, n, pb.NVFP4, P(codes), P(bs), P(rs), P(x), 2, shard_rows, 64, 100,
                                       ctypes.byref(ix)) == 0

    def index_search(part, k):
        qs = np.ascontiguousarray(q[part * 16:(part + 1) * 16])
        dist = np.zeros((16, k), np.float32)
        ords = np.zeros((16, k), np.uint64)
        cnt = np.zeros(16, np.uint32)
        assert lib.AnnB200IndexSearch(ix, P(qs), 16, None, 0, k, P(dist), P(ords), P(cnt)) == 0
        return dist.view(np.uint32).tolist(), ords.tolist(), cnt.tolist()

    h = synth.to_half_bits(x)

    def typed(part):
        return pb.search_typed([dict(dtype=pb.F16, metric=pb.L2, dims=d, k=5 + part, codes=h[part::4],
                                     queries=q[part * 16:(part + 1) * 16])])

    try:
        want = [(index_search(p, 10 + p), typed(p)) for p in range(4)]
        got = [None] * 4
        errors = []

        def run(p):
            try:
                for _ in range(3):
                    got[p] = (index_search(p, 10 + p), typed(p))
                    assert got[p] == want[p]
            except Exception as e:              # surfaced below, with the thread's part
                errors.append((p, repr(e)))

        threads = [threading.Thread(target=run, args=(p,)) for p in range(4)]
        for t in threads:
            t.start()
        for t in threads:
            t.join(300)
        assert not errors, errors
        assert got == want
    finally:
        lib.AnnB200IndexDestroy(ix)


def test_rescore_gather_kernel(cuda):
    # AnnB200RescoreGather: rows fetched by ordinal, the restated ExactDistance
    import torch
    import pgvector_b200 as pb
    lib = pb.load()
    rng = np.random.default_rng(17)
    for d in (768, 37, 1100):                   # one, a partial, and three row chunks
        n, nq, stride = 3000, 4, 50
        x = (rng.standard_normal((n, d)) * 10 ** rng.uniform(-2, 2, (n, 1))).astype(np.float32)
        q = rng.standard_normal((nq, d)).astype(np.float32)
        ords = rng.integers(0, n, (nq, stride)).astype(np.uint64)
        counts = np.array([50, 0, 23, 1], dtype=np.uint32)
        xd, qd = torch.from_numpy(x).to(cuda), torch.from_numpy(q).to(cuda)
        od = torch.from_numpy(ords.view(np.int64)).to(cuda)
        cd = torch.from_numpy(counts.view(np.int32)).to(cuda)
        out = torch.full((nq, stride), -1.0, dtype=torch.float32, device=cuda)
        assert lib.AnnB200RescoreGather(ctypes.c_void_p(qd.data_ptr()), nq, d, ctypes.c_void_p(xd.data_ptr()),
                                        ctypes.c_void_p(od.data_ptr()), stride, ctypes.c_void_p(cd.data_ptr()),
                                        ctypes.c_void_p(out.data_ptr()),
                                        ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)) == 0
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        for i in range(nq):
            c = int(counts[i])
            want = oracle.exact_distance_f64(x[ords[i, :c].astype(np.int64)], q[i])
            assert np.array_equal(got[i, :c].view(np.uint32), want.view(np.uint32)), (d, i)
            assert np.all(got[i, c:] == -1.0)


@pytest.mark.parametrize('mapped', ['1', '0'])
def test_quantized_index_rows_in_place_or_copied(cuda, monkeypatch, capfd, mapped):
    # the quantized route with the FP32 rows read in place by the device
    # (registered host memory) and copied through staging: both equal the
    # restated route
    import pgvector_b200 as pb
    lib = pb.load()
    n, d = 30000, 128
    x = synth.mixture(n, d, 50, seed=61)
    q = synth.mixture_queries(40, d, 50, seed=62)
    codes, rs = oracle.quantize_fp8(x)
    monkeypatch.setenv('ANN_B200_QUANT_MAPPED', mapped)
    monkeypatch.setenv('ANN_B200_DEBUG', '1')
    monkeypatch.setenv('ANN_B200_QUANT_STAGE_MB', '16')     # several chunks
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    ix = ctypes.c_void_p()
    shard_rows = (ctypes.c_uint64 * 3)(10000, 15000, 5000)
    assert lib.AnnB200IndexCreateQuant(0, d, n, pb.E4M3, P(codes), None, P(rs), P(x), 3, shard_rows, 32, 150,
                                       ctypes.byref(ix)) == 0
    try:
        assert ('read in place' in capfd.readouterr().err) == (mapped == '1')
        ords_f = np.sort(np.random.default_rng(63).choice(n, 4000, replace=False)).astype(np.uint64)
        for k, filt in ((10, None), (40, ords_f)):
            dist = np.zeros((40, k), np.float32)
            ords = np.zeros((40, k), np.uint64)
            cnt = np.zeros(40, np.uint32)
            assert lib.AnnB200IndexSearch(ix, P(q), 40, None if filt is None else P(filt),
                                          0 if filt is None else len(filt), k, P(dist), P(ords), P(cnt)) == 0
            want = oracle.quant_index_search(oracle.E4M3, x, codes, q, k, [0, 10000, 25000, n], ordinals=filt,
                                             row_scales=rs, quant_slack=32, slack_ratio=150, threads=8)
            for i in range(40):
                assert cnt[i] == len(want[i])
                assert [int(o) for o in ords[i, :cnt[i]]] == [o for o, _ in want[i]], (k, i)
                assert dist[i, :cnt[i]].view(np.uint32).tolist() == [w.view(np.uint32).item() for _, w in want[i]]
    finally:
        lib.AnnB200IndexDestroy(ix)


def test_quantized_index_registration_cap_and_release(cuda, monkeypatch, capfd):
    # the registration cap sends a large row array to the copy path; two
    # indexes over one array: the second cannot register the pages again,
    # copies instead and answers the same; once both are destroyed the pages
    # register again (the first index released them)
    import pgvector_b200 as pb
    lib = pb.load()
    n, d = 12000, 96
    x = synth.mixture(n, d, 30, seed=71)
    q = synth.mixture_queries(24, d, 30, seed=72)
    codes, rs = oracle.quantize_fp8(x)
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    monkeypatch.setenv('ANN_B200_DEBUG', '1')

    def create():
        ix = ctypes.c_void_p()
        st = lib.AnnB200IndexCreateQuant(0, d, n, pb.E4M3, P(codes), None, P(rs), P(x), 0, None, 32, 100,
                                         ctypes.byref(ix))
        assert st == 0, (st, lib.AnnB200LastError(), capfd.readouterr().err)
        return ix, capfd.readouterr().err

    def answer(ix):
        dist = np.zeros((24, 10), np.float32)
        ords = np.zeros((24, 10), np.uint64)
        cnt = np.zeros(24, np.uint32)
        assert lib.AnnB200IndexSearch(ix, P(q), 24, None, 0, 10, P(dist), P(ords), P(cnt)) == 0
        return dist.view(np.uint32).tolist(), ords.tolist(), cnt.tolist()

    monkeypatch.setenv('ANN_B200_QUANT_MAP_MAX_MB', '1')          # the rows take 4.6 MB
    capped, err = create()
    assert 'registration cap' in err and 'read in place' not in err
    monkeypatch.delenv('ANN_B200_QUANT_MAP_MAX_MB')
    first, err1 = create()
    second, err2 = create()
    try:
        assert 'read in place' in err1
        assert 'registration failed' in err2 and 'read in place' not in err2
        a, b, c = answer(first), answer(second), answer(capped)
        assert a == b == c
        want = oracle.quant_index_search(oracle.E4M3, x, codes, q, 10, [0, n], row_scales=rs, quant_slack=32,
                                         slack_ratio=100, threads=8)
        assert a[1] == [[o for o, _ in w] + [0] * (10 - len(w)) for w in want]
    finally:
        lib.AnnB200IndexDestroy(first)
        lib.AnnB200IndexDestroy(second)
        lib.AnnB200IndexDestroy(capped)
    third, err3 = create()
    lib.AnnB200IndexDestroy(third)
    assert 'read in place' in err3


def shard_bitsets(n, shards, ordinals):
    """Per-shard bitsets (uint32 words, bit r of shard s = row first_s + r)
    of a sorted ordinal list, over write_index_dir's shard bounds."""
    bounds = [n * i // shards for i in range(shards + 1)]
    out = []
    for s in range(shards):
        lo, hi = bounds[s], bounds[s + 1]
        sel = ordinals[(ordinals >= lo) & (ordinals < hi)] - lo
        bits = np.zeros(((hi - lo + 31) // 32) * 32, dtype=np.uint8)
        bits[sel.astype(np.int64)] = 1
        out.append(np.packbits(bits, bitorder='little').view(np.uint32))
    return out, bounds


def test_same_filter_groups_and_bitset_forms(backends, tmp_path):
    # jobs sharing one filter's arrays run as one batched search (the
    # tensor-core path from 16 queries); the filter's per-shard bitsets are
    # expanded on the device instead of uploading ordinals; answers equal
    # the cpu backend's, job by job
    rng = np.random.default_rng(17)
    n, d, shards = 40000, 64, 3
    x = synth.mixture(n, d, 40, seed=17)
    keys = rng.choice(np.arange(-10 ** 9, 10 ** 9), n, replace=False)
    skeys, rows = synth.write_index_dir(str(tmp_path / 'grp'), keys, x, shards=shards)
    cpu, ours = backends
    assert load(cpu, 'cpu_g', str(tmp_path / 'grp')) == 0
    assert load(ours, 'b200_g', str(tmp_path / 'grp')) == 0
    q = synth.mixture_queries(80, d, 40, seed=18)
    ords_a = np.sort(rng.choice(n, 9000, replace=False)).astype(np.uint64)
    ords_b = np.sort(rng.choice(n, 700, replace=False)).astype(np.uint64)
    keys_c = np.sort(rng.choice(skeys, 4000, replace=False))
    bits_a, _ = shard_bitsets(n, shards, ords_a)
    jobs = Jobs()
    for i in range(24):                    # group 1: one ordinal array, with its bitsets
        jobs.add('IX', q[i], (10, 40, 100)[i % 3], ordinals=ords_a, bitsets=bits_a)
    for i in range(24, 44):                # group 2: one key array
        jobs.add('IX', q[i], 25, keys=keys_c)
    for i in range(44, 50):                # group 3: a small ordinal array, interleaved with unfiltered jobs
        jobs.add('IX', q[i], 30, ordinals=ords_b)
        jobs.add('IX', q[i + 20], 12)
    jobs.add('IX', q[70], 30, ordinals=np.array(ords_b))   # same values, its own array: its own search
    assert_same_as_cpu(backends, jobs, 'cpu_g', 'b200_g')
    # bitsets alone (a filter the server keeps only as bitsets): the same
    # answers as the ordinal list they encode
    alone, listed = Jobs(), Jobs()
    for i in range(20):
        alone.add('IX', q[i], 33, bitsets=bits_a)
        listed.add('IX', q[i], 33, ordinals=ords_a)
    got = alone.run(ours, rename={'IX': 'b200_g'})
    want = listed.run(ours, rename={'IX': 'b200_g'})
    assert got == want and all(g[0] == 0 and len(g[2]) == 33 for g in got)


def test_bitsets_kept_on_device(cuda):
    # AnnB200IndexKeepBitsets / AnnB200IndexSearchBitsets(ANNB200_BITSETS_DEVICE):
    # the cached-bitmap form kept on the device answers as the ordinal list,
    # including shards with no bitset and shards whose rows are not a
    # multiple of 32
    import pgvector_b200 as pb
    lib = pb.load()
    rng = np.random.default_rng(19)
    n, d, shards = 30001, 48, 4
    x = synth.mixture(n, d, 30, seed=19)
    q = synth.mixture_queries(40, d, 30, seed=20)
    ords = np.sort(rng.choice(n, 6000, replace=False)).astype(np.uint64)
    bits, bounds = shard_bitsets(n, shards, ords)
    bits[2] = None
    ords = ords[(ords < bounds[2]) | (ords >= bounds[3])]
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    ix = ctypes.c_void_p()
    assert lib.AnnB200IndexCreate(0, d, n, P(x), ctypes.byref(ix)) == 0
    try:
        assert lib.AnnB200IndexDevice(ix) == 0
        first = np.array(bounds[:-1], dtype=np.uint64)
        count = np.diff(np.array(bounds, dtype=np.uint64))
        host = (ctypes.c_void_p * shards)(*[None if b is None else b.ctypes.data for b in bits])
        dev = (ctypes.c_void_p * shards)()
        assert lib.AnnB200IndexKeepBitsets(ix, shards, host, P(count), dev) == 0
        assert dev[2] is None and all(dev[s] for s in (0, 1, 3))

        def search(kind, k):
            dist = np.zeros((40, k), np.float32)
            o = np.zeros((40, k), np.uint64)
            cnt = np.zeros(40, np.uint32)
            if kind == 'ords':
                st = lib.AnnB200IndexSearch(ix, P(q), 40, P(ords), len(ords), k, P(dist), P(o), P(cnt))
            else:
                st = lib.AnnB200IndexSearchBitsets(ix, P(q), 40, shards, dev if kind == 'device' else host, P(first),
                                                   P(count), 1 if kind == 'device' else 0, k, P(dist), P(o), P(cnt))
            assert st == 0
            return dist.view(np.uint32).tolist(), o.tolist(), cnt.tolist()
        for k in (10, 100):
            assert search('device', k) == search('ords', k) == search('host', k)
        lib.AnnB200IndexDropBitsets(ix, shards, dev)
        assert all(dev[s] is None for s in range(shards))
    finally:
        lib.AnnB200IndexDestroy(ix)


def test_fp16_copy_route_library(cuda):
    # AnnB200IndexCreateQuant(ANNB200_F16, codes NULL): the FP32 rows kept as
    # FP16 on the device (made there, round to nearest), each shard's k + slack
    # nearest by the FP16 rows, their FP32 rows re-scored: equal to the
    # restated route over the same FP16 rows
    import pgvector_b200 as pb
    lib = pb.load()
    n, d = 24000, 72
    x = synth.mixture(n, d, 40, seed=81)
    q = synth.mixture_queries(40, d, 40, seed=82)
    h = x.astype(np.float16)
    P = lambda a: a.ctypes.data_as(ctypes.c_void_p)
    ix = ctypes.c_void_p()
    shard_rows = (ctypes.c_uint64 * 2)(9000, 15000)
    assert lib.AnnB200IndexCreateQuant(0, d, n, pb.F16, None, None, None, P(x), 2, shard_rows, 32, 120,
                                       ctypes.byref(ix)) == 0
    try:
        assert lib.AnnB200IndexCopyRoute(ix) == 1
        filt = np.sort(np.random.default_rng(83).choice(n, 3000, replace=False)).astype(np.uint64)
        for k, ords in ((10, None), (50, filt)):
            dist = np.zeros((40, k), np.float32)
            o = np.zeros((40, k), np.uint64)
            cnt = np.zeros(40, np.uint32)
            assert lib.AnnB200IndexSearch(ix, P(q), 40, None if ords is None else P(ords),
                                          0 if ords is None else len(ords), k, P(dist), P(o), P(cnt)) == 0
            want = oracle.quant_index_search(oracle.F16, x, h.view(np.uint16), q, k, [0, 9000, n], ordinals=ords,
                                             quant_slack=32, slack_ratio=120, threads=8)
            for i in range(40):
                assert cnt[i] == len(want[i])
                assert [int(v) for v in o[i, :cnt[i]]] == [w for w, _ in want[i]], (k, i)
                assert dist[i, :cnt[i]].view(np.uint32).tolist() == [w.view(np.uint32).item() for _, w in want[i]]
    finally:
        lib.AnnB200IndexDestroy(ix)


def test_float16_directory_served_from_fp16_copy(backends, tmp_path):
    # a "dtype float16" directory: the worker keeps an FP16 copy on the
    # device and answers by the FP16 route (route ANN_ROUTE_EXACT), its hits
    # those of the restated route
    rng = np.random.default_rng(85)
    n, d = 20000, 40
    x = synth.mixture(n, d, 30, seed=85)
    keys = rng.choice(np.arange(-10 ** 8, 10 ** 8), n, replace=False)
    skeys, rows = synth.write_index_dir(str(tmp_path / 'h'), keys, x, shards=2, dtype='float16')
    cpu, ours = backends
    assert load(ours, 'b200_h', str(tmp_path / 'h')) == 0
    q = synth.mixture_queries(20, d, 30, seed=86)
    jobs = Jobs()
    for i in range(20):
        jobs.add('IX', q[i], 15)
    got = jobs.run(ours, rename={'IX': 'b200_h'})
    # the worker's defaults: --quant-slack 256, --slack-ratio 100 (AnnIndexConfig)
    want = oracle.quant_index_search(oracle.F16, rows, rows.astype(np.float16).view(np.uint16), q, 15,
                                     [0, n // 2, n], quant_slack=256, slack_ratio=100, threads=8)
    for (status, route, hits), w in zip(got, want):
        assert status == 0 and route == 2
        assert [h[2] for h in hits] == [o for o, _ in w]
        assert [h[1] for h in hits] == [v.view(np.uint32).item() for _, v in w]
        assert [h[0] for h in hits] == [int(skeys[o]) for o, _ in w]
