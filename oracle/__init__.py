"""CPU oracle for the exact gather-scan -- TEST INFRASTRUCTURE ONLY.

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this package, as the checker. The product (pgvector_b200) never imports it.

Two libraries:
  * liboracle.so  -- this repo's C restatement (oracle/oracle.c): decoders,
    quantizers and exact search for every storage format and metric.
  * _ref/libannref.so -- the reference's own cpu.c / indexfile.c compiled
    from the reference sources by oracle/Makefile (absent when the reference
    tree is not on this machine). Used to pin the restatement and as the
    timed CPU baseline.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, 'liboracle.so')
REF_SO = os.path.join(HERE, '_ref', 'libannref.so')

F32, F16, E4M3, NVFP4, BIT = 0, 1, 2, 3, 4

_lib = None
_ref = None

P = ctypes.c_void_p
u32, u64, i32, i64, f64 = ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int32, ctypes.c_int64, ctypes.c_double


def build(reference=None):
    """make -C oracle (and the reference library when its sources exist)."""
    # the reference tree: ANN_REFERENCE, else a `reference` directory beside
    # this repository
    ref = reference or os.environ.get('ANN_REFERENCE') or os.path.join(os.path.dirname(os.path.dirname(HERE)),
                                                                       'reference')
    subprocess.run(['make', '-s', '-C', HERE, 'all'], check=True)
    if os.path.isdir(os.path.join(ref, 'ann', 'server')):
        subprocess.run(['make', '-s', '-C', HERE, 'ref', 'REF=' + ref], check=True)
        if os.path.exists(os.path.join(os.path.dirname(HERE), 'pgvector_b200', 'libannb200.so')):
            subprocess.run(['make', '-s', '-C', HERE, 'worker', 'REF=' + ref], check=True)
            # the reference worker with the typed search operation (both backends)
            from . import worker_typed
            worker_typed.build(ref)


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(ORACLE_SO):
            subprocess.run(['make', '-s', '-C', HERE, 'all'], check=True)
        L = ctypes.CDLL(ORACLE_SO)
        L.orc_half_to_float.restype = ctypes.c_float
        L.orc_half_to_float.argtypes = [ctypes.c_uint16]
        L.orc_float_to_half.restype = ctypes.c_uint16
        L.orc_float_to_half.argtypes = [ctypes.c_float]
        L.orc_e4m3.restype = ctypes.c_float
        L.orc_e4m3.argtypes = [ctypes.c_uint8]
        L.orc_e2m1.restype = ctypes.c_float
        L.orc_e2m1.argtypes = [ctypes.c_uint8]
        L.orc_row_bytes.restype = u64
        L.orc_row_bytes.argtypes = [u32, u32]
        L.orc_search.restype = ctypes.c_int
        L.orc_search.argtypes = [u32, u32, u64, P, P, P, P, u32, P, u64, u32, u32, ctypes.c_int, u64,
                                 P, P, P, P, ctypes.c_int]
        L.orc_search_lists.restype = ctypes.c_int
        L.orc_search_lists.argtypes = [u32, u32, u64, P, P, P, P, P, u32, P, u32, P, u32, u32, u32, P, P, P,
                                       ctypes.c_int]
        L.orc_quantize_fp8.restype = None
        L.orc_quantize_fp8.argtypes = [P, u64, u32, P, P]
        L.orc_quantize_nvfp4.restype = None
        L.orc_quantize_nvfp4.argtypes = [P, u64, u32, P, P, P]
        L.orc_decode_rows.restype = None
        L.orc_decode_rows.argtypes = [u32, u32, u64, u64, P, P, P, P, ctypes.c_int]
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(P)


def row_bytes(dtype, dims):
    return int(lib().orc_row_bytes(dtype, dims))


def search(dtype, dims, codes, queries, k, metric, ids=None, block_scales=None, row_scales=None,
           window=False, cap=None, threads=None):
    """Exact search; returns (dist [nq][cap] f64, id [nq][cap] i64, count [nq], status [nq])."""
    codes = np.ascontiguousarray(codes)
    rows = codes.shape[0]
    queries = np.ascontiguousarray(queries)
    nq = queries.shape[0]
    ids_a = None if ids is None else np.ascontiguousarray(ids, dtype=np.uint32)
    n = rows if ids_a is None else ids_a.shape[0]
    cap = int(cap if cap is not None else (max(n, 1) if window else max(k, 1)))
    dist = np.full((nq, cap), np.inf)
    out_id = np.full((nq, cap), -1, dtype=np.int64)
    count = np.zeros(nq, dtype=np.uint32)
    status = np.zeros(nq, dtype=np.int32)
    bs = None if block_scales is None else np.ascontiguousarray(block_scales, dtype=np.uint8)
    rs = None if row_scales is None else np.ascontiguousarray(row_scales, dtype=np.float32)
    lib().orc_search(dtype, dims, rows, _p(codes), _p(bs), _p(rs), _p(queries), nq, _p(ids_a),
                     0 if ids_a is None else ids_a.shape[0], k, metric, 1 if window else 0, cap,
                     _p(dist), _p(out_id), _p(count), _p(status), threads or os.cpu_count() or 1)
    return dist, out_id, count, status


def search_lists(dtype, dims, codes, queries, offsets, probes, k, metric, row_ids=None, block_scales=None,
                 row_scales=None, threads=None):
    """IVF list gather: query q scans the rows of lists probes[q]; strict top-k."""
    codes = np.ascontiguousarray(codes)
    queries = np.ascontiguousarray(queries, dtype=np.float32)
    offsets = np.ascontiguousarray(offsets, dtype=np.uint64)
    probes = np.ascontiguousarray(probes, dtype=np.uint32)
    nq, nprobe = probes.shape
    dist = np.full((nq, max(k, 1)), np.inf)
    out_id = np.full((nq, max(k, 1)), -1, dtype=np.int64)
    count = np.zeros(nq, dtype=np.uint32)
    rid = None if row_ids is None else np.ascontiguousarray(row_ids, dtype=np.int64)
    bs = None if block_scales is None else np.ascontiguousarray(block_scales, dtype=np.uint8)
    rs = None if row_scales is None else np.ascontiguousarray(row_scales, dtype=np.float32)
    lib().orc_search_lists(dtype, dims, codes.shape[0], _p(codes), _p(bs), _p(rs), _p(rid), _p(offsets),
                           offsets.shape[0] - 1, _p(probes), nprobe, _p(queries), nq, k, metric, _p(dist),
                           _p(out_id), _p(count), threads or os.cpu_count() or 1)
    return dist, out_id, count


def decode_rows(dtype, dims, codes, block_scales=None, row_scales=None, first=0, count=None, threads=None):
    codes = np.ascontiguousarray(codes)
    count = codes.shape[0] - first if count is None else count
    out = np.empty((count, dims), dtype=np.float32)
    bs = None if block_scales is None else np.ascontiguousarray(block_scales, dtype=np.uint8)
    rs = None if row_scales is None else np.ascontiguousarray(row_scales, dtype=np.float32)
    lib().orc_decode_rows(dtype, dims, first, count, _p(codes), _p(bs), _p(rs), _p(out),
                          threads or os.cpu_count() or 1)
    return out


def exact_distance_f64(rows, query):
    """The reference's FP32 re-score of a quantized scan's candidates
    (ExactDistance, ann/server/cuvs.c:2930-2942): each difference and square
    in FP64, summed in dimension order (cumsum adds in order), the FP64
    square root rounded to FP32. Pinned by construction: the reference keeps
    this function static in its GPU backend, which does not build here."""
    delta = np.asarray(rows, dtype=np.float32).astype(np.float64) - \
        np.asarray(query, dtype=np.float32).astype(np.float64)
    sq = delta * delta
    if sq.shape[-1] == 0:
        return np.zeros(sq.shape[:-1], dtype=np.float32)
    return np.sqrt(np.cumsum(sq, axis=-1)[..., -1]).astype(np.float32)


def quant_index_search(dtype, vectors, codes, queries, k, bounds, ordinals=None, block_scales=None,
                       row_scales=None, quant_slack=256, slack_ratio=100, threads=1):
    """The reference's quantized scan route for a loaded index (SearchGather,
    ann/server/cuvs.c:4585-4930): per index shard [bounds[s], bounds[s+1]),
    the min(k + slack, eligible) rows nearest by the exact L2 distance of the
    decoded rows (slack = max(quant_slack, k * slack_ratio / 100), GatherSlack
    cuvs.c:4286-4296; this restatement breaks ties by ordinal), re-scored by
    exact_distance_f64 of their FP32 rows; the k best over all shards by
    (distance, ordinal), which is the per-shard (distance, key) sort cut at k
    and tree-merged (cuvs.c:4919-4930). Returns per query a list of
    (ordinal, FP32 distance)."""
    queries = np.ascontiguousarray(queries, dtype=np.float32)
    dims = queries.shape[1]
    want = k + max(quant_slack, k * slack_ratio // 100)
    out = []
    for q in queries:
        cand = []
        for s in range(len(bounds) - 1):
            lo, hi = int(bounds[s]), int(bounds[s + 1])
            if ordinals is None:
                local = np.arange(hi - lo, dtype=np.uint32)
            else:
                o = np.asarray(ordinals, dtype=np.uint64)
                local = (o[(o >= lo) & (o < hi)] - lo).astype(np.uint32)
            kk = min(want, len(local))
            if kk == 0 or k == 0:
                continue
            bs = None if block_scales is None else block_scales[lo:hi]
            rs = None if row_scales is None else row_scales[lo:hi]
            _, ids, cnt, _ = search(dtype, dims, codes[lo:hi], q[None], kk, 0, ids=local, block_scales=bs,
                                    row_scales=rs, threads=threads)
            cand += [lo + int(i) for i in ids[0, :cnt[0]]]
        cand = np.array(cand, dtype=np.int64)
        if len(cand) == 0:
            out.append([])
            continue
        dist = exact_distance_f64(vectors[cand], q)
        order = np.lexsort((cand, dist))[:k]
        out.append([(int(cand[i]), dist[i]) for i in order])
    return out


def quantize_fp8(vectors):
    v = np.ascontiguousarray(vectors, dtype=np.float32)
    rows, dims = v.shape
    codes = np.zeros((rows, (dims + 15) // 16 * 16), dtype=np.uint8)
    scale = np.zeros(rows, dtype=np.float32)
    lib().orc_quantize_fp8(_p(v), rows, dims, _p(codes), _p(scale))
    return codes, scale


def quantize_nvfp4(vectors):
    v = np.ascontiguousarray(vectors, dtype=np.float32)
    rows, dims = v.shape
    blocks = (dims + 15) // 16
    packed = np.zeros((rows, blocks * 8), dtype=np.uint8)
    sc = np.zeros((rows, blocks), dtype=np.uint8)
    row = np.zeros(rows, dtype=np.float32)
    lib().orc_quantize_nvfp4(_p(v), rows, dims, _p(packed), _p(sc), _p(row))
    return packed, sc, row


def half_to_float(h):
    L = lib()
    return np.array([L.orc_half_to_float(int(x)) for x in np.asarray(h, dtype=np.uint16).ravel()],
                    dtype=np.float32).reshape(np.shape(h))


def float_to_half(f):
    L = lib()
    return np.array([L.orc_float_to_half(float(x)) for x in np.asarray(f, dtype=np.float32).ravel()],
                    dtype=np.uint16).reshape(np.shape(f))


# ---------------------------------------------------------------- reference

class AnnCandidate(ctypes.Structure):
    _fields_ = [('id', ctypes.c_uint32), ('distance', ctypes.c_double)]


class AnnGatheredJob(ctypes.Structure):
    _fields_ = [('rows', ctypes.c_uint32), ('dimensions', ctypes.c_uint32), ('k', ctypes.c_uint32),
                ('metric', ctypes.c_uint32), ('query', ctypes.POINTER(ctypes.c_float)),
                ('vectors', ctypes.POINTER(ctypes.c_float)), ('results', ctypes.POINTER(AnnCandidate)),
                ('nresults', ctypes.c_uint32), ('status', ctypes.c_int)]


class AnnIndexHit(ctypes.Structure):
    _fields_ = [('key', ctypes.c_int64), ('distance', ctypes.c_float), ('ordinal', ctypes.c_uint64)]


def ref_available():
    return os.path.exists(REF_SO)


def ref():
    """The reference's compiled CPU backend (oracle/_ref/libannref.so)."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_SO):
            raise FileNotFoundError(REF_SO + ' (build with make -C oracle ref)')
        L = ctypes.CDLL(REF_SO)
        L.AnnGatheredExact.restype = None
        L.AnnGatheredExact.argtypes = [ctypes.POINTER(AnnGatheredJob)]
        L.AnnIndexTreeMerge.restype = ctypes.c_uint32
        L.AnnIndexTreeMerge.argtypes = [ctypes.POINTER(ctypes.POINTER(AnnIndexHit)), ctypes.POINTER(ctypes.c_uint32),
                                        ctypes.c_uint32, ctypes.c_uint32, ctypes.POINTER(AnnIndexHit)]
        _ref = L
    return _ref


def ref_gathered_exact(query, vectors, k, metric):
    """The reference worker's AnnGatheredExact (ann/server/cpu.c:218-276) on one
    job: returns (status, [(id, distance)]) in the reference's output order."""
    q = np.ascontiguousarray(query, dtype=np.float32)
    v = np.ascontiguousarray(vectors, dtype=np.float32)
    rows = v.shape[0] if v.ndim == 2 else 0
    res = (AnnCandidate * max(rows, 1))()
    job = AnnGatheredJob()
    job.rows, job.dimensions, job.k, job.metric = rows, q.shape[0], k, metric
    job.query = q.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    job.vectors = v.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
    job.results = res
    ref().AnnGatheredExact(ctypes.byref(job))
    return job.status, [(res[i].id, res[i].distance) for i in range(job.nresults)]


def ref_tree_merge(lists, k):
    """The reference's AnnIndexTreeMerge (ann/server/indexfile.c:3235-3258) over
    lists of (key, distance) sorted by (distance, key); returns merged list."""
    n = len(lists)
    bufs, heads = [], (ctypes.POINTER(AnnIndexHit) * n)()
    counts = (ctypes.c_uint32 * n)()
    for i, lst in enumerate(lists):
        buf = (AnnIndexHit * max(k, len(lst), 1))()
        for j, (key, dist) in enumerate(lst):
            buf[j].key, buf[j].distance, buf[j].ordinal = key, dist, key
        bufs.append(buf)
        heads[i] = ctypes.cast(buf, ctypes.POINTER(AnnIndexHit))
        counts[i] = len(lst)
    out = (AnnIndexHit * max(k, 1))()
    m = ref().AnnIndexTreeMerge(heads, counts, n, k, out)
    return [(out[i].key, out[i].distance) for i in range(m)]
