"""pgvector_b200: B200-native exact gather-scan behind the ANN worker's backend ABI.

Host-side mirror of the reference worker's interface for this path:

  * ``search_gathered(jobs)``  - the backend's search_gathered over gathered
    jobs (ann/server/backend.h:45-62,130; ann/server/cpu.c:218-283): one query
    against caller-supplied FP32 rows, results hold every row within the
    gathered tolerance of the k-th distance, sorted by (distance, id).
  * ``Shard`` / ``Shard.search`` - a device-resident shard in fp32, fp16
    (halfvec), FP8-E4M3, NVFP4 or bit format, searched for a query batch over
    a candidate row list (the loaded-index gather scan,
    ann/server/cuvs.c:4585-4930).
  * ``merge_topk`` - the on-device merge of per-shard lists
    (AnnIndexTreeMerge, ann/server/indexfile.c:3235-3258).
  * ``bitmap_rows`` - filter bitmap to row list (expand_*,
    ann/server/cuvs.c:1910-1968).

All compute runs in libannb200.so (AOT sm_100a CUDA); there is no CPU path.
Tensors are torch CUDA tensors; torch only provides device memory and streams.
"""
import ctypes

import numpy as np

from . import _abi
from ._lib import (OK, INVALID, UNSUPPORTED, NOMEM, BACKEND_ERROR, AnnB200Error, check, load)

F32, F16, E4M3, NVFP4, BIT = 0, 1, 2, 3, 4
L2, IP, COSINE, HAMMING = 0, 1, 2, 3
SHARD_HOST = 1
WINDOW, FORCE_SIMT, FORCE_F16, BOUNDS_EXCHANGE = 1, 2, 8, 32

DTYPE_NAMES = {'f32': F32, 'float32': F32, 'f16': F16, 'float16': F16, 'halfvec': F16, 'e4m3': E4M3,
               'fp8': E4M3, 'nvfp4': NVFP4, 'bit': BIT}


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def _stream(stream=None):
    import torch
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def device_count():
    return load().AnnB200DeviceCount()


class Shard:
    """A shard of rows on one GPU; codes (and scales) are torch CUDA tensors
    kept alive by this object."""

    def __init__(self, dtype, dims, codes, block_scales=None, row_scales=None, first_id=0, stream=None):
        lib = load()
        self.dtype = DTYPE_NAMES.get(dtype, dtype)
        self.dims = int(dims)
        self.codes, self.block_scales, self.row_scales = codes, block_scales, row_scales
        self.rows = int(codes.shape[0])
        self.first_id = int(first_id)
        self.device = codes.device.index if codes.device.index is not None else 0
        handle = ctypes.c_void_p()
        check(lib.AnnB200ShardCreate(self.device, self.dtype, self.dims, self.rows, _ptr(codes),
                                     _ptr(block_scales), _ptr(row_scales), self.first_id, 0, _stream(stream),
                                     ctypes.byref(handle)))
        self._handle = handle

    def close(self):
        if getattr(self, '_handle', None):
            load().AnnB200ShardDestroy(self._handle)
            self._handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def search(self, queries, k, metric, rows=None, window=False, force_simt=False, out_cap=None,
               stream=None, status=None, force_f16=False):
        """Exact search of a query batch; returns (dist f64 [nq][cap], id i64
        [nq][cap], count u32 [nq]) CUDA tensors."""
        import torch
        nq = int(queries.shape[0])
        nrows = int(rows.shape[0]) if rows is not None else self.rows
        cap = int(out_cap if out_cap is not None else (max(nrows, 1) if window else max(k, 1)))
        dev = queries.device
        dist = torch.empty((nq, cap), dtype=torch.float64, device=dev)
        ids = torch.empty((nq, cap), dtype=torch.int64, device=dev)
        count = torch.empty((nq,), dtype=torch.int32, device=dev)
        flags = (WINDOW if window else 0) | (FORCE_SIMT if force_simt else 0) | (FORCE_F16 if force_f16 else 0)
        if rows is not None and rows.numel() == 0:
            # an empty list is a non-NULL pointer with no entries (NULL means every row)
            rows = torch.zeros((1,), dtype=torch.int32, device=dev)
        check(load().AnnB200Search(self._handle, _ptr(queries), nq, _ptr(rows), nrows if rows is not None else 0,
                                   int(k), int(metric), flags, cap, _ptr(dist), _ptr(ids), _ptr(count),
                                   _ptr(status), _stream(stream)))
        return dist, ids, count

    def search_sharded(self, comm, queries, k, metric, rows=None, stream=None, status=None, force_simt=False,
                       bounds_exchange=False):
        """One rank of a row-sharded search (AnnB200SearchSharded): every rank
        of `comm` calls this with its own shard and candidate rows and the
        same queries; each gets the k best over all ranks' rows. Returns
        (dist, id, count) CUDA tensors like search()."""
        import torch
        nq = int(queries.shape[0])
        nrows = int(rows.shape[0]) if rows is not None else self.rows
        cap = max(int(k), 1)
        dev = queries.device
        dist = torch.empty((nq, cap), dtype=torch.float64, device=dev)
        ids = torch.empty((nq, cap), dtype=torch.int64, device=dev)
        count = torch.empty((nq,), dtype=torch.int32, device=dev)
        if rows is not None and rows.numel() == 0:
            rows = torch.zeros((1,), dtype=torch.int32, device=dev)
        check(load().AnnB200SearchSharded(self._handle, comm.handle if comm is not None else None, _ptr(queries), nq,
                                          _ptr(rows), nrows if rows is not None else 0, int(k), int(metric),
                                          (FORCE_SIMT if force_simt else 0) | (BOUNDS_EXCHANGE if bounds_exchange else 0),
                                          cap, _ptr(dist), _ptr(ids), _ptr(count), _ptr(status), _stream(stream)))
        return dist, ids, count

    def search_bitmap(self, comm, queries, k, metric, words, nbits, stream=None, status=None, force_simt=False,
                      bounds_exchange=False):
        """AnnB200SearchBitmap: search_sharded (comm None: one GPU) over the
        rows whose bits are set in a u32 device bitmap of nbits rows, the
        expansion and the search in one call. Returns (dist, id, count,
        rows selected)."""
        import torch
        nq = int(queries.shape[0])
        cap = max(int(k), 1)
        dev = queries.device
        dist = torch.empty((nq, cap), dtype=torch.float64, device=dev)
        ids = torch.empty((nq, cap), dtype=torch.int64, device=dev)
        count = torch.empty((nq,), dtype=torch.int32, device=dev)
        n = ctypes.c_uint64()
        check(load().AnnB200SearchBitmap(self._handle, comm.handle if comm is not None else None, _ptr(queries), nq,
                                         _ptr(words), int(nbits), int(k), int(metric),
                                         (FORCE_SIMT if force_simt else 0) | (BOUNDS_EXCHANGE if bounds_exchange else 0),
                                         cap, _ptr(dist), _ptr(ids), _ptr(count), _ptr(status), ctypes.byref(n),
                                         _stream(stream)))
        return dist, ids, count, n.value

    def search_lists_sharded(self, comm, queries, k, metric, offsets, probes, row_ids=None, stream=None,
                             status=None, force_simt=False):
        """One rank of a sharded IVF list search (AnnB200SearchListsSharded):
        this rank's share of the lists, then the exchange and merge."""
        import torch
        nq = int(queries.shape[0])
        nlists = int(offsets.shape[0]) - 1
        nprobe = int(probes.shape[1]) if probes.dim() == 2 else 0
        cap = max(int(k), 1)
        dev = queries.device
        dist = torch.empty((nq, cap), dtype=torch.float64, device=dev)
        ids = torch.empty((nq, cap), dtype=torch.int64, device=dev)
        count = torch.empty((nq,), dtype=torch.int32, device=dev)
        check(load().AnnB200SearchListsSharded(self._handle, comm.handle if comm is not None else None,
                                               _ptr(queries), nq, _ptr(offsets), nlists, _ptr(probes), nprobe,
                                               _ptr(row_ids), int(k), int(metric), FORCE_SIMT if force_simt else 0,
                                               cap, _ptr(dist), _ptr(ids), _ptr(count), _ptr(status),
                                               _stream(stream)))
        return dist, ids, count

    def search_lists(self, queries, k, metric, offsets, probes, row_ids=None, stream=None, status=None,
                     force_simt=False):
        """IVF list gather: each query's k nearest among the rows of the lists
        it probes. offsets: int64 [nlists+1] row runs of the lists; probes:
        int32 [nq][nprobe] list numbers; row_ids: optional int64 [rows] global
        ids. Returns (dist, id, count) CUDA tensors like search()."""
        import torch
        nq = int(queries.shape[0])
        nlists = int(offsets.shape[0]) - 1
        nprobe = int(probes.shape[1]) if probes.dim() == 2 else 0
        cap = max(int(k), 1)
        dev = queries.device
        dist = torch.empty((nq, cap), dtype=torch.float64, device=dev)
        ids = torch.empty((nq, cap), dtype=torch.int64, device=dev)
        count = torch.empty((nq,), dtype=torch.int32, device=dev)
        check(load().AnnB200SearchLists(self._handle, _ptr(queries), nq, _ptr(offsets), nlists, _ptr(probes), nprobe,
                                        _ptr(row_ids), int(k), int(metric), FORCE_SIMT if force_simt else 0, cap,
                                        _ptr(dist), _ptr(ids),
                                        _ptr(count), _ptr(status), _stream(stream)))
        return dist, ids, count

    def probe_lists(self, queries, nprobe, metric, stream=None, status=None):
        """IVF coarse probe on a shard of list centroids (row l = list l's
        centre): each query's nprobe nearest lists as an int32 [nq][nprobe]
        CUDA tensor of u32 list numbers (-1 = UINT32_MAX past the number of
        lists), ordered by (distance, list) -- the probe table search_lists
        takes."""
        import torch
        nq = int(queries.shape[0])
        probes = torch.empty((nq, max(int(nprobe), 1)), dtype=torch.int32, device=queries.device)
        check(load().AnnB200ProbeLists(self._handle, _ptr(queries), nq, int(nprobe), int(metric), _ptr(probes),
                                       _ptr(status), _stream(stream)))
        return probes

    def score_matrix(self, queries, metric, rows=None, force_simt=False, stream=None, force_f16=False):
        """Approximate distances [nq][n] (squared for L2) and each query's
        error bound, as the scan computes them."""
        import torch
        nq = int(queries.shape[0])
        n = int(rows.shape[0]) if rows is not None else self.rows
        out = torch.empty((nq, max(n, 1)), dtype=torch.float32, device=queries.device)
        err = torch.empty((nq,), dtype=torch.float64, device=queries.device)
        check(load().AnnB200ScoreMatrix(self._handle, _ptr(queries), nq, _ptr(rows), n if rows is not None else 0,
                                        int(metric), (FORCE_SIMT if force_simt else 0) | (FORCE_F16 if force_f16 else 0),
                                        _ptr(out), _ptr(err),
                                        _stream(stream)))
        return out[:, :n], err


class Comm:
    """One rank's NCCL communicator in libannb200 (AnnB200CommCreate): the
    all-gather of the row-sharded searches. comm_id: the 128 bytes
    Comm.unique_id() returned on one rank, shared with all ranks."""

    def __init__(self, device, nranks, rank, comm_id):
        handle = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(bytes(comm_id), 128)
        check(load().AnnB200CommCreate(int(device), int(nranks), int(rank), buf, ctypes.byref(handle)))
        self.handle = handle
        self.rank, self.nranks, self.device = int(rank), int(nranks), int(device)

    @staticmethod
    def unique_id():
        buf = ctypes.create_string_buffer(128)
        check(load().AnnB200CommId(buf))
        return buf.raw

    def abort(self):
        """End this rank's part of the group at once (peers gone)."""
        if getattr(self, 'handle', None):
            load().AnnB200CommAbort(self.handle)

    def close(self):
        if getattr(self, 'handle', None):
            load().AnnB200CommDestroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def merge_topk(dist, ids, counts, k, window=False, out_cap=None, stream=None):
    """Merge [nlists][nq][list_cap] per-shard results on the device."""
    import torch
    nlists, nq, list_cap = (int(x) for x in dist.shape)
    cap = int(out_cap if out_cap is not None else (nlists * list_cap if window else max(k, 1)))
    od = torch.empty((nq, cap), dtype=torch.float64, device=dist.device)
    oi = torch.empty((nq, cap), dtype=torch.int64, device=dist.device)
    oc = torch.empty((nq,), dtype=torch.int32, device=dist.device)
    check(load().AnnB200MergeTopk(_ptr(dist), _ptr(ids), _ptr(counts), nlists, nq, list_cap, int(k),
                                  WINDOW if window else 0, cap, _ptr(od), _ptr(oi), _ptr(oc), _stream(stream)))
    return od, oi, oc


def bitmap_rows(words, nbits, stream=None):
    """Row numbers of the set bits of a u32 bitmap (CUDA tensor), ascending."""
    import torch
    rows = torch.empty((max(int(nbits), 1),), dtype=torch.int32, device=words.device)
    n = ctypes.c_uint64()
    check(load().AnnB200BitmapRows(_ptr(words), int(nbits), _ptr(rows), ctypes.byref(n), _stream(stream)))
    return rows[:n.value]


def bitmap_rows_static(words, nbits, rows, stream=None):
    """bitmap_rows for callers that must not allocate device memory: writes
    the row numbers into the caller's `rows` tensor (int32, >= nbits long)
    using the library's fixed scratch array; returns the count. At most 2^31
    rows; concurrent calls on one device must be serialised."""
    n = ctypes.c_uint64()
    check(load().AnnB200BitmapRowsStatic(_ptr(words), int(nbits), _ptr(rows), ctypes.byref(n), _stream(stream)))
    return n.value


def backend():
    """The AnnBackend vtable AnnB200Backend() returns."""
    return load().AnnB200Backend().contents


def search_gathered(jobs):
    """Run gathered jobs through the backend: jobs are (query, vectors, k,
    metric) with float32 numpy arrays; returns [(status, [(id, distance)])]."""
    n = len(jobs)
    arr = (_abi.AnnGatheredJob * n)()
    keep = []
    for i, (query, vectors, k, metric) in enumerate(jobs):
        q = np.ascontiguousarray(query, dtype=np.float32)
        v = np.ascontiguousarray(vectors, dtype=np.float32).reshape(-1, q.shape[0]) if q.shape[0] else \
            np.zeros((0, 0), np.float32)
        rows = v.shape[0]
        res = (_abi.AnnCandidate * max(rows, 1))()
        keep += [q, v, res]
        arr[i].rows, arr[i].dimensions, arr[i].k, arr[i].metric = rows, q.shape[0], int(k), int(metric)
        arr[i].query = q.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        arr[i].vectors = v.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        arr[i].results = res
    backend().search_gathered(arr, n)
    out = []
    for i in range(n):
        out.append((arr[i].status, [(arr[i].results[j].id, arr[i].results[j].distance)
                                    for j in range(arr[i].nresults)]))
    return out


def search_typed(jobs):
    """Typed gathered jobs (AnnB200SearchTyped): jobs are dicts with dtype,
    metric, queries (float32 [nq, dims], or packed-bit uint8 [nq, bytes] for
    Hamming), codes (the rows in dtype's format: float32, float16 / int16
    bits, or uint8 codes [rows, row-bytes]), dims, k, and block_scales /
    row_scales where the format has them; cap defaults to the rows. Returns
    per job (status, [[(row, distance), ...] per query])."""
    lib = load()
    n = len(jobs)
    arr = (_abi.AnnB200TypedJob * n)()
    keep = []
    caps = []
    for i, j in enumerate(jobs):
        q = np.ascontiguousarray(j['queries'])
        c = np.ascontiguousarray(j['codes'])
        nq, rows = q.shape[0], c.shape[0]
        cap = int(j.get('cap', max(rows, 1)))
        dist = np.zeros(max(nq * cap, 1), np.float64)
        ids = np.zeros(max(nq * cap, 1), np.uint32)
        cnt = np.zeros(max(nq, 1), np.uint32)
        bs = None if j.get('block_scales') is None else np.ascontiguousarray(j['block_scales'], dtype=np.uint8)
        rs = None if j.get('row_scales') is None else np.ascontiguousarray(j['row_scales'], dtype=np.float32)
        keep += [q, c, dist, ids, cnt, bs, rs]
        a = arr[i]
        a.dtype, a.metric, a.dimensions, a.rows = int(j['dtype']), int(j['metric']), int(j['dims']), rows
        a.nq, a.k, a.cap = nq, int(j['k']), cap
        a.queries, a.codes = q.ctypes.data, c.ctypes.data
        a.block_scales = None if bs is None else bs.ctypes.data
        a.row_scales = None if rs is None else rs.ctypes.data
        a.distances, a.ids, a.nresults = dist.ctypes.data, ids.ctypes.data, cnt.ctypes.data
        caps.append((nq, cap, dist, ids, cnt))
    lib.AnnB200SearchTyped(arr, n)
    out = []
    for i, (nq, cap, dist, ids, cnt) in enumerate(caps):
        out.append((arr[i].status, [[(int(ids[q * cap + r]), float(dist[q * cap + r])) for r in range(cnt[q])]
                                    for q in range(nq)]))
    del keep
    return out


__all__ = ['Shard', 'search_typed', 'merge_topk', 'bitmap_rows', 'bitmap_rows_static', 'backend', 'search_gathered', 'device_count', 'load', 'check',
           'AnnB200Error', 'F32', 'F16', 'E4M3', 'NVFP4', 'BIT', 'L2', 'IP', 'COSINE', 'HAMMING', 'WINDOW',
           'FORCE_SIMT', 'FORCE_F16', 'BOUNDS_EXCHANGE', 'OK', 'INVALID', 'UNSUPPORTED', 'NOMEM', 'BACKEND_ERROR']
