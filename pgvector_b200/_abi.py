"""ctypes layouts of the worker backend ABI (include/annb200_backend.h).

Field order and C types follow the reference worker's backend.h
(ann/server/backend.h:30-151 in chenqin/pgvector), so a Python caller can
drive AnnB200Backend() exactly as the worker's lane threads do.
"""
import ctypes


class AnnCandidate(ctypes.Structure):
    _fields_ = [('id', ctypes.c_uint32), ('distance', ctypes.c_double)]


class AnnGatheredJob(ctypes.Structure):
    _fields_ = [('rows', ctypes.c_uint32), ('dimensions', ctypes.c_uint32), ('k', ctypes.c_uint32),
                ('metric', ctypes.c_uint32), ('query', ctypes.POINTER(ctypes.c_float)),
                ('vectors', ctypes.POINTER(ctypes.c_float)), ('results', ctypes.POINTER(AnnCandidate)),
                ('nresults', ctypes.c_uint32), ('status', ctypes.c_int)]


class AnnB200TypedJob(ctypes.Structure):
    """AnnB200TypedJob of annb200.h: one typed gathered job."""
    _fields_ = [('dtype', ctypes.c_uint32), ('metric', ctypes.c_uint32), ('dimensions', ctypes.c_uint32),
                ('rows', ctypes.c_uint32), ('nq', ctypes.c_uint32), ('k', ctypes.c_uint32),
                ('cap', ctypes.c_uint32), ('reserved', ctypes.c_uint32), ('queries', ctypes.c_void_p),
                ('codes', ctypes.c_void_p), ('block_scales', ctypes.c_void_p), ('row_scales', ctypes.c_void_p),
                ('distances', ctypes.c_void_p), ('ids', ctypes.c_void_p), ('nresults', ctypes.c_void_p),
                ('status', ctypes.c_int)]


class AnnIndex(ctypes.Structure):
    _fields_ = [('generation', ctypes.c_uint64), ('rows', ctypes.c_uint32), ('dimensions', ctypes.c_uint32),
                ('vectors', ctypes.POINTER(ctypes.c_float)), ('backend_state', ctypes.c_void_p)]


BUILD = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.POINTER(AnnIndex), ctypes.c_uint64, ctypes.c_uint32,
                         ctypes.c_uint32, ctypes.POINTER(ctypes.c_float))
SEARCH = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.POINTER(AnnIndex), ctypes.POINTER(ctypes.c_float), ctypes.c_uint32,
                          ctypes.POINTER(ctypes.c_uint32), ctypes.c_uint32, ctypes.c_uint32,
                          ctypes.POINTER(AnnCandidate), ctypes.POINTER(ctypes.c_uint32))
DESTROY = ctypes.CFUNCTYPE(None, ctypes.POINTER(AnnIndex))
SEARCH_GATHERED = ctypes.CFUNCTYPE(None, ctypes.POINTER(AnnGatheredJob), ctypes.c_uint32)
DEVICE_JOBS = ctypes.CFUNCTYPE(ctypes.c_uint64)
LOST = ctypes.CFUNCTYPE(ctypes.c_char_p)


class AnnIndexHit(ctypes.Structure):
    _fields_ = [('key', ctypes.c_int64), ('distance', ctypes.c_float), ('ordinal', ctypes.c_uint64)]


class AnnIndexJob(ctypes.Structure):
    _fields_ = [('name', ctypes.c_char * 64), ('dimensions', ctypes.c_uint32), ('k', ctypes.c_uint32),
                ('query', ctypes.POINTER(ctypes.c_float)), ('filter', ctypes.POINTER(ctypes.c_int64)),
                ('nfilter', ctypes.c_uint32), ('filtered', ctypes.c_int),
                ('ordinals', ctypes.POINTER(ctypes.c_uint64)), ('bitsets', ctypes.c_void_p),
                ('deviceBitsets', ctypes.c_void_p), ('deviceRows', ctypes.c_void_p),
                ('results', ctypes.POINTER(AnnIndexHit)), ('nresults', ctypes.c_uint32),
                ('route', ctypes.c_uint32), ('status', ctypes.c_int),
                ('exclude', ctypes.POINTER(ctypes.c_uint64)), ('nexclude', ctypes.c_uint32),
                ('ownedOrdinals', ctypes.POINTER(ctypes.c_uint64))]


LOAD_INDEX = ctypes.CFUNCTYPE(ctypes.c_int, ctypes.c_char_p, ctypes.c_char_p)
SEARCH_INDEX = ctypes.CFUNCTYPE(None, ctypes.POINTER(AnnIndexJob), ctypes.c_uint32)


class AnnBackend(ctypes.Structure):
    _fields_ = [('name', ctypes.c_char_p), ('metrics', ctypes.c_uint32), ('filters', ctypes.c_uint32),
                ('algorithm', ctypes.c_char_p), ('storage', ctypes.c_char_p), ('exact', ctypes.c_int),
                ('min_rows', ctypes.c_uint32), ('max_k', ctypes.c_uint32), ('build', BUILD), ('search', SEARCH),
                ('destroy', DESTROY), ('search_gathered', SEARCH_GATHERED), ('device_jobs', ctypes.c_void_p),
                ('load_index', ctypes.c_void_p), ('search_index', ctypes.c_void_p), ('lost', ctypes.c_void_p),
                ('scan_preferred', ctypes.c_void_p),
                # after the reference's last slot: the typed search operation's jobs
                ('search_typed', ctypes.c_void_p)]
