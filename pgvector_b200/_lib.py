"""ctypes binding of libannb200.so (the C ABI in include/annb200.h).

The library is built in-tree by pgvector_b200.build; there is no fallback:
loading fails loudly when it is missing.
"""
import ctypes
import os

from ._abi import AnnBackend

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, 'libannb200.so')

# AnnStatus values (reference ann/server/backend.h:12-28)
OK, INVALID, UNSUPPORTED, STALE, NOMEM, BACKEND_ERROR = 0, 1, 2, 3, 4, 5
STATUS_NAMES = {0: 'ANN_OK', 1: 'ANN_INVALID', 2: 'ANN_UNSUPPORTED', 3: 'ANN_STALE',
                4: 'ANN_NOMEM', 5: 'ANN_BACKEND_ERROR'}

c_void_p, c_uint32, c_uint64, c_int64, c_int, c_double = (
    ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_int64, ctypes.c_int, ctypes.c_double)

# name -> (restype, argtypes); every symbol include/annb200.h and
# include/annb200_backend.h declare.
SIGNATURES = {
    'AnnB200LastError': (ctypes.c_char_p, []),
    'AnnB200DeviceCount': (c_int, []),
    'AnnB200ShardCreate': (c_int, [c_int, c_uint32, c_uint32, c_uint64, c_void_p, c_void_p, c_void_p,
                                   c_int64, c_uint32, c_void_p, ctypes.POINTER(c_void_p)]),
    'AnnB200ShardAssign': (c_int, [c_void_p, c_uint32, c_uint32, c_uint64, c_void_p, c_void_p, c_void_p,
                                   c_int64, c_void_p]),
    'AnnB200ShardDestroy': (None, [c_void_p]),
    'AnnB200Search': (c_int, [c_void_p, c_void_p, c_uint32, c_void_p, c_uint64, c_uint32, c_uint32,
                              c_uint32, c_uint32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    'AnnB200SearchLists': (c_int, [c_void_p, c_void_p, c_uint32, c_void_p, c_uint32, c_void_p, c_uint32,
                                   c_void_p, c_uint32, c_uint32, c_uint32, c_uint32, c_void_p, c_void_p,
                                   c_void_p, c_void_p, c_void_p]),
    'AnnB200ProbeLists': (c_int, [c_void_p, c_void_p, c_uint32, c_uint32, c_uint32, c_void_p, c_void_p, c_void_p]),
    'AnnB200IndexCreate': (c_int, [ctypes.c_int, c_uint32, c_uint64, c_void_p, ctypes.POINTER(c_void_p)]),
    'AnnB200IndexCreateQuant': (c_int, [ctypes.c_int, c_uint32, c_uint64, c_uint32, c_void_p, c_void_p, c_void_p,
                                        c_void_p, c_uint32, c_void_p, c_uint32, c_uint32,
                                        ctypes.POINTER(c_void_p)]),
    'AnnB200RescoreRows': (c_int, [c_void_p, c_uint32, c_uint32, c_void_p, c_uint32, c_void_p, c_void_p,
                                   c_void_p]),
    'AnnB200RescoreGather': (c_int, [c_void_p, c_uint32, c_uint32, c_void_p, c_void_p, c_uint32, c_void_p,
                                     c_void_p, c_void_p]),
    'AnnB200IndexDestroy': (None, [c_void_p]),
    'AnnB200IndexSearchBitsets': (c_int, [c_void_p, c_void_p, c_uint32, c_uint32, c_void_p, c_void_p, c_void_p,
                                          c_uint32, c_uint32, c_void_p, c_void_p, c_void_p]),
    'AnnB200IndexDevice': (c_int, [c_void_p]),
    'AnnB200IndexCopyRoute': (c_int, [c_void_p]),
    'AnnB200IndexKeepBitsets': (c_int, [c_void_p, c_uint32, c_void_p, c_void_p, c_void_p]),
    'AnnB200IndexDropBitsets': (None, [c_void_p, c_uint32, c_void_p]),
    'AnnB200IndexCreateSharded': (c_int, [c_int, c_void_p, c_uint32, c_uint64, c_void_p, ctypes.POINTER(c_void_p)]),
    'AnnB200SearchTyped': (c_int, [c_void_p, c_uint32]),
    'AnnB200SearchBatch': (c_int, [c_void_p, c_void_p, c_uint32, c_void_p]),
    'AnnB200IndexSearch': (c_int, [c_void_p, c_void_p, c_uint32, c_void_p, c_uint64, c_uint32, c_void_p, c_void_p,
                                   c_void_p]),
    'AnnB200MergeTopk': (c_int, [c_void_p, c_void_p, c_void_p, c_uint32, c_uint32, c_uint32, c_uint32,
                                 c_uint32, c_uint32, c_void_p, c_void_p, c_void_p, c_void_p]),
    'AnnB200BitmapRows': (c_int, [c_void_p, c_uint64, c_void_p, ctypes.POINTER(c_uint64), c_void_p]),
    'AnnB200BitmapRowsFrom': (c_int, [c_void_p, c_uint64, c_uint32, c_void_p, ctypes.POINTER(c_uint64), c_void_p]),
    'AnnB200BitmapRowsStatic': (c_int, [c_void_p, c_uint64, c_void_p, ctypes.POINTER(c_uint64), c_void_p]),
    'AnnB200Backend': (ctypes.POINTER(AnnBackend), []),
    'AnnB200LaunchCount': (ctypes.c_ulonglong, []),
    'AnnB200ScoreMatrix': (c_int, [c_void_p, c_void_p, c_uint32, c_void_p, c_uint64, c_uint32, c_uint32,
                                   c_void_p, c_void_p, c_void_p]),
    'AnnB200StageTimes': (c_int, [c_void_p, c_void_p, c_uint32, c_int]),
    'AnnB200StageTiming': (c_int, [c_int]),
    'AnnB200CommId': (c_int, [c_void_p]),
    'AnnB200CommCreate': (c_int, [c_int, c_int, c_int, c_void_p, ctypes.POINTER(c_void_p)]),
    'AnnB200CommCreateAll': (c_int, [c_int, c_void_p, c_void_p]),
    'AnnB200CommDestroy': (None, [c_void_p]),
    'AnnB200CommAbort': (None, [c_void_p]),
    'AnnB200CommRank': (c_int, [c_void_p]),
    'AnnB200CommSize': (c_int, [c_void_p]),
    'AnnB200SearchListsSharded': (c_int, [c_void_p, c_void_p, c_void_p, c_uint32, c_void_p, c_uint32, c_void_p,
                                          c_uint32, c_void_p, c_uint32, c_uint32, c_uint32, c_uint32, c_void_p,
                                          c_void_p, c_void_p, c_void_p, c_void_p]),
    'AnnB200SearchSharded': (c_int, [c_void_p, c_void_p, c_void_p, c_uint32, c_void_p, c_uint64, c_uint32, c_uint32,
                                     c_uint32, c_uint32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
    'AnnB200SearchBitmap': (c_int, [c_void_p, c_void_p, c_void_p, c_uint32, c_void_p, c_uint64, c_uint32, c_uint32,
                                    c_uint32, c_uint32, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p, c_void_p]),
}

_lib = None


class AnnB200Error(RuntimeError):
    def __init__(self, status, message):
        super().__init__('%s: %s' % (STATUS_NAMES.get(status, status), message))
        self.status = status


def load():
    """The loaded library (building it first if this checkout has no build)."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        from . import build
        build.build()
    lib = ctypes.CDLL(LIB_PATH)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def check(status):
    if status != OK:
        raise AnnB200Error(status, load().AnnB200LastError().decode(errors='replace'))
    return status
