"""ctypes binding of the C ABI declared in include/dsa_topk_indexer.h."""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdsa_topk_indexer.so")

DSA_OK = 0
DSA_ERR_INVALID_ARG = 1
DSA_ERR_MISALIGNED = 2
DSA_ERR_CUDA = 3
DSA_ERR_NO_DEVICE = 4
DSA_ERR_TOO_LARGE = 5
DSA_NOALLOC_MAX_BATCH = 65536

DSA_STATUS_WAIT_TIMEOUT = 0x1
DSA_STATUS_BAD_PAGE = 0x2
DSA_STATUS_SEQ_CLAMPED = 0x4
DSA_STATUS_BAD_RECORD = 0x8

# Decode-queue record format (dsa_decode_queue_apply).
DSA_QUEUE_HEADER_WORDS = 8
DSA_QUEUE_ADMIT = 1
DSA_QUEUE_APPEND_PAGE = 2
DSA_QUEUE_SET_LEN = 3
DSA_QUEUE_RETIRE = 4

# (name, restype, argtypes) for every function the header declares.
_P, _I64, _I32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
SIGNATURES = [
    ("dsa_topk_indexer_launch", _I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    ("dsa_topk_indexer_scores", _I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _I64, _P]),
    ("dsa_topk_indexer_partial", _I32, [_P, _P, _P, _P, _P, _I64, _I64, _P, _P, _I64, _I64, _I64, _P]),
    ("dsa_topk_indexer_merge", _I32, [_P, _P, _I64, _P, _P, _P, _I64, _I64, _P]),
    ("dsa_topk_indexer_launch_noalloc", _I32, [_P, _P, _P, _P, _P, _P, _I64, _I64, _I64, _P]),
    ("dsa_topk_indexer_set_test_fault", _I32, [_I32, _I64]),
    ("dsa_topk_indexer_set_device", _I32, [_I32]),
    ("dsa_topk_indexer_status", _I32, [_I32, ctypes.POINTER(ctypes.c_uint32), _I32]),
    ("dsa_topk_indexer_error_string", ctypes.c_char_p, [_I32]),
    ("dsa_topk_indexer_last_launch_count", _I32, []),
    ("dsa_topk_indexer_last_path", ctypes.c_char_p, []),
    ("dsa_index_cache_write", _I32, [_P, _I32, _P, _P, _I64, _I64, _P]),
    ("dsa_peer_region_bytes", _I32, [_I64, ctypes.POINTER(ctypes.c_int64)]),
    ("dsa_peer_alloc", _I32, [_I64, ctypes.POINTER(ctypes.c_void_p), _P]),
    ("dsa_peer_open", _I32, [_P, ctypes.POINTER(ctypes.c_void_p)]),
    ("dsa_peer_close", _I32, [_P]),
    ("dsa_peer_free", _I32, [_P]),
    ("dsa_peer_merge", _I32, [_P, _I32, _I32, ctypes.c_uint32, _I64, _P, _I64, _I32, _I64, _P]),
    ("dsa_decode_queue_apply", _I32, [_P, _I64, _P, _P, _I64, _I64, _P, _P, _I64, _P]),
    ("dsa_sparse_attention_launch", _I32, [_P, _P, _P, _P, _P, ctypes.c_float, _P, _P, _I64, _I64, _I64, _P]),
    ("dsa_topk_indexer_set_timing", _I32, [_I32]),
    ("dsa_topk_indexer_kernel_ms", _I32, [ctypes.POINTER(ctypes.c_float)]),
]

_lib = None


def load():
    """Loads the CUDA library; raises if it has not been built (no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"DSA indexer CUDA library missing at {LIB_PATH}; build it with "
                "__graft_entry__.build() (there is no CPU fallback)")
        lib = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
    return _lib


def error_string(code):
    return load().dsa_topk_indexer_error_string(int(code)).decode()


def check(code, what):
    if code != DSA_OK:
        raise RuntimeError(f"{what} failed: {error_string(code)} (code {code})")
