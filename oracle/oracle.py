"""ctypes wrapper of the C oracle (dsa_oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg, always as the checker. The shipped library never
routes through it.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
TOPK = 2048
_lib = None


def build(force=False):
    src = os.path.join(HERE, "dsa_oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(src) > os.path.getmtime(LIB_PATH):
        subprocess.run(["make", "-C", HERE, "-B" if force else "-s", "liboracle.so"], check=True,
                       stdout=subprocess.DEVNULL)
    return LIB_PATH


def load():
    global _lib
    if _lib is None:
        build()
        lib = ctypes.CDLL(LIB_PATH)
        P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        lib.oracle_indexer.argtypes = [P, P, P, P, P, I64, I64, P, I]
        lib.oracle_scores.argtypes = [P, P, P, P, P, I64, I64, P, I64, I]
        lib.oracle_topk_from_scores.argtypes = [P, I64, P, P, I64, I64, P, I]
        lib.oracle_fp8_gemm_nt.argtypes = [P, P, I, I, P]
        lib.oracle_e4m3_to_f32.argtypes = [ctypes.c_uint8]
        lib.oracle_e4m3_to_f32.restype = ctypes.c_float
        for f in (lib.oracle_indexer, lib.oracle_scores, lib.oracle_topk_from_scores):
            f.restype = ctypes.c_int
        _lib = lib
    return _lib


def _u8(a):
    """Bytes view of a tensor/array (fp8 tensors are viewed as uint8)."""
    if hasattr(a, "detach"):
        import torch
        t = a.detach().cpu().contiguous()
        if t.element_size() == 1 and t.dtype != torch.uint8:
            t = t.view(torch.uint8)
        return np.ascontiguousarray(t.numpy())
    return np.ascontiguousarray(a)


def _np(a, dtype):
    if hasattr(a, "detach"):
        a = a.detach().cpu().numpy()
    return np.ascontiguousarray(a, dtype=dtype)


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _threads(n):
    return n if n and n > 0 else (os.cpu_count() or 1)


def indexer(q, k_cache, weights, seq_lens, block_table, nthreads=0):
    """Top-2048 physical slots [B, 2048] int32 (reference semantics)."""
    q8, kc = _u8(q), _u8(k_cache)
    w, sl, bt = _np(weights, np.float32), _np(seq_lens, np.int32), _np(block_table, np.int32)
    B, max_pages = bt.shape
    out = np.empty((B, TOPK), dtype=np.int32)
    rc = load().oracle_indexer(_p(q8), _p(kc), _p(w), _p(sl), _p(bt), B, max_pages, _p(out), _threads(nthreads))
    if rc:
        raise MemoryError("oracle_indexer: allocation failed")
    return out


def scores(q, k_cache, weights, seq_lens, block_table, stride=None, nthreads=0):
    """fp32 scores [B, stride]; -inf past each row's length."""
    q8, kc = _u8(q), _u8(k_cache)
    w, sl, bt = _np(weights, np.float32), _np(seq_lens, np.int32), _np(block_table, np.int32)
    B, max_pages = bt.shape
    stride = stride or max_pages * 64
    out = np.empty((B, stride), dtype=np.float32)
    load().oracle_scores(_p(q8), _p(kc), _p(w), _p(sl), _p(bt), B, max_pages, _p(out), stride, _threads(nthreads))
    return out


def topk_from_scores(sc, seq_lens, block_table, nthreads=0):
    sc = np.ascontiguousarray(sc, dtype=np.float32)
    sl, bt = _np(seq_lens, np.int32), _np(block_table, np.int32)
    B, max_pages = bt.shape
    out = np.empty((B, TOPK), dtype=np.int32)
    rc = load().oracle_topk_from_scores(_p(sc), sc.shape[1], _p(sl), _p(bt), B, max_pages, _p(out),
                                        _threads(nthreads))
    if rc:
        raise MemoryError("oracle_topk_from_scores: allocation failed")
    return out


def fp8_gemm_nt(a, b):
    """d[m, n] = sum_k e4m3(a[m, k]) * e4m3(b[n, k]) for byte matrices with 128 columns."""
    a8, b8 = _u8(a), _u8(b)
    d = np.empty((a8.shape[0], b8.shape[0]), dtype=np.float32)
    load().oracle_fp8_gemm_nt(_p(a8), _p(b8), a8.shape[0], b8.shape[0], _p(d))
    return d


def e4m3_table():
    lib = load()
    return np.array([lib.oracle_e4m3_to_f32(i) for i in range(256)], dtype=np.float32)
