"""B200 (sm_100a) DSA lightning-indexer top-K.

Host-side mirror of the reference operator interface
(`dsa_topk_indexer_fp8_h64_d128_topk2048_ps64`, entry point
`kernel.cu::launch_topk_c`, destination-passing style; reference
solution/cuda/kernel.cu:818-891). Every call goes through the C ABI of
include/dsa_topk_indexer.h; there is no CPU fallback: if the CUDA library is
missing, calls raise.

The package directory name is not a Python identifier; import it with
``importlib.import_module("karnbirkhera-mlsys2026-dsa_topk_indexer_b200")``.
"""
import ctypes

from . import _lib
from ._lib import (DSA_STATUS_BAD_PAGE, DSA_STATUS_BAD_RECORD, DSA_STATUS_SEQ_CLAMPED,  # noqa: F401
                   DSA_STATUS_WAIT_TIMEOUT)

HEADS = 64
HEAD_DIM = 128
PAGE_SIZE = 64
PAGE_BYTES = 8448
TOPK = 2048

__all__ = ["launch_topk_c", "indexer_scores", "indexer_partial", "indexer_merge", "sparse_attention",
           "decode_queue_apply", "device_status",
           "last_launch_count", "HEADS", "HEAD_DIM", "PAGE_SIZE", "PAGE_BYTES", "TOPK"]


def _torch():
    import torch
    return torch


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _stream(device):
    return ctypes.c_void_p(_torch().cuda.current_stream(device).cuda_stream)


def _select(lib, device):
    """Makes the tensors' device current for the library's CUDA runtime."""
    _lib.check(lib.dsa_topk_indexer_set_device(int(device.index if device.index is not None else
                                                   _torch().cuda.current_device())), "set_device")


def _require(cond, msg):
    if not cond:
        raise RuntimeError(msg)


def _check_inputs(q, kc, w, sl, bt):
    torch = _torch()
    dev = q.device
    _require(dev.type == "cuda", "q_index_fp8 must be a CUDA tensor")
    for name, t in (("k_index_cache_fp8", kc), ("weights", w), ("seq_lens", sl), ("block_table", bt)):
        _require(t.device == dev, f"{name} must be on {dev}")
        _require(t.is_contiguous(), f"{name} must be contiguous")
    _require(q.is_contiguous(), "q_index_fp8 must be contiguous")
    _require(q.element_size() == 1 and q.dim() == 3 and q.shape[1] == HEADS and q.shape[2] == HEAD_DIM,
             "q_index_fp8 must be [B, 64, 128] fp8_e4m3 (or uint8)")
    B = q.shape[0]
    _require(kc.element_size() == 1 and kc.numel() % PAGE_BYTES == 0 and kc.numel() // PAGE_BYTES == kc.shape[0],
             "k_index_cache_fp8 must be [num_pages, 64, 1, 132] (8448 bytes per page) of a 1-byte dtype")
    _require(w.dtype == torch.float32 and tuple(w.shape) == (B, HEADS), "weights must be float32 [B, 64]")
    _require(sl.dtype == torch.int32 and tuple(sl.shape) == (B,), "seq_lens must be int32 [B]")
    _require(bt.dtype == torch.int32 and bt.dim() == 2 and bt.shape[0] == B and bt.shape[1] >= 1,
             "block_table must be int32 [B, max_num_pages]")
    return B, bt.shape[1], kc.shape[0]


def launch_topk_c(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, topk_indices):
    """Writes the top-2048 physical KV slots of every query into `topk_indices`.

    Same tensor signature, argument meaning and destination-passing contract
    as the reference entry point (solution/cuda/kernel.cu:818-824): rank
    r < min(seq_len, 2048) holds block_table[b, pos // 64] * 64 + pos % 64 for
    the r-th best logical position, the rest hold -1. Runs asynchronously on
    the current CUDA stream. Raises RuntimeError on bad arguments (the
    reference raises through TORCH_CHECK). Unlike the reference, there is no
    max_num_pages * 64 <= 8192 limit.
    """
    torch = _torch()
    B, max_pages, num_pages = _check_inputs(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table)
    _require(topk_indices.device == q_index_fp8.device and topk_indices.is_contiguous()
             and topk_indices.dtype == torch.int32 and tuple(topk_indices.shape) == (B, TOPK),
             "topk_indices must be a contiguous int32 [B, 2048] tensor on the same device")
    lib = _lib.load()
    _select(lib, q_index_fp8.device)
    with torch.cuda.device(q_index_fp8.device):
        rc = lib.dsa_topk_indexer_launch(
            _ptr(q_index_fp8), _ptr(k_index_cache_fp8), _ptr(weights), _ptr(seq_lens), _ptr(block_table),
            _ptr(topk_indices), B, max_pages, num_pages, _stream(q_index_fp8.device))
    _lib.check(rc, "launch_topk_c")


def indexer_scores(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, scores=None):
    """fp32 scores [B, max_num_pages*64] of the same scoring path (-inf past seq_len)."""
    torch = _torch()
    B, max_pages, num_pages = _check_inputs(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table)
    if scores is None:
        scores = torch.empty((B, max_pages * PAGE_SIZE), dtype=torch.float32, device=q_index_fp8.device)
    _require(scores.dtype == torch.float32 and scores.is_contiguous() and scores.dim() == 2
             and scores.shape[0] == B and scores.shape[1] >= max_pages * PAGE_SIZE,
             "scores must be contiguous float32 [B, >= max_num_pages*64]")
    lib = _lib.load()
    _select(lib, q_index_fp8.device)
    with torch.cuda.device(q_index_fp8.device):
        rc = lib.dsa_topk_indexer_scores(
            _ptr(q_index_fp8), _ptr(k_index_cache_fp8), _ptr(weights), _ptr(seq_lens), _ptr(block_table),
            _ptr(scores), scores.shape[1], B, max_pages, num_pages, _stream(q_index_fp8.device))
    _lib.check(rc, "indexer_scores")
    return scores


def indexer_partial(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table, key_begin, key_end,
                    cand_scores=None, cand_pos=None):
    """Best 2048 (score, logical position) candidates among keys [key_begin, key_end)."""
    torch = _torch()
    B, max_pages, num_pages = _check_inputs(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table)
    dev = q_index_fp8.device
    if cand_scores is None:
        cand_scores = torch.empty((B, TOPK), dtype=torch.float32, device=dev)
    if cand_pos is None:
        cand_pos = torch.empty((B, TOPK), dtype=torch.int32, device=dev)
    _require(cand_scores.is_contiguous() and cand_scores.dtype == torch.float32 and tuple(cand_scores.shape) == (B, TOPK)
             and cand_pos.is_contiguous() and cand_pos.dtype == torch.int32 and tuple(cand_pos.shape) == (B, TOPK),
             "cand_scores / cand_pos must be contiguous [B, 2048] float32 / int32")
    lib = _lib.load()
    _select(lib, dev)
    with torch.cuda.device(dev):
        rc = lib.dsa_topk_indexer_partial(
            _ptr(q_index_fp8), _ptr(k_index_cache_fp8), _ptr(weights), _ptr(seq_lens), _ptr(block_table),
            int(key_begin), int(key_end), _ptr(cand_scores), _ptr(cand_pos), B, max_pages, num_pages,
            _stream(dev))
    _lib.check(rc, "indexer_partial")
    return cand_scores, cand_pos


def indexer_merge(cand_scores, cand_pos, seq_lens, block_table, topk_indices=None):
    """Merges [nparts, B, 2048] candidate lists into final top-2048 physical slots."""
    torch = _torch()
    _require(cand_scores.dim() == 3 and cand_scores.shape[2] == TOPK and cand_pos.shape == cand_scores.shape,
             "candidates must be [nparts, B, 2048]")
    nparts, B = cand_scores.shape[0], cand_scores.shape[1]
    dev = cand_scores.device
    if topk_indices is None:
        topk_indices = torch.empty((B, TOPK), dtype=torch.int32, device=dev)
    _require(block_table.dtype == torch.int32 and block_table.shape[0] == B and block_table.is_contiguous(),
             "block_table must be contiguous int32 [B, max_num_pages]")
    lib = _lib.load()
    _select(lib, dev)
    with torch.cuda.device(dev):
        rc = lib.dsa_topk_indexer_merge(_ptr(cand_scores.contiguous()), _ptr(cand_pos.contiguous()), nparts,
                                        _ptr(seq_lens), _ptr(block_table), _ptr(topk_indices), B,
                                        block_table.shape[1], _stream(dev))
    _lib.check(rc, "indexer_merge")
    return topk_indices


def index_cache_write(k, slots, k_index_cache_fp8):
    """Quantises index-K vectors into the paged FP8 cache the indexer reads
    (in place): k [T, 128] bfloat16 or float32, slots [T] int64 (page * 64 +
    offset; negative = skip), k_index_cache_fp8 [num_pages, 64, 1, 132]
    (uint8 or float8 view), all on one CUDA device. Per token: scale =
    max|x| / 448 (1 for an all-zero vector), bytes = e4m3(x * 448 / max|x|)."""
    torch = _torch()
    _require(k.dim() == 2 and k.shape[1] == 128 and k.is_contiguous(), "k must be contiguous [T, 128]")
    _require(k.dtype in (torch.bfloat16, torch.float32), "k must be bfloat16 or float32")
    _require(slots.dtype == torch.int64 and slots.dim() == 1 and slots.shape[0] == k.shape[0]
             and slots.is_contiguous(), "slots must be contiguous int64 [T]")
    _require(k_index_cache_fp8.is_contiguous() and k_index_cache_fp8.numel() * k_index_cache_fp8.element_size()
             % 8448 == 0, "k_index_cache_fp8 must be contiguous pages of 8448 bytes")
    dev = k.device
    _require(slots.device == dev and k_index_cache_fp8.device == dev, "tensors must share one device")
    num_pages = k_index_cache_fp8.numel() * k_index_cache_fp8.element_size() // 8448
    lib = _lib.load()
    _select(lib, dev)
    with torch.cuda.device(dev):
        rc = lib.dsa_index_cache_write(_ptr(k), 0 if k.dtype == torch.bfloat16 else 1, _ptr(slots),
                                       _ptr(k_index_cache_fp8), k.shape[0], num_pages, _stream(dev))
    _lib.check(rc, "index_cache_write")
    return k_index_cache_fp8


def sparse_attention(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale, output=None, lse=None):
    """Sparse MLA attention over the slots the indexer selected (the consumer
    of ``topk_indices``, operator dsa_sparse_attention_h16_ckv512_kpe64_
    topk2048_ps64). q_nope [T,16,512], q_pe [T,16,64], ckv_cache
    [pages,64,512], kpe_cache [pages,64,64] bfloat16; sparse_indices [T, L]
    int32 slots (-1 = none); sm_scale a float. Writes (and returns)
    output [T,16,512] bfloat16 and lse [T,16] float32 (log2 of the softmax
    denominator; -inf and a zero row when a token has no valid slot)."""
    torch = _torch()
    dev = q_nope.device
    _require(dev.type == "cuda", "q_nope must be a CUDA tensor")
    for name, t, shape in (("q_nope", q_nope, (16, 512)), ("q_pe", q_pe, (16, 64))):
        _require(t.dtype == torch.bfloat16 and t.dim() == 3 and tuple(t.shape[1:]) == shape,
                 f"{name} must be bfloat16 [T, {shape[0]}, {shape[1]}]")
    T = q_nope.shape[0]
    _require(q_pe.shape[0] == T, "q_pe must have as many tokens as q_nope")
    for name, t, d in (("ckv_cache", ckv_cache, 512), ("kpe_cache", kpe_cache, 64)):
        _require(t.dtype == torch.bfloat16 and t.dim() == 3 and t.shape[1] == 64 and t.shape[2] == d,
                 f"{name} must be bfloat16 [num_pages, 64, {d}]")
    _require(ckv_cache.shape[0] == kpe_cache.shape[0], "ckv_cache and kpe_cache must have the same pages")
    _require(sparse_indices.dtype == torch.int32 and sparse_indices.dim() == 2 and sparse_indices.shape[0] == T,
             "sparse_indices must be int32 [T, L]")
    if output is None:
        output = torch.empty(T, 16, 512, dtype=torch.bfloat16, device=dev)
    if lse is None:
        lse = torch.empty(T, 16, dtype=torch.float32, device=dev)
    _require(output.dtype == torch.bfloat16 and tuple(output.shape) == (T, 16, 512), "output must be bf16 [T,16,512]")
    _require(lse.dtype == torch.float32 and tuple(lse.shape) == (T, 16), "lse must be float32 [T,16]")
    for name, t in (("q_nope", q_nope), ("q_pe", q_pe), ("ckv_cache", ckv_cache), ("kpe_cache", kpe_cache),
                    ("sparse_indices", sparse_indices), ("output", output), ("lse", lse)):
        _require(t.device == dev, f"{name} must be on {dev}")
        _require(t.is_contiguous(), f"{name} must be contiguous")
    lib = _lib.load()
    _select(lib, dev)
    with torch.cuda.device(dev):
        rc = lib.dsa_sparse_attention_launch(_ptr(q_nope), _ptr(q_pe), _ptr(ckv_cache), _ptr(kpe_cache),
                                             _ptr(sparse_indices), ctypes.c_float(float(sm_scale)), _ptr(output),
                                             _ptr(lse), T, sparse_indices.shape[1], ckv_cache.shape[0],
                                             _stream(dev))
    _lib.check(rc, "sparse_attention")
    return output, lse


def decode_queue_apply(record, req_len, req_block_table, seq_lens, block_table):
    """Applies one decode-queue record on the device (C ABI
    dsa_decode_queue_apply): the record's events update the request table
    (req_len [S] int32, -1 = free; req_block_table [S, max_pages] int32),
    then every batch row's request advances and its length and visible
    block-table entries are written to seq_lens [C] / block_table
    [C, max_pages] (rows past the batch: length 0). All int32, contiguous,
    on one CUDA device; record [W] int32 in the layout the C header gives
    (decode_queue.QueueRecord builds it)."""
    torch = _torch()
    dev = record.device
    _require(dev.type == "cuda", "record must be a CUDA tensor")
    for name, t in (("record", record), ("req_len", req_len), ("req_block_table", req_block_table),
                    ("seq_lens", seq_lens), ("block_table", block_table)):
        _require(t.dtype == torch.int32 and t.is_contiguous() and t.device == dev,
                 f"{name} must be contiguous int32 on {dev}")
    _require(req_block_table.dim() == 2 and req_block_table.shape[0] == req_len.numel(),
             "req_block_table must be [num_slots, max_pages]")
    _require(block_table.dim() == 2 and block_table.shape[1] == req_block_table.shape[1]
             and block_table.shape[0] == seq_lens.numel(), "block_table must be [capacity, max_pages]")
    lib = _lib.load()
    _select(lib, dev)
    with torch.cuda.device(dev):
        rc = lib.dsa_decode_queue_apply(_ptr(record), record.numel(), _ptr(req_len), _ptr(req_block_table),
                                        req_len.numel(), req_block_table.shape[1], _ptr(seq_lens), _ptr(block_table),
                                        seq_lens.numel(), _stream(dev))
    _lib.check(rc, "decode_queue_apply")


def device_status(device=0, clear=True):
    """Status bits the kernels raised on `device` since the last clear."""
    v = ctypes.c_uint32(0)
    _lib.check(_lib.load().dsa_topk_indexer_status(int(device), ctypes.byref(v), 1 if clear else 0),
               "device_status")
    return v.value


def last_launch_count():
    return _lib.load().dsa_topk_indexer_last_launch_count()


def last_path():
    """Schedule of the last top-K call on this thread: "cluster",
    "cluster-split", "cluster-tail", "prefill+cluster" or "noalloc"."""
    return _lib.load().dsa_topk_indexer_last_path().decode()


def set_kernel_timing(on):
    """Turns per-kernel timing events on or off (profiling only)."""
    _lib.load().dsa_topk_indexer_set_timing(1 if on else 0)


def last_kernel_ms():
    """Device time of the dominant kernel of the last call on this thread
    (timing must have been on for it); waits for that call."""
    import ctypes
    v = ctypes.c_float(0.0)
    rc = _lib.load().dsa_topk_indexer_kernel_ms(ctypes.byref(v))
    if rc != 0:
        raise RuntimeError(_lib.load().dsa_topk_indexer_error_string(rc).decode())
    return float(v.value)
