"""GPU: the no-allocation entry point, for callers that cannot allocate device
memory (code running inside an allocator or memory-pool callback, or a server
that has reserved all of HBM up front). Batches up to 256 rows rank their rows
inside the kernel; larger ones keep the longest-first row order in a fixed
array inside the library instead of a per-stream workspace. Its results must
equal those of the regular entry point. Consecutive calls with different
inputs (two of them above 256 rows) check that whatever the shared array holds
from the previous call does not leak into the next one.

Kept in its own file, collected last, so a run that stops at the first
failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from conftest import package, workloads
from parity import check_all

pytestmark = pytest.mark.gpu


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _call(lib, name, w, out):
    fn = getattr(lib, name)
    rc = fn(_ptr(w.q), _ptr(w.k_cache), _ptr(w.weights), _ptr(w.seq_lens), _ptr(w.block_table), _ptr(out),
            w.batch, w.max_pages, w.num_pages, ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    return rc


def test_noalloc_matches_regular_entry_two_calls():
    assert torch.cuda.is_available()
    pkg = package()
    lib = pkg._lib.load()
    assert lib.dsa_topk_indexer_set_device(0) == 0
    W = workloads()
    # First input: 64 rows up to 32k keys -> more clusters than one wave, so
    # the row order is planned into the scratch array. Second input: other
    # rows and lengths, reusing the same array.
    cases = [W.config(1, seed=41), W.custom([9000, 40, 0, 131072, 2049, 777] * 20, seed=42),
             W.custom([5000, 100, 2049, 0, 700] * 60, seed=43), W.custom([300, 4100, 64] * 100, seed=44)]
    for w_cpu in cases:
        w = w_cpu.to("cuda")
        ref = torch.full((w.batch, 2048), -7, dtype=torch.int32, device="cuda")
        got = torch.full((w.batch, 2048), -9, dtype=torch.int32, device="cuda")
        assert _call(lib, "dsa_topk_indexer_launch", w, ref) == 0
        assert _call(lib, "dsa_topk_indexer_launch_noalloc", w, got) == 0
        torch.cuda.synchronize()
        ref_np, got_np = ref.cpu().numpy(), got.cpu().numpy()
        # Same kernels on the same inputs: identical, which is within the
        # parity tolerance used everywhere else; also check against the oracle.
        assert np.array_equal(got_np, ref_np)
        ref_o = oracle.indexer(w_cpu.q, w_cpu.k_cache, w_cpu.weights, w_cpu.seq_lens, w_cpu.block_table)
        sc = oracle.scores(w_cpu.q, w_cpu.k_cache, w_cpu.weights, w_cpu.seq_lens, w_cpu.block_table)
        rows = [sc[b, :max(0, min(int(s), w_cpu.max_pages * 64))] for b, s in enumerate(w_cpu.seq_lens.tolist())]
        fails = check_all(got_np, ref_o, rows, w_cpu.seq_lens.numpy(), w_cpu.block_table.numpy(), w_cpu.num_pages)
        assert not fails, fails[:3]
    assert pkg.device_status(0) == 0
    # The no-allocation call reports its own schedule and, with timing on,
    # its own kernel time (not an earlier call's).
    w = cases[0].to("cuda")
    got = torch.empty((w.batch, 2048), dtype=torch.int32, device="cuda")
    pkg.set_kernel_timing(True)
    try:
        assert _call(lib, "dsa_topk_indexer_launch", w, got) == 0
        assert _call(lib, "dsa_topk_indexer_launch_noalloc", w, got) == 0
        assert pkg.last_path() == "noalloc"
        assert pkg.last_kernel_ms() > 0.0
    finally:
        pkg.set_kernel_timing(False)
    torch.cuda.synchronize()


def test_noalloc_rejects_batch_above_capacity():
    pkg = package()
    lib = pkg._lib.load()
    P = ctypes.c_void_p
    ok = P(256)
    rc = lib.dsa_topk_indexer_launch_noalloc(ok, ok, ok, ok, ok, ok, pkg._lib.DSA_NOALLOC_MAX_BATCH + 1, 4, 16, None)
    assert rc == pkg._lib.DSA_ERR_TOO_LARGE
    assert b"65536" in lib.dsa_topk_indexer_error_string(rc)
