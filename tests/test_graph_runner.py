"""Decode-loop graph runner: bucket logic (CPU) and replays equal to direct
calls across changing batches (GPU)."""
import numpy as np
import pytest
import torch

from conftest import package, workloads


def _mod():
    return __import__("importlib").import_module(package().__name__ + ".graph_runner")


def test_buckets():
    m = _mod()
    assert m.bucket_sizes(64) == [1, 2, 4, 8, 16, 32, 64]
    assert m.bucket_sizes(100) == [1, 2, 4, 8, 16, 32, 64, 128]
    assert m.bucket_for(33, m.bucket_sizes(64)) == 64
    assert m.bucket_for(1, [4, 8]) == 4
    with pytest.raises(ValueError):
        m.bucket_for(65, m.bucket_sizes(64))


@pytest.mark.gpu
def test_replays_equal_direct_calls():
    pkg = package()
    m = _mod()
    W = workloads()
    full = W.config(1, device="cuda")  # 64 requests over one pool
    runner = m.GraphRunner(full.k_cache, max_batch=64, max_pages=full.max_pages)
    g = torch.Generator().manual_seed(5)
    for step, B in enumerate([64, 7, 33, 1, 64, 20]):
        rows = torch.randperm(64, generator=g)[:B].cuda()
        q, w, sl = full.q[rows], full.weights[rows], full.seq_lens[rows]
        bt = full.block_table[rows]
        got = runner(q, w, sl, bt).clone()
        ref = torch.empty((B, 2048), dtype=torch.int32, device="cuda")
        pkg.launch_topk_c(q.contiguous(), full.k_cache, w.contiguous(), sl.contiguous(), bt.contiguous(), ref)
        torch.cuda.synchronize()
        assert torch.equal(got, ref), (step, B)
    assert set(runner.graphs) <= {1, 8, 32, 64}
    assert pkg.device_status(0) == 0


@pytest.mark.gpu
def test_decode_step_runner_equals_direct_calls():
    """Indexer + sparse attention in one graph per bucket: replays equal the
    two direct calls across changing batches (top-K bit for bit; the
    attention within its parity tolerance, since the padded bucket may split
    the index lists differently from a direct call on B rows)."""
    pkg = package()
    m = _mod()
    W = workloads()
    lens = [3000, 9000, 700, 16000, 64, 2500, 5000, 1, 12000, 4100, 800, 2048, 2049]
    full = W.custom(lens, seed=21, device="cuda")
    pages = full.num_pages
    g = torch.Generator(device="cuda").manual_seed(6)
    ckv = torch.randn((pages, 64, 512), generator=g, device="cuda").to(torch.bfloat16)
    kpe = torch.randn((pages, 64, 64), generator=g, device="cuda").to(torch.bfloat16)
    qn_all = torch.randn((len(lens), 16, 512), generator=g, device="cuda").to(torch.bfloat16)
    qp_all = torch.randn((len(lens), 16, 64), generator=g, device="cuda").to(torch.bfloat16)
    runner = m.DecodeStepRunner(full.k_cache, ckv, kpe, 0.07, max_batch=16, max_pages=full.max_pages)
    gc = torch.Generator().manual_seed(7)
    for step, B in enumerate([13, 3, 9, 1, 13]):
        rows = torch.randperm(len(lens), generator=gc)[:B].cuda()
        q, w, sl, bt = full.q[rows], full.weights[rows], full.seq_lens[rows], full.block_table[rows]
        qn, qp = qn_all[rows], qp_all[rows]
        topk, out, lse = (t.clone() for t in runner(q, w, sl, bt, qn, qp))
        ref_topk = torch.empty((B, 2048), dtype=torch.int32, device="cuda")
        pkg.launch_topk_c(q.contiguous(), full.k_cache, w.contiguous(), sl.contiguous(), bt.contiguous(), ref_topk)
        ref_out, ref_lse = pkg.sparse_attention(qn.contiguous(), qp.contiguous(), ckv, kpe, ref_topk, 0.07)
        torch.cuda.synchronize()
        assert torch.equal(topk, ref_topk), (step, B)
        assert torch.allclose(out.float(), ref_out.float(), atol=1e-2, rtol=1e-2), (step, B)
        assert torch.allclose(lse, ref_lse, atol=1e-3, rtol=1e-5, equal_nan=False), (step, B)
    assert pkg.device_status(0) == 0
