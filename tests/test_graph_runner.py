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
