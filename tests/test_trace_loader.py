"""FlashInfer-Bench workload files: loading (CPU) and a run through the
indexer with the parity check (GPU)."""
import json
import os

import pytest
import torch
from safetensors.torch import save_file

from conftest import package, workloads


def _write(dirname, name, seq_lens, pages, seed):
    g = torch.Generator().manual_seed(seed)
    max_pages = max(1, max((s + 63) // 64 for s in seq_lens))
    perm = torch.randperm(pages, generator=g).to(torch.int32)
    bt = torch.zeros((len(seq_lens), max_pages), dtype=torch.int32)
    off = 0
    for i, s in enumerate(seq_lens):
        n = (s + 63) // 64
        bt[i, :n] = perm[off:off + n]
        off += n
    path = os.path.join(dirname, name + ".safetensors")
    save_file({"block_table": bt, "seq_lens": torch.tensor(seq_lens, dtype=torch.int32)}, path)
    return path


def test_load_safetensors_workload(tmp_path):
    W = workloads()
    p = _write(str(tmp_path), "wl_a", [100, 3000, 0, 2049], 100, 1)
    w = W.load_safetensors_workload(p, seed=3)
    assert w.batch == 4 and w.max_pages == 47 and w.q.dtype == torch.float8_e4m3fn
    assert w.num_pages == int(w.block_table.max()) + 1
    assert w.k_cache.shape == (w.num_pages, 64, 1, 132) and w.weights.shape == (4, 64)
    w2 = W.load_safetensors_workload(p, seed=3, k_init="randint")
    assert w2.k_cache.dtype == torch.uint8 and int(w2.k_cache.max()) > 200  # full byte range
    with pytest.raises(ValueError):
        W.load_safetensors_workload(p, k_init="bogus")


def test_loader_rejects_bad_files(tmp_path):
    W = workloads()
    p = os.path.join(str(tmp_path), "bad.safetensors")
    save_file({"seq_lens": torch.tensor([5], dtype=torch.int32)}, p)
    with pytest.raises(ValueError):
        W.load_safetensors_workload(p)


@pytest.mark.gpu
def test_trace_runner_parity(tmp_path, capsys):
    pkg = package()
    _write(str(tmp_path), "wl_a", [100, 3000, 0, 2049], 100, 1)
    _write(str(tmp_path), "wl_b", [9000, 64], 200, 2)
    import check_traces  # tests/: the runner with the oracle parity hook
    rows = check_traces.main([str(tmp_path), "--iters", "3"])
    assert [r["workload"] for r in rows] == ["wl_a", "wl_b"]
    assert all(r["parity"] == "pass" for r in rows), rows
