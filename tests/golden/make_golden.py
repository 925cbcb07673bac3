"""Generates the golden fixtures in this directory.

Inputs are regenerated from seeds by the package's workload generators
(their SHA-256 is stored and checked, so a change in the generator or the RNG
is detected instead of silently comparing different data); the known-answer
case is built explicitly. Outputs come from the PyTorch restatement of the
reference definition (oracle/reference_torch.py), i.e. the grader's
dequantisation quoted at methodology/framework/CLAUDE (16).md:505-517 and the
math of methodology/checkpoints/kernel_naive.cu:92-113.

Run:  python tests/golden/make_golden.py
"""
import hashlib
import importlib
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
wl = importlib.import_module("karnbirkhera-mlsys2026-dsa_topk_indexer_b200.workloads")
import reference_torch as rt  # noqa: E402

E4M3_ONE, E4M3_FOUR = 0x38, 0x48  # 1.0 and 4.0 (reference diagnostic_tests/run_tmem2_p11.py:87-91)


def kat_diag():
    """Known answer: Q head h = e_h (1.0 on the diagonal), logical page 0 has
    token t = e_t, logical page 1 has token t = 4 e_t, all scales 1 and
    weights (h+1)/64. So score(pos t) = (t+1)/64 and score(pos 64+t) =
    4(t+1)/64, exact in fp32, with exact ties (e.g. pos 3 and pos 64) that the
    smaller position must win. Physical pages are swapped (block_table [1, 0])."""
    q = torch.zeros((1, 64, 128), dtype=torch.uint8)
    for h in range(64):
        q[0, h, h] = E4M3_ONE
    kc = torch.zeros((2, 8448), dtype=torch.uint8)
    for phys, val in ((1, E4M3_ONE), (0, E4M3_FOUR)):
        for t in range(64):
            kc[phys, t * 128 + t] = val
        kc[phys, 8192:] = torch.ones(64, dtype=torch.float32).view(torch.uint8)
    w = (torch.arange(64, dtype=torch.float32) + 1) / 64
    return wl.Workload("kat_diag", q.view(torch.float8_e4m3fn), kc.view(2, 64, 1, 132), w.view(1, 64),
                       torch.tensor([128], dtype=torch.int32), torch.tensor([[1, 0]], dtype=torch.int32))


def cases():
    yield kat_diag(), None
    yield wl.config(0), {"kind": "config", "idx": 0}
    edge = [0, 1, 63, 64, 65, 127, 2047, 2048, 2049, 5000]
    yield wl.custom(edge, seed=11, max_pages=100), {"kind": "custom", "seq_lens": edge, "seed": 11, "max_pages": 100}
    lu = [3000, 2048, 4100]
    yield (wl.custom(lu, seed=12, scale_dist="loguniform"),
           {"kind": "custom", "seq_lens": lu, "seed": 12, "scale_dist": "loguniform"})
    yield (wl.make_shared("prefill_mini", 24, 2112, 40, 13),
           {"kind": "shared", "n_queries": 24, "total_keys": 2112, "pool_pages": 40, "seed": 13})


def input_digest(w):
    h = hashlib.sha256()
    for t in (w.q.view(torch.uint8), w.k_cache.view(torch.uint8), w.weights, w.seq_lens, w.block_table):
        h.update(t.contiguous().numpy().tobytes())
    return h.hexdigest()


def main():
    for w, spec in cases():
        out, rows = rt.indexer(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, return_scores=True)
        scores = np.concatenate([r.numpy().astype(np.float32) for r in rows]) if rows else np.zeros(0, np.float32)
        payload = {"out": out.numpy(), "scores": scores, "digest": np.array(input_digest(w))}
        if spec is None:  # explicit inputs are small: store them
            payload.update(q=w.q.view(torch.uint8).numpy(), k_cache=w.k_cache.view(torch.uint8).numpy(),
                           weights=w.weights.numpy(), seq_lens=w.seq_lens.numpy(), block_table=w.block_table.numpy())
        else:
            payload["spec"] = np.array(repr(spec))
        path = os.path.join(HERE, f"{w.name if spec is None or spec['kind'] != 'custom' else 'custom_' + str(spec['seed'])}.npz")
        np.savez_compressed(path, **payload)
        print(path, os.path.getsize(path), "bytes")


if __name__ == "__main__":
    main()
