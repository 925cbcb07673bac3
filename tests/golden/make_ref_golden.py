"""Golden fixtures from the REFERENCE's own CUDA kernel, run on a B200.

The reference's `launch_topk_c` (solution/cuda/kernel.cu:818-891 of the
reference repository) is compiled from its sources by oracle/build_ref.py
into oracle/_ref/ (test infrastructure, git-ignored, built on the development
machine and carried to the GPU machine). This script runs it on inputs that
its host code accepts (max_pages * 64 <= 8192, kernel.cu:858-859, and every
block-table entry a valid page id, since its scoring kernel reads all of
them) and stores its outputs as `refkernel_*.npz`. The fixtures have the
same layout as make_golden.py's, so tests/test_oracle.py pins the oracle to
the reference kernel itself and the GPU golden test compares this library
with it. The score rows stored beside the outputs (for the near-tie rule)
come from the PyTorch restatement (oracle/reference_torch.py).

With --time it also times the reference kernel beside this library's on
config 0 and config 3 (direct calls on the current stream, CUDA events,
256 MB L2 flush before every call, about 1.5 s of calls per arm with the
SM clocks and throttle reasons sampled meanwhile) and prints one JSON line
per config. With --time-only it skips writing the fixtures.

Run on a GPU machine:  python tests/golden/make_ref_golden.py [--time] [--out DIR]
(--out writes the fixtures elsewhere, e.g. a folder the GPU machine returns.)
"""
import importlib
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))
wl = importlib.import_module("karnbirkhera-mlsys2026-dsa_topk_indexer_b200.workloads")
import build_ref  # noqa: E402  (oracle/build_ref.py)
import reference_torch as rt  # noqa: E402
from make_golden import input_digest  # noqa: E402

CFG3_ROWS = [0, 1, 63, 64, 1000, 2046, 2047, 2048, 2049, 4095, 5000, 6143, 7000, 8190, 8191]


def select_rows(w, rows):
    idx = torch.as_tensor(rows)
    return wl.Workload(w.name, w.q[idx].contiguous(), w.k_cache, w.weights[idx].contiguous(),
                       w.seq_lens[idx].contiguous(), w.block_table[idx].contiguous())


def cases():
    yield "refkernel_cfg0", wl.config(0), {"kind": "config", "idx": 0}
    yield ("refkernel_cfg3_rows", select_rows(wl.config(3), CFG3_ROWS),
           {"kind": "config_rows", "idx": 3, "rows": CFG3_ROWS})
    edge = [1, 65, 2047, 2048, 2049, 8192, 5000, 128]
    yield ("refkernel_edge", wl.custom(edge, seed=21, max_pages=128),
           {"kind": "custom", "seq_lens": edge, "seed": 21, "max_pages": 128})
    lu = [3000, 2048, 4100, 8000]
    yield ("refkernel_loguniform", wl.custom(lu, seed=22, scale_dist="loguniform", max_pages=128),
           {"kind": "custom", "seq_lens": lu, "seed": 22, "scale_dist": "loguniform", "max_pages": 128})


def run_ref(ref, w):
    d = w.to("cuda")
    out = torch.full((w.batch, 2048), -7, dtype=torch.int32, device="cuda")
    ref.launch_topk_c(d.q, d.k_cache, d.weights, d.seq_lens, d.block_table, out)
    torch.cuda.synchronize()
    return out.cpu()


def make(ref, out_dir):
    for name, w, spec in cases():
        assert w.max_pages * 64 <= 8192
        out = run_ref(ref, w).numpy()
        _, rows = rt.indexer(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, return_scores=True)
        scores = np.concatenate([r.numpy().astype(np.float32) for r in rows])
        path = os.path.join(out_dir, name + ".npz")
        np.savez_compressed(path, out=out, scores=scores, digest=np.array(input_digest(w)), spec=np.array(repr(spec)),
                            source=np.array("reference kernel.cu launch_topk_c on B200"))
        print(path, os.path.getsize(path), "bytes", flush=True)


def time_call(fn, flush, min_seconds=1.5, warmup=3):
    """Median device time of fn() (CUDA events on the current stream, 256 MB
    L2 flush before every call) over enough calls to run about min_seconds,
    with the GPU's clocks sampled by nvidia-smi meanwhile (bench.py's
    ClockSampler: reads only, changes no setting). Returns (ms, clocks)."""
    from bench import ClockSampler  # repository root
    for _ in range(warmup):
        flush.zero_()
        fn()
    torch.cuda.synchronize()
    st = torch.cuda.current_stream()
    a0, b0 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a0.record(st)
    for _ in range(5):
        flush.zero_()
        fn()
    b0.record(st)
    torch.cuda.synchronize()
    iters = max(20, int(min_seconds * 1e3 / max(a0.elapsed_time(b0) / 5, 1e-3)))
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(iters)]
    with ClockSampler(torch.cuda.current_device()) as clk:
        for a, b in ev:
            flush.zero_()
            a.record(st)
            fn()
            b.record(st)
        torch.cuda.synchronize()
    return sorted(a.elapsed_time(b) for a, b in ev)[iters // 2], dict(clk.summary(), calls=iters)


def head_to_head(ref):
    """Reference kernel vs this library on configs 0 and 3 (the configs the
    reference's host code accepts), one JSON line per config with both arms'
    clock records."""
    pkg = importlib.import_module("karnbirkhera-mlsys2026-dsa_topk_indexer_b200")
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    for idx in (0, 3):
        w = wl.config(idx, device="cuda")
        o_ref = torch.empty((w.batch, 2048), dtype=torch.int32, device="cuda")
        o_our = torch.empty_like(o_ref)
        t_ref, c_ref = time_call(lambda: ref.launch_topk_c(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table,
                                                           o_ref), flush)
        t_our, c_our = time_call(lambda: pkg.launch_topk_c(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table,
                                                           o_our), flush)
        same = float((o_ref == o_our).float().mean())
        print(json.dumps({"config": idx, "rows": w.batch, "reference_ms_median": t_ref, "ours_ms_median": t_our,
                          "speedup": t_ref / t_our, "identical_slot_fraction": same,
                          "reference_clocks": c_ref, "ours_clocks": c_our}), flush=True)
        del w, o_ref, o_our
        torch.cuda.empty_cache()


if __name__ == "__main__":
    ref = build_ref.load_ref()
    out_dir = sys.argv[sys.argv.index("--out") + 1] if "--out" in sys.argv else HERE
    os.makedirs(out_dir, exist_ok=True)
    if "--time-only" not in sys.argv:
        make(ref, out_dir)
    if "--time" in sys.argv or "--time-only" in sys.argv:
        head_to_head(ref)
