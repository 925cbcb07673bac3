"""Runs the indexer over a directory of FlashInfer-Bench workload files.

    python -m <package>.trace_runner DIR [--k-init normal|randint] [--iters N]

Every `*.safetensors` file in DIR (structural tensors block_table and
seq_lens, see workloads.load_safetensors_workload) becomes one workload;
q, weights and the K pages are synthesised. For each workload the indexer
runs on the current GPU; the output prints one JSON line with the shapes and
the median device time over N calls (CUDA events). `main(..., on_result=f)`
calls f(workload, topk_indices_on_host, record) for each workload before the
line is printed (tests/check_traces.py uses it to check every result against
the CPU oracle).
"""
import argparse
import glob
import importlib
import json
import os


def main(argv=None, on_result=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("dir")
    ap.add_argument("--k-init", choices=["normal", "randint"], default="normal")
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--seed", type=int, default=0)
    args = ap.parse_args(argv)
    import torch
    pkg = importlib.import_module(__package__)
    wl = importlib.import_module(__package__ + ".workloads")
    files = sorted(glob.glob(os.path.join(args.dir, "*.safetensors")))
    if not files:
        raise SystemExit(f"no *.safetensors files in {args.dir}")
    rows = []
    for path in files:
        w = wl.load_safetensors_workload(path, seed=args.seed, k_init=args.k_init)
        d = w.to("cuda")
        out = torch.empty((w.batch, 2048), dtype=torch.int32, device="cuda")
        pkg.launch_topk_c(d.q, d.k_cache, d.weights, d.seq_lens, d.block_table, out)
        torch.cuda.synchronize()
        times = []
        for _ in range(args.iters):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            pkg.launch_topk_c(d.q, d.k_cache, d.weights, d.seq_lens, d.block_table, out)
            b.record()
            b.synchronize()
            times.append(a.elapsed_time(b))
        rec = {"workload": w.name, "batch": w.batch, "max_num_pages": w.max_pages, "num_pages": w.num_pages,
               "visible_keys": w.visible_keys(), "ms_median": sorted(times)[len(times) // 2],
               "schedule": pkg.last_path()}
        if on_result is not None:
            on_result(w, out.cpu(), rec)
        print(json.dumps(rec), flush=True)
        rows.append(rec)
    return rows


if __name__ == "__main__":
    main()
