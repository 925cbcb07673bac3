"""Runs the indexer over a directory of FlashInfer-Bench workload files.

    python -m <package>.trace_runner DIR [--k-init normal|randint] [--check] [--iters N]

Every `*.safetensors` file in DIR (structural tensors block_table and
seq_lens, see workloads.load_safetensors_workload) becomes one workload;
q, weights and the K pages are synthesised. For each workload the indexer
runs on the current GPU; the output prints one JSON line with the shapes, the
median device time over N calls (CUDA events) and, with --check, the result
of the parity rule against the CPU oracle (oracle/, present in a source
checkout only; test infrastructure).
"""
import argparse
import glob
import importlib
import json
import os
import sys


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("dir")
    ap.add_argument("--k-init", choices=["normal", "randint"], default="normal")
    ap.add_argument("--check", action="store_true")
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
        if args.check:
            root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
            for p in (os.path.join(root, "oracle"), os.path.join(root, "tests")):
                if p not in sys.path:
                    sys.path.insert(0, p)
            import oracle  # test infrastructure: the CPU restatement
            from parity import check_all
            ref = oracle.indexer(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table)
            sc = oracle.scores(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table)
            sl = w.seq_lens.clamp(0, w.max_pages * 64).tolist()
            fails = check_all(out.cpu().numpy(), ref, [sc[i, :s] for i, s in enumerate(sl)], w.seq_lens.numpy(),
                              w.block_table.numpy(), w.num_pages)
            rec["parity"] = "pass" if not fails else f"{len(fails)} failures"
        print(json.dumps(rec), flush=True)
        rows.append(rec)
    return rows


if __name__ == "__main__":
    main()
