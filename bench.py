"""Benchmark of the B200 DSA indexer: queries/s on BASELINE config 2 (the
large decode batch the metric is quoted on at 1/2/4/8 B200: 512 requests of
16k..131k keys) by default, one JSON line on rank 0.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--config C] [--impl ours|reference]

A step = one indexer call over the whole batch. `value` is device time (CUDA
events on the launching stream, L2 flushed before every step); `e2e` is the
same call fed from pinned host buffers (q, weights, seq_lens, block_table
host->device, top-K device->host inside the timed region; the paged K cache
is the serving system's resident device state). Under torchrun the one
global batch is split: decode configs by request (balanced by total length,
no collective), the long-context config 4 along the key axis (partial top-K,
then the candidate lists exchanged and merged over NVLink peer memory by the
library's own kernels, or through NCCL with --exchange alltoall|allgather);
both are strong scaling (the global batch is fixed).
"""
import argparse
import importlib
import json
import math
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG_NAME = "karnbirkhera-mlsys2026-dsa_topk_indexer_b200"
sys.path.insert(0, ROOT)

METRIC = "indexer queries/s at 1/2/4/8 B200; % of HBM BW (decode) / FP8 TC peak (prefill)"
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return FALLBACK_HBM_GBS, FALLBACK_BF16_TFLOPS, "fallback"


def traffic_per_launch(config, kernel):
    """DRAM bytes per launch of `kernel` on `config` from the committed ncu
    summaries (profiles/traffic.json), or None."""
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if not os.path.exists(p):
        return None
    return json.load(open(p)).get(f"cfg{config}:{kernel}")


DOMINANT = {"cluster": "dsa::indexer_kernel<0>", "cluster-split": "dsa::indexer_kernel<0>",
            "cluster-tail": "dsa::indexer_kernel<0>",
            "prefill+cluster": "dsa::prefill_kernel<0> + dsa::indexer_kernel<0>"}
DOMINANT_PARTIAL = {"cluster": "dsa::indexer_kernel<2>", "cluster-split": "dsa::indexer_kernel<2>",
                    "cluster-tail": "dsa::indexer_kernel<2>",
                    "prefill+cluster": "dsa::prefill_kernel<2> + dsa::indexer_kernel<2>"}
PREFILL_CONFIGS = (3, 4)
# Configs whose single sequence is split along the key axis across ranks
# (every rank holds the same inputs; partial top-K, NCCL all-gather, merge).
KEY_SHARDED_CONFIGS = (4,)
FLOP_PER_KEY = 64 * 128 * 2  # one query row against one key: 64 heads x 128-dim dot products


class L2Flush:
    """Empties L2 of the step's data before every timed step by writing a
    256 MB buffer (more than the 126 MB L2). The write leaves dirty lines in
    L2 whose write-back overlaps the timed step; that cost is kept (reading
    another buffer afterwards removes it on large steps but slowed the B=1
    decode call by ~10 us, so the plain write is the measurement)."""
    NOTE = "flushed (256 MB write) before every timed step"

    def __init__(self, torch, dev):
        self.w = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device=dev)

    def __call__(self):
        self.w.zero_()


class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index):
        self.dev = device_index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.dev), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc is not None:
            time.sleep(0.2)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [ln for ln in out.splitlines() if ln.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in getattr(self, "lines", []):
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": mx, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


def cpu_reference_run(w, budget_s, max_queries=None):
    """Times the PyTorch CPU restatement of the reference (oracle/
    reference_torch.py) on a bounded sample of the workload: its first n
    queries (with only the K pages they read, copied to host memory),
    repeated until about `budget_s` seconds of CPU work have run. Returns
    (queries/s, queries timed, seconds, threads, passes)."""
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import reference_torch as rt  # CPU baseline only
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    # probe one query to size the sample
    one, _ = w.compact([0], "cpu")
    t0 = time.perf_counter()
    rt.indexer(one.q, one.k_cache, one.weights, one.seq_lens, one.block_table)
    t1 = time.perf_counter() - t0
    n = max(1, min(w.batch if max_queries is None else max_queries, int(budget_s / max(t1, 1e-4))))
    cpu, _ = w.compact(list(range(n)), "cpu")
    done, passes = 0, 0
    t0 = time.perf_counter()
    while True:
        rt.indexer(cpu.q, cpu.k_cache, cpu.weights, cpu.seq_lens, cpu.block_table)
        done += n
        passes += 1
        dt = time.perf_counter() - t0
        if dt >= budget_s:
            break
    return done / dt, done, dt, threads, passes


def cpu_port_rate(fn, units_per_call, budget_s):
    """Times fn() (a call of the CPU restatement in oracle/reference_torch.py
    on a bounded sample covering `units_per_call` units) until about
    `budget_s` seconds have run, on all host threads. Returns (units/s,
    threads, calls)."""
    import torch
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    calls = 0
    t0 = time.perf_counter()
    while True:
        fn()
        calls += 1
        dt = time.perf_counter() - t0
        if dt >= budget_s:
            break
    return units_per_call * calls / dt, threads, calls


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--batch-scale", type=float, default=1.0,
                    help="profiling only: run the config with its batch scaled down (ncu captures)")
    ap.add_argument("--op", choices=["indexer", "cache_write", "sparse_attention", "decode_loop"], default="indexer",
                    help="cache_write: the index-K cache writer (FP8 quantiser); sparse_attention: the "
                         "consumer of topk_indices (sparse MLA attention over the selected slots); "
                         "decode_loop: a decode loop over --config's requests through the device work "
                         "queue and through the per-step graph runner")
    ap.add_argument("--attn-tokens", type=int, default=128, help="sparse_attention: query tokens per step")
    ap.add_argument("--tokens", type=int, default=1 << 20, help="cache_write: tokens per step")
    ap.add_argument("--exchange", choices=["peer", "alltoall", "allgather"], default="peer",
                    help="key-sharded configs at N>1: how the per-rank candidate lists meet (peer: NVLink "
                         "peer memory, the library's own kernels; alltoall / allgather: NCCL)")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)

    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    wl = importlib.import_module(PKG_NAME + ".workloads")

    if args.impl == "reference":
        return reference_arm(args, rank, wl)
    if args.op == "cache_write":
        return cache_write_bench(args, rank, local)
    if args.op == "sparse_attention":
        return sparse_attention_bench(args, rank, local)
    if args.op == "decode_loop":
        return decode_loop_bench(args, rank, local)

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    pkg = importlib.import_module(PKG_NAME)
    pkg._lib.load()

    key_sharded = world > 1 and args.config in KEY_SHARDED_CONFIGS
    # Every rank builds the same global workload (same seed); request-sharded
    # ranks then keep their share of the rows, balanced by total length.
    w = wl.config(args.config, device=dev, seed=args.config, scale_batch=args.batch_scale)
    global_batch = w.batch
    global_kbytes = w.kcache_bytes()
    if world > 1 and not key_sharded:
        sh = importlib.import_module(PKG_NAME + ".sharding")
        w = w.rows(sh.request_shards(w.seq_lens, world)[rank])
    B = w.batch
    out = torch.empty((B, 2048), dtype=torch.int32, device=dev)
    flush = L2Flush(torch, dev)
    stream = torch.cuda.current_stream(dev)

    peer_ex = None
    if key_sharded:
        sh = importlib.import_module(PKG_NAME + ".sharding")
        counts = {}

        def pfn(*a):
            r = pkg.indexer_partial(*a)
            counts["p"] = pkg.last_launch_count()
            counts["path"] = pkg.last_path()
            if counts.get("timing"):  # the merge call after this one resets the kernel timer
                counts["kms"] = pkg.last_kernel_ms()
            return r

        def mfn(*a):
            r = pkg.indexer_merge(*a)
            counts["m"] = pkg.last_launch_count()
            return r

        # exchange="peer": candidate lists exchanged and merged over NVLink
        # peer memory by the library's own kernels (no NCCL on the data path).
        peer_ex = sh.PeerExchange(B, dev) if args.exchange == "peer" and world > 1 else None

        def run_sharded(q, kc, wt, sl, bt):
            out.copy_(sh.key_sharded_topk(q, kc, wt, sl, bt, partial_fn=pfn, merge_fn=mfn,
                                          exchange=args.exchange if peer_ex else
                                          ("alltoall" if args.exchange == "peer" else args.exchange),
                                          peer=peer_ex))
            if peer_ex is not None:
                counts["m"] = pkg.last_launch_count()
            return counts["p"] + counts["m"]

        def call():
            return run_sharded(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table)
    elif B > 0:
        def call():
            pkg.launch_topk_c(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, out)
            return pkg.last_launch_count()
    else:  # a rank with no rows of the global batch (more ranks than rows)
        def call():
            return 0

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    # Warm-up runs on the stream the step is later captured on: the library
    # creates its per-stream workspace on the first call, outside capture.
    cap_stream = torch.cuda.Stream(dev)
    cap_stream.wait_stream(stream)
    with torch.cuda.stream(cap_stream):
        for _ in range(args.warmup):
            flush()
            call()
    torch.cuda.synchronize()
    pkg.device_status(local, clear=True)

    # The step is captured once into a CUDA graph, so the device-timed region
    # measures the kernels, not Python launch overhead (the e2e region below
    # keeps direct calls). Key-sharded steps (NCCL collectives, milliseconds
    # long) are launched directly.
    graph = None
    if key_sharded:
        per_step = call()
        torch.cuda.synchronize()
    else:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=cap_stream):
            per_step = call()
        torch.cuda.synchronize()

    # ---------------- device-timed region ----------------
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    launches = 0
    barrier()
    torch.cuda.synchronize()
    with ClockSampler(local) as clk:
        for i in range(args.steps):
            flush()
            starts[i].record(stream)
            if graph is not None:
                graph.replay()
            else:
                call()
            ends[i].record(stream)
            launches += per_step
        torch.cuda.synchronize()
    barrier()
    step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    ms = sum(step_ms) / len(step_ms)
    status = pkg.device_status(local, clear=True)

    # ---------------- dominant-kernel time (roofline) ----------------
    # The library brackets the call's dominant kernel with CUDA events on
    # the launching stream; a separate pass of the same K steps (the events
    # keep the bracketed kernel from overlapping its neighbours).
    pkg.set_kernel_timing(True)
    kms = []
    if key_sharded:
        counts["timing"] = True
    for i in range(args.steps if B > 0 else 0):
        flush()
        call()
        kms.append(counts["kms"] if key_sharded else pkg.last_kernel_ms())
    pkg.set_kernel_timing(False)
    if key_sharded:
        counts["timing"] = False
    path = (counts["path"] if key_sharded else pkg.last_path()) if B > 0 else "idle"
    kernel_ms = sum(kms) / len(kms) if kms else 0.0

    # ---------------- end-to-end region (host buffers) ----------------
    # A serving loop stages the step's small inputs (q, weights, seq_lens,
    # block table) in one pinned host buffer and moves them with one copy;
    # the result comes back with another. Both copies are inside the timed
    # region; the K cache is resident device state.
    def align(n):
        return (n + 255) // 256 * 256
    parts = [w.q.view(torch.uint8).reshape(-1), w.weights.view(torch.uint8).reshape(-1),
             w.seq_lens.view(torch.uint8).reshape(-1), w.block_table.view(torch.uint8).reshape(-1)]
    offs, off = [], 0
    for t in parts:
        offs.append(off)
        off = align(off + t.numel())
    h_in = torch.empty(off, dtype=torch.uint8).pin_memory()
    for t, o in zip(parts, offs):
        h_in[o:o + t.numel()].copy_(t.cpu())

    def views(d_in):
        return (d_in[offs[0]:offs[0] + parts[0].numel()].view(torch.float8_e4m3fn).view(w.q.shape),
                d_in[offs[1]:offs[1] + parts[1].numel()].view(torch.float32).view(w.weights.shape),
                d_in[offs[2]:offs[2] + parts[2].numel()].view(torch.int32).view(w.seq_lens.shape),
                d_in[offs[3]:offs[3] + parts[3].numel()].view(torch.int32).view(w.block_table.shape))
    # Two sets of device inputs / outputs and host result buffers, so that a
    # pipelined step's copies can overlap the neighbouring steps' kernels.
    d_ins = [torch.empty(off, dtype=torch.uint8, device=dev) for _ in range(2)]
    outs = [out, torch.empty_like(out)]
    h_outs = [torch.empty((B, 2048), dtype=torch.int32).pin_memory() for _ in range(2)]
    h2d = sum(t.numel() for t in parts)
    d2h = h_outs[0].numel() * 4

    def compute(b):
        d_q, d_w, d_sl, d_bt = views(d_ins[b])
        if key_sharded:
            run_sharded(d_q, w.k_cache, d_w, d_sl, d_bt)
            if b:
                outs[1].copy_(out)
        elif B > 0:
            pkg.launch_topk_c(d_q, w.k_cache, d_w, d_sl, d_bt, outs[b])

    # Serial (every step: H2D, kernel, D2H, one after the other, L2 flushed
    # before each step outside its timing) when the step's K pages would fit
    # in L2; pipelined when they are far larger than L2 (no flush needed):
    # the inputs of step i+1 go up on one copy stream and the result of step
    # i-1 comes back on another while step i runs; K steps are timed as one
    # span, every step's copies inside it.
    # Unique K bytes a step touches: its visible pages, at most the pool.
    footprint = min(w.k_cache.numel() * w.k_cache.element_size(), w.kcache_bytes())
    pipelined = not key_sharded and footprint > 2 * torch.cuda.get_device_properties(dev).L2_cache_size
    if not pipelined:
        def e2e_call():
            d_ins[0].copy_(h_in, non_blocking=True)
            compute(0)
            h_outs[0].copy_(outs[0], non_blocking=True)

        for _ in range(3):
            flush()
            e2e_call()
        torch.cuda.synchronize()
        es = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        ee = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        barrier()
        torch.cuda.synchronize()
        for i in range(args.steps):
            flush()
            es[i].record(stream)
            e2e_call()
            ee[i].record(stream)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = sum(s.elapsed_time(e) for s, e in zip(es, ee)) / args.steps
        last = 0
    else:
        s_in, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev)
        ev_in = [torch.cuda.Event() for _ in range(2)]
        ev_k = [torch.cuda.Event() for _ in range(2)]
        ev_out = [torch.cuda.Event() for _ in range(2)]

        def run_steps(n):
            for i in range(n):
                b = i & 1
                with torch.cuda.stream(s_in):
                    if i >= 2:
                        s_in.wait_event(ev_k[b])  # step i-2's kernel has read d_ins[b]
                    d_ins[b].copy_(h_in, non_blocking=True)
                    ev_in[b].record(s_in)
                stream.wait_event(ev_in[b])
                if i >= 2:
                    stream.wait_event(ev_out[b])  # step i-2's result has left outs[b]
                compute(b)
                ev_k[b].record(stream)
                with torch.cuda.stream(s_out):
                    s_out.wait_event(ev_k[b])
                    h_outs[b].copy_(outs[b], non_blocking=True)
                    ev_out[b].record(s_out)
            stream.wait_stream(s_out)

        run_steps(4)
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        s_in.wait_stream(stream)
        run_steps(args.steps)
        e1.record(stream)
        torch.cuda.synchronize()
        barrier()
        e2e_ms = e0.elapsed_time(e1) / args.steps
        last = (args.steps - 1) & 1
    assert torch.equal(h_outs[last], out.cpu()), "e2e output mismatch"
    e2e_mode = ("pipelined: step i+1's inputs copied and step i-1's result read back while step i runs "
                "(two copy streams, double-buffered; K pages far larger than L2, no flush)") if pipelined else \
        "serial: H2D, call, D2H per step; L2 flushed before every step"

    # max over ranks
    t = torch.tensor([ms, e2e_ms, kernel_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max, e2e_max, kms_max = float(t[0]), float(t[1]), float(t[2])
    # Roofline of the slowest rank's dominant kernel: that rank's bytes.
    kb = torch.tensor([float(kernel_ms), float(w.kcache_bytes())], dtype=torch.float64, device=dev)
    if world > 1 and not key_sharded:
        allk = [torch.zeros_like(kb) for _ in range(world)]
        dist.all_gather(allk, kb)
        kb = max(allk, key=lambda x: float(x[0]))
    kbytes = int(kb[1])
    hbm, bf16, peak_src = peaks()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        qps, n, dt, threads, passes = cpu_reference_run(w, budget_s=10.0)
        cpu = {"value": qps, "unit": "queries/s", "cores": threads, "kind": "port",
               "sample": f"{n} queries ({passes} passes over the first {n // passes} of {B} queries of {w.name}, "
                         f"their K pages copied to host memory) through the PyTorch CPU restatement "
                         f"(oracle/reference_torch.py), {dt:.2f} s"}

    if rank == 0:
        kernel = (DOMINANT_PARTIAL.get(path, path) + " (partial, key range)") if key_sharded else DOMINANT.get(path, path)
        tr = traffic_per_launch(args.config, kernel)
        if tr is not None and not key_sharded and args.config not in PREFILL_CONFIGS and kbytes != global_kbytes:
            # The table holds the whole batch's launch; a rank's launch moves its
            # share (DRAM traffic grows with the K bytes a launch reads).
            tr = int(round(tr * kbytes / global_kbytes))
        if args.config in PREFILL_CONFIGS:
            # K is L2-resident (one sequence): the contraction on the tensor
            # cores bounds the kernel. B200's dense fp8 rate is twice bf16.
            # Key-sharded: each rank's partial kernel scores 1/world of the keys.
            flops = (kbytes // 132) * FLOP_PER_KEY // (world if key_sharded else 1)
            achieved = flops / (kms_max * 1e-3) / 1e12
            roof = {"bound": "tensor", "achieved": achieved, "peak": 2 * bf16, "unit": "TFLOP/s",
                    "frac": achieved / (2 * bf16), "traffic": tr,
                    "peak_source": f"2 x {peak_src} bf16 dense (fp8 dense rate)",
                    "algorithmic_flops_per_launch": flops}
        else:
            achieved = kbytes / (kms_max * 1e-3) / 1e9
            # Beside the K-cache bytes (the roofline unit): every byte the call
            # touches once (q, weights, seq_lens, block table, output).
            total = (kbytes + w.q.numel() + w.weights.numel() * 4 + w.seq_lens.numel() * 4
                     + w.block_table.numel() * 4 + B * 2048 * 4)
            roof = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                    "traffic": tr, "peak_source": peak_src, "algorithmic_bytes_per_launch": kbytes,
                    "total_bytes_per_launch": total}
        roof.update({"kernel": kernel, "kernel_ms": kms_max, "schedule": path,
                     "kernel_timing": "CUDA events on the launching stream around the kernel, "
                                      "separate pass of the same steps"})
        line = {
            "metric": METRIC, "value": global_batch / (ms_max * 1e-3), "unit": "queries/s",
            "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None,
            "dtype": "fp8_e4m3 (fp32 accumulate)", "data": "synthetic",
            "config": {"workload": w.name + ("" if args.batch_scale == 1.0 else f" (batch x{args.batch_scale})"),
                       "batch_per_gpu": B, "global_batch": global_batch,
                       "visible_keys_per_gpu": w.visible_keys() // (world if key_sharded else 1),
                       "global_kcache_bytes": global_kbytes,
                       "max_pages": w.max_pages,
                       "pool_pages": w.num_pages,
                       "parallelism": (f"key-sharded x{world} (candidate lists read over NVLink peer memory by a "
                                       "fused merge kernel that stores each row into every rank; no NCCL on the "
                                       "data path)" if args.exchange == "peer" else
                                       f"key-sharded x{world} (NCCL all-to-all of candidate lists, merge, all-gather "
                                       "of results)" if args.exchange == "alltoall" else
                                       f"key-sharded x{world} (NCCL all-gather of candidate lists + merge)")
                       if key_sharded
                       else f"request-sharded x{world} (rows split by total length, no collective)",
                       "l2": L2Flush.NOTE},
            "e2e": {"value": global_batch / (e2e_max * 1e-3), "unit": "queries/s",
                    "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h, "ms_per_step": e2e_max, "mode": e2e_mode,
                    "kcache": "resident in HBM (persistent serving state)"},
            "roofline": roof,
            "gpu_launches": launches,
            "clocks": clk.summary(),
            "status_word": status,
            "step_ms_min_median_max": [min(step_ms), statistics.median(step_ms), max(step_ms)],
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    del graph
    if peer_ex is not None:
        peer_ex.close()  # every rank together, before the group goes away
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def cache_write_bench(args, rank, local):
    """The index-K cache writer: `--tokens` bf16 vectors of 128 values,
    quantised into a paged FP8 cache at a random permutation of its slots
    (every page gets all 64 of its tokens). HBM-bound: per token 256 B read,
    8 B slot read, 132 B written. One process; rank 0 prints."""
    import torch
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pkg = importlib.import_module(PKG_NAME)
    T = args.tokens
    pages = (T + 63) // 64
    g = torch.Generator(device=dev)
    g.manual_seed(7)
    k = (torch.randn((T, 128), generator=g, device=dev) * 0.5).to(torch.bfloat16)
    slots = torch.randperm(pages * 64, generator=g, device=dev)[:T].to(torch.int64)
    cache = torch.zeros((pages, 64, 1, 132), dtype=torch.uint8, device=dev)
    flush = L2Flush(torch, dev)
    for _ in range(max(3, args.warmup)):
        flush()
        pkg.index_cache_write(k, slots, cache)
    torch.cuda.synchronize()
    st = torch.cuda.current_stream(dev)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        for a, b in ev:
            flush()
            a.record(st)
            pkg.index_cache_write(k, slots, cache)
            b.record(st)
        torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in ev) / args.steps
    cpu = None
    if not args.no_cpu_baseline:
        # The reference has no writer; the CPU restatement on 65536 tokens.
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import reference_torch as rt  # CPU baseline only
        n = min(T, 65536)
        ks, ss = k[:n].cpu(), slots[:n].cpu() % (((n + 63) // 64) * 64)
        cc = torch.zeros(((n + 63) // 64, 64, 1, 132), dtype=torch.uint8)
        rate, threads, calls = cpu_port_rate(lambda: rt.cache_write(ks, ss, cc), n, 10.0)
        cpu = {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": f"{n} tokens per call, {calls} calls (oracle/reference_torch.py cache_write)"}
    hbm, _, peak_src = peaks()
    algo = T * (256 + 8 + 132)
    achieved = algo / (ms * 1e-3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": "index-K cache writer tokens/s", "value": T / (ms * 1e-3), "unit": "tokens/s",
            "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 -> fp8_e4m3",
            "data": "synthetic",
            "config": {"workload": f"{T} tokens into {pages} pages, random slot permutation",
                       "l2": L2Flush.NOTE},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": None, "peak_source": peak_src,
                         "algorithmic_bytes_per_launch": algo, "kernel": "dsa::cache_write_kernel<true>"},
            "gpu_launches": args.steps, "clocks": clk.summary(), "cpu_baseline": cpu}), flush=True)


def decode_loop_bench(args, rank, local):
    """A decode loop over the requests of `--config` (1 or 2; default 2):
    every step each request grows by one token, taking the next free page of
    the pool when it crosses a page boundary, and the indexer runs over the
    whole batch. q and weights are device tensors, as the model produces
    them. Two host paths, the same device work:
      graph_runner  every step copies seq_lens and the full block table from
                    pinned host memory into the graph's buffers (double-
                    buffered host arrays), then replays the indexer graph;
      decode_queue  every step copies one record (the step's page appends and
                    the batch list) and replays [apply + gather, indexer];
                    the request table stays in device memory.
    K steps timed as one span with CUDA events on the caller's stream (steps
    not synchronised); config 2's K pages are far larger than L2, other
    configs get the L2 flush between steps. Both paths end with bit-equal
    outputs (checked). One process; rank 0 prints."""
    import numpy as np
    import torch
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    wl = importlib.import_module(PKG_NAME + ".workloads")
    gr = importlib.import_module(PKG_NAME + ".graph_runner")
    dqm = importlib.import_module(PKG_NAME + ".decode_queue")
    cfg = 2 if args.config not in (1, 2) else args.config
    w = wl.config(cfg, device=dev)
    B, K, Wm = w.batch, args.steps, max(3, args.warmup)
    total = Wm + K
    sl0 = w.seq_lens.cpu().numpy().astype(np.int64)
    bt0 = w.block_table.cpu().numpy()
    np0 = (sl0 + 63) // 64
    max_pages = int(max(bt0.shape[1], int((sl0 + total + 63).max()) // 64 + 1))
    used = np.zeros(w.num_pages, dtype=bool)
    for b in range(B):
        used[bt0[b, :np0[b]]] = True
    free = np.flatnonzero(~used).astype(np.int64)
    flush = L2Flush(torch, dev) if cfg != 2 else (lambda: None)
    cur = torch.cuda.current_stream(dev)

    def appends(lens, npg):
        """Rows whose next token needs a new page (each takes the next free page)."""
        return np.flatnonzero(lens + 1 > 64 * npg)

    # ---- graph runner: full seq_lens / block table from pinned host memory every step
    runner = gr.GraphRunner(w.k_cache, max_batch=B, max_pages=max_pages, buckets=[B])
    lens, npg, fp = sl0.copy(), np0.copy(), 0
    host = []
    for _ in range(2):
        bt_h = torch.zeros((B, max_pages), dtype=torch.int32).pin_memory()
        bt_h[:, :bt0.shape[1]] = torch.from_numpy(bt0)
        host.append([bt_h, torch.zeros(B, dtype=torch.int32).pin_memory(), None])
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
    for i in range(total):
        if i == Wm:
            torch.cuda.synchronize()
            ev[0].record(cur)
            t0 = time.perf_counter()
        bt_h, sl_h, done = host[i % 2]
        if done is not None:
            done.synchronize()
        rows = appends(lens, npg)
        # Both host copies get the new pages; the other copy may still be in
        # flight for the previous step, which does not read these entries.
        for h in host:
            h[0][rows, npg[rows]] = torch.from_numpy(free[fp:fp + rows.size].astype(np.int32))
        fp += rows.size
        npg[rows] += 1
        lens += 1
        sl_h.copy_(torch.from_numpy(lens.astype(np.int32)))
        flush()
        out_a = runner(w.q, w.weights, sl_h, bt_h)
        e = torch.cuda.Event()
        e.record(runner.stream)
        host[i % 2][2] = e
    ev[1].record(cur)
    torch.cuda.synchronize()
    t_host_a = (time.perf_counter() - t0) / K
    ms_a = ev[0].elapsed_time(ev[1]) / K
    out_a = out_a.clone()
    h2d_a = B * 4 + B * max_pages * 4

    # ---- device work queue: one record per step, the request table on the device
    dq = dqm.DecodeQueue(w.k_cache, num_slots=B, max_pages=max_pages, max_batch=B, buckets=[B],
                         record_words=int(np0.sum()) + 8 * B + 64)
    for b in range(B):
        dq.admit(b, int(sl0[b]), bt0[b, :np0[b]])
    slots = np.arange(B)
    lens, npg, fp = sl0.copy(), np0.copy(), 0
    rec_words = 0
    for i in range(total):
        if i == Wm:
            torch.cuda.synchronize()
            ev[0].record(cur)
            t0 = time.perf_counter()
        rows = appends(lens, npg)
        for r, pid in zip(rows.tolist(), free[fp:fp + rows.size].tolist()):
            dq.append_page(r, pid)
        fp += rows.size
        npg[rows] += 1
        lens += 1
        if i >= Wm:
            rec_words += dq.table.record_words(B)
        flush()
        out_b = dq.step(slots, w.q, w.weights)
    ev[1].record(cur)
    torch.cuda.synchronize()
    t_host_b = (time.perf_counter() - t0) / K
    ms_b = ev[0].elapsed_time(ev[1]) / K
    same = bool(torch.equal(out_b, out_a))
    if rank == 0:
        print(json.dumps({
            "metric": "decode-loop queries/s (indexer step with its per-step host-to-device input transfer)",
            "value": B / (ms_b * 1e-3), "unit": "queries/s", "n_gpus": 1, "steps": K, "warmup": Wm,
            "ms_per_step": ms_b, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "fp8_e4m3 (fp32 accumulate)", "data": "synthetic",
            "config": {"workload": w.name + " decode loop (+1 token per request per step)", "batch": B,
                       "max_pages": max_pages, "l2": "K pages far larger than L2" if cfg == 2 else L2Flush.NOTE},
            "decode_queue": {"ms_per_step": ms_b, "h2d_bytes_per_step": 4 * rec_words / K,
                             "host_ms_per_step": t_host_b * 1e3},
            "graph_runner": {"ms_per_step": ms_a, "value": B / (ms_a * 1e-3), "h2d_bytes_per_step": h2d_a,
                             "host_ms_per_step": t_host_a * 1e3},
            "outputs_equal": same, "gpu_launches": 3 * K}), flush=True)


def sparse_attention_bench(args, rank, local):
    """Sparse MLA attention over 2048 selected slots per token (the consumer
    of topk_indices): `--attn-tokens` tokens, 16 heads, a 1.2 GB pool of
    bf16 latent (512) + rope (64) rows, slots drawn uniformly from the pool
    (no reuse between tokens: the worst case for L2). HBM-bound gather:
    per token 2048 x 1152 B of rows + 18 KB q + 16 KB out + 8 KB indices.
    `value` is device-timed with inputs resident; `e2e` copies q and indices
    from pinned host memory and the output and lse back every step."""
    import torch
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    pkg = importlib.import_module(PKG_NAME)
    T, L, pages = args.attn_tokens, 2048, 16384
    g = torch.Generator(device=dev)
    g.manual_seed(11)
    q_nope = torch.randn((T, 16, 512), generator=g, device=dev).to(torch.bfloat16)
    q_pe = torch.randn((T, 16, 64), generator=g, device=dev).to(torch.bfloat16)
    ckv = torch.randn((pages, 64, 512), generator=g, device=dev).to(torch.bfloat16)
    kpe = torch.randn((pages, 64, 64), generator=g, device=dev).to(torch.bfloat16)
    idx = torch.randint(0, pages * 64, (T, L), generator=g, device=dev, dtype=torch.int32)
    out = torch.empty((T, 16, 512), dtype=torch.bfloat16, device=dev)
    lse = torch.empty((T, 16), dtype=torch.float32, device=dev)
    scale = 1.0 / math.sqrt(192.0)
    flush = L2Flush(torch, dev)
    st = torch.cuda.current_stream(dev)
    # Warm-up on the capture stream (the library allocates its split buffers
    # for that stream outside capture), then one CUDA graph of the call, so
    # the device-timed region holds the kernel and not Python launch overhead.
    cap = torch.cuda.Stream(dev)
    cap.wait_stream(st)
    with torch.cuda.stream(cap):
        for _ in range(max(3, args.warmup)):
            flush()
            pkg.sparse_attention(q_nope, q_pe, ckv, kpe, idx, scale, out, lse)
    torch.cuda.synchronize()
    launches = pkg.last_launch_count()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=cap):
        pkg.sparse_attention(q_nope, q_pe, ckv, kpe, idx, scale, out, lse)
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    with ClockSampler(local) as clk:
        for a, b in ev:
            flush()
            a.record(st)
            graph.replay()
            b.record(st)
        torch.cuda.synchronize()
    ms = sum(a.elapsed_time(b) for a, b in ev) / args.steps
    del graph
    # End to end: inputs from pinned host memory, results back to it.
    h_qn, h_qp, h_idx = q_nope.cpu().pin_memory(), q_pe.cpu().pin_memory(), idx.cpu().pin_memory()
    h_out, h_lse = torch.empty_like(out, device="cpu").pin_memory(), torch.empty_like(lse, device="cpu").pin_memory()
    d_qn, d_qp, d_idx = torch.empty_like(q_nope), torch.empty_like(q_pe), torch.empty_like(idx)
    ev2 = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    for i in range(args.steps + 3):
        flush()
        a, b = ev2[i - 3] if i >= 3 else (None, None)
        if a is not None:
            a.record(st)
        d_qn.copy_(h_qn, non_blocking=True)
        d_qp.copy_(h_qp, non_blocking=True)
        d_idx.copy_(h_idx, non_blocking=True)
        pkg.sparse_attention(d_qn, d_qp, ckv, kpe, d_idx, scale, out, lse)
        h_out.copy_(out, non_blocking=True)
        h_lse.copy_(lse, non_blocking=True)
        if b is not None:
            b.record(st)
    torch.cuda.synchronize()
    ms_e2e = sum(a.elapsed_time(b) for a, b in ev2) / args.steps
    h2d = h_qn.numel() * 2 + h_qp.numel() * 2 + h_idx.numel() * 4
    d2h = h_out.numel() * 2 + h_lse.numel() * 4
    cpu = None
    if not args.no_cpu_baseline:
        # The reference has no code for this operator; the CPU restatement on
        # 8 tokens of the same workload.
        sys.path.insert(0, os.path.join(ROOT, "oracle"))
        import reference_torch as rt  # CPU baseline only
        n = min(T, 8)
        c_qn, c_qp, c_ix = q_nope[:n].cpu(), q_pe[:n].cpu(), idx[:n].cpu()
        c_ckv, c_kpe = ckv.cpu(), kpe.cpu()
        rate, threads, calls = cpu_port_rate(lambda: rt.sparse_attention(c_qn, c_qp, c_ckv, c_kpe, c_ix, scale),
                                             n, 10.0)
        cpu = {"value": rate, "unit": "tokens/s", "cores": threads, "kind": "port",
               "sample": f"{n} tokens x 2048 slots per call, {calls} calls (oracle/reference_torch.py sparse_attention)"}
    hbm, _, peak_src = peaks()
    algo = T * (L * 1152 + 16 * 576 * 2 + 16 * 512 * 2 + 16 * 4 + L * 4)
    achieved = algo / (ms * 1e-3) / 1e9
    if rank == 0:
        print(json.dumps({
            "metric": "sparse attention tokens/s (2048 slots each)", "value": T / (ms * 1e-3), "unit": "tokens/s",
            "n_gpus": 1, "steps": args.steps, "warmup": max(3, args.warmup), "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (fp32 accumulate)",
            "data": "synthetic",
            "config": {"workload": f"{T} tokens x 2048 slots, 16 heads, ckv 512 + kpe 64, pool {pages} pages",
                       "l2": L2Flush.NOTE},
            "e2e": {"value": T / (ms_e2e * 1e-3), "unit": "tokens/s", "ms_per_step": ms_e2e,
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                         "frac": achieved / hbm, "traffic": None, "peak_source": peak_src,
                         "algorithmic_bytes_per_launch": algo, "kernel": "dsa::sparse_attention_kernel"},
            "gpu_launches": args.steps * launches, "clocks": clk.summary(), "cpu_baseline": cpu}), flush=True)


def reference_arm(args, rank, wl):
    """The reference's CPU path (the PyTorch restatement of its definition,
    all host threads) on the same workload, metric and config; rank 0 only.
    Each step is a bounded sample: the first n queries of the batch, n sized
    so that the whole run takes about 150 s."""
    if rank != 0:
        return
    import torch
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import reference_torch as rt  # the reference arm's CPU implementation
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    # The same seeded workload as the GPU arm (generated on the GPU when there
    # is one: the generators are seeded per device); the sampled rows and the
    # K pages they read are copied to host memory once.
    gen_dev = "cuda" if torch.cuda.is_available() else "cpu"
    w = wl.config(args.config, device=gen_dev, seed=args.config)
    per_step = 150.0 / (args.steps + args.warmup)
    one, _ = w.compact([0], "cpu")
    t0 = time.perf_counter()
    rt.indexer(one.q, one.k_cache, one.weights, one.seq_lens, one.block_table)
    t1 = time.perf_counter() - t0
    n = max(1, min(w.batch, int(per_step / max(t1, 1e-4))))
    cpu, _ = w.compact(list(range(n)), "cpu")
    global_batch = w.batch
    del w
    if gen_dev == "cuda":
        torch.cuda.empty_cache()
    times = []
    for i in range(args.warmup + args.steps):
        t0 = time.perf_counter()
        rt.indexer(cpu.q, cpu.k_cache, cpu.weights, cpu.seq_lens, cpu.block_table)
        dt = time.perf_counter() - t0
        if i >= args.warmup:
            times.append(dt)
    value = n * len(times) / sum(times)
    line = {
        "metric": METRIC, "value": value, "unit": "queries/s", "n_gpus": int(os.environ.get("WORLD_SIZE", "1")),
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1e3 * sum(times) / len(times),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "fp32", "data": "synthetic",
        "impl": "reference",
        "config": {"workload": cpu.name, "global_batch": global_batch},
        "cpu_baseline": {"value": value, "unit": "queries/s", "cores": threads, "kind": "port",
                         "sample": f"the first {n} queries of the batch per step (their K pages in host memory), "
                                   "PyTorch CPU restatement of the reference definition "
                                   "(oracle/reference_torch.py)"},
        "e2e": {"value": value, "unit": "queries/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
