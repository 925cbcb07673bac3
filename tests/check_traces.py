"""Runs the trace runner over a directory of contest workload files and
checks every result against the CPU oracle with the parity rule (test
infrastructure: the oracle is the checker, never the thing measured).

    python tests/check_traces.py DIR [--k-init normal|randint] [--iters N]
"""
import importlib
import os
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
for p in (ROOT, HERE, os.path.join(ROOT, "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

import oracle  # noqa: E402  (the CPU restatement)
from parity import check_all  # noqa: E402

PKG = "karnbirkhera-mlsys2026-dsa_topk_indexer_b200"


def parity_hook(w, out, rec):
    """Adds "parity": "pass" or "<n> failures" to the runner's record."""
    ref = oracle.indexer(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table)
    sc = oracle.scores(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table)
    sl = w.seq_lens.clamp(0, w.max_pages * 64).tolist()
    fails = check_all(out.numpy(), ref, [sc[i, :s] for i, s in enumerate(sl)], w.seq_lens.numpy(),
                      w.block_table.numpy(), w.num_pages)
    rec["parity"] = "pass" if not fails else f"{len(fails)} failures"


def main(argv=None):
    runner = importlib.import_module(PKG + ".trace_runner")
    return runner.main(argv, on_result=parity_hook)


if __name__ == "__main__":
    main()
