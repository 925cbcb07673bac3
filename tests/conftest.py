import ast
import glob
import importlib
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_NAME = "karnbirkhera-mlsys2026-dsa_topk_indexer_b200"
for p in (ROOT, os.path.join(ROOT, "oracle"), os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


def package():
    return importlib.import_module(PKG_NAME)


def workloads():
    return importlib.import_module(PKG_NAME + ".workloads")


@pytest.fixture(scope="session")
def pkg():
    return package()


@pytest.fixture(scope="session")
def wl():
    return workloads()


def load_golden(name):
    """Returns (Workload, expected_out [B,2048], score rows list) for a fixture."""
    import torch
    from make_golden import input_digest  # tests/golden/make_golden.py
    d = np.load(os.path.join(ROOT, "tests", "golden", name + ".npz"))
    W = workloads()
    if "spec" in d:
        spec = ast.literal_eval(str(d["spec"]))
        kind = spec.pop("kind")
        if kind == "config":
            w = W.config(spec["idx"])
        elif kind == "config_rows":
            full = W.config(spec["idx"])
            idx = torch.as_tensor(spec["rows"])
            w = W.Workload(full.name, full.q[idx].contiguous(), full.k_cache, full.weights[idx].contiguous(),
                           full.seq_lens[idx].contiguous(), full.block_table[idx].contiguous())
        elif kind == "custom":
            w = W.custom(spec.pop("seq_lens"), **spec)
        else:
            w = W.make_shared("fixture", spec["n_queries"], spec["total_keys"], spec["pool_pages"], spec["seed"])
    else:
        w = W.Workload(name, torch.from_numpy(d["q"]).view(torch.float8_e4m3fn), torch.from_numpy(d["k_cache"]),
                       torch.from_numpy(d["weights"]), torch.from_numpy(d["seq_lens"]),
                       torch.from_numpy(d["block_table"]))
    digest = str(d["digest"])
    if input_digest(w) != digest:
        raise AssertionError(f"fixture {name}: regenerated inputs differ from the recorded ones "
                             "(generator or RNG changed); rerun tests/golden/make_golden.py")
    sl = np.clip(w.seq_lens.numpy(), 0, w.max_pages * 64)
    rows, off = [], 0
    for n in sl:
        rows.append(d["scores"][off:off + n])
        off += n
    return w, d["out"], rows


def golden_names():
    return sorted(os.path.splitext(os.path.basename(p))[0]
                  for p in glob.glob(os.path.join(ROOT, "tests", "golden", "*.npz")))


sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
