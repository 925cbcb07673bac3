"""GPU: the contest harness's solution slot (solution/), built from source
the way the harness builds it, then called like the harness calls it.

The packed solution (solution/pack.py -> solution.json: config.toml's spec
plus every source inlined, flat) is unpacked into a fresh directory and
compiled
  - by torch.utils.cpp_extension.load on kernel.cu, the reference's
    `binding = "torch"` path (solution/cuda/binding.py pins
    TORCH_CUDA_ARCH_LIST=10.0a first, as the reference's binding.py does);
  - by tvm_ffi.cpp.load, the harness's default tvm-ffi builder path.
Each build's `launch_topk_c` (destination-passing, six tensors) must match
the oracle on config 0 and on short / empty / boundary rows, and raise on a
malformed output tensor. Building takes a few minutes of nvcc time.
"""
import importlib.util
import json
import os

import numpy as np
import pytest
import torch

import oracle
from conftest import ROOT, workloads
from parity import check_all

pytestmark = pytest.mark.gpu


def _unpack(dst):
    spec = importlib.util.spec_from_file_location("solution_pack", os.path.join(ROOT, "solution", "pack.py"))
    pack = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(pack)
    doc = json.load(open(pack.pack()))
    os.makedirs(dst, exist_ok=True)
    for s in doc["sources"]:
        with open(os.path.join(dst, s["path"]), "w") as f:
            f.write(s["content"])
    return doc


def _cases():
    W = workloads()
    return [W.config(0), W.custom([4096, 1000, 0, 2049, 64, 1], seed=61)]


def _check(fn, w_cpu):
    w = w_cpu.to("cuda")
    out = torch.full((w.batch, 2048), -7, dtype=torch.int32, device="cuda")
    fn(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, out)
    torch.cuda.synchronize()
    sc = oracle.scores(w_cpu.q, w_cpu.k_cache, w_cpu.weights, w_cpu.seq_lens, w_cpu.block_table)
    ref = oracle.topk_from_scores(sc, w_cpu.seq_lens, w_cpu.block_table)
    sl = np.clip(w_cpu.seq_lens.numpy(), 0, w_cpu.max_pages * 64)
    rows = [sc[b, :sl[b]] for b in range(w_cpu.batch)]
    fails = check_all(out.cpu().numpy(), ref, rows, w_cpu.seq_lens.numpy(), w_cpu.block_table.numpy(),
                      w_cpu.num_pages)
    assert not fails, fails[:3]
    return out


@pytest.fixture(scope="module")
def unpacked(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("solution"))
    doc = _unpack(os.path.join(d, "src"))
    assert doc["spec"]["entry_point"] == "kernel.cu::launch_topk_c"
    assert doc["spec"]["destination_passing_style"] is True
    return d, doc


def test_torch_builder(unpacked):
    d, doc = unpacked
    assert doc["spec"]["binding"] == "torch"
    src = os.path.join(d, "src")
    exec(open(os.path.join(src, "binding.py")).read(), {})  # as the harness imports binding.py
    assert os.environ["TORCH_CUDA_ARCH_LIST"] == "10.0a"
    from torch.utils.cpp_extension import load
    os.makedirs(os.path.join(d, "torch_build"), exist_ok=True)
    mod = load(name="dsa_solution_torch", sources=[os.path.join(src, "kernel.cu")],
               build_directory=os.path.join(d, "torch_build"), verbose=False)
    for w in _cases():
        _check(mod.launch_topk_c, w)
    w = _cases()[1].to("cuda")
    with pytest.raises(RuntimeError, match="topk_indices"):
        mod.launch_topk_c(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table,
                          torch.empty((w.batch, 100), dtype=torch.int32, device="cuda"))


def test_tvm_ffi_builder(unpacked):
    tvm_ffi_cpp = pytest.importorskip("tvm_ffi.cpp")
    d, _ = unpacked
    src = os.path.join(d, "src")
    os.makedirs(os.path.join(d, "tvm_build"), exist_ok=True)
    # The tvm-ffi builder targets the detected device's generic architecture
    # (compute_100) unless TVM_FFI_CUDA_ARCH_LIST names one; tcgen05 and TMA
    # need the arch-specific sm_100a target.
    os.environ["TVM_FFI_CUDA_ARCH_LIST"] = "10.0a"
    mod = tvm_ffi_cpp.load("dsa_solution_tvm", cuda_files=[os.path.join(src, "kernel.cu")],
                           extra_cuda_cflags=["-O3"], build_directory=os.path.join(d, "tvm_build"))
    fn = mod["launch_topk_c"]
    for w in _cases():
        _check(fn, w)
