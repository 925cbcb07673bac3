"""GPU: the TVM-FFI export `launch_topk_c` (the solution-slot binding) gives
the same result as the torch binding; both end in the same C ABI."""
import os

import pytest
import torch

from conftest import package, workloads

pytestmark = pytest.mark.gpu


def test_tvm_ffi_export_matches_torch_binding():
    tvm_ffi = pytest.importorskip("tvm_ffi")
    pkg = package()
    so = os.path.join(os.path.dirname(pkg.__file__), "libdsa_topk_indexer_tvmffi.so")
    assert os.path.exists(so), "TVM-FFI binding not built"
    f = tvm_ffi.load_module(so)["launch_topk_c"]
    w = workloads().custom([3000, 100, 0, 9000], seed=4).to("cuda")
    a = torch.empty((w.batch, 2048), dtype=torch.int32, device="cuda")
    b = torch.full((w.batch, 2048), -7, dtype=torch.int32, device="cuda")
    pkg.launch_topk_c(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, a)
    torch.cuda.synchronize()
    f(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, b)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    with pytest.raises(Exception, match="topk_indices"):
        f(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, b[:, :100].contiguous())
