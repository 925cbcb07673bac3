"""GPU: the bounded-wait abort path of the indexer kernel.

Every pipeline wait gives up after a time limit, raises
DSA_STATUS_WAIT_TIMEOUT and ends the kernel early (waiting, bounded, for its
own loads and MMAs in flight, then freeing its tensor memory) instead of
hanging the GPU. The library's test hook makes every CTA skip the loads of
one of its tiles, so the waits for that tile run out after a short limit;
nothing faults and nothing waits without a bound. The call must return with
the status bit set, and a normal call right after it on the same stream must
pass parity (its kernels allocate tensor memory again and run the whole
pipeline).
"""
import time

import numpy as np
import pytest
import torch

import oracle
from conftest import workloads
from parity import check_all

pytestmark = pytest.mark.gpu


def _parity(pkg, w, out):
    sc = oracle.scores(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table)
    ref = oracle.topk_from_scores(sc, w.seq_lens, w.block_table)
    sl = np.clip(w.seq_lens.numpy(), 0, w.max_pages * 64)
    rows = [sc[b, :sl[b]] for b in range(w.batch)]
    return check_all(out, ref, rows, w.seq_lens.numpy(), w.block_table.numpy(), w.num_pages)


# skip 0: the first tile of every CTA never arrives. skip 31: an odd tile at
# the end of the epilogue's first 16-pair check interval, so one epilogue
# group gives up while the other waits at the shared check barrier (the group
# that gave up must still arrive there). One-CTA clusters so each row's CTA
# streams all its tiles (24, 71 and 157 here: the 24-tile row never reaches
# tile 31 and completes normally).
@pytest.mark.parametrize("skip", [0, 31])
def test_wait_timeout_aborts_and_next_call_is_clean(pkg, skip, monkeypatch):
    monkeypatch.setenv("DSA_TOPK_CLUSTER", "1")
    lib = pkg._lib.load()
    w = workloads().custom([3000, 9000, 20000], seed=51)
    d = w.to("cuda")
    out = torch.full((w.batch, 2048), -7, dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()
    pkg.device_status(0, clear=True)
    assert lib.dsa_topk_indexer_set_test_fault(skip, 1_000_000) == 0  # 1 ms wait limit
    try:
        t0 = time.perf_counter()
        pkg.launch_topk_c(d.q, d.k_cache, d.weights, d.seq_lens, d.block_table, out)
        torch.cuda.synchronize()
        elapsed = time.perf_counter() - t0
    finally:
        assert lib.dsa_topk_indexer_set_test_fault(-1, 0) == 0
    assert pkg.device_status(0, clear=True) & pkg.DSA_STATUS_WAIT_TIMEOUT
    assert elapsed < 5.0
    # The same stream, a normal call: full pipeline, parity with the oracle.
    out.fill_(-7)
    pkg.launch_topk_c(d.q, d.k_cache, d.weights, d.seq_lens, d.block_table, out)
    torch.cuda.synchronize()
    assert pkg.device_status(0, clear=True) == 0
    fails = _parity(pkg, w, out.cpu().numpy())
    assert not fails, fails[:3]


def test_test_fault_hook_rejects_bad_limits(pkg):
    lib = pkg._lib.load()
    assert lib.dsa_topk_indexer_set_test_fault(-2, 0) != 0
    assert lib.dsa_topk_indexer_set_test_fault(0, 10) != 0          # below 100 us
    assert lib.dsa_topk_indexer_set_test_fault(0, 3_000_000_000) != 0  # above 2 s
    assert lib.dsa_topk_indexer_set_test_fault(-1, 0) == 0
