"""GPU: the shared-sequence (prefill) path against the oracle.

Batches of 256 rows or more first go through the shared-sequence kernel,
which serves every group of four consecutive rows whose block-table entries
agree over their visible keys (one K stream and one N = 128 MMA per row pair and tile) and
leaves the other rows to the per-row kernel. These tests mix both kinds of
group in one batch, including groups that agree on every page but the last
visible one, and batches whose size is not a multiple of four.
"""
import numpy as np
import pytest
import torch

import oracle
from conftest import workloads
from parity import check_all

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _prefill_on(monkeypatch):
    """By default the stage runs only when the block table must share pages
    (more entries than four times the pool's pages); these tests turn it on
    for every batch of 256+ rows (DSA_TOPK_PREFILL=1)."""
    monkeypatch.setenv("DSA_TOPK_PREFILL", "1")


def _check(pkg, w, monkeypatch=None, prefill=True):
    if monkeypatch is not None and not prefill:
        monkeypatch.setenv("DSA_TOPK_PREFILL", "0")
    d = w.to("cuda")
    out = torch.full((w.batch, 2048), -7, dtype=torch.int32, device="cuda")
    pkg.device_status(0, clear=True)
    pkg.launch_topk_c(d.q, d.k_cache, d.weights, d.seq_lens, d.block_table, out)
    torch.cuda.synchronize()
    path = pkg.last_path()
    assert pkg.device_status(0, clear=True) == 0
    o = out.cpu().numpy()
    sc = oracle.scores(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table)
    ref = oracle.topk_from_scores(sc, w.seq_lens, w.block_table)
    sl = np.clip(w.seq_lens.numpy(), 0, w.max_pages * 64)
    rows = [sc[b, :sl[b]] for b in range(w.batch)]
    fails = check_all(o, ref, rows, w.seq_lens.numpy(), w.block_table.numpy(), w.num_pages)
    assert not fails, fails[:5]
    return o, path


def _mixed(n_rows, total_keys, seed):
    """A causal sequence of n_rows query rows over total_keys keys whose
    pages are stored twice (an identical copy at other page ids). Groups
    whose rows all use the original pages are shared; in the others some
    rows read the copy, so their block-table rows differ (the outputs differ
    only in the slot ids, which the oracle follows)."""
    W = workloads()
    n_pages = (total_keys + 63) // 64
    w = W.make_shared("mixed", n_rows, total_keys, 2 * n_pages + 8, seed)
    flat = w.k_cache.view(w.k_cache.shape[0], -1)
    orig = w.block_table[0, :n_pages].to(torch.int64)
    used = set(orig.tolist())
    free = [p for p in range(w.k_cache.shape[0]) if p not in used][:n_pages]
    copy = torch.tensor(free, dtype=torch.int64)
    flat[copy] = flat[orig]
    bt = w.block_table.clone()
    g = torch.Generator().manual_seed(seed)
    for r0 in range(0, n_rows, 4):
        kind = int(torch.randint(0, 4, (1,), generator=g))
        r = min(r0 + 1, n_rows - 1)
        npg = (int(w.seq_lens[r]) + 63) // 64
        if kind == 1:    # one row reads the copy everywhere
            bt[r, :n_pages] = copy.to(torch.int32)
        elif kind == 2 and npg > 0:  # one row differs only at its last visible page
            bt[r, npg - 1] = int(copy[npg - 1])
        # kind 0 / 3: shared
    w.block_table = bt.contiguous()
    return w


@pytest.mark.parametrize("n_rows,total_keys", [(256, 6000), (258, 3000), (261, 20000)])
def test_mixed_shared_and_independent_groups(pkg, n_rows, total_keys):
    w = _mixed(n_rows, total_keys, seed=n_rows)
    _, path = _check(pkg, w)
    assert path == "prefill+cluster"


def test_prefill_off_matches_oracle(pkg, monkeypatch):
    """The same causal batch through the per-row kernel alone."""
    w = workloads().make_shared("causal", 256, 9000, 160, 5)
    _, path = _check(pkg, w, monkeypatch, prefill=False)
    assert path != "prefill+cluster"


def test_prefill_short_rows_and_empty(pkg):
    """Rows of 0..300 keys (one or two tiles, empty rows, rows shorter than a
    page) in shared groups."""
    w = workloads().make_shared("short", 300, 300, 8, 6)
    w.seq_lens[:40] = 0
    w.seq_lens[40:44] = torch.tensor([1, 63, 64, 65], dtype=torch.int32)
    _check(pkg, w)


def test_prefill_partial_merge_equals_direct(pkg):
    """Key-range partial lists (served by the shared-sequence kernel in
    partial mode) merged equal the one-shot result bit for bit."""
    w = workloads().make_shared("pm", 256, 40000, 700, 8)
    d = w.to("cuda")
    direct = torch.empty((w.batch, 2048), dtype=torch.int32, device="cuda")
    pkg.launch_topk_c(d.q, d.k_cache, d.weights, d.seq_lens, d.block_table, direct)
    bounds = [(0, 12800), (12800, 25600), (25600, 40000)]
    cs = torch.empty((3, w.batch, 2048), dtype=torch.float32, device="cuda")
    cp = torch.empty((3, w.batch, 2048), dtype=torch.int32, device="cuda")
    for i, (lo, hi) in enumerate(bounds):
        pkg.indexer_partial(d.q, d.k_cache, d.weights, d.seq_lens, d.block_table, lo, hi, cs[i], cp[i])
        assert pkg.last_path() == "prefill+cluster"
    merged = pkg.indexer_merge(cs, cp, d.seq_lens, d.block_table)
    torch.cuda.synchronize()
    assert pkg.device_status(0, clear=True) == 0
    assert np.array_equal(merged.cpu().numpy(), direct.cpu().numpy())


def test_prefill_nan_input_bytes(pkg):
    """e4m3 NaN bytes on the shared-sequence path: one key seen by every row,
    and one NaN head in the queries of a whole group (rows in both the first
    and second slot of each row pair, whose scores take different code: the
    second row hands its TMEM columns back before its last heads are
    reduced). relu maps every NaN product to 0, as on the per-row kernel."""
    w = workloads().make_shared("nan", 256, 6000, 100, 9)
    page = int(w.block_table[0, 3])
    w.k_cache[page, 10, 0, 5] = 0x7F            # key 3*64+10, visible to every row
    q8 = w.q.view(torch.uint8)
    # group 2 (rows 8..11: first / second slot of both pairs); heads 3, 22
    # and 54 are heads whose relu takes the x + |x| form, in the first (3,
    # 22) and the second half (54) of the 64
    for r, h in ((8, 3), (9, 22), (10, 37), (11, 54)):
        q8[r, h, 40] = 0x7F
    q8[201, 62, 0] = 0xFF                        # a second-slot row of another group
    _, path = _check(pkg, w)
    assert path == "prefill+cluster"
