"""Parity rule for the indexer output (shared by the CPU and GPU tests).

Rule: scores agree within rtol 1e-2 / atol 1e-3; the
top-K index set is identical except for positions whose score lies within
that tolerance of the k-th value; padding (-1) is bit-exact. Because both
outputs are sorted best-first, the score at every rank must also agree within
the tolerance, which checks the order without being sensitive to the order of
near-tied keys.
"""
import numpy as np

RTOL, ATOL = 1e-2, 1e-3
PAGE, TOPK = 64, 2048


def _close(a, b):
    return np.abs(a - b) <= ATOL + RTOL * np.abs(b)


def slots_to_positions(slots, bt_row, n_valid, num_pages):
    """Maps physical slots back to logical positions of one row (-1 if the
    slot is not one of the row's first n_valid keys)."""
    npg = (n_valid + PAGE - 1) // PAGE
    inv = np.full(num_pages, -1, dtype=np.int64)
    inv[bt_row[:npg]] = np.arange(npg)
    slots = np.asarray(slots, dtype=np.int64)
    page = slots // PAGE
    ok = (slots >= 0) & (page < num_pages)
    pos = np.full(slots.shape, -1, dtype=np.int64)
    pos[ok] = inv[page[ok]] * PAGE + slots[ok] % PAGE
    pos[(pos < 0) | (pos >= n_valid) | ~ok] = -1
    pos[ok & (inv[np.where(ok, page, 0)] < 0)] = -1
    return pos


def check_row(out_row, ref_row, ref_scores, seq_len, bt_row, num_pages, max_pages):
    """Returns None if the row passes, else a message."""
    n_valid = max(0, min(int(seq_len), max_pages * PAGE))
    k = min(TOPK, n_valid)
    out_row = np.asarray(out_row)
    ref_row = np.asarray(ref_row)
    if not (out_row[k:] == -1).all():
        return f"padding: expected -1 at ranks >= {k}"
    if not (ref_row[k:] == -1).all():
        return "reference padding broken"
    if k == 0:
        return None
    pos = slots_to_positions(out_row[:k], bt_row, n_valid, num_pages)
    if (pos < 0).any():
        return f"{int((pos < 0).sum())} output slots are not visible keys of this row"
    if len(np.unique(pos)) != k:
        return "duplicate slots"
    ref_pos = slots_to_positions(ref_row[:k], bt_row, n_valid, num_pages)
    sc = np.asarray(ref_scores[:n_valid], dtype=np.float64)
    got, want = sc[pos], sc[ref_pos]
    bad = ~_close(got, want)
    if bad.any():
        r = int(np.nonzero(bad)[0][0])
        return f"rank {r}: score {got[r]:.7g} vs reference {want[r]:.7g}"
    kth = want[-1]
    extra = np.setdiff1d(pos, ref_pos)
    missing = np.setdiff1d(ref_pos, pos)
    for p in np.concatenate([extra, missing]):
        if not _close(sc[p], kth):
            return f"position {int(p)} (score {sc[p]:.7g}) differs from the reference set; k-th score {kth:.7g}"
    return None


def check_all(out, ref, ref_scores_rows, seq_lens, block_table, num_pages):
    out, ref = np.asarray(out), np.asarray(ref)
    bt = np.asarray(block_table)
    sl = np.asarray(seq_lens)
    max_pages = bt.shape[1]
    fails = []
    for b in range(out.shape[0]):
        msg = check_row(out[b], ref[b], ref_scores_rows[b], sl[b], bt[b], num_pages, max_pages)
        if msg:
            fails.append(f"row {b}: {msg}")
    return fails


def exact_match_fraction(out, ref):
    return float((np.asarray(out) == np.asarray(ref)).mean())
