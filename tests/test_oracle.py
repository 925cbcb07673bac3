"""CPU: pins the C oracle before it is trusted as the GPU path's checker."""
import numpy as np
import pytest
import torch

import oracle
import reference_torch as rt
from conftest import golden_names, load_golden
from parity import check_all


def test_e4m3_table_matches_torch():
    tab = oracle.e4m3_table()
    ref = torch.arange(256, dtype=torch.uint8).view(torch.float8_e4m3fn).to(torch.float32).numpy()
    nan = np.isnan(ref)
    assert (np.isnan(tab) == nan).all()
    assert (tab[~nan] == ref[~nan]).all()
    # the reference's probe constants (diagnostic_tests/run_tmem2_p11.py:87-91)
    assert tab[0x38] == 1.0 and tab[0x48] == 4.0


def _diag_tile(byte):
    t = np.zeros((64, 128), dtype=np.uint8)
    t[np.arange(64), np.arange(64)] = byte
    return t


@pytest.mark.parametrize("kbyte,val", [(0x38, 1.0), (0x48, 4.0)])
def test_fp8_gemm_known_answer(kbyte, val):
    """The reference's tcgen05 probe pattern: diagonal Q and K tiles give a
    diagonal product (methodology/diagnostic_tests/tmem2_probe.cu:1-40)."""
    d = oracle.fp8_gemm_nt(_diag_tile(0x38), _diag_tile(kbyte))
    assert np.array_equal(d, np.eye(64, dtype=np.float32) * val)


@pytest.mark.parametrize("name", golden_names())
def test_oracle_matches_golden(name):
    w, expected, rows = load_golden(name)
    got = oracle.indexer(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table)
    fails = check_all(got, expected, rows, w.seq_lens.numpy(), w.block_table.numpy(), w.num_pages)
    assert not fails, fails[:5]
    sc = oracle.scores(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table)
    for b, r in enumerate(rows):
        np.testing.assert_allclose(sc[b, :len(r)], r, rtol=1e-5, atol=1e-6)
        assert np.isneginf(sc[b, len(r):]).all()


def test_kat_exact_order():
    """Exact known answer incl. tie-break by smaller position (pos 3 beats pos 64)."""
    w, expected, _ = load_golden("kat_diag")
    got = oracle.indexer(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table)
    assert np.array_equal(got, expected)
    # score(pos t) = (t+1)/64, score(pos 64+t) = 4(t+1)/64; slot = bt[pos>>6]*64 + pos%64, bt = [1, 0]
    keys = sorted(range(128), key=lambda p: (-(p % 64 + 1) * (4 if p >= 64 else 1), p))
    slots = [(1 if p < 64 else 0) * 64 + p % 64 for p in keys]
    assert got[0, :128].tolist() == slots and (got[0, 128:] == -1).all()


def test_padding_and_empty_rows():
    W = __import__("conftest").workloads()
    w = W.custom([0, 5, 2047, 2048, 3000], seed=5, max_pages=60)
    got = oracle.indexer(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table)
    for b, sl in enumerate([0, 5, 2047, 2048, 3000]):
        k = min(sl, 2048)
        assert (got[b, k:] == -1).all() and (got[b, :k] >= 0).all()
        assert len(set(got[b, :k].tolist())) == k


def test_topk_from_scores_stable_ties():
    """Equal scores rank by ascending position (stable descending sort)."""
    sc = np.zeros((1, 4096), dtype=np.float32)
    sc[0, 1::3] = 1.0  # 1365 ones, then zeros fill the rest in position order
    bt = np.arange(64, dtype=np.int32).reshape(1, 64)
    out = oracle.topk_from_scores(sc, np.array([4096], np.int32), bt)
    ones = list(range(1, 4096, 3))
    zeros = [p for p in range(4096) if p % 3 != 1]
    assert out[0].tolist() == (ones + zeros)[:2048]


def test_oracle_vs_torch_random():
    W = __import__("conftest").workloads()
    w = W.custom([1500, 4500, 9000, 64], seed=21)
    a = oracle.indexer(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table)
    b, rows = rt.indexer(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, return_scores=True)
    fails = check_all(a, b.numpy(), [r.numpy() for r in rows], w.seq_lens.numpy(), w.block_table.numpy(),
                      w.num_pages)
    assert not fails, fails[:5]


def test_shared_causal_restatement_agrees():
    W = __import__("conftest").workloads()
    w = W.make_shared("t", 16, 2100, 40, 3)
    a = rt.indexer_shared_causal(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, chunk=5)
    b, rows = rt.indexer(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, return_scores=True)
    fails = check_all(a.numpy(), b.numpy(), [r.numpy() for r in rows], w.seq_lens.numpy(),
                      w.block_table.numpy(), w.num_pages)
    assert not fails, fails[:5]
