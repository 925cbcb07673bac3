"""GPU parity: the CUDA path through the C ABI against the oracle.

Bar: scores within rtol 1e-2 / atol 1e-3 (tests/parity.py), index sets equal
except at near-ties of the k-th score, -1 padding bit-exact; known-answer
cases bit-exact.
"""
import numpy as np
import pytest
import torch

import oracle
from conftest import golden_names, load_golden, workloads
from parity import check_all

pytestmark = pytest.mark.gpu
RTOL, ATOL = 1e-2, 1e-3


@pytest.fixture(scope="module", autouse=True)
def _cuda(pkg):
    assert torch.cuda.is_available(), "GPU tests need a CUDA device"
    pkg.device_status(0, clear=True)
    yield
    torch.cuda.synchronize()


def run(pkg, w, stream=None):
    d = w.to("cuda")
    out = torch.full((w.batch, 2048), -7, dtype=torch.int32, device="cuda")
    if stream is None:
        pkg.launch_topk_c(d.q, d.k_cache, d.weights, d.seq_lens, d.block_table, out)
    else:
        with torch.cuda.stream(stream):
            pkg.launch_topk_c(d.q, d.k_cache, d.weights, d.seq_lens, d.block_table, out)
    torch.cuda.synchronize()
    return out.cpu().numpy()


def oracle_rows(w):
    sc = oracle.scores(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table)
    sl = np.clip(w.seq_lens.numpy(), 0, w.max_pages * 64)
    return [sc[b, :sl[b]] for b in range(w.batch)], sc


def oracle_ref(w):
    """The oracle's top-K [B, 2048] and per-row scores (one scoring pass)."""
    rows, sc = oracle_rows(w)
    return oracle.topk_from_scores(sc, w.seq_lens, w.block_table), rows


def assert_parity(pkg, w, out=None):
    out = run(pkg, w) if out is None else out
    ref, rows = oracle_ref(w)
    fails = check_all(out, ref, rows, w.seq_lens.numpy(), w.block_table.numpy(), w.num_pages)
    assert not fails, fails[:5]
    assert pkg.device_status(0) == 0
    return out, ref


@pytest.mark.parametrize("name", golden_names())
def test_golden(pkg, name):
    w, expected, rows = load_golden(name)
    out = run(pkg, w)
    fails = check_all(out, expected, rows, w.seq_lens.numpy(), w.block_table.numpy(), w.num_pages)
    assert not fails, fails[:5]
    assert pkg.device_status(0) == 0


def test_kat_bit_exact(pkg):
    """Diagonal tiles (the reference's tcgen05 probe pattern): exact scores,
    exact ties broken by the smaller position."""
    w, expected, _ = load_golden("kat_diag")
    out = run(pkg, w)
    assert np.array_equal(out, expected)


def test_kat_scores_exact(pkg):
    w, _, rows = load_golden("kat_diag")
    d = w.to("cuda")
    sc = pkg.indexer_scores(d.q, d.k_cache, d.weights, d.seq_lens, d.block_table).cpu().numpy()
    assert np.array_equal(sc[0, :128], rows[0])


@pytest.mark.parametrize("sls", [[4096], [1, 63, 64, 65, 127, 128, 129], [2047, 2048, 2049, 0, 300],
                                 [40000, 7, 130000]])
def test_scores_within_tolerance(pkg, sls):
    W = workloads()
    w = W.custom(sls, seed=len(sls))
    d = w.to("cuda")
    got = pkg.indexer_scores(d.q, d.k_cache, d.weights, d.seq_lens, d.block_table).cpu().numpy()
    _, ref = oracle_rows(w)
    fin = np.isfinite(ref)
    np.testing.assert_allclose(got[fin], ref[fin], rtol=RTOL, atol=ATOL)
    assert np.array_equal(np.isneginf(got), ~fin)


@pytest.mark.parametrize("sls", [[0], [1], [5, 0, 77], [64 * 3 + 1] * 5, [2047, 2048, 2049],
                                 [8191, 8192, 8193], [33000], [131072]])
def test_edge_lengths(pkg, sls):
    W = workloads()
    assert_parity(pkg, W.custom(sls, seed=7))


def test_unused_block_table_tail(pkg):
    """max_num_pages far above the longest row; tail entries are never read."""
    W = workloads()
    w = W.custom([100, 3000], seed=8, max_pages=400)
    w.block_table[:, 100:] = -12345  # invalid ids past every row's pages
    assert_parity(pkg, w)


def test_config0(pkg):
    assert_parity(pkg, workloads().config(0))


def test_config1(pkg):
    assert_parity(pkg, workloads().config(1))


def test_config2_subset(pkg):
    """Config 2 rows (16k..131k keys) at reduced batch."""
    assert_parity(pkg, workloads().config(2, scale_batch=8 / 512))


def _rows(w, idx):
    return w.rows(idx)


# Configs 3 and 4 are causal rows of one sequence: by default they take the
# shared-sequence kernel ("prefill+cluster"); DSA_TOPK_PREFILL=0 keeps them on
# the per-row kernel alone.
@pytest.mark.parametrize("prefill", ["default", "0"])
def test_config3_full(pkg, prefill, monkeypatch):
    if prefill == "0":
        monkeypatch.setenv("DSA_TOPK_PREFILL", "0")
    assert_parity(pkg, workloads().config(3))
    assert (pkg.last_path() == "prefill+cluster") == (prefill == "default")


@pytest.mark.parametrize("prefill", ["default", "0"])
def test_config4_full(pkg, prefill, monkeypatch):
    """All 2048 rows of config 4 (131072-key causal context, log-uniform
    scales) against the oracle."""
    if prefill == "0":
        monkeypatch.setenv("DSA_TOPK_PREFILL", "0")
    w = workloads().config(4)
    out, _ = assert_parity(pkg, w)
    assert (pkg.last_path() == "prefill+cluster") == (prefill == "default")
    assert (out >= 0).all()  # every row has >= 2048 visible keys
    assert (np.diff(np.sort(out, axis=1), axis=1) > 0).all()  # unique per row


def test_config2_full(pkg):
    """All 512 rows of config 2 (~4.98 GB of K read from a 10.1 GB pool) on
    the GPU against the oracle. The oracle runs on a compacted copy (only the
    pages the rows read, renumbered); its slots are mapped back."""
    w = workloads().config(2, device="cuda")
    out = torch.empty((w.batch, 2048), dtype=torch.int32, device="cuda")
    pkg.launch_topk_c(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, out)
    torch.cuda.synchronize()
    assert pkg.device_status(0) == 0
    o = out.cpu().numpy()
    bt = w.block_table.cpu().numpy()
    sl = w.seq_lens.cpu().numpy()
    assert (o >= 0).all()
    assert (np.diff(np.sort(o, axis=1), axis=1) > 0).all()
    c, used = w.compact(None, "cpu")
    num_pages = w.num_pages
    del w
    torch.cuda.empty_cache()
    ref_c, rows = oracle_ref(c)
    ref = np.where(ref_c >= 0, used[np.maximum(ref_c, 0) // 64] * 64 + ref_c % 64, -1)
    fails = check_all(o, ref, rows, sl, bt, num_pages)
    assert not fails, fails[:5]


def test_partial_merge_equals_direct(pkg):
    """Key-axis sharding: per-range partial top-K + merge is bit-identical to
    the one-shot indexer (same scores, same exact selection)."""
    w = workloads().custom([50000, 131072, 3000, 0], seed=9)
    d = w.to("cuda")
    direct = run(pkg, w)
    L = 131072
    parts = 4
    bounds = [(L * i // parts, L * (i + 1) // parts) for i in range(parts)]
    cs = torch.empty((parts, w.batch, 2048), dtype=torch.float32, device="cuda")
    cp = torch.empty((parts, w.batch, 2048), dtype=torch.int32, device="cuda")
    for i, (lo, hi) in enumerate(bounds):
        pkg.indexer_partial(d.q, d.k_cache, d.weights, d.seq_lens, d.block_table, lo, hi, cs[i], cp[i])
    merged = pkg.indexer_merge(cs, cp, d.seq_lens, d.block_table)
    torch.cuda.synchronize()
    assert np.array_equal(merged.cpu().numpy(), direct)


@pytest.mark.parametrize("nparts", [1, 2])
def test_merge_out_of_range_position_is_missing(pkg, nparts):
    """A candidate position past the row's block-table span is treated as
    missing by the merge (no read past the row) and flagged. The lists stay
    best-first: the corrupted entry is row 0's last (worst) candidate; with
    two parts the second list is empty (all missing)."""
    w = workloads().custom([3000, 5000], seed=14)
    d = w.to("cuda")
    direct = run(pkg, w)
    cs = torch.full((nparts, 2, 2048), float("-inf"), dtype=torch.float32, device="cuda")
    cp = torch.full((nparts, 2, 2048), -1, dtype=torch.int32, device="cuda")
    pkg.indexer_partial(d.q, d.k_cache, d.weights, d.seq_lens, d.block_table, 0, 1 << 30, cs[0], cp[0])
    cp[0, 0, 2047] = w.max_pages * 64 + 5  # row 0's worst candidate now points past its pages
    pkg.device_status(0, clear=True)
    merged = pkg.indexer_merge(cs, cp, d.seq_lens, d.block_table)
    torch.cuda.synchronize()
    assert pkg.device_status(0) & pkg.DSA_STATUS_BAD_PAGE
    m = merged.cpu().numpy()
    assert np.array_equal(m[1], direct[1])
    assert np.array_equal(m[0, :-1], direct[0, :-1]) and m[0, -1] == -1


def test_partial_unaligned_ranges(pkg):
    w = workloads().custom([9000, 5000], seed=10)
    d = w.to("cuda")
    direct = run(pkg, w)
    bounds = [(0, 1000), (1000, 4097), (4097, 9000)]
    cs = torch.empty((3, 2, 2048), dtype=torch.float32, device="cuda")
    cp = torch.empty((3, 2, 2048), dtype=torch.int32, device="cuda")
    for i, (lo, hi) in enumerate(bounds):
        pkg.indexer_partial(d.q, d.k_cache, d.weights, d.seq_lens, d.block_table, lo, hi, cs[i], cp[i])
    merged = pkg.indexer_merge(cs, cp, d.seq_lens, d.block_table)
    torch.cuda.synchronize()
    assert np.array_equal(merged.cpu().numpy(), direct)


def test_deterministic_and_side_stream(pkg):
    w = workloads().config(1, scale_batch=0.25)
    a = run(pkg, w)
    b = run(pkg, w, stream=torch.cuda.Stream())
    assert np.array_equal(a, b)


def test_nan_input_bytes_relu_to_zero(pkg):
    """e4m3 NaN bytes (0x7F) in a key and in one query head: the affected
    head products are NaN and relu maps them to 0, as the reference's
    fmaxf(x, 0) epilogue does (the oracle: x > 0 ? x : 0)."""
    w = workloads().custom([3000, 5000], seed=15)
    page = int(w.block_table[0, 3])
    w.k_cache[page, 10, 0, 5] = 0x7F           # one key of row 0
    q8 = w.q.view(torch.uint8)
    q8[1, 7, 3] = 0x7F                          # head 7 of row 1, every key
    assert_parity(pkg, w)


def test_bad_page_id_flags_status(pkg):
    """An out-of-range page id is zero-filled by the TMA bounds check and
    reported in the status word; the kernel does not fault."""
    w = workloads().custom([3000], seed=12)
    w.block_table[0, 5] = w.num_pages + 1000
    run(pkg, w)
    assert pkg.device_status(0) & pkg.DSA_STATUS_BAD_PAGE


def test_seq_len_clamped_flags_status(pkg):
    w = workloads().custom([1000], seed=13)
    w.seq_lens[0] = 5000  # longer than max_pages * 64 = 1024
    out = run(pkg, w)
    assert pkg.device_status(0) & pkg.DSA_STATUS_SEQ_CLAMPED
    assert (out[0, :1024] >= 0).all() and (out[0, 1024:] == -1).all()


@pytest.mark.parametrize("g", [1, 2, 3, 5, 8, 16])
def test_forced_cluster_sizes_l2_resident(pkg, g, monkeypatch):
    """Cluster sizes 1 to 16 on a shared, L2-resident K (an epilogue-bound
    pipeline where ring stages are refilled fastest): rows of 71 tiles, so up
    to 8 CTAs per row reuse every ring stage; the cluster-wide ordering ranks
    each CTA's survivors against every other CTA's bucket table (16: the
    largest cluster, a non-portable size)."""
    monkeypatch.setenv("DSA_TOPK_CLUSTER", str(g))
    w = workloads().make_shared("l2res", 192, 9000, 160, 21)
    assert_parity(pkg, _rows(w, list(range(0, 192, 3))))


@pytest.mark.parametrize("g", [2, 4, 8, 16])
def test_cluster_select_small_rows(pkg, g, monkeypatch):
    """Rows of up to a few thousand keys spread over 2 to 16 CTAs: every key
    is a candidate (no CTA fills its buffer), so the cluster select runs on
    totals around and below 2048 and 4096, including rows with fewer keys
    than CTAs and an empty row."""
    monkeypatch.setenv("DSA_TOPK_CLUSTER", str(g))
    w = workloads().custom([1, 700, 2047, 2048, 2049, 3000, 4095, 4096, 4097, 4200, 6000, 0], seed=91)
    assert_parity(pkg, w)


@pytest.mark.parametrize("tail", ["0", "1"])
def test_cluster_tail_launch(pkg, tail, monkeypatch):
    """A batch of 300 rows at two CTAs per row: two waves of 148 clusters and
    a partial one of 4 rows, which run as a second launch at 8 CTAs per row
    (tail=1) or in the last wave of the single launch (tail=0)."""
    monkeypatch.setenv("DSA_TOPK_TAIL", tail)
    g = torch.Generator().manual_seed(93)
    sl = torch.randint(1, 9000, (300,), generator=g).to(torch.int32)
    w = workloads().custom(sl.tolist(), seed=94)
    assert_parity(pkg, w)
    assert (pkg.last_path() == "cluster-tail") == (tail == "1")


def test_cluster_tail_launch_ranked_in_kernel(pkg):
    """128 rows at four CTAs per row (rows ranked inside the kernel, no plan
    launch): a wave of 74 clusters, then 54 rows as a second launch at five
    CTAs per row."""
    g = torch.Generator().manual_seed(95)
    sl = torch.randint(1, 20000, (128,), generator=g).to(torch.int32)
    w = workloads().custom(sl.tolist(), seed=96)
    assert_parity(pkg, w)
    assert pkg.last_path() == "cluster-tail"


@pytest.mark.parametrize("split", ["0", "1"])
def test_cluster_two_class_launch(pkg, split, monkeypatch):
    """Cluster path on a batch that needs more clusters than fit at once:
    the longest rows at the default cluster size and the rest at two CTAs
    each, launched concurrently on two streams (split=1), or all rows at one
    size in longest-first order (split=0)."""
    monkeypatch.setenv("DSA_TOPK_SPLIT", split)
    w = workloads().custom([32768, 600, 0, 17000, 2049, 9000, 100, 24000] * 8, seed=31)
    assert_parity(pkg, w)


@pytest.mark.parametrize("kind", ["uniform", "loguniform"])
def test_two_class_launch_decided_on_device(pkg, kind):
    """64 rows, in-kernel ranking: the kernel decides between the two-class
    split and all rows in waves from the lengths (uniform long rows take
    waves, log-uniform ones the split); both must be parity-green."""
    g = torch.Generator().manual_seed(81)
    u = torch.rand(64, generator=g, dtype=torch.float64)
    if kind == "uniform":
        sl = (16384 + u * (131072 - 16384)).floor().to(torch.int32)
    else:
        sl = torch.exp(np.log(512) + u * (np.log(32768) - np.log(512))).floor().to(torch.int32)
    assert_parity(pkg, workloads().custom(sl.tolist(), seed=82))


@pytest.mark.parametrize("cfg", [1, 3])
def test_cluster_kernel_path(pkg, cfg, monkeypatch):
    """The one-launch cluster kernel (the schedule when the two-class and
    last-wave launches are off, and that of the no-allocation entry point)
    stays parity-green."""
    monkeypatch.setenv("DSA_TOPK_SPLIT", "0")
    monkeypatch.setenv("DSA_TOPK_TAIL", "0")
    w = workloads().config(cfg)
    if cfg == 3:
        w = _rows(w, list(range(0, 8192, 37)))
    assert_parity(pkg, w)
    assert pkg.last_path() == "cluster"


def _schedules(pkg, w, settings, monkeypatch):
    """Output of the same batch under each setting (a dict of switches)."""
    outs = []
    for env in settings:
        for k in ("DSA_TOPK_CLUSTER", "DSA_TOPK_SPLIT", "DSA_TOPK_TAIL", "DSA_TOPK_PREFILL"):
            monkeypatch.delenv(k, raising=False)
        for k, v in env.items():
            monkeypatch.setenv(k, v)
        outs.append((env, run(pkg, w), pkg.last_path()))
    return outs


def test_schedules_bit_identical_decode(pkg, monkeypatch):
    """Every key's score comes from one routine and the selection is exact,
    so the decode schedules agree bit for bit: cluster sizes 1 to 8, the
    two-class split and the last-wave launch on and off."""
    g = torch.Generator().manual_seed(71)
    u = torch.rand(160, generator=g, dtype=torch.float64)
    sl = torch.exp(np.log(300) + u * (np.log(40000) - np.log(300))).floor().to(torch.int32)
    sl[:5] = torch.tensor([0, 1, 2047, 2048, 2049], dtype=torch.int32)
    w = workloads().custom(sl.tolist(), seed=72)
    settings = [{}, {"DSA_TOPK_SPLIT": "0", "DSA_TOPK_TAIL": "0"}, {"DSA_TOPK_TAIL": "0"}] + \
               [{"DSA_TOPK_CLUSTER": str(c)} for c in (1, 2, 3, 4, 8)]
    outs = _schedules(pkg, w, settings, monkeypatch)
    base = outs[0][1]
    for env, o, path in outs[1:]:
        assert np.array_equal(o, base), (env, path)
    assert len({p for _, _, p in outs}) >= 2  # more than one schedule really ran
    assert_parity(pkg, w, base)


def test_schedules_bit_identical_prefill(pkg, monkeypatch):
    """The shared-sequence kernel and the per-row kernel (at two cluster
    sizes) agree bit for bit on a causal batch."""
    w = workloads().make_shared("xpath", 260, 12000, 200, 73)
    settings = [{"DSA_TOPK_PREFILL": "1"}, {"DSA_TOPK_PREFILL": "0"},
                {"DSA_TOPK_PREFILL": "0", "DSA_TOPK_CLUSTER": "4"}]
    outs = _schedules(pkg, w, settings, monkeypatch)
    assert outs[0][2] == "prefill+cluster" and outs[1][2] != "prefill+cluster"
    for env, o, path in outs[1:]:
        assert np.array_equal(o, outs[0][1]), (env, path)
    assert_parity(pkg, w, outs[0][1])
