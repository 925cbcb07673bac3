"""Sparse MLA attention over the indexer's selected slots (the consumer of
topk_indices).

CPU: the restatement in oracle/reference_torch.py against a per-token,
per-head loop of the same math (softmax over the valid slots, values = the
latent rows, base-2 lse), its edge cases, and the C ABI's argument checks.
GPU: the CUDA kernel against the restatement on seeded inputs (single CTA
per token and split lists combined on the device, -1 padding, a token with
no valid slot, duplicated and out-of-range slots), repeated launches (the
split counters reset themselves), and the indexer -> attention chain on one
page pool. Tolerance (floating point; the kernel rounds P and the output to
bf16): |out - ref| <= 1e-2 + 1e-2 |ref|, |lse - ref| <= 1e-3 + 1e-5 |ref|.
"""
import ctypes
import math

import pytest
import torch

from conftest import package

import reference_torch as rt  # oracle/ is on sys.path (conftest)

OUT_ATOL, OUT_RTOL = 1e-2, 1e-2
LSE_ATOL, LSE_RTOL = 1e-3, 1e-5
SM_SCALE = 1.0 / math.sqrt(192.0)


def _inputs(T, L, pages, seed, pad_frac=0.0, tail_pad=None):
    g = torch.Generator().manual_seed(seed)
    q_nope = torch.randn((T, 16, 512), generator=g).to(torch.bfloat16)
    q_pe = torch.randn((T, 16, 64), generator=g).to(torch.bfloat16)
    ckv = torch.randn((pages, 64, 512), generator=g).to(torch.bfloat16)
    kpe = torch.randn((pages, 64, 64), generator=g).to(torch.bfloat16)
    idx = torch.randint(0, pages * 64, (T, L), generator=g, dtype=torch.int32)
    if pad_frac > 0:
        idx[torch.rand((T, L), generator=g) < pad_frac] = -1
    if tail_pad is not None:  # the indexer's layout: valid entries first, -1 after
        for t in range(T):
            n = int(tail_pad[t])
            idx[t, n:] = -1
    return q_nope, q_pe, ckv, kpe, idx


def _naive(q_nope, q_pe, ckv, kpe, idx, scale):
    T = q_nope.shape[0]
    ckv2 = ckv.reshape(-1, 512).double()
    kpe2 = kpe.reshape(-1, 64).double()
    out = torch.zeros(T, 16, 512)
    lse = torch.full((T, 16), float("-inf"))
    for t in range(T):
        v = [int(s) for s in idx[t] if 0 <= int(s) < ckv2.shape[0]]
        if not v:
            continue
        sel = torch.tensor(v)
        for h in range(16):
            logit = (ckv2[sel] @ q_nope[t, h].double() + kpe2[sel] @ q_pe[t, h].double()) * scale
            p = torch.softmax(logit, 0)
            out[t, h] = (p @ ckv2[sel]).float()
            lse[t, h] = float(torch.logsumexp(logit, 0) / math.log(2.0))
    return out, lse


def _close(got, ref, atol, rtol):
    both_inf = torch.isinf(ref) & torch.isinf(got) & (torch.sign(ref) == torch.sign(got))
    err = (got - ref).abs()
    ok = both_inf | (err <= atol + rtol * ref.abs())
    return bool(ok.all()), float(torch.where(both_inf, torch.zeros_like(err), err).max())


def test_oracle_matches_per_head_loop():
    q_nope, q_pe, ckv, kpe, idx = _inputs(5, 300, 12, 0, pad_frac=0.3)
    idx[2] = -1                     # no valid slot
    idx[3, :10] = idx[3, 10]        # duplicated slot counts every time
    idx[4, 5] = 12 * 64 + 3         # out of range: ignored
    out, lse = rt.sparse_attention(q_nope, q_pe, ckv, kpe, idx, SM_SCALE, chunk=2)
    ref_out, ref_lse = _naive(q_nope, q_pe, ckv, kpe, idx, SM_SCALE)
    assert _close(out, ref_out, 1e-5, 1e-5)[0]
    assert _close(lse, ref_lse, 1e-5, 1e-6)[0]
    assert torch.all(out[2] == 0) and torch.all(torch.isneginf(lse[2]))


def test_oracle_single_slot_returns_its_row():
    q_nope, q_pe, ckv, kpe, idx = _inputs(2, 64, 4, 1)
    idx[:] = -1
    idx[0, 17] = 77
    out, lse = rt.sparse_attention(q_nope, q_pe, ckv, kpe, idx, SM_SCALE)
    assert torch.allclose(out[0], ckv.reshape(-1, 512)[77].float().expand(16, 512))
    logit = (q_nope[0].double() @ ckv.reshape(-1, 512)[77].double() +
             q_pe[0].double() @ kpe.reshape(-1, 64)[77].double()) * SM_SCALE
    assert torch.allclose(lse[0].double(), logit / math.log(2.0), atol=1e-5)


def test_abi_argument_errors_without_gpu():
    lib = package()._lib.load()
    P, ok = ctypes.c_void_p, ctypes.c_void_p(16)
    f = lib.dsa_sparse_attention_launch
    assert f(ok, ok, ok, ok, ok, 0.1, ok, ok, 4, 2048, 0, None) == 1     # no pages
    assert f(None, ok, ok, ok, ok, 0.1, ok, ok, 4, 2048, 8, None) == 1   # null q
    assert f(ok, ok, ok, ok, ok, 0.1, ok, ok, -1, 2048, 8, None) == 1    # negative T
    assert f(P(24), ok, ok, ok, ok, 0.1, ok, ok, 4, 2048, 8, None) == 2  # misaligned q
    assert f(ok, ok, ok, ok, ok, 0.1, ok, ok, 4, 65537, 8, None) == 5    # list too long
    assert f(None, None, None, None, None, 0.1, None, None, 0, 2048, 8, None) == 0  # no tokens


def test_torch_wrapper_validates_before_launch():
    pkg = package()
    q_nope, q_pe, ckv, kpe, idx = _inputs(2, 64, 2, 2)
    with pytest.raises(RuntimeError, match="CUDA tensor"):
        pkg.sparse_attention(q_nope, q_pe, ckv, kpe, idx, SM_SCALE)


# ---------------------------------------------------------------- GPU


def _run_gpu(q_nope, q_pe, ckv, kpe, idx, scale=SM_SCALE):
    pkg = package()
    d = torch.device("cuda:0")
    out, lse = pkg.sparse_attention(q_nope.to(d), q_pe.to(d), ckv.to(d), kpe.to(d), idx.to(d), scale)
    torch.cuda.synchronize()
    return out.float().cpu(), lse.cpu()


def _check(q_nope, q_pe, ckv, kpe, idx, scale=SM_SCALE):
    out, lse = _run_gpu(q_nope, q_pe, ckv, kpe, idx, scale)
    ref_out, ref_lse = rt.sparse_attention(q_nope, q_pe, ckv, kpe, idx, scale)
    ok_o, e_o = _close(out, ref_out, OUT_ATOL, OUT_RTOL)
    ok_l, e_l = _close(lse, ref_lse, LSE_ATOL, LSE_RTOL)
    assert ok_o, f"output max abs error {e_o}"
    assert ok_l, f"lse max abs error {e_l}"
    return out, lse


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 7, 64, 148, 300])
def test_gpu_matches_oracle_full_lists(T):
    # 148 tokens (one per SM) run one CTA per token; the others split every
    # list across CTAs (1 and 7 tokens many ways, 64 and 300 two and four
    # ways) and combine on the device.
    _check(*_inputs(T, 2048, 2000, 10 + T))


@pytest.mark.gpu
def test_gpu_padding_and_edge_slots():
    pkg = package()
    pkg.device_status(0, clear=True)
    T = 40
    lens = torch.tensor([0, 1, 63, 64, 65, 2047, 2048] + [int(x) for x in torch.randint(0, 2049, (T - 7,))])
    q_nope, q_pe, ckv, kpe, idx = _inputs(T, 2048, 600, 3, tail_pad=lens)
    idx[8, 100:140] = idx[8, 99]             # duplicates
    idx[9, 5] = 600 * 64 + 1                 # past the pool: ignored, flagged
    idx[10, ::3] = -1                        # holes in the middle
    out, lse = _check(q_nope, q_pe, ckv, kpe, idx)
    assert torch.all(out[0] == 0) and torch.all(torch.isneginf(lse[0]))
    assert pkg.device_status(0, clear=True) & pkg.DSA_STATUS_BAD_PAGE


@pytest.mark.gpu
@pytest.mark.parametrize("L", [1, 100, 640, 4096])
def test_gpu_list_lengths(L):
    # 4096 entries need at least two splits (2048 per CTA at most).
    _check(*_inputs(9, L, 400, 20 + L, pad_frac=0.1))


@pytest.mark.gpu
def test_gpu_large_logits_and_repeat_launches():
    # Sharp softmax (large scale) and three launches on one stream: the split
    # counters must come back to zero each time.
    inputs = _inputs(3, 2048, 300, 5)
    first = _check(*inputs, scale=0.5)
    for _ in range(2):
        again = _run_gpu(*inputs, scale=0.5)
        assert torch.equal(again[0], first[0]) and torch.equal(again[1], first[1])


@pytest.mark.gpu
def test_gpu_indexer_then_attention_chain():
    """The indexer's topk_indices (physical slots, -1 padded) feed the
    attention directly: both caches share one page pool and block table."""
    pkg = package()
    from conftest import workloads
    w = workloads().custom([1500, 4096, 700, 9000], seed=11)  # short rows end in -1
    d = torch.device("cuda:0")
    topk = torch.empty((w.batch, 2048), dtype=torch.int32, device=d)
    pkg.launch_topk_c(w.q.to(d), w.k_cache.to(d), w.weights.to(d), w.seq_lens.to(d), w.block_table.to(d), topk)
    torch.cuda.synchronize()
    topk = topk.cpu()
    assert int((topk[0] >= 0).sum()) == 1500 and int((topk[3] >= 0).sum()) == 2048
    q_nope, q_pe, ckv, kpe, _ = _inputs(w.batch, 1, w.num_pages, 7)
    _check(q_nope, q_pe, ckv, kpe, topk)


@pytest.mark.gpu
def test_gpu_empty_lists():
    # L = 0: every token has no slot (output 0, lse -inf); T = 0 is a no-op.
    q_nope, q_pe, ckv, kpe, _ = _inputs(5, 1, 8, 30)
    out, lse = _run_gpu(q_nope, q_pe, ckv, kpe, torch.empty((5, 0), dtype=torch.int32))
    assert torch.all(out == 0) and torch.all(torch.isneginf(lse))
    pkg = package()
    d = torch.device("cuda:0")
    e_out, e_lse = pkg.sparse_attention(q_nope[:0].to(d), q_pe[:0].to(d), ckv.to(d), kpe.to(d),
                                        torch.empty((0, 2048), dtype=torch.int32, device=d), SM_SCALE)
    torch.cuda.synchronize()
    assert e_out.shape == (0, 16, 512) and e_lse.shape == (0, 16)


@pytest.mark.gpu
def test_gpu_graph_capture_after_warmup():
    """A split shape is warmed up on a stream (the library allocates its
    split buffers there), captured into a CUDA graph, and replayed on new
    inputs copied into the same buffers: replays equal direct calls."""
    pkg = package()
    d = torch.device("cuda:0")
    a = [t.to(d) for t in _inputs(6, 2048, 500, 40)]   # 6 tokens: lists split across CTAs
    b = [t.to(d) for t in _inputs(6, 2048, 500, 41)]
    bufs = [t.clone() for t in a]                       # the graph's input buffers
    s = torch.cuda.Stream(d)
    s.wait_stream(torch.cuda.current_stream(d))
    with torch.cuda.stream(s):
        out, lse = pkg.sparse_attention(*bufs, SM_SCALE)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        pkg.sparse_attention(*bufs, SM_SCALE, output=out, lse=lse)
    for src in (b, a, b):
        for dst_t, src_t in zip(bufs, src):
            dst_t.copy_(src_t)
        g.replay()
        torch.cuda.synchronize()
        want = pkg.sparse_attention(*src, SM_SCALE)
        torch.cuda.synchronize()
        assert torch.equal(out, want[0]) and torch.equal(lse, want[1])
    del g
