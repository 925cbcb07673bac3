"""Index-K cache writer (the producer of the page format the indexer reads).

CPU: the restatement in oracle/reference_torch.py against the format's
dequantisation (f32(e4m3) * scale, the reference's reading of a page,
solution/cuda/kernel.cu:22-25): error within half an e4m3 step of the
token's scale. GPU: the CUDA writer bit-exact against the restatement, and
the indexer on a cache written by the CUDA writer equal to the oracle on the
same cache.
"""
import numpy as np
import pytest
import torch

import oracle
from conftest import package, workloads
from parity import check_all

import reference_torch as rt  # oracle/ is on sys.path (conftest)


def _inputs(T, dtype, seed, pages=40):
    g = torch.Generator().manual_seed(seed)
    k = torch.randn((T, 128), generator=g) * torch.exp(torch.randn((T, 1), generator=g) * 2)
    k[3] = 0.0                          # all-zero vector: scale 1
    k[5] = 0.0
    k[5, 7] = -3.0e-3                   # one value: it maps to -448
    k[7] = torch.linspace(-1, 1, 128)   # exact ties of the rounding are possible
    k = k.to(dtype)
    slots = torch.randperm(pages * 64, generator=g)[:T].to(torch.int64)
    slots[1] = -1                       # skipped token
    return k, slots


def test_oracle_writer_dequantises_within_half_step():
    k, slots = _inputs(200, torch.float32, 1)
    cache = torch.zeros((40, 64, 1, 132), dtype=torch.uint8)
    rt.cache_write(k, slots, cache)
    flat = cache.view(40, 8448)
    for t in range(200):
        s = int(slots[t])
        if s < 0:
            continue
        page, off = s >> 6, s & 63
        q = flat[page, off * 128:(off + 1) * 128].view(torch.float8_e4m3fn).to(torch.float32)
        scale = flat[page, 8192 + off * 4:8192 + off * 4 + 4].view(torch.float32)[0]
        back = q * scale
        x = k[t]
        # e4m3 has 3 mantissa bits: relative step 1/8 for normals; absolute
        # step 2^-9 * scale below the normal range.
        tol = torch.maximum(x.abs() / 16, torch.full_like(x, 2.0 ** -10) * scale) * 1.0001
        assert (back - x).abs().le(tol).all(), t
        if float(x.abs().max()) > 0:
            assert abs(float(scale) - float(x.abs().max()) / 448) <= 1e-6 * float(scale)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_cuda_writer_bit_exact(dtype):
    pkg = package()
    k, slots = _inputs(1000, dtype, 2, pages=40)
    ref = torch.zeros((40, 64, 1, 132), dtype=torch.uint8)
    rt.cache_write(k, slots, ref)
    got = torch.zeros_like(ref).cuda()
    pkg.index_cache_write(k.cuda(), slots.cuda(), got)
    torch.cuda.synchronize()
    assert torch.equal(got.cpu(), ref)
    assert pkg.device_status(0) == 0


@pytest.mark.gpu
def test_cuda_writer_out_of_range_slot_flags_status():
    pkg = package()
    k, slots = _inputs(64, torch.float32, 3, pages=2)
    slots = slots % 128
    slots[9] = 2 * 64 + 5  # page 2 of a 2-page cache
    cache = torch.zeros((2, 64, 1, 132), dtype=torch.uint8, device="cuda")
    pkg.device_status(0, clear=True)
    pkg.index_cache_write(k.cuda(), slots.cuda(), cache)
    torch.cuda.synchronize()
    assert pkg.device_status(0, clear=True) & pkg._lib.DSA_STATUS_BAD_PAGE


@pytest.mark.gpu
def test_indexer_on_written_cache():
    """Write a sequence's K through the CUDA writer, then run the indexer on
    that cache: same parity bar as every other workload."""
    pkg = package()
    W = workloads()
    seq_lens = [3000, 700, 5000]
    w = W.custom(seq_lens, seed=4)            # block tables and queries
    T = w.num_pages * 64
    g = torch.Generator().manual_seed(5)
    kv = (torch.randn((T, 128), generator=g) * 0.7).to(torch.bfloat16)
    slots = torch.arange(T, dtype=torch.int64)
    cache = torch.zeros_like(w.k_cache).cuda()
    pkg.index_cache_write(kv.cuda(), slots.cuda(), cache)
    torch.cuda.synchronize()
    ww = type(w)("written", w.q, cache.cpu(), w.weights, w.seq_lens, w.block_table)
    d = ww.to("cuda")
    out = torch.empty((ww.batch, 2048), dtype=torch.int32, device="cuda")
    pkg.launch_topk_c(d.q, d.k_cache, d.weights, d.seq_lens, d.block_table, out)
    torch.cuda.synchronize()
    ref = oracle.indexer(ww.q, ww.k_cache, ww.weights, ww.seq_lens, ww.block_table)
    sc = oracle.scores(ww.q, ww.k_cache, ww.weights, ww.seq_lens, ww.block_table)
    rows = [sc[b, :s] for b, s in enumerate(seq_lens)]
    fails = check_all(out.cpu().numpy(), ref, rows, ww.seq_lens.numpy(), ww.block_table.numpy(), ww.num_pages)
    assert not fails, fails[:3]
