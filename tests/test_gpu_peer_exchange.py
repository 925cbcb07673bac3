"""GPU: the key-axis exchange over peer memory (dsa_peer_*).

On one GPU the protocol is emulated with several regions standing for the
ranks: every rank's phase is issued in order on one stream (all ready
signals, then all merges, then all done signals, then all waits), so no wait
ever depends on a launch that comes after it. The merged rows must equal
dsa_topk_indexer_merge over the same lists bit for bit in every rank's
output. A wait on a flag that nothing sets runs out (1 ms) and reports
DSA_STATUS_WAIT_TIMEOUT without a fault. With two GPUs, two processes run
the real exchange over NVLink and must match the NCCL all-to-all path."""
import ctypes
import os

import pytest
import torch

from conftest import package, workloads

pytestmark = pytest.mark.gpu


def _sharding():
    return __import__("importlib").import_module(package().__name__ + ".sharding")


class _Regions:
    """n peer regions on the current GPU (each a 'rank'), freed on close."""

    def __init__(self, lib, n, batch):
        sh = _sharding()
        self.lib, self.batch, self.ptrs = lib, batch, []
        nbytes = ctypes.c_int64(0)
        assert lib.dsa_peer_region_bytes(batch, ctypes.byref(nbytes)) == 0
        L = batch * 2048 * 4
        self.views = []
        for _ in range(n):
            p, h = ctypes.c_void_p(), (ctypes.c_char * 64)()
            assert lib.dsa_peer_alloc(nbytes.value, ctypes.byref(p), h) == 0
            self.ptrs.append(p.value)
            reg = torch.as_tensor(sh._DeviceBytes(p.value, nbytes.value), device="cuda")
            self.views.append((reg[:L].view(torch.float32).view(batch, 2048),
                               reg[L:2 * L].view(torch.int32).view(batch, 2048),
                               reg[2 * L:3 * L].view(torch.int32).view(batch, 2048)))
        self.bases = torch.tensor(self.ptrs, dtype=torch.int64, device="cuda")

    def run(self, bt, epoch, phases_in_order=(1, 2, 4, 8), wait_ns=0):
        n = len(self.ptrs)
        st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
        for ph in phases_in_order:
            for r in range(n):
                assert self.lib.dsa_peer_merge(ctypes.c_void_p(self.bases.data_ptr()), n, r, epoch, self.batch,
                                               ctypes.c_void_p(bt.data_ptr()), bt.shape[1], ph, wait_ns, st) == 0

    def close(self):
        torch.cuda.synchronize()
        for p in self.ptrs:
            self.lib.dsa_peer_free(ctypes.c_void_p(p))


@pytest.mark.parametrize("nranks", [2, 3])
def test_peer_protocol_emulated_on_one_gpu(pkg, nranks):
    sh = _sharding()
    w = workloads().make_shared("peer", 67, 20000, 400, 5).to("cuda")
    B, mp = w.batch, w.max_pages
    lib = pkg._lib.load()
    regs = _Regions(lib, nranks, B)
    try:
        ranges = sh.key_ranges(mp * 64, nranks)
        for epoch in (1, 2):
            if epoch == 2:  # a second step with other queries: the step counters move on
                w.q = w.q.flip(0).contiguous()
            for r, (lo, hi) in enumerate(ranges):
                cs, cp, _ = regs.views[r]
                pkg.indexer_partial(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, lo, hi, cs, cp)
            pkg.device_status(0, clear=True)
            regs.run(w.block_table, epoch)
            torch.cuda.synchronize()
            assert pkg.device_status(0, clear=True) == 0
            cs_all = torch.stack([v[0] for v in regs.views])
            cp_all = torch.stack([v[1] for v in regs.views])
            ref = pkg.indexer_merge(cs_all, cp_all, w.seq_lens, w.block_table)
            direct = torch.empty_like(ref)
            pkg.launch_topk_c(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, direct)
            torch.cuda.synchronize()
            assert torch.equal(ref, direct)
            for r in range(nranks):
                assert torch.equal(regs.views[r][2], ref), (epoch, r)
    finally:
        regs.close()


def test_peer_wait_runs_out_without_fault(pkg):
    """Flags that nothing sets: the merge and the final wait give up after
    1 ms with DSA_STATUS_WAIT_TIMEOUT, the merge CTAs write nothing, and a
    normal step afterwards is correct."""
    w = workloads().make_shared("peerto", 8, 5000, 100, 6).to("cuda")
    lib = pkg._lib.load()
    regs = _Regions(lib, 2, w.batch)
    try:
        regs.views[0][2].fill_(-7)
        pkg.device_status(0, clear=True)
        # ready flags of epoch 5 are never raised: only phases 2 and 8 run
        regs.run(w.block_table, 5, phases_in_order=(2, 8), wait_ns=1_000_000)
        torch.cuda.synchronize()
        assert pkg.device_status(0, clear=True) & pkg.DSA_STATUS_WAIT_TIMEOUT
        assert (regs.views[0][2] == -7).all()
        for r, (lo, hi) in enumerate(_sharding().key_ranges(w.max_pages * 64, 2)):
            cs, cp, _ = regs.views[r]
            pkg.indexer_partial(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, lo, hi, cs, cp)
        regs.run(w.block_table, 6)
        torch.cuda.synchronize()
        assert pkg.device_status(0, clear=True) == 0
        direct = torch.empty_like(regs.views[0][2])
        pkg.launch_topk_c(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, direct)
        torch.cuda.synchronize()
        assert torch.equal(regs.views[0][2], direct) and torch.equal(regs.views[1][2], direct)
    finally:
        regs.close()


def _two_gpu_child(rank, port):
    import datetime
    import torch.distributed as dist
    os.environ["NCCL_NVLS_ENABLE"] = "0"  # plain peer traffic only
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=2,
                            timeout=datetime.timedelta(seconds=60))
    try:
        pkg, sh = package(), _sharding()
        dev = torch.device("cuda", rank)
        w = workloads().make_shared("peer2", 96, 40000, 800, 7).to(dev)
        ref = sh.key_sharded_topk(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, exchange="alltoall")
        direct = torch.empty_like(ref)
        pkg.launch_topk_c(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, direct)
        ex = sh.PeerExchange(w.batch, dev)
        for _ in range(3):
            got = sh.key_sharded_topk(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table, exchange="peer",
                                      peer=ex).clone()
            torch.cuda.synchronize(dev)
            assert torch.equal(got, ref) and torch.equal(got, direct)
        assert pkg.device_status(rank) == 0
        ex.close()
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(600)
def test_peer_exchange_two_gpus():
    """Two processes on two GPUs: the peer exchange equals the NCCL all-to-all
    path and the one-GPU call, three steps in a row."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    mp.spawn(_two_gpu_child, args=(port,), nprocs=2, join=True)
