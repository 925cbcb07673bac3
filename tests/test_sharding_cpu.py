"""CPU: multi-rank host logic over gloo (world size 2). The per-rank scoring
is the oracle restricted to the rank's key range, so the sharded result must
equal the one-shot oracle result exactly."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from conftest import workloads, package

PAGE, TOPK = 64, 2048


def _pack(score, pos):
    u = np.frombuffer(np.float32(score).tobytes(), dtype=np.uint32)[0]
    u = (~u) & 0xFFFFFFFF if u & 0x80000000 else u | 0x80000000
    return (int(u) << 32) | (0xFFFFFFFF - int(pos))


def oracle_partial(q, kc, w, sl, bt, lo, hi):
    """Best 2048 (score, position) per row among keys [lo, hi), best first."""
    sc = oracle.scores(q, kc, w, sl, bt)
    B = sc.shape[0]
    cs = torch.full((B, TOPK), float("-inf"))
    cp = torch.full((B, TOPK), -1, dtype=torch.int32)
    for b in range(B):
        n = min(int(sl[b]), bt.shape[1] * PAGE)
        pos = np.arange(lo, min(hi, n))
        keys = sorted(((_pack(sc[b, p], p), p) for p in pos), reverse=True)[:TOPK]
        for r, (_, p) in enumerate(keys):
            cs[b, r] = float(sc[b, p])
            cp[b, r] = int(p)
    return cs, cp


def oracle_merge(cs_all, cp_all, sl, bt):
    W, B, _ = cs_all.shape
    out = torch.full((B, TOPK), -1, dtype=torch.int32)
    for b in range(B):
        keys = []
        for r in range(W):
            for s, p in zip(cs_all[r, b].tolist(), cp_all[r, b].tolist()):
                if p >= 0:
                    keys.append((_pack(s, p), p))
        keys.sort(reverse=True)
        for i, (_, p) in enumerate(keys[:TOPK]):
            out[b, i] = int(bt[b, p // PAGE]) * PAGE + p % PAGE
    return out


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


SHARD_LENS = [5000, 2100, 700, 0, 3333]  # 5 rows: the all-to-all blocks are uneven


def _worker(rank, world, port, result_q, exchange):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        W = workloads()
        sh = __import__("importlib").import_module(package().__name__ + ".sharding")
        w = W.custom(SHARD_LENS, seed=31)
        got = sh.key_sharded_topk(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table,
                                  partial_fn=oracle_partial, merge_fn=oracle_merge, exchange=exchange)
        result_q.put((rank, got.numpy()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["allgather", "alltoall"])
def test_key_sharded_merge_equals_one_shot(exchange):
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, exchange)) for r in range(world)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    W = workloads()
    w = W.custom(SHARD_LENS, seed=31)
    ref = oracle.indexer(w.q, w.k_cache, w.weights, w.seq_lens, w.block_table)
    for r in range(world):
        assert np.array_equal(results[r], ref)


def test_request_shards_balanced_and_complete(pkg):
    sh = __import__("importlib").import_module(pkg.__name__ + ".sharding")
    sl = torch.tensor([100, 5000, 300, 4000, 4100, 0, 7, 9000])
    bins = sh.request_shards(sl, 3)
    allidx = torch.cat(bins).sort().values
    assert torch.equal(allidx, torch.arange(8))
    loads = [int(sl[b].sum()) for b in bins]
    assert max(loads) - min(loads) <= int(sl.max())


@pytest.mark.parametrize("L,world", [(131072, 8), (8192, 2), (1000, 4), (129, 2)])
def test_key_ranges_cover_and_align(pkg, L, world):
    sh = __import__("importlib").import_module(pkg.__name__ + ".sharding")
    rs = sh.key_ranges(L, world)
    assert rs[0][0] == 0 and rs[-1][1] == L
    for (a, b), (c, d) in zip(rs, rs[1:]):
        assert b == c and a <= b
    for a, _ in rs:
        assert a % 128 == 0


def test_peer_exchange_needs_its_region():
    """exchange="peer" without a PeerExchange is an error, not a silent
    fallback to another exchange."""
    import importlib
    sh = importlib.import_module(package().__name__ + ".sharding")
    with socket.socket() as so:
        so.bind(("127.0.0.1", 0))
        port = so.getsockname()[1]
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=0, world_size=1)
    try:
        with pytest.raises(ValueError, match="PeerExchange"):
            sh.key_sharded_topk(None, None, None, None, torch.zeros((1, 4), dtype=torch.int32), exchange="peer")
    finally:
        dist.destroy_process_group()
