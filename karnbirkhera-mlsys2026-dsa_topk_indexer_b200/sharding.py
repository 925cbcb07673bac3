"""Multi-GPU partitioning of the indexer (one process per GPU).

Decode batches split by request with no collective (`request_shards`).
Long sequences split along the key axis: every rank scores its key range and
keeps a best-2048 candidate list, and the lists meet and are merged
(`key_sharded_topk`): over NVLink peer memory by this library's own kernels
(`PeerExchange`: each rank merges its share of the rows straight from every
rank's lists and stores them into every rank's output), or through NCCL
(all-to-all by row or all-gather, then the merge kernel). The reference has
no multi-GPU path; this is the partitioning its north star asks for.
"""
import torch

PAGE, TOPK = 64, 2048


def request_shards(seq_lens, world):
    """Splits request indices into `world` bins of similar total length
    (longest-first greedy). Returns a list of sorted index tensors."""
    sl = torch.as_tensor(seq_lens).clamp(min=0).to(torch.int64).cpu()
    order = torch.argsort(sl, descending=True, stable=True).tolist()
    loads = [0] * world
    bins = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (loads[k], k))
        bins[r].append(i)
        loads[r] += int(sl[i])
    return [torch.tensor(sorted(b), dtype=torch.int64) for b in bins]


def key_ranges(max_len, world, align=2 * PAGE):
    """Contiguous, tile-aligned key ranges [lo, hi) covering [0, max_len)."""
    tiles = (int(max_len) + align - 1) // align
    out = []
    for r in range(world):
        lo = (tiles * r // world) * align
        hi = (tiles * (r + 1) // world) * align
        out.append((lo, min(hi, int(max_len)) if r < world - 1 else int(max_len)))
    return out


def _default_partial(q, kc, w, sl, bt, lo, hi):
    import importlib
    pkg = importlib.import_module(__package__)
    return pkg.indexer_partial(q, kc, w, sl, bt, lo, hi)


def _default_merge(cs, cp, sl, bt):
    import importlib
    pkg = importlib.import_module(__package__)
    return pkg.indexer_merge(cs, cp, sl, bt)


class _DeviceBytes:
    """A raw device allocation seen through the CUDA array interface, so that
    torch can view it without copying (the owner keeps it alive)."""

    def __init__(self, ptr, nbytes):
        self.__cuda_array_interface__ = {"shape": (int(nbytes),), "typestr": "|u1", "data": (int(ptr), False),
                                         "version": 3, "strides": None}


class PeerExchange:
    """The key-axis exchange and merge over NVLink peer memory, no NCCL on the
    data path (C ABI dsa_peer_*; protocol in include/dsa_topk_indexer.h).

    Every rank of `group` builds one for the same batch size (a collective:
    the CUDA IPC handles are exchanged once with all_gather_object). Per step:
    write the rank's partial lists into `cand_scores` / `cand_pos` (pass them
    to indexer_partial), then `merge(block_table)` runs [signal ready, merge
    this rank's rows from every rank's lists and store them into every rank's
    output, signal done, wait for every rank] on the current stream and
    returns `out` [B, 2048] int32, valid until the next merge. Call `close()`
    on every rank together before the process group goes away."""

    def __init__(self, batch, device, group=None, wait_ns=0):
        import ctypes
        import importlib
        import torch.distributed as dist
        self.pkg = importlib.import_module(__package__)
        self.lib = self.pkg._lib.load()
        self.group, self.device, self.batch, self.wait_ns = group, torch.device(device), int(batch), int(wait_ns)
        if self.device.index is None:
            self.device = torch.device("cuda", torch.cuda.current_device())
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        self.pkg._select(self.lib, self.device)
        nbytes = ctypes.c_int64(0)
        self.pkg._lib.check(self.lib.dsa_peer_region_bytes(self.batch, ctypes.byref(nbytes)), "peer_region_bytes")
        ptr, handle = ctypes.c_void_p(), (ctypes.c_char * 64)()
        with torch.cuda.device(self.device):
            self.pkg._lib.check(self.lib.dsa_peer_alloc(nbytes.value, ctypes.byref(ptr), handle), "peer_alloc")
        self.own = ptr.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        self.opened, bases = [], []
        for r, h in enumerate(handles):
            if r == self.rank:
                bases.append(self.own)
                continue
            p = ctypes.c_void_p()
            with torch.cuda.device(self.device):
                self.pkg._lib.check(self.lib.dsa_peer_open(h, ctypes.byref(p)), "peer_open")
            self.opened.append(p.value)
            bases.append(p.value)
        self._views(bases, nbytes.value)
        self.epoch = 0

    def _views(self, bases, nbytes):
        """Device array of the region bases and tensor views of this rank's region."""
        self.bases = torch.tensor([b - (1 << 64) if b >= (1 << 63) else b for b in bases], dtype=torch.int64,
                                  device=self.device)
        region = torch.as_tensor(_DeviceBytes(self.own, nbytes), device=self.device)
        L = self.batch * TOPK * 4
        self.cand_scores = region[:L].view(torch.float32).view(self.batch, TOPK)
        self.cand_pos = region[L:2 * L].view(torch.int32).view(self.batch, TOPK)
        self.out = region[2 * L:3 * L].view(torch.int32).view(self.batch, TOPK)

    def merge(self, block_table, phases=15):
        """One step of the protocol (all phases by default) on the current
        stream; returns `out`."""
        import ctypes
        if (block_table.dim() != 2 or block_table.shape[0] != self.batch or block_table.dtype != torch.int32
                or block_table.device != self.device):
            raise RuntimeError(f"block_table must be int32 [{self.batch}, max_pages] on {self.device}")
        if phases & 1:
            self.epoch += 1
        bt = block_table.contiguous()
        stream = torch.cuda.current_stream(self.device).cuda_stream
        with torch.cuda.device(self.device):
            rc = self.lib.dsa_peer_merge(ctypes.c_void_p(self.bases.data_ptr()), self.world, self.rank, self.epoch,
                                         self.batch, ctypes.c_void_p(bt.data_ptr()), bt.shape[1], phases,
                                         self.wait_ns, ctypes.c_void_p(stream))
        self.pkg._lib.check(rc, "peer_merge")
        return self.out

    def close(self):
        """Unmaps the peers' regions and frees this rank's, after every rank
        has finished with them (barriers on the process group)."""
        import torch.distributed as dist
        if self.own is None:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for p in self.opened:
            self.lib.dsa_peer_close(p)
        dist.barrier(group=self.group)
        with torch.cuda.device(self.device):
            self.lib.dsa_peer_free(self.own)
        self.own, self.opened = None, []


def key_sharded_topk(q, kc, w, seq_lens, block_table, group=None, partial_fn=None, merge_fn=None, max_len=None,
                     exchange="alltoall", peer=None):
    """Top-2048 physical slots of every row, the key axis split over the ranks
    of `group`. Every rank holds the full inputs (the K cache pages of its
    range must be resident) and returns the same full result.

    exchange="allgather": every rank gathers every rank's [B, 2048]
    candidate lists and merges all B rows. exchange="alltoall": rank r
    receives only the lists of its B/world rows (all-to-all), merges those,
    and the [B, 2048] int32 results are all-gathered: (world-1)/world of one
    rank's lists cross the links instead of world-1 times all of them, and
    the merge work is split world ways. exchange="peer": the same split of
    the merge with no collective library, over NVLink peer memory (`peer`, a
    PeerExchange for this batch size; the partial lists are written straight
    into its region and the result is its `out`, valid until the next call)."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if max_len is None:
        max_len = int(block_table.shape[1]) * PAGE
    lo, hi = key_ranges(max_len, world)[rank]
    if exchange == "peer":
        if peer is None:
            raise ValueError('exchange="peer" needs a PeerExchange (peer=)')
        import importlib
        pkg = importlib.import_module(__package__)
        fn = partial_fn or pkg.indexer_partial  # written straight into this rank's region
        fn(q, kc, w, seq_lens, block_table, lo, hi, peer.cand_scores, peer.cand_pos)
        return peer.merge(block_table)
    partial_fn = partial_fn or _default_partial
    merge_fn = merge_fn or _default_merge
    cs, cp = partial_fn(q, kc, w, seq_lens, block_table, lo, hi)
    B = cs.shape[0]
    if exchange == "allgather":
        cs_all = torch.empty((world * B, TOPK), dtype=cs.dtype, device=cs.device)
        cp_all = torch.empty((world * B, TOPK), dtype=cp.dtype, device=cp.device)
        dist.all_gather_into_tensor(cs_all, cs.contiguous(), group=group)
        dist.all_gather_into_tensor(cp_all, cp.contiguous(), group=group)
        return merge_fn(cs_all.view(world, B, TOPK), cp_all.view(world, B, TOPK), seq_lens, block_table)
    if exchange != "alltoall":
        raise ValueError(f"exchange must be 'allgather' or 'alltoall', not {exchange!r}")
    # Rows [bounds[r], bounds[r+1]) are merged on rank r.
    bounds = [B * r // world for r in range(world + 1)]
    sizes = [bounds[r + 1] - bounds[r] for r in range(world)]
    mine = sizes[rank]
    cs_in = torch.empty((world * mine, TOPK), dtype=cs.dtype, device=cs.device)
    cp_in = torch.empty((world * mine, TOPK), dtype=cp.dtype, device=cp.device)
    dist.all_to_all_single(cs_in, cs.contiguous(), [mine] * world, sizes, group=group)
    dist.all_to_all_single(cp_in, cp.contiguous(), [mine] * world, sizes, group=group)
    r0, r1 = bounds[rank], bounds[rank + 1]
    per = (B + world - 1) // world  # equal all-gather blocks; short blocks padded
    part = torch.full((per, TOPK), -1, dtype=torch.int32, device=cs.device)
    if mine > 0:
        part[:mine] = merge_fn(cs_in.view(world, mine, TOPK), cp_in.view(world, mine, TOPK),
                               seq_lens[r0:r1].contiguous(), block_table[r0:r1].contiguous())
    gathered = torch.empty((world * per, TOPK), dtype=torch.int32, device=cs.device)
    dist.all_gather_into_tensor(gathered, part, group=group)
    g = gathered.view(world, per, TOPK)
    return torch.cat([g[r, :sizes[r]] for r in range(world)], dim=0)
