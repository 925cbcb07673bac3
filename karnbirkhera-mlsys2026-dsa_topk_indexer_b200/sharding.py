"""Multi-GPU partitioning of the indexer (one process per GPU).

Decode batches split by request with no collective (`request_shards`).
Long sequences split along the key axis: every rank scores its key range and
keeps a best-2048 candidate list, the lists are all-gathered (NCCL over
NVLink on GPUs) and merged (`key_sharded_topk`). The reference has no
multi-GPU path; this is the partitioning its north star asks for.
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


def key_sharded_topk(q, kc, w, seq_lens, block_table, group=None, partial_fn=None, merge_fn=None, max_len=None,
                     exchange="alltoall"):
    """Top-2048 physical slots of every row, the key axis split over the ranks
    of `group`. Every rank holds the full inputs (the K cache pages of its
    range must be resident) and returns the same full result.

    exchange="allgather": every rank gathers every rank's [B, 2048]
    candidate lists and merges all B rows. exchange="alltoall": rank r
    receives only the lists of its B/world rows (all-to-all), merges those,
    and the [B, 2048] int32 results are all-gathered: (world-1)/world of one
    rank's lists cross the links instead of world-1 times all of them, and
    the merge work is split world ways."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if max_len is None:
        max_len = int(block_table.shape[1]) * PAGE
    lo, hi = key_ranges(max_len, world)[rank]
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
