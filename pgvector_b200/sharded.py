"""Row-sharded search across ranks (one process per GPU).

The reference spreads an index over GPUs as contiguous row-range shards and
tree-merges the per-shard top-k lists on the host (shard placement
ann/server/cuvs.c:2845-2862, AnnIndexTreeMerge
ann/server/indexfile.c:3235-3258). Here each rank owns one contiguous range,
searches it on its GPU, and the per-rank lists are combined by one NCCL
all-gather followed by the on-device merge -- the only collective on the
path. The exchange lives in libannb200 (AnnB200SearchSharded, with its own
NCCL communicator: comm_from_process_group); torch.distributed only carries
the communicator's id from rank 0 to the others. gather_lists and
search_sharded are the same exchange through torch.distributed, kept for
the CPU (gloo) tests of the host logic.
"""


def shard_bounds(rows, world, align=32):
    """Row boundaries of `world` contiguous shards; inner boundaries are
    multiples of `align` so each shard's slice of a u32 filter bitmap starts
    on a word."""
    b = [(rows * r // world) // align * align for r in range(world)] + [rows]
    return b


def ivf_shard(offsets, world, rank, align=32):
    """This rank's share of a list-major IVF shard (offsets: the nlists + 1
    row offsets of its lists): rows [lo, hi) in equal shares, the lists
    l0 .. l1-1 that meet them, and those lists' offsets clipped to the range
    (local, from 0). Lists are cut at the boundaries, so one very large list
    does not unbalance the ranks; a list held by two ranks is searched on
    both and the merge joins the halves. Returns (lo, hi, l0, l1, local
    offsets as int64 numpy)."""
    import numpy as np
    offsets = np.asarray(offsets, dtype=np.int64)
    b = shard_bounds(int(offsets[-1]), world, align)
    lo, hi = b[rank], b[rank + 1]
    l0 = int(np.searchsorted(offsets, lo, side='right')) - 1
    l1 = max(l0 + 1, int(np.searchsorted(offsets, hi, side='left')))
    return lo, hi, l0, l1, np.clip(offsets[l0:l1 + 1], lo, hi) - lo


def local_probes(probes, l0, l1):
    """A probe table ([nq][nprobe] global list numbers, numpy) in a rank's
    list numbering: lists l0 .. l1-1 become 0 .. l1-l0-1, the others
    padding (UINT32_MAX)."""
    import numpy as np
    p = np.asarray(probes).astype(np.int64)
    return np.where((p >= l0) & (p < l1), p - l0, 0xffffffff).astype(np.uint32)


def bitmap_slice(words, lo, hi):
    """The words covering rows [lo, hi) (lo a multiple of 32) and the bit count."""
    return words[lo // 32:(hi + 31) // 32], hi - lo


def gather_lists(dist_t, ids_t, count_t, group=None):
    """All-gather every rank's [nq][k] results into [world][nq][k] tensors
    (rank-major, the layout AnnB200MergeTopk takes). The three result tensors
    travel packed in one byte buffer: one collective a step."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    parts = [t.contiguous() for t in (dist_t, ids_t, count_t)]
    flat = [p.reshape(-1).view(torch.uint8) for p in parts]
    send = torch.cat(flat)
    if dist.get_backend(group) == 'nccl':
        buf = torch.empty((world, send.numel()), dtype=torch.uint8, device=send.device)
        dist.all_gather_into_tensor(buf, send, group=group)
    else:
        chunks = [torch.empty_like(send) for _ in range(world)]
        dist.all_gather(chunks, send, group=group)
        buf = torch.stack(chunks)
    out, off = [], 0
    for p, f in zip(parts, flat):
        n = f.numel()
        out.append(buf[:, off:off + n].contiguous().view(p.dtype).view((world,) + tuple(p.shape)))
        off += n
    return out


def search_sharded(shard, queries, k, metric, rows, group=None, merge=None):
    """Search this rank's shard and merge all ranks' results; every rank
    returns the merged (dist, id, count). `merge` defaults to the device
    merge; `rows` is this rank's candidate list (or None for all rows)."""
    import torch.distributed as dist
    d, i, c = shard.search(queries, k, metric, rows=rows)
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return d, i, c
    gd, gi, gc = gather_lists(d, i, c, group)
    if merge is None:
        from . import merge_topk as merge
    return merge(gd, gi, gc, k)


def comm_from_process_group(device, group=None):
    """This rank's libannb200 NCCL communicator over the ranks of a
    torch.distributed group: rank 0 makes the id, a broadcast hands it to
    the others (the only use of torch.distributed here), and every rank
    joins with its device."""
    import torch.distributed as dist
    from . import Comm
    world, rank = dist.get_world_size(group), dist.get_rank(group)
    box = [Comm.unique_id() if rank == 0 else None]
    dist.broadcast_object_list(box, src=0, group=group)
    return Comm(device, world, rank, box[0])
