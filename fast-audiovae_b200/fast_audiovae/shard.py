"""Multi-GPU decoding by independent shards (one process per GPU).

The decoder has no cross-stream reduction: each stream or clip owns its
history (the reference's streaming.py:61-72, gpu.py:202-210), so N GPUs decode
N disjoint, contiguous shards with no collective on the data path. A stream's
history lives on its GPU for the stream's lifetime. ``torch.distributed`` only
carries host-side bookkeeping here: collecting a caller's results in input
order, and the max of per-rank timings.
"""
from __future__ import annotations


def shard_range(n_items, world, rank):
    """Contiguous share [start, stop) of rank ``rank`` among ``world`` ranks (sizes differ by at most one)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("rank must lie in [0, world)")
    if n_items < 0:
        raise ValueError("n_items must be non-negative")
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def _world(group):
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


def decode_clips(decoder, clips, *, group=None, gather=True):
    """Batch-decode this rank's contiguous share of ``clips`` on its GPU.

    Returns this rank's audio list, or with ``gather`` every clip's audio in
    input order on every rank (host-side object gather; the decode itself
    exchanges nothing).
    """
    world, rank = _world(group)
    start, stop = shard_range(len(clips), world, rank)
    mine = list(clips[start:stop])
    # Clips of equal length decode together (one launch per layer per chunk).
    local = [None] * len(mine)
    by_length = {}
    for i, clip in enumerate(mine):
        by_length.setdefault(clip.shape[-1], []).append(i)
    for idx in by_length.values():
        for i, audio in zip(idx, decoder.decode_many([mine[i] for i in idx])):
            local[i] = audio
    if not gather or world == 1:
        return local
    import torch.distributed as dist
    parts = [None] * world
    dist.all_gather_object(parts, (start, local), group=group)
    return [audio for _, part in sorted(parts, key=lambda p: p[0]) for audio in part]


def max_over_ranks(value, group=None):
    """The maximum of a per-rank float (e.g. a device time) over all ranks."""
    world, _ = _world(group)
    if world == 1:
        return float(value)
    import torch
    import torch.distributed as dist
    t = torch.tensor([float(value)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
