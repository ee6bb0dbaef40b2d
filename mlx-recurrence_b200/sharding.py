"""Data-parallel placement of the scans over ranks (one process per GPU).

The recurrences are independent per (batch row, head) and per (batch row,
channel), so a multi-GPU job gives each rank a contiguous range of batch rows
and runs it with no exchange at all. Collectives appear only around the work:
a max-over-ranks reduction of timings and, for checking, gathering the
ranks' result rows. Works with any torch.distributed backend (NCCL on GPUs,
gloo on CPU).
"""

from __future__ import annotations

import torch


def shard_batch(B, rank, world):
    """Contiguous batch range [b0, b1) of ``rank`` out of ``world``; ranks
    below B % world take one extra row."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    per, rem = divmod(B, world)
    b0 = rank * per + min(rank, rem)
    return b0, b0 + per + (1 if rank < rem else 0)


def max_over_ranks(values, device=None):
    """Element-wise maximum of a list of floats over all ranks (float64)."""
    import torch.distributed as dist
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def gather_rows(t, B):
    """Concatenate every rank's batch rows (dim 0) into the full [B, ...]
    tensor on every rank. Shards may differ by one row; they are padded to the
    largest shard for the collective and trimmed afterwards."""
    import torch.distributed as dist
    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return t
    world = dist.get_world_size()
    sizes = [shard_batch(B, r, world) for r in range(world)]
    rows = max(b1 - b0 for b0, b1 in sizes)
    pad = torch.zeros((rows,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    pad[: t.shape[0]] = t
    out = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(out, pad.contiguous())
    return torch.cat([o[: b1 - b0] for o, (b0, b1) in zip(out, sizes)], dim=0)
