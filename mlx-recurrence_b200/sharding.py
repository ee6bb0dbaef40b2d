"""Data-parallel placement of the scans over ranks (one process per GPU).

The recurrences are independent per (batch row, head) for SSD, GLA and Gated
DeltaNet and per (batch row, channel) for RG-LRU and rotLRU, so a multi-GPU
job gives each rank a rectangular block of those units - a contiguous range
of batch rows times a contiguous range of heads (channels) - and runs it with
no exchange at all. When the world size divides the batch the blocks are
whole batch ranges; otherwise the heads (channels) are split as well, so that
every rank has work whenever there are at least as many units as ranks.
Channel ranges keep the lane rule of the scans (RG-LRU channels in multiples
of 32, rotLRU pairs in multiples of 16). Collectives appear only around the
work: a max-over-ranks reduction of timings and, for checking, gathering the
ranks' blocks. Works with any torch.distributed backend (NCCL on GPUs, gloo on
CPU).
"""

from __future__ import annotations

import torch


def shard_range(n, rank, world):
    """Contiguous range [i0, i1) of ``rank`` out of ``world`` over n items;
    ranks below n % world take one extra item."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    per, rem = divmod(n, world)
    i0 = rank * per + min(rank, rem)
    return i0, i0 + per + (1 if rank < rem else 0)


def shard_batch(B, rank, world):
    """Contiguous batch range [b0, b1) of ``rank`` out of ``world``."""
    return shard_range(B, rank, world)


def rank_grid(B, U, world, quantum=1):
    """(wb, wu): the ranks laid out as wb batch groups times wu unit groups
    (wb * wu == world) over a [B, U] grid of units whose unit axis is split in
    multiples of ``quantum``. Every rank gets a nonempty block; among the
    layouts that allow it, the one with the smallest largest block wins, and
    on a tie the one with more batch groups (whole batch rows per rank)."""
    if U % quantum != 0:
        raise ValueError(f"unit axis {U} is not a multiple of its split quantum {quantum}")
    G = U // quantum
    best = None
    for wb in range(1, world + 1):
        if world % wb:
            continue
        wu = world // wb
        if wb > B or wu > G:
            continue
        cost = -(-B // wb) * (-(-G // wu))
        key = (cost, -wb)
        if best is None or key < best[0]:
            best = (key, (wb, wu))
    if best is None:
        raise ValueError(f"{world} ranks cannot each get work from {B} batch rows x {G} unit groups")
    return best[1]


def block_of(B, U, rank, world, quantum=1):
    """Block (b0, b1, u0, u1) of ``rank``: batch rows [b0, b1) times units
    [u0, u1) (u0, u1 multiples of ``quantum``). Consecutive ranks walk the
    unit axis first, so a batch group's ranks are neighbours."""
    wb, wu = rank_grid(B, U, world, quantum)
    rb, ru = divmod(rank, wu)
    b0, b1 = shard_range(B, rb, wb)
    g0, g1 = shard_range(U // quantum, ru, wu)
    return b0, b1, g0 * quantum, g1 * quantum


def max_over_ranks(values, device=None):
    """Element-wise maximum of a list of floats over all ranks (float64)."""
    import torch.distributed as dist
    t = torch.tensor(list(values), dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return t.tolist()


def _world():
    import torch.distributed as dist
    if dist.is_available() and dist.is_initialized():
        return dist.get_world_size()
    return 1


def gather_blocks(t, B, U, quantum=1, axis=2):
    """Every rank's block of a [B, ..., U * s, ...] tensor (batch on dim 0, the
    unit axis on ``axis`` with s values per unit, s = its extent / the block's
    unit count) assembled into the full tensor on every rank."""
    import torch.distributed as dist
    world = _world()
    if world == 1:
        return t
    blocks = [block_of(B, U, r, world, quantum) for r in range(world)]
    rank = dist.get_rank()
    b0, b1, u0, u1 = blocks[rank]
    s = t.shape[axis] // (u1 - u0)
    rows = max(bb1 - bb0 for bb0, bb1, _, _ in blocks)
    cols = max(uu1 - uu0 for _, _, uu0, uu1 in blocks) * s
    pshape = list(t.shape)
    pshape[0], pshape[axis] = rows, cols
    pad = torch.zeros(pshape, dtype=t.dtype, device=t.device)
    idx = [slice(None)] * t.dim()
    idx[0], idx[axis] = slice(0, t.shape[0]), slice(0, t.shape[axis])
    pad[tuple(idx)] = t
    out = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(out, pad.contiguous())
    fshape = list(t.shape)
    fshape[0], fshape[axis] = B, U * s
    full = torch.empty(fshape, dtype=t.dtype, device=t.device)
    for o, (bb0, bb1, uu0, uu1) in zip(out, blocks):
        dst = [slice(None)] * t.dim()
        src = [slice(None)] * t.dim()
        dst[0], dst[axis] = slice(bb0, bb1), slice(uu0 * s, uu1 * s)
        src[0], src[axis] = slice(0, bb1 - bb0), slice(0, (uu1 - uu0) * s)
        full[tuple(dst)] = o[tuple(src)]
    return full


def sum_unit_param(g, B, U, quantum=1):
    """A per-unit parameter's gradient (dim 0 = the rank's unit range) summed
    over ranks into the full [U, ...] gradient (ranks holding the same units
    for different batch rows add up)."""
    import torch.distributed as dist
    world = _world()
    if world == 1:
        return g
    _, _, u0, u1 = block_of(B, U, dist.get_rank(), world, quantum)
    full = torch.zeros((U,) + tuple(g.shape[1:]), dtype=torch.promote_types(g.dtype, torch.float32),
                       device=g.device)
    full[u0:u1] = g
    dist.all_reduce(full)
    return full


def gather_rows(t, B):
    """Concatenate every rank's batch rows (dim 0) into the full [B, ...]
    tensor on every rank (whole-batch-range blocks)."""
    import torch.distributed as dist
    world = _world()
    if world == 1:
        return t
    sizes = [shard_batch(B, r, world) for r in range(world)]
    rows = max(b1 - b0 for b0, b1 in sizes)
    pad = torch.zeros((rows,) + tuple(t.shape[1:]), dtype=t.dtype, device=t.device)
    pad[: t.shape[0]] = t
    out = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(out, pad.contiguous())
    return torch.cat([o[: b1 - b0] for o, (b0, b1) in zip(out, sizes)], dim=0)
