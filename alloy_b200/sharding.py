"""Partitioning a Mamba-2 layer across the GPUs of one node.

Every (batch row, head group) of the mixer is independent: no state or
activation crosses between them inside the path (alloy/models/mamba_block.py
only couples heads through the shared B/C of a group, :463-468).  A layer is
therefore split with no collective inside the path:

* prefill: by head group when the groups divide over the ranks (each rank
  reads the x channels of its heads and its groups' B/C columns), otherwise
  by heads inside the groups (each rank reads all B/C of its groups);
* decode: by batch rows.

``allgather_heads`` is the one collective, used only when a caller needs the
whole y replicated (e.g. before an out-projection that is not sharded).
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

__all__ = ["HeadShard", "head_shard", "batch_shard", "allgather_heads"]


@dataclass(frozen=True)
class HeadShard:
    head_begin: int
    head_count: int
    group_begin: int
    group_count: int


def head_shard(n_heads: int, n_groups: int, world: int, rank: int) -> HeadShard:
    """This rank's heads: whole head groups when ``n_groups % world == 0``,
    else an equal run of heads inside the groups (``n_heads % world == 0``)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of {world}")
    if n_heads % n_groups:
        raise ValueError("n_heads must be a multiple of n_groups")
    hpg = n_heads // n_groups
    if n_groups % world == 0:
        gpr = n_groups // world
        g0 = rank * gpr
        return HeadShard(g0 * hpg, gpr * hpg, g0, gpr)
    if n_heads % world:
        raise ValueError(f"{n_heads} heads do not split over {world} ranks")
    hpr = n_heads // world
    h0 = rank * hpr
    g0 = h0 // hpg
    g1 = (h0 + hpr - 1) // hpg
    return HeadShard(h0, hpr, g0, g1 - g0 + 1)


def batch_shard(batch: int, world: int, rank: int) -> tuple[int, int]:
    """(begin, count) of this rank's batch rows (the first ranks take one more
    when the batch does not divide)."""
    base, extra = divmod(batch, world)
    begin = rank * base + min(rank, extra)
    return begin, base + (1 if rank < extra else 0)


def allgather_heads(y_local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """Gather per-rank head slices ``[B, L, H/world, P]`` into ``[B, L, H, P]``.

    Rank r's slice holds heads [r*H/world, (r+1)*H/world).  The gather is one
    contiguous all-gather into a head-major ``[world, B, L, H/world, P]``
    buffer, then a permute (a copy) to the caller's layout.
    """
    import torch.distributed as dist
    if world == 1:
        return y_local
    y_local = y_local.contiguous()
    B, L, hl, P = y_local.shape
    buf = torch.empty((world * B, L, hl, P), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(buf, y_local, group=group)
    return buf.view(world, B, L, hl, P).permute(1, 2, 0, 3, 4).reshape(B, L, world * hl, P)
