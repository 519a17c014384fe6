"""Head sharding of a layer over the ranks of one node.

The flat operator has no exchange step: the heads of a layer (and the batch entries of a CFG pair) are
independent, so each rank runs its own contiguous block of heads through the single-GPU path and the
outputs are gathered once per head at the end.  The reference's runner loops over ``(head, q, k, v)``
jobs in one process (h3/htrc_flat_runner.py:179-200); here the jobs are split by rank.  The gather is one
``all_gather_into_tensor`` per local head slot, so it can run on a side stream while the next head
computes.
"""
from __future__ import annotations

import torch


def heads_of_rank(n_heads: int, rank: int, world: int) -> range:
    """The contiguous block of heads rank ``rank`` of ``world`` computes."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of world {world}")
    if n_heads % world:
        raise ValueError(f"{n_heads} heads do not split over {world} ranks")
    per = n_heads // world
    return range(rank * per, (rank + 1) * per)


def gather_slot(local: torch.Tensor, out: torch.Tensor | None = None, group=None) -> torch.Tensor:
    """Gather the i-th local head of every rank: ``local`` [N, D] -> [world, N, D] (rank-major)."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    if out is None:
        out = torch.empty((world, *local.shape), dtype=local.dtype, device=local.device)
    # the concatenated [world * N, D] form is accepted by every backend (gloo rejects the stacked one)
    dist.all_gather_into_tensor(out.view(world * local.shape[0], *local.shape[1:]), local.contiguous(), group=group)
    return out


def assemble(slots: list[torch.Tensor], n_heads: int) -> torch.Tensor:
    """Gathered slots (``slots[i]`` = [world, N, D], the i-th local head of each rank) -> [n_heads, N, D]
    in head order: head ``r * per + i`` is ``slots[i][r]``."""
    if not slots:
        raise ValueError("no slots")
    world = int(slots[0].shape[0])
    per = len(slots)
    if per * world != n_heads:
        raise ValueError(f"{per} slots x {world} ranks != {n_heads} heads")
    return torch.stack(slots, dim=1).reshape(n_heads, *slots[0].shape[1:])
