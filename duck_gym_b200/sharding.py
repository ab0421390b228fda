"""Environment sharding across ranks (one process per GPU).

Environments are independent, so a multi-GPU run needs no physics
communication: each rank owns a contiguous slice of the environments, with its
own batch on its own device, and per-rank seeds so that the ranks draw
different inputs.  The only collectives are the timing barrier and the
max-over-ranks reduction of the measured time.
"""

from __future__ import annotations

from dataclasses import dataclass


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    first: int     # first global environment index owned by this rank
    count: int     # environments owned by this rank

    @property
    def stop(self):
        return self.first + self.count


def shard(total: int, rank: int, world: int) -> Shard:
    """Contiguous slice of `total` environments for `rank` of `world`
    (strong scaling: sizes differ by at most one)."""
    if world < 1 or not 0 <= rank < world or total < world:
        raise ValueError("need 0 <= rank < world <= total")
    base, extra = divmod(total, world)
    first = rank * base + min(rank, extra)
    return Shard(rank, world, first, base + (1 if rank < extra else 0))


def weak_shard(per_rank: int, rank: int, world: int) -> Shard:
    """Weak scaling: every rank owns `per_rank` environments."""
    return Shard(rank, world, rank * per_rank, per_rank)


def rank_seed(seed: int, rank: int) -> int:
    """Seed of a rank's input draws (distinct per rank, reproducible)."""
    return seed + 1000 * rank


def max_over_ranks(value: float, device=None) -> float:
    """Max of a float over all ranks of the default process group (the value
    itself when no group is initialised)."""
    import torch
    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()) or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
