"""Data parallelism over views: one process per GPU, views (or whole clips) sharded across ranks.

Every rank holds the full Gaussian set, renders its share of the views and differentiates its
share of the loss; the one exchange is a sum of the per-Gaussian parameter gradients
(``allreduce_gradients``: one flat bucket, NCCL over NVLink on GPUs, gloo on CPU tests).
Per-clip workloads (each clip its own Gaussians) shard whole clips and need no exchange.

The reference is single-process (no torch.distributed anywhere in nbardy/dynaworld); this is the
scaling layer this library adds around its render call.
"""
from __future__ import annotations

import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class Shard:
    rank: int
    world: int
    start: int  # first view of this rank
    stop: int   # one past the last view

    @property
    def count(self) -> int:
        return self.stop - self.start


def shard_views(n_views: int, world: int, rank: int, views_per_set: int = 1, shared_set: bool = True) -> Shard:
    """Contiguous, balanced split of ``n_views`` views.

    With per-set (per-clip) Gaussians (``shared_set=False``) the split is on set boundaries so each
    rank owns whole sets.  Ranks may get zero views when there are fewer units than ranks.
    """
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    unit = 1 if shared_set else max(1, views_per_set)
    if n_views % unit:
        raise ValueError(f"{n_views} views do not divide into sets of {unit}")
    units = n_views // unit
    base, extra = divmod(units, world)
    first = rank * base + min(rank, extra)
    count = base + (1 if rank < extra else 0)
    return Shard(rank, world, first * unit, (first + count) * unit)


def flatten(tensors: list[torch.Tensor]) -> torch.Tensor:
    return torch.cat([t.reshape(-1) for t in tensors]) if tensors else torch.zeros(0)


def unflatten_into(flat: torch.Tensor, tensors: list[torch.Tensor]) -> None:
    off = 0
    for t in tensors:
        n = t.numel()
        t.copy_(flat[off:off + n].view_as(t))
        off += n


def allreduce_gradients(grads: list[torch.Tensor | None], group=None) -> None:
    """Sums the gradients over ranks in place with one all_reduce of a flat fp32 bucket.

    Every rank must pass the same list of shapes in the same order (None entries are skipped on
    every rank alike).  Ranks that rendered no view pass zero gradients.
    """
    live = [g for g in grads if g is not None]
    if not live or not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    flat = flatten([g.float() for g in live])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    unflatten_into(flat, live)


def env_rank_world() -> tuple[int, int, int]:
    """(rank, local_rank, world_size) from torchrun's environment (1 process when unset)."""
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))
