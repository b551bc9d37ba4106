"""Data parallelism over views: one process per GPU, views (or whole clips) sharded across ranks.

Every rank holds the full Gaussian set, renders its share of the views and differentiates its
share of the loss; the one exchange is a sum of the per-Gaussian parameter gradients, NCCL over
NVLink on GPUs (gloo on CPU tests).  The render backward writes every parameter gradient into one
flat buffer (the gradients are views of it), so the sum is an in-place all-reduce of that buffer
with no gather or scatter copies.  ``GradientAllReduce`` launches it from inside the backward,
bucket by bucket as the chain-rule kernel finishes each range of Gaussians, on NCCL's stream;
``allreduce_gradients`` does the same for gradients already computed.  Per-clip workloads (each
clip its own Gaussians) shard whole clips and need no exchange.

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


def shared_span(tensors: list[torch.Tensor]) -> torch.Tensor | None:
    """One flat tensor covering ``tensors`` exactly when they are contiguous, non-overlapping,
    gap-free views of one storage (the render backward's gradient buffer), else None."""
    if not tensors:
        return None
    first = tensors[0]
    storage = first.untyped_storage().data_ptr()
    if any(t.untyped_storage().data_ptr() != storage or t.dtype != first.dtype or not t.is_contiguous()
           for t in tensors):
        return None
    spans = sorted((t.storage_offset(), t.numel()) for t in tensors)
    for (o0, n0), (o1, _n1) in zip(spans, spans[1:]):
        if o0 + n0 != o1:
            return None
    lo = spans[0][0]
    hi = spans[-1][0] + spans[-1][1]
    return torch.empty(0, dtype=first.dtype, device=first.device).set_(first.untyped_storage(), lo, (hi - lo,))


def allreduce_gradients(grads: list[torch.Tensor | None], group=None) -> None:
    """Sums the gradients over ranks in place.

    Gradients from the render backward are views of one flat buffer and are reduced in place with
    one all_reduce of it; other lists go through one flat fp32 copy.  Every rank must pass the same
    list of shapes in the same order (None entries are skipped on every rank alike).  Ranks that
    rendered no view pass zero gradients.
    """
    live = [g for g in grads if g is not None]
    if not live or not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    span = shared_span(live) if all(g.dtype == torch.float32 for g in live) else None
    if span is not None:
        dist.all_reduce(span, op=dist.ReduceOp.SUM, group=group)
        return
    flat = flatten([g.float() for g in live])
    dist.all_reduce(flat, op=dist.ReduceOp.SUM, group=group)
    unflatten_into(flat, live)


class GradientAllReduce:
    """Sums the render backward's parameter gradients over the ranks from inside the backward.

    Installed with ``render.set_gradient_reducer``; the backward then computes the chain rule in
    ``buckets`` ranges of Gaussians and hands each range's gradient rows to ``reduce`` as soon as
    its kernel is queued, so the all-reduce of one range overlaps the chain rule of the next.
    ``finish`` makes the current stream wait for every bucket (no host wait).  Only for scenes whose
    one Gaussian set every rank shares (per-clip sets need no exchange).
    """

    def __init__(self, group=None, buckets: int = 4):
        self.group = group
        self.buckets = max(1, int(buckets))
        self._works: list = []

    def active(self) -> bool:
        return dist.is_available() and dist.is_initialized() and dist.get_world_size(self.group) > 1

    def reduce(self, views: list[torch.Tensor]) -> None:
        for v in views:
            if v.numel():
                self._works.append(dist.all_reduce(v, op=dist.ReduceOp.SUM, group=self.group, async_op=True))

    def finish(self) -> None:
        works, self._works = self._works, []
        for w in works:
            w.wait()


def env_rank_world() -> tuple[int, int, int]:
    """(rank, local_rank, world_size) from torchrun's environment (1 process when unset)."""
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))
