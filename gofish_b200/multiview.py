"""Data-parallel multi-view training step over ranks (one process per GPU).

Views of one scene are independent: each rank renders its own share of the
views against a replicated copy of the Gaussians, accumulates the
per-Gaussian gradients of its views, and one all-reduce (sum) per step gives
every rank the gradient of the whole batch.  No other exchange is needed.
The reference is single-GPU (no torch.distributed anywhere); this module is
the multi-GPU layer its training loop would call.
"""

from __future__ import annotations

from typing import Callable, Sequence

import torch
import torch.distributed as dist


def shard_views(num_views: int, rank: int, world: int) -> list[int]:
    """Views of this rank: round-robin, so every rank gets floor or ceil of num_views / world."""
    if world <= 0 or not (0 <= rank < world):
        raise ValueError("invalid rank/world")
    return list(range(rank, num_views, world))


class GradientBucket:
    """The gradients of ``params`` as views into one flat buffer, so that a
    training step's all-reduce is a single collective over every parameter
    (for a Gaussian scene: positions, rotations, scales, opacities and SH,
    59 floats per Gaussian at SH degree 3).

    ``attach()`` zeroes the buffer and sets each parameter's ``.grad`` to
    its view; autograd then accumulates the step's gradients in place."""

    def __init__(self, params: Sequence[torch.Tensor]):
        self.params = list(params)
        if not self.params:
            raise ValueError("no parameters")
        sizes = [p.numel() for p in self.params]
        first = self.params[0]
        self.flat = torch.zeros(sum(sizes), dtype=first.dtype, device=first.device)
        self.views = []
        offset = 0
        for p, n in zip(self.params, sizes):
            self.views.append(self.flat[offset:offset + n].view(p.shape))
            offset += n

    def attach(self) -> None:
        self.flat.zero_()
        for p, v in zip(self.params, self.views):
            p.grad = v

    def allreduce(self, group=None) -> None:
        """Sums the bucket over the ranks (no-op on one rank)."""
        for p, v in zip(self.params, self.views):
            if p.grad is not v:
                raise RuntimeError("a gradient left its bucket view; call attach() before backward")
        allreduce_gradients([self.flat], group)


def allreduce_gradients(grads: Sequence[torch.Tensor], group=None) -> None:
    """Sums each gradient tensor over the ranks in place (one collective per tensor)."""
    if not dist.is_available() or not dist.is_initialized() or dist.get_world_size(group) == 1:
        return
    for g in grads:
        dist.all_reduce(g, op=dist.ReduceOp.SUM, group=group)


def multiview_step(render_view: Callable[[int], Sequence[torch.Tensor]], views: Sequence[int],
                   accum: Sequence[torch.Tensor], group=None) -> None:
    """Runs ``render_view(v)`` (forward + loss + backward of view v, returning
    its gradient tensors) for this rank's views, sums the gradients into
    ``accum`` (zeroed first) and all-reduces them over the ranks."""
    for a in accum:
        a.zero_()
    for v in views:
        grads = render_view(v)
        for a, g in zip(accum, grads):
            a.add_(g)
    allreduce_gradients(accum, group)
