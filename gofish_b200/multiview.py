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
    its view; autograd then accumulates the step's gradients in place.

    ``early`` names parameters whose gradient is complete before the others
    in the step's last backward (the SH gradient of the tracer comes out of
    the render backward, before the full-shape VJP that produces the
    position, rotation, scale and opacity gradients).  They sit at the end
    of the buffer.  After ``arm()``, called before the last backward of a
    step, the accumulation of the last of them starts an asynchronous
    all-reduce of that tail, which overlaps the rest of the backward;
    ``allreduce()`` then reduces the head and orders the stream after both.
    Every rank must arm before the same backward.  An early parameter must
    receive exactly one gradient in the armed backward (one producer): the
    all-reduce starts at its first accumulation, so a second contribution
    would arrive after the reduction had read the buffer, and raises.  For the tracer
    the SH coefficients and the positions qualify: both come only out of the
    render's backward (the per-view footprint reads the positions detached)."""

    def __init__(self, params: Sequence[torch.Tensor], early: Sequence[torch.Tensor] = ()):
        params = list(params)
        if not params:
            raise ValueError("no parameters")
        early_ids = {id(p) for p in early}
        if not early_ids <= {id(p) for p in params}:
            raise ValueError("early parameters must be among the bucket's parameters")
        late = [p for p in params if id(p) not in early_ids]
        tail = [p for p in params if id(p) in early_ids]
        self.params = params
        first = params[0]
        self.head_numel = sum(p.numel() for p in late)
        self.flat = torch.zeros(self.head_numel + sum(p.numel() for p in tail), dtype=first.dtype,
                                device=first.device)
        view_of = {}
        offset = 0
        for p in late + tail:
            view_of[id(p)] = self.flat[offset:offset + p.numel()].view(p.shape)
            offset += p.numel()
        self.views = [view_of[id(p)] for p in params]
        self._early = tail
        self._pending: set[int] = set()
        self._armed = False
        self._group = None
        self._work = None
        self._hooks = [p.register_post_accumulate_grad_hook(self._on_accumulated) for p in tail]

    def attach(self) -> None:
        self.flat.zero_()
        for p, v in zip(self.params, self.views):
            p.grad = v

    def arm(self, group=None) -> None:
        """The next backward is the step's last: start the tail's all-reduce
        as soon as its gradients are accumulated."""
        if not self._early or not _distributed(group):
            return
        self._armed = True
        self._group = group
        self._pending = {id(p) for p in self._early}

    def _on_accumulated(self, param: torch.Tensor) -> None:
        if not self._armed:
            return
        if self._work is not None:
            raise RuntimeError("an early parameter received another gradient after its all-reduce started: early "
                               "parameters must have one gradient producer in the armed backward")
        self._pending.discard(id(param))
        if not self._pending and self._work is None:
            self._work = dist.all_reduce(self.flat[self.head_numel:], op=dist.ReduceOp.SUM, group=self._group,
                                         async_op=True)

    def allreduce(self, group=None) -> None:
        """Sums the bucket over the ranks (no-op on one rank)."""
        for p, v in zip(self.params, self.views):
            if p.grad is not v:
                raise RuntimeError("a gradient left its bucket view; call attach() before backward")
        work, self._work, self._armed = self._work, None, False
        if work is None:
            allreduce_gradients([self.flat], group)
            return
        if self.head_numel > 0:
            dist.all_reduce(self.flat[:self.head_numel], op=dist.ReduceOp.SUM, group=group)
        work.wait()


def _distributed(group=None) -> bool:
    return dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1


def allreduce_gradients(grads: Sequence[torch.Tensor], group=None) -> None:
    """Sums each gradient tensor over the ranks in place (one collective per tensor)."""
    if not _distributed(group):
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
