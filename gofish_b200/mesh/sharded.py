"""The mesh opacity query sharded over the ranks of one node.

Query points (and bisection edges) are independent, so each rank evaluates a
contiguous slice of them with the Gaussians and cameras replicated, and one
all-gather at the end assembles the [Q] results on every rank: the only
exchange of the sharded query.  With the NCCL backend the gather runs on the
GPU over NVLink; with gloo (CPU tests) on host tensors.

``shard_bounds`` and ``gather_shards`` are the pieces the sharded entry points
share; ``evaluate_field_sharded`` and ``refine_crossings_sharded`` wrap the
single-rank ``evaluate_field`` and ``refine_crossings``.
"""

from __future__ import annotations

import numpy as np
import torch
import torch.distributed as dist


def shard_bounds(total: int, rank: int, world: int) -> tuple[int, int]:
    """[lo, hi) of rank's contiguous slice of ``total`` units (sizes differ by at most one)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    return total * rank // world, total * (rank + 1) // world


def _group_info(group) -> tuple[int, int, torch.device]:
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if dist.get_backend(group) == "nccl":
        device = torch.device("cuda", torch.cuda.current_device())
    else:
        device = torch.device("cpu")
    return rank, world, device


def gather_shards_tensor(local: torch.Tensor, total: int, group=None) -> torch.Tensor:
    """The full [total, ...] tensor on every rank, from each rank's
    contiguous slice ``local`` (rank order; slices as shard_bounds cuts
    them), without leaving the device: slices are padded to the longest one
    for the all-gather (as bytes per row, so any dtype gathers exactly) and
    trimmed after.  ``local`` must be on the backend's device (CUDA for
    NCCL, CPU for gloo)."""
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    lo, hi = shard_bounds(total, rank, world)
    if local.shape[0] != hi - lo:
        raise ValueError(f"rank {rank} holds {local.shape[0]} rows, its shard has {hi - lo}")
    longest = max(shard_bounds(total, r, world)[1] - shard_bounds(total, r, world)[0] for r in range(world))
    row_shape = tuple(local.shape[1:])
    row_bytes = local.element_size() * int(np.prod(row_shape, dtype=np.int64))
    padded = torch.zeros((longest, row_bytes), dtype=torch.uint8, device=local.device)
    if local.shape[0]:
        padded[: local.shape[0]] = local.contiguous().view(torch.uint8).reshape(local.shape[0], row_bytes)
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    rows = [parts[r][: shard_bounds(total, r, world)[1] - shard_bounds(total, r, world)[0]] for r in range(world)]
    full = torch.cat(rows, dim=0).contiguous()
    return full.view(local.dtype).reshape((total,) + row_shape)


def gather_shards(local: np.ndarray, total: int, group=None) -> np.ndarray:
    """gather_shards_tensor for host arrays: the full [total, ...] array on every rank."""
    _rank, _world, device = _group_info(group)
    local = np.ascontiguousarray(local)
    full = gather_shards_tensor(torch.from_numpy(local).to(device), total, group)
    return np.ascontiguousarray(full.cpu().numpy())


def evaluate_field_sharded(raster, shape, cameras, points: np.ndarray, device, group=None):
    """evaluate_field over this rank's slice of ``points``, gathered: every
    rank returns (minimum opacity [Q] float32, observed [Q] uint8) for all Q
    points, identical to a single-rank evaluate_field."""
    from .field import evaluate_field

    rank, world, _ = _group_info(group)
    q = int(np.asarray(points).reshape(-1, 3).shape[0])
    lo, hi = shard_bounds(q, rank, world)
    minimum, observed = evaluate_field(raster, shape, cameras, np.asarray(points).reshape(-1, 3)[lo:hi], device)
    return gather_shards(minimum, q, group), gather_shards(observed, q, group)


def refine_crossings_sharded(raster, shape, cameras, endpoints: np.ndarray, fields: np.ndarray, device, group=None):
    """refine_crossings over this rank's slice of the edges, gathered: every
    rank returns the [E,3] refined vertices of all edges."""
    from .bisection import refine_crossings

    rank, world, _ = _group_info(group)
    e = int(np.asarray(endpoints).shape[0])
    lo, hi = shard_bounds(e, rank, world)
    vertices = refine_crossings(raster, shape, cameras, np.asarray(endpoints)[lo:hi], np.asarray(fields)[lo:hi],
                                device)
    return gather_shards(np.asarray(vertices, dtype=np.float32).reshape(hi - lo, 3), e, group)
