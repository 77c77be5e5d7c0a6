"""Sign-preserving bisection of Marching-Tetrahedra crossing edges
(gofish/mesh/bisection.py:25-128).

Each edge is bracketed by a solid endpoint (O >= 1/2) and a free one.  Each
of ROUNDS rounds evaluates the field at the bracket midpoint through the
bisection table and moves the endpoint of the same sign there; an exact tie
(O == 1/2) collapses the bracket.  Unobserved midpoints count as solid.  The
refined vertex is the final midpoint.  Edges are independent, so batching
does not change any output.
"""

from __future__ import annotations

import numpy as np
import torch

from .cameras import TrainingCamera
from .field import camera_inputs
from .shape import EffectiveShape

ROUNDS = 8
DEVICE_HEADROOM_BYTES = 1536 << 20
MAX_BATCH_EDGES = 1 << 24
BATCH_EDGE_QUANTUM = 1 << 16
BYTES_PER_EDGE = 1024  # conservative device bytes per edge


def batch_size(edge_count: int, free_bytes: int, camera_bytes: int) -> int:
    """All edges in one batch when they fit; otherwise the largest multiple of
    BATCH_EDGE_QUANTUM that fits (bisection.py:31-39)."""
    budget = free_bytes - camera_bytes - DEVICE_HEADROOM_BYTES
    if budget < BYTES_PER_EDGE:
        raise MemoryError("not enough device memory for the bisection camera table")
    fit = budget // BYTES_PER_EDGE
    if fit < edge_count:
        fit = max(BATCH_EDGE_QUANTUM, (fit // BATCH_EDGE_QUANTUM) * BATCH_EDGE_QUANTUM)
    return int(min(edge_count, MAX_BATCH_EDGES, fit))


def _padded_batch(endpoints: np.ndarray, fields: np.ndarray, start: int, end: int, capacity: int):
    """Copy of edges [start, end) padded to ``capacity`` by repeating the last edge."""
    count = end - start
    ends = np.empty((capacity, 2, 3), dtype="<f4")
    vals = np.empty((capacity, 2), dtype="<f4")
    ends[:count] = endpoints[start:end]
    vals[:count] = fields[start:end]
    if count < capacity:
        ends[count:] = ends[count - 1]
        vals[count:] = vals[count - 1]
    return ends, vals


def bracket(ends: torch.Tensor, fields: torch.Tensor):
    """(solid, free) endpoints of crossing edges; raises unless every edge is
    a finite sign crossing of 1/2 - O."""
    f0, f1 = fields[:, 0], fields[:, 1]
    crossing = ((f0 <= 0.0) & (f1 >= 0.0)) | ((f1 <= 0.0) & (f0 >= 0.0))
    if not (bool(torch.isfinite(fields).all().item()) and bool(crossing.all().item())):
        raise ValueError("bisection input edges are not finite sign crossings")
    swap = (f0 > 0.0)[:, None]
    solid = torch.where(swap, ends[:, 1], ends[:, 0]).contiguous()
    free = torch.where(swap, ends[:, 0], ends[:, 1]).contiguous()
    return solid, free


def bisect(raster, token: int, solid: torch.Tensor, free: torch.Tensor) -> torch.Tensor:
    """ROUNDS rounds on one batch; returns the refined midpoints."""
    for round_index in range(ROUNDS):
        mid = torch.add(solid, free).mul_(0.5).contiguous()
        above_u8, observed_u8, exact_u8 = raster.evaluate_bisection_round(token, mid, round_index)
        observed = observed_u8.bool()
        above = above_u8.bool() | ~observed
        exact = exact_u8.bool() & observed
        solid = torch.where(above[:, None], mid, solid).contiguous()
        free = torch.where(((~above) | exact)[:, None], mid, free).contiguous()
    return torch.add(solid, free).mul_(0.5).contiguous()


def refine_crossings(raster, shape: EffectiveShape, cameras: list[TrainingCamera], endpoints: np.ndarray,
                     endpoint_fields: np.ndarray, device: torch.device) -> np.ndarray:
    """Refined vertex [E, 3] float32 of every crossing edge; ``endpoints`` is
    [E, 2, 3] and ``endpoint_fields`` [E, 2] holds 1/2 - O at them."""
    edge_count = int(endpoints.shape[0])
    packed = torch.from_numpy(shape.packed_density()).to(device).contiguous()
    sigma = torch.from_numpy(np.array(shape.sigma_max, dtype=np.float32, order="C", copy=True)).to(device)
    free_bytes, _ = torch.cuda.mem_get_info(device)
    camera_bytes = 0
    for cam in cameras:
        camera_bytes += int(cam.ray_direction.numel()) * 4
        if cam.physical_mask is not None:
            camera_bytes += int(cam.physical_mask.numel()) * int(cam.physical_mask.element_size())
    capacity = batch_size(edge_count, int(free_bytes), camera_bytes)

    vertices = np.empty((edge_count, 3), dtype="<f4")
    token = None
    released = False
    try:
        for start in range(0, edge_count, capacity):
            end = min(edge_count, start + capacity)
            ends_np, vals_np = _padded_batch(endpoints, endpoint_fields, start, end, capacity)
            solid, free = bracket(torch.from_numpy(ends_np).to(device), torch.from_numpy(vals_np).to(device))
            if token is None:
                # The camera table is staged once and reused by every batch.
                probe = torch.add(solid, free).mul_(0.5).contiguous()
                token = raster.begin_bisection_table(packed, sigma.contiguous(), probe)
                for cam in cameras:
                    raster.stage_bisection_camera(token, *camera_inputs(cam, device))
                raster.seal_bisection_table(token)
            refined = bisect(raster, token, solid, free)
            if not bool(torch.isfinite(refined).all().item()):
                raise ValueError("refined vertices are not finite")
            vertices[start:end] = refined[:end - start].cpu().numpy()
            if end < edge_count:
                raster.reset_bisection_batch(token)
        if token is not None:
            raster.release_bisection_table(token)
        released = True
    finally:
        if token is not None and not released:
            try:
                raster.release_bisection_table(token)
            except RuntimeError:
                pass
    return vertices
