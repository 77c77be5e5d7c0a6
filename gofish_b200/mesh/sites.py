# Portions derived from GOF (https://github.com/autonomousvision/gaussian-opacity-fields)
# by way of tuallen/GOFish, distributed under the Gaussian-Splatting License (Inria / MPII;
# non-commercial research and evaluation use).

"""Tetrahedralization sites: each retained Gaussian's centre and the eight
corners of its support box (gofish/mesh/sites.py:43-83).

For B = R S' and the opacity-adaptive support radius r, the support
ellipsoid is mu + B u with |u| <= r; its oriented box has corners
mu + B (r s) for s in {-1, +1}^3, listed x-major then y then z.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np

from .shape import DEAD_OPACITY, EffectiveShape

SIGNS = np.array([[x, y, z] for x in (-1.0, 1.0) for y in (-1.0, 1.0) for z in (-1.0, 1.0)], dtype=np.float64)
# The renderer's minimum kernel response (float32) and the radius it implies.
KERNEL_MIN_RESPONSE = float(np.float32(0.0113))
RADIUS_CAP = math.sqrt(-2.0 * math.log(KERNEL_MIN_RESPONSE))
SITES_PER_GAUSSIAN = 9


@dataclass
class Sites:
    points: np.ndarray  # [M, 3] float32
    scale: np.ndarray  # [M, 1] float32, owner's sigma_max * r
    owner: np.ndarray  # [M] int64

    @property
    def count(self) -> int:
        return int(self.points.shape[0])


def support_radius(opacity: np.ndarray) -> np.ndarray:
    """min(RADIUS_CAP, sqrt(2 ln(255 o))) in float64; opacities must exceed 1/255."""
    o = np.asarray(opacity, dtype=np.float64).reshape(-1)
    if not (np.isfinite(o).all() and np.all(o > DEAD_OPACITY)):
        raise ValueError("site opacities must be finite and above 1/255")
    r = np.minimum(RADIUS_CAP, np.sqrt(2.0 * np.log(255.0 * o)))
    if not (np.isfinite(r).all() and np.all(r > 0.0)):
        raise ValueError("support radius is not finite and positive")
    return r


def support_box_sites(positions: np.ndarray, factor: np.ndarray, radius: np.ndarray) -> np.ndarray:
    """[N, 9, 3] float64: the centre, then the eight corners in SIGNS order."""
    mu = np.asarray(positions, dtype=np.float64)
    B = np.asarray(factor, dtype=np.float64)
    r = np.asarray(radius, dtype=np.float64).reshape(-1)
    offsets = r[:, None, None] * SIGNS[None, :, :]               # [N, 8, 3] in the canonical frame
    corners = mu[:, None, :] + np.einsum("nij,nkj->nki", B, offsets, optimize=False)
    return np.concatenate((mu[:, None, :], corners), axis=1)


def generate_sites(shape: EffectiveShape) -> Sites:
    opacity = np.asarray(shape.density[:, 0], dtype=np.float64)
    if not np.array_equal(shape.retained, opacity > DEAD_OPACITY):
        raise ValueError("retained Gaussians differ from opacity > 1/255")
    keep = np.flatnonzero(shape.retained)
    if keep.size == 0:
        raise ValueError("no Gaussian has opacity above 1/255")
    r = support_radius(opacity[keep])
    pts = support_box_sites(shape.positions[keep].astype("<f4"), shape.factor[keep].astype("<f4"), r).astype("<f4")
    scale = np.asarray(shape.sigma_max[keep, 0], dtype=np.float64) * r
    return Sites(points=np.ascontiguousarray(pts.reshape(-1, 3)),
                 scale=np.repeat(scale.astype("<f4"), SITES_PER_GAUSSIAN).reshape(-1, 1),
                 owner=np.repeat(keep.astype("<i8"), SITES_PER_GAUSSIAN))


def generate_sites_cuda(shape: EffectiveShape, device) -> Sites:
    """generate_sites on the GPU (gf_mesh_sites): the same sites, scales and
    owners, as CUDA tensors on ``device``.  ``shape`` may hold numpy arrays
    or tensors; one host read of the kept count sizes the outputs."""
    import ctypes

    import torch

    from .. import _native

    def dev(a, shape_):
        t = a if isinstance(a, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(a))
        return t.to(device=device, dtype=torch.float32).reshape(shape_).contiguous()

    n = int(shape.positions.shape[0])
    positions = dev(shape.positions, (n, 3))
    factor = dev(shape.factor, (n, 9))
    density = dev(shape.density, (n,))
    sigma = dev(shape.sigma_max, (n,))
    points = torch.empty((9 * n, 3), dtype=torch.float32, device=device)
    scale = torch.empty((9 * n,), dtype=torch.float32, device=device)
    owner = torch.empty((9 * n,), dtype=torch.int64, device=device)
    count = torch.zeros(1, dtype=torch.int32, device=device)
    status = torch.zeros(1, dtype=torch.int32, device=device)
    with torch.cuda.device(device):
        stream = torch.cuda.current_stream(device).cuda_stream
        _native.check(_native.load().gf_mesh_sites(positions.data_ptr(), factor.data_ptr(), density.data_ptr(),
                                                   sigma.data_ptr(), ctypes.c_uint32(n), points.data_ptr(),
                                                   scale.data_ptr(), owner.data_ptr(), count.data_ptr(),
                                                   status.data_ptr(), stream), "mesh sites")
    kept = int(count.item())
    if int(status.item()) != 0:
        raise ValueError("support radius is not finite and positive")
    if kept == 0:
        raise ValueError("no Gaussian has opacity above 1/255")
    m = SITES_PER_GAUSSIAN * kept
    return Sites(points=points[:m], scale=scale[:m].reshape(m, 1), owner=owner[:m])
