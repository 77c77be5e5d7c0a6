"""Calibrated Mip filtering, per-view part: the pixel footprint
(threedgut_tracer/view_observation_filter.py:1-381).

For one render the pixel variance gamma is pulled back through the active
camera as the minimum-norm 3-D covariance Q_v = gamma J^+ J^+^T (so that
J Q_v J^T = gamma I); the renderer draws Sigma + Q_v with the
mass-preserving opacity factor m = sqrt(det S0 / det(S0 + gamma I)),
S0 = J Sigma J^T.  Q_v, J and the observed flags come from one sm_100a kernel
(gf_view_q6) in float64, with J rounded to float32 as the full-shape
operator receives it.
"""

from __future__ import annotations

import math
from typing import Any

import torch

from . import _native
from ._native import GfShapeCamera

FILTER_VARIANCE_PIXELS = 0.3


def _select(conf, path: str, default):
    node = conf
    for part in path.split("."):
        if node is None:
            return default
        node = node.get(part) if isinstance(node, dict) else getattr(node, part, None)
    return default if node is None else node


def pixel_footprint_variance(conf) -> float:
    """gamma of ``conf`` (0 when render.gofish.scene_sensor_factorization is off)."""
    if not bool(_select(conf, "render.gofish.scene_sensor_factorization", True)):
        return 0.0
    gamma = float(_select(conf, "render.gofish.pixel_footprint_variance", FILTER_VARIANCE_PIXELS))
    if not (math.isfinite(gamma) and gamma >= 0.0):
        raise ValueError("render.gofish.pixel_footprint_variance must be finite and >= 0")
    return gamma


def footprint_covariance(jacobian: torch.Tensor, pixel_variance: float = FILTER_VARIANCE_PIXELS) -> torch.Tensor:
    """Q_v = gamma J^+ J^+^T in float64 for full-rank Jacobians [N,2,3]."""
    pinv = torch.linalg.pinv(jacobian.detach().to(torch.float64))
    return float(pixel_variance) * pinv @ pinv.transpose(1, 2)


def mass_preserving_factor(covariance: torch.Tensor, jacobian: torch.Tensor,
                           pixel_variance: float = FILTER_VARIANCE_PIXELS) -> torch.Tensor:
    """m = sqrt(det S0 / det(S0 + gamma I)), S0 = J Sigma J^T, float64 [N]."""
    j = jacobian.detach().to(torch.float64)
    s0 = j @ covariance.detach().to(torch.float64) @ j.transpose(1, 2)
    eye = torch.eye(2, dtype=torch.float64, device=s0.device)
    return torch.sqrt(torch.linalg.det(s0) / torch.linalg.det(s0 + float(pixel_variance) * eye))


def shape_camera(gpu_batch: Any) -> GfShapeCamera:
    """The active camera of a batch (one camera-to-world pose, global shutter,
    OPENCV_FISHEYE or ideal pinhole), as the C ABI takes it."""
    if getattr(gpu_batch, "rays_in_world_space", False):
        raise RuntimeError("view observation filter requires camera-space rays")
    poses = getattr(gpu_batch, "T_to_world", None)
    if not torch.is_tensor(poses) or tuple(poses.shape) != (1, 4, 4):
        raise RuntimeError("view observation filter requires exactly one active pose")
    end = getattr(gpu_batch, "T_to_world_end", None)
    if end is not None and not torch.equal(poses, end):
        raise RuntimeError("view observation filter is scoped to global shutter")
    cam = GfShapeCamera()
    cam.c2w[:] = [float(v) for v in poses[0].detach().float().reshape(-1).cpu().tolist()]
    fish = getattr(gpu_batch, "intrinsics_OpenCVFisheyeCameraModelParameters", None)
    if fish is not None:
        cam.fisheye = 1
        cam.focal_length[:] = [float(v) for v in torch.as_tensor(fish["focal_length"]).reshape(-1)[:2]]
        cam.radial[:] = [float(v) for v in torch.as_tensor(fish["radial_coeffs"]).reshape(-1)[:4]]
        cam.max_angle = float(torch.as_tensor(fish["max_angle"]).reshape(-1)[0])
        return cam
    pin = getattr(gpu_batch, "intrinsics_OpenCVPinholeCameraModelParameters", None)
    if pin is None:
        raise RuntimeError("view observation filter supports OPENCV_FISHEYE and ideal pinhole")
    focal = [float(v) for v in torch.as_tensor(pin["focal_length"]).reshape(-1)]
    if len(focal) not in (1, 2):
        raise RuntimeError("ideal pinhole focal_length must contain one or two values")
    for name in ("radial_coeffs", "tangential_coeffs", "thin_prism_coeffs"):
        if name not in pin:
            raise RuntimeError(f"ideal pinhole Q requires explicit zero {name}; distorted OPENCV is unsupported")
        values = torch.as_tensor(pin[name]).reshape(-1)
        if not bool(torch.isfinite(values).all()) or bool(torch.count_nonzero(values)):
            raise RuntimeError("view observation filter does not approximate distorted OPENCV with an "
                               "ideal-pinhole Jacobian")
    cam.fisheye = 0
    cam.focal_length[:] = [focal[0], focal[-1]]
    cam.max_angle = math.pi
    return cam


@torch.no_grad()
def current_view_q6(positions: torch.Tensor, gpu_batch: Any, pixel_variance: float = FILTER_VARIANCE_PIXELS, *,
                    host_sync_free: bool = False):
    """(q6 float64 [N,6], jacobian float32 [N,2,3], observed bool [N]) of the
    active view (view_observation_filter.py:232-330)."""
    if positions.ndim != 2 or positions.shape[1] != 3:
        raise RuntimeError("positions must be [N,3]")
    cam = shape_camera(gpu_batch)
    pos = positions.detach().float().contiguous()
    n = pos.shape[0]
    q6 = torch.empty((n, 6), dtype=torch.float64, device=pos.device)
    jac = torch.empty((n, 2, 3), dtype=torch.float32, device=pos.device)
    obs = torch.empty(n, dtype=torch.uint8, device=pos.device)
    lib = _native.load()
    import ctypes
    _native.check(lib.gf_view_q6(pos.data_ptr(), n, ctypes.byref(cam), float(pixel_variance), q6.data_ptr(),
                                 jac.data_ptr(), obs.data_ptr(), torch.cuda.current_stream(pos.device).cuda_stream),
                  "current_view_q6")
    return q6, jac, obs.bool()


def build_intrinsic_view_shape(scales, quaternion, density, positions, gpu_batch, *,
                               pixel_footprint_variance: float = FILTER_VARIANCE_PIXELS, frame_id=None,
                               defer_check: bool = False):
    """C = Sigma + Q_v, its factors and the m-compensated density of one view
    (``defer_check``: see build_full_shape)."""
    from .footprint_shape_operator import build_full_shape

    del frame_id
    q6, jacobian, observed = current_view_q6(positions, gpu_batch, pixel_footprint_variance)
    return build_full_shape(scales, quaternion, density, q6, jacobian, observed, mass_preserving=True,
                            pixel_variance=pixel_footprint_variance, defer_check=defer_check)


__all__ = ["FILTER_VARIANCE_PIXELS", "footprint_covariance", "mass_preserving_factor", "build_intrinsic_view_shape",
           "current_view_q6", "pixel_footprint_variance", "shape_camera"]
