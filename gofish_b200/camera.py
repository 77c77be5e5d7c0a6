"""Camera models of the tracer and the calibrated fisheye ray generator.

``fromOpenCVFisheyeCameraModelParameters`` / ``fromOpenCVPinholeCameraModelParameters``
keep the names and argument meaning of the reference's pybind factories
(threedgut_tracer/bindings.cpp:36-79).  ``first_branch_rays`` restates the
reference's Kannala-Brandt inverse on the first monotone branch
(gofish/camera/domain.py:37-113), used to build per-pixel camera rays.
"""

from __future__ import annotations

import dataclasses
import enum
import math
from typing import Iterable, Sequence

import numpy as np

from ._native import GF_CAMERA_OPENCV_FISHEYE, GF_CAMERA_OPENCV_PINHOLE, GfCamera


class ShutterType(enum.IntEnum):
    """cameraModels.h:51-57."""

    ROLLING_TOP_TO_BOTTOM = 0
    ROLLING_LEFT_TO_RIGHT = 1
    ROLLING_BOTTOM_TO_TOP = 2
    ROLLING_RIGHT_TO_LEFT = 3
    GLOBAL = 4


class PolynomialType(enum.IntEnum):
    """FThetaProjectionParameters::PolynomialType (bindings.cpp:133-135)."""

    PIXELDIST_TO_ANGLE = 0
    ANGLE_TO_PIXELDIST = 1


@dataclasses.dataclass(frozen=True)
class CameraModelParameters:
    """Native camera model (the reference's TSensorModel)."""

    model: int
    shutter_type: ShutterType
    resolution: tuple[int, int]
    principal_point: tuple[float, float]
    focal_length: tuple[float, float]
    radial_coeffs: tuple[float, ...]
    tangential_coeffs: tuple[float, float] = (0.0, 0.0)
    thin_prism_coeffs: tuple[float, float, float, float] = (0.0, 0.0, 0.0, 0.0)
    max_angle: float = 0.0

    def native(self, width: int, height: int) -> GfCamera:
        cam = GfCamera()
        cam.model = int(self.model)
        cam.width = int(width)
        cam.height = int(height)
        cam.shutter = int(self.shutter_type)
        cam.principal_point[:] = [float(v) for v in self.principal_point]
        cam.focal_length[:] = [float(v) for v in self.focal_length]
        radial = [float(v) for v in self.radial_coeffs] + [0.0] * (6 - len(self.radial_coeffs))
        cam.radial[:] = radial[:6]
        cam.tangential[:] = [float(v) for v in self.tangential_coeffs]
        cam.thin_prism[:] = [float(v) for v in self.thin_prism_coeffs]
        cam.max_angle = float(np.float32(self.max_angle))
        return cam


def _f32(values: Iterable[float], n: int) -> tuple[float, ...]:
    arr = np.asarray(list(np.asarray(values, dtype=np.float64).reshape(-1)), dtype=np.float32)
    if arr.size != n:
        raise ValueError(f"expected {n} values, got {arr.size}")
    return tuple(float(v) for v in arr)


def fromOpenCVFisheyeCameraModelParameters(resolution, shutter_type, principal_point, focal_length, radial_coeffs,
                                           max_angle) -> CameraModelParameters:
    """bindings.cpp:60-79 (the resolution argument is carried but, as in the
    reference, the raster size of a call comes from its ray tensor)."""
    res = tuple(int(v) for v in np.asarray(resolution).reshape(-1))
    return CameraModelParameters(GF_CAMERA_OPENCV_FISHEYE, ShutterType(int(shutter_type)), res,
                                 _f32(principal_point, 2), _f32(focal_length, 2), _f32(radial_coeffs, 4),
                                 max_angle=float(np.float32(max_angle)))


def fromOpenCVPinholeCameraModelParameters(resolution, shutter_type, principal_point, focal_length, radial_coeffs,
                                           tangential_coeffs, thin_prism_coeffs) -> CameraModelParameters:
    """bindings.cpp:36-58."""
    res = tuple(int(v) for v in np.asarray(resolution).reshape(-1))
    return CameraModelParameters(GF_CAMERA_OPENCV_PINHOLE, ShutterType(int(shutter_type)), res,
                                 _f32(principal_point, 2), _f32(focal_length, 2), _f32(radial_coeffs, 6),
                                 _f32(tangential_coeffs, 2), _f32(thin_prism_coeffs, 4))


# --------------------------------------------------------------------------- Kannala-Brandt domain
def radial_value(theta: float, coefficients: Sequence[float]) -> float:
    """rho(theta) = theta (1 + k1 t^2 + k2 t^4 + k3 t^6 + k4 t^8) (domain.py:37-40)."""
    k1, k2, k3, k4 = (float(v) for v in coefficients)
    y = theta * theta
    return theta * (1.0 + y * (k1 + y * (k2 + y * (k3 + y * k4))))


def radial_derivative(theta: float, coefficients: Sequence[float]) -> float:
    k1, k2, k3, k4 = (float(v) for v in coefficients)
    y = theta * theta
    return 1.0 + y * (3.0 * k1 + y * (5.0 * k2 + y * (7.0 * k3 + y * 9.0 * k4)))


def monotone_branch_limit(coefficients: Sequence[float]) -> float:
    """Open upper limit of the first increasing branch of rho on [0, pi] (domain.py:49-66)."""
    k1, k2, k3, k4 = (float(v) for v in coefficients)
    poly = np.asarray([9.0 * k4, 7.0 * k3, 5.0 * k2, 3.0 * k1, 1.0], dtype=np.float64)
    nonzero = np.flatnonzero(np.abs(poly) > 0.0)
    roots = np.roots(poly[int(nonzero[0]):])
    roots_y = sorted(float(r.real) for r in roots
                     if abs(float(r.imag)) <= 1.0e-10 * max(1.0, abs(float(r.real))) and float(r.real) > 0.0)
    folds = [math.sqrt(v) for v in roots_y if math.sqrt(v) < math.pi]
    limit = math.nextafter(folds[0] if folds else math.pi, 0.0)
    while radial_derivative(limit, (k1, k2, k3, k4)) <= 0.0:
        limit = math.nextafter(limit, 0.0)
    return limit


def first_branch_rays(points: np.ndarray, focal, principal, coefficients, max_angle: float, iterations: int = 48):
    """Unit camera rays of native pixel coordinates ``points`` [M,2] by float64
    bisection of rho on [0, max_angle] (domain.py:78-113).  Points outside the
    branch get the forward ray and ``valid = False``."""
    work = np.asarray(points, dtype=np.float64)
    focal = np.asarray(focal, dtype=np.float64)
    principal = np.asarray(principal, dtype=np.float64)
    normalized = (work - principal) / focal
    distorted = np.linalg.norm(normalized, axis=-1)
    cap = float(max_angle)
    cap_radius = radial_value(cap, coefficients)
    finite = np.isfinite(normalized).all(axis=-1) & np.isfinite(distorted)
    valid = finite & (distorted < cap_radius)
    lo = np.zeros_like(distorted)
    hi = np.full_like(distorted, cap)
    k1, k2, k3, k4 = (float(v) for v in coefficients)
    for _ in range(iterations):
        mid = 0.5 * (lo + hi)
        y = mid * mid
        value = mid * (1.0 + y * (k1 + y * (k2 + y * (k3 + y * k4))))
        move_lo = value < distorted
        lo = np.where(move_lo, mid, lo)
        hi = np.where(move_lo, hi, mid)
    theta = 0.5 * (lo + hi)
    safe = np.where(distorted > 0.0, distorted, 1.0)
    azimuth = normalized / safe[..., None]
    rays = np.concatenate([np.sin(theta)[..., None] * azimuth, np.cos(theta)[..., None]], axis=-1)
    forward = np.zeros_like(rays)
    forward[..., 2] = 1.0
    rays = np.where((distorted == 0.0)[..., None], forward, rays)
    rays = np.where(valid[..., None], rays, forward)
    return rays.astype(np.float32), valid


@dataclasses.dataclass(frozen=True)
class FisheyeCamera:
    """A calibrated OPENCV_FISHEYE camera and its raster."""

    width: int
    height: int
    focal: tuple[float, float]
    principal: tuple[float, float]
    coefficients: tuple[float, float, float, float]
    max_angle: float

    def model(self) -> CameraModelParameters:
        return fromOpenCVFisheyeCameraModelParameters(
            np.array([self.width, self.height], dtype=np.uint64), ShutterType.GLOBAL,
            np.array(self.principal, dtype=np.float32), np.array(self.focal, dtype=np.float32),
            np.array(self.coefficients, dtype=np.float32), self.max_angle)

    def intrinsics(self) -> dict:
        """The batch's ``intrinsics_OpenCVFisheyeCameraModelParameters`` record."""
        return {"resolution": [self.width, self.height], "shutter_type": "GLOBAL",
                "principal_point": list(self.principal), "focal_length": list(self.focal),
                "radial_coeffs": list(self.coefficients), "max_angle": float(self.max_angle)}

    def rays(self):
        """Sensor-frame rays at pixel centres: origins [1,H,W,3] (zero),
        directions [1,H,W,3] and the physical mask [1,H,W,1] (bool)."""
        u = np.arange(self.width, dtype=np.float64) + 0.5
        v = np.arange(self.height, dtype=np.float64) + 0.5
        uu, vv = np.meshgrid(u, v)
        pts = np.stack([uu.reshape(-1), vv.reshape(-1)], axis=1)
        d, valid = first_branch_rays(pts, self.focal, self.principal, self.coefficients, self.max_angle)
        d = d.reshape(1, self.height, self.width, 3)
        o = np.zeros_like(d)
        return o, d, valid.reshape(1, self.height, self.width, 1)


def fisheye_camera(width: int, height: int, fov_deg: float, coefficients=(0.0, 0.0, 0.0, 0.0)) -> FisheyeCamera:
    """Camera whose half field of view fov/2 lands on the inscribed radius
    min(W,H)/2: f = (min(W,H)/2) / rho(fov/2).  Requires the first monotone
    branch of rho to extend past fov/2."""
    half = math.radians(fov_deg) / 2.0
    coeffs = tuple(float(np.float32(c)) for c in coefficients)
    if monotone_branch_limit(coeffs) <= half:
        raise ValueError("distortion polynomial folds before the requested field of view")
    radius = min(width, height) / 2.0
    f = float(np.float32(radius / radial_value(half, coeffs)))
    return FisheyeCamera(int(width), int(height), (f, f), (width / 2.0, height / 2.0), coeffs,
                         float(np.float32(half)))


EQUISOLID_KB4 = (-1.0 / 24.0, 1.0 / 1920.0, -1.0 / 322560.0, 1.0 / 92897280.0)
"""Kannala-Brandt coefficients of the equisolid model r = 2 f sin(theta/2):
the Taylor series of 2 sin(t/2) = t (1 - t^2/24 + t^4/1920 - t^6/322560 + t^8/92897280 ...)."""


def random_kb_coefficients(rng: np.random.Generator, fov_deg: float, spread: float = 0.05):
    """k1..k4 ~ U(-spread, spread), redrawn until the first monotone branch
    extends past fov/2."""
    half = math.radians(fov_deg) / 2.0
    while True:
        k = tuple(float(np.float32(v)) for v in rng.uniform(-spread, spread, size=4))
        if monotone_branch_limit(k) > half:
            return k
