"""One camera frame as the renderers take it, and its native camera model and
sensor poses.

``Batch`` carries the fields of the reference's training/inference batch that
the tracer reads (``rays_ori``/``rays_dir`` [1,H,W,3] camera-space rays,
``T_to_world`` [1,4,4] camera-to-world pose, one intrinsics dictionary, the
optional physical field-of-view mask).  ``create_camera_parameters`` restates
the reference's ``Tracer.__create_camera_parameters`` and
``__create_sensor_pose_from_R_T`` (threedgut_tracer/tracer.py:536-672): the
world-to-camera pose is the float64 inverse of the 4x4 camera-to-world matrix,
sent to the renderer as [t, quaternion (x, y, z, w)] in float32 with the end
pose equal to the start pose for a global shutter.
"""

from __future__ import annotations

import dataclasses
import math
from typing import Any, NamedTuple, Optional

import numpy as np

from .camera import (CameraModelParameters, ShutterType, fromOpenCVFisheyeCameraModelParameters,
                     fromOpenCVPinholeCameraModelParameters)


@dataclasses.dataclass
class Batch:
    """One frame: camera-space rays, camera-to-world pose and intrinsics."""

    rays_ori: Any                       # [1,H,W,3] float32
    rays_dir: Any                       # [1,H,W,3] float32
    T_to_world: Any                     # [1,4,4] camera-to-world
    intrinsics_OpenCVFisheyeCameraModelParameters: Optional[dict] = None
    intrinsics_OpenCVPinholeCameraModelParameters: Optional[dict] = None
    intrinsics: Optional[Any] = None    # [fx, fy, cx, cy] ideal pinhole
    T_to_world_end: Optional[Any] = None
    physical_fov_mask: Optional[Any] = None   # [1,H,W,1] bool
    physical_fov_key: Optional[str] = None
    rays_in_world_space: bool = False


class SensorPose3D(NamedTuple):
    """World-to-sensor poses [t(3), q(x, y, z, w)] at the start and end of the
    exposure, with their relative timestamps."""

    T_world_sensors: list
    timestamps_us: list


def so3_to_quaternion_xyzw(R: np.ndarray) -> np.ndarray:
    """Unit quaternion (x, y, z, w) of a rotation matrix (Shepperd's method:
    the largest of w, x, y, z is taken from the trace or a diagonal entry, the
    others from the off-diagonal sums and differences).  q and -q give the same
    rotation, and the renderer's rotation matrix is even in q."""
    m = np.asarray(R, dtype=np.float64)
    tr = m[0, 0] + m[1, 1] + m[2, 2]
    if tr > 0.0:
        s = math.sqrt(tr + 1.0) * 2.0
        w, x, y, z = 0.25 * s, (m[2, 1] - m[1, 2]) / s, (m[0, 2] - m[2, 0]) / s, (m[1, 0] - m[0, 1]) / s
    elif m[0, 0] > m[1, 1] and m[0, 0] > m[2, 2]:
        s = math.sqrt(1.0 + m[0, 0] - m[1, 1] - m[2, 2]) * 2.0
        w, x, y, z = (m[2, 1] - m[1, 2]) / s, 0.25 * s, (m[0, 1] + m[1, 0]) / s, (m[0, 2] + m[2, 0]) / s
    elif m[1, 1] > m[2, 2]:
        s = math.sqrt(1.0 + m[1, 1] - m[0, 0] - m[2, 2]) * 2.0
        w, x, y, z = (m[0, 2] - m[2, 0]) / s, (m[0, 1] + m[1, 0]) / s, 0.25 * s, (m[1, 2] + m[2, 1]) / s
    else:
        s = math.sqrt(1.0 + m[2, 2] - m[0, 0] - m[1, 1]) * 2.0
        w, x, y, z = (m[1, 0] - m[0, 1]) / s, (m[0, 2] + m[2, 0]) / s, (m[1, 2] + m[2, 1]) / s, 0.25 * s
    q = np.array([x, y, z, w], dtype=np.float64)
    return q / np.linalg.norm(q)


def _world_to_camera(pose) -> tuple[np.ndarray, np.ndarray]:
    """(R, t) of the inverse of a camera-to-world pose (tracer.py:596-602)."""
    c2w = np.zeros((4, 4), dtype=np.float64)
    c2w[:3, :4] = np.asarray(pose.detach().cpu().numpy() if hasattr(pose, "detach") else pose,
                             dtype=np.float64).reshape(-1, 4)[:3, :4]
    c2w[3, 3] = 1.0
    w2c = np.linalg.inv(c2w)
    return w2c[:3, :3], w2c[:3, 3]


def _pose7(R: np.ndarray, t: np.ndarray) -> np.ndarray:
    return np.concatenate([np.asarray(t, dtype=np.float32),
                           so3_to_quaternion_xyzw(R.astype(np.float32).astype(np.float64)).astype(np.float32)])


def _shutter(K: dict) -> ShutterType:
    name = K.get("shutter_type", "GLOBAL")
    return ShutterType[name] if isinstance(name, str) else ShutterType(int(name))


def create_camera_parameters(gpu_batch) -> tuple[CameraModelParameters, SensorPose3D]:
    """Native camera model and sensor poses of ``gpu_batch`` (tracer.py:562-672)."""
    if getattr(gpu_batch, "rays_in_world_space", False):
        R_start = R_end = np.eye(3)
        T_start = T_end = np.zeros(3)
    else:
        start = gpu_batch.T_to_world
        start = start.reshape(-1, 4, 4)[0] if hasattr(start, "reshape") else np.asarray(start).reshape(-1, 4, 4)[0]
        R_start, T_start = _world_to_camera(start)
        end = getattr(gpu_batch, "T_to_world_end", None)
        if end is None:
            R_end, T_end = R_start, T_start
        else:
            end = end.reshape(-1, 4, 4)[0] if hasattr(end, "reshape") else np.asarray(end).reshape(-1, 4, 4)[0]
            R_end, T_end = _world_to_camera(end)
    p0 = _pose7(R_start, T_start)
    p1 = p0 if (R_end is R_start and T_end is T_start) else _pose7(R_end, T_end)
    poses = SensorPose3D([p0, p1], [0, 1])

    if (K := getattr(gpu_batch, "intrinsics", None)) is not None:
        fx, fy, cx, cy = (float(v) for v in K[:4])
        w, h = int(2 * cx), int(2 * cy)
        fov_x, fov_y = 2.0 * math.atan(w / (2.0 * fx)), 2.0 * math.atan(h / (2.0 * fy))
        cam = fromOpenCVPinholeCameraModelParameters(
            np.array([w, h], dtype=np.uint32), ShutterType.GLOBAL, np.array([w, h], dtype=np.float32) / 2,
            np.array([w / (2.0 * math.tan(fov_x * 0.5)), h / (2.0 * math.tan(fov_y * 0.5))], dtype=np.float32),
            np.zeros(6, np.float32), np.zeros(2, np.float32), np.zeros(4, np.float32))
        return cam, poses
    if (K := getattr(gpu_batch, "intrinsics_OpenCVPinholeCameraModelParameters", None)) is not None:
        cam = fromOpenCVPinholeCameraModelParameters(
            K["resolution"], _shutter(K), K["principal_point"], K["focal_length"], K["radial_coeffs"],
            K["tangential_coeffs"], K.get("thin_prism_coeffs", np.zeros(4, np.float32)))
        return cam, poses
    if (K := getattr(gpu_batch, "intrinsics_OpenCVFisheyeCameraModelParameters", None)) is not None:
        cam = fromOpenCVFisheyeCameraModelParameters(K["resolution"], _shutter(K), K["principal_point"],
                                                     K["focal_length"], K["radial_coeffs"], K["max_angle"])
        return cam, poses
    raise ValueError("camera intrinsics unavailable or unsupported (OPENCV_FISHEYE and pinhole are rendered)")


__all__ = ["Batch", "SensorPose3D", "create_camera_parameters", "so3_to_quaternion_xyzw"]
