"""Training cameras as the opacity field consumes them
(gofish/mesh/cameras.py:39-52: frame number, one ray origin, calibrated ray
directions, physical-domain mask, sensor model and start/end poses).  The
reference builds them from a checkpoint's dataset; ``fisheye_training_camera``
builds one from a calibrated fisheye camera and a pose."""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

from ..camera import FisheyeCamera


@dataclass
class SensorPose3D:
    T_world_sensors: list  # two world->sensor [t, q(x,y,z,w)] float32 tensors [7] (start, end)
    timestamps_us: list


@dataclass
class TrainingCamera:
    frame_number: int
    ray_origin: torch.Tensor  # [3] float32
    ray_direction: torch.Tensor  # [1, H, W, 3] float32
    physical_mask: torch.Tensor | None  # [H, W] uint8 or None
    sensor: object  # CameraModelParameters
    poses: SensorPose3D


def fisheye_training_camera(frame_number: int, camera: FisheyeCamera, pose7, masked: bool = True,
                            timestamp_us: int = 0, rays=None) -> TrainingCamera:
    """Global-shutter camera at ``pose7`` with its first-branch rays and, when
    ``masked``, the physical mask of pixels whose ray lies inside max_angle.
    ``rays`` (the ``camera.rays()`` triple) lets views of one camera share a
    ray table computed once."""
    _origin, direction, valid = camera.rays() if rays is None else rays
    pose = torch.as_tensor(np.asarray(pose7, dtype=np.float32).reshape(7))
    mask = torch.from_numpy(valid.reshape(camera.height, camera.width).astype(np.uint8)) if masked else None
    return TrainingCamera(
        frame_number=int(frame_number),
        ray_origin=torch.zeros(3, dtype=torch.float32),
        ray_direction=torch.from_numpy(np.ascontiguousarray(direction, dtype=np.float32)),
        physical_mask=mask,
        sensor=camera.model(),
        poses=SensorPose3D(T_world_sensors=[pose, pose.clone()], timestamps_us=[timestamp_us, timestamp_us]),
    )
