"""Host side of the inference path: batch -> native camera and pose
(threedgut_tracer/tracer.py:536-672), the inference-orbit workload and its
physical-mip camera records."""

import math

import numpy as np
import pytest
import torch

from gofish_b200 import scene as S
from gofish_b200.batch import Batch, create_camera_parameters, so3_to_quaternion_xyzw
from gofish_b200.camera import GF_CAMERA_OPENCV_FISHEYE, GF_CAMERA_OPENCV_PINHOLE, ShutterType
from gofish_b200.inference import SHAPE_MODES, InferenceTracer


def _rot(q_xyzw):
    x, y, z, w = q_xyzw
    return S.quaternion_to_matrix(np.array([[w, x, y, z]]))[0]


@pytest.mark.parametrize("trace_case", ["w", "x", "y", "z"])
def test_quaternion_of_rotation_every_branch(trace_case):
    # a rotation whose largest quaternion component is the named one
    angle = {"w": 0.3, "x": 2.9, "y": 2.9, "z": 2.9}[trace_case]
    axis = {"w": [1.0, 2.0, 3.0], "x": [1.0, 0.1, 0.2], "y": [0.1, 1.0, 0.2], "z": [0.1, 0.2, 1.0]}[trace_case]
    axis = np.asarray(axis) / np.linalg.norm(axis)
    q = np.concatenate([axis * math.sin(angle / 2), [math.cos(angle / 2)]])
    R = _rot(q)
    got = so3_to_quaternion_xyzw(R)
    assert abs(np.linalg.norm(got) - 1.0) < 1e-12
    np.testing.assert_allclose(_rot(got), R, atol=1e-12)
    assert "xyzw"[int(np.argmax(np.abs(got)))] == trace_case


def test_camera_parameters_round_trip_the_pose():
    rng = np.random.default_rng(5)
    cam = S.fisheye_camera(64, 48, 205.0, S.EQUISOLID_KB4)
    for _ in range(20):
        q = rng.standard_normal(4)
        pose = S.pose_world_to_sensor(rng.uniform(-3, 3, 3), q / np.linalg.norm(q))
        batch = Batch(None, None, torch.from_numpy(S.pose_to_c2w(pose)[None]).float(),
                      intrinsics_OpenCVFisheyeCameraModelParameters=cam.intrinsics())
        model, poses = create_camera_parameters(batch)
        p0, p1 = poses.T_world_sensors
        assert p1 is p0 and poses.timestamps_us == [0, 1]
        np.testing.assert_allclose(_rot(p0[3:]), _rot(pose[3:]), atol=1e-6)
        np.testing.assert_allclose(p0[:3], pose[:3], atol=2e-6)
        assert model.model == GF_CAMERA_OPENCV_FISHEYE and model.shutter_type == ShutterType.GLOBAL
        assert model.max_angle == pytest.approx(math.radians(102.5), abs=1e-6)
        assert model.resolution == (64, 48)


def test_camera_parameters_pinhole_intrinsics_and_end_pose():
    c2w = np.eye(4)
    c2w[:3, 3] = [1.0, 2.0, 3.0]
    end = c2w.copy()
    end[:3, 3] = [1.5, 2.0, 3.0]
    batch = Batch(None, None, torch.from_numpy(c2w[None]).float(), intrinsics=[100.0, 90.0, 32.0, 24.0],
                  T_to_world_end=torch.from_numpy(end[None]).float())
    model, poses = create_camera_parameters(batch)
    assert model.model == GF_CAMERA_OPENCV_PINHOLE and model.resolution == (64, 48)
    np.testing.assert_allclose(model.focal_length, (100.0, 90.0), rtol=1e-6)
    np.testing.assert_allclose(poses.T_world_sensors[0][:3], [-1.0, -2.0, -3.0])
    np.testing.assert_allclose(poses.T_world_sensors[1][:3], [-1.5, -2.0, -3.0])
    with pytest.raises(ValueError):
        create_camera_parameters(Batch(None, None, torch.eye(4)[None]))


def test_inference_orbit_workload_places_large_gaussians_beside_the_path():
    w = S.workload_inference(n=20_000, frames=12, size=64)
    assert w.k_buffer == 32 and len(w.poses) == 12
    big = w.big_rows
    assert big.size == 1000 and np.unique(big).size == 1000
    assert np.median(w.scene.scales[big]) > 5 * np.median(w.scene.scales)
    p = w.scene.positions[big].astype(np.float64)
    ring = np.hypot(p[:, 0], p[:, 1])
    # distance to the 2 m ring: within 1 m (plus the 0.1 m outward jitter)
    assert np.all(np.hypot(ring - 2.0, p[:, 2]) <= math.hypot(1.0, 0.1) + 1e-5)
    # equisolid 205 deg: f puts 102.5 deg on the inscribed radius
    assert w.camera.max_angle == pytest.approx(math.radians(102.5), abs=1e-6)
    # every camera looks outward from the ring
    for k, pose in enumerate(w.poses):
        c2w = S.pose_to_c2w(pose)
        yaw = 2 * math.pi * k / 12
        np.testing.assert_allclose(c2w[:3, 3], [2 * math.cos(yaw), 2 * math.sin(yaw), 0.0], atol=1e-5)
        np.testing.assert_allclose(c2w[:3, 2], [math.cos(yaw), math.sin(yaw), 0.0], atol=1e-5)


def test_mip_camera_records_follow_the_valid_mask():
    cam = S.fisheye_camera(40, 30, 205.0, S.EQUISOLID_KB4)
    _o, _d, valid = cam.rays()
    valid = valid[0, :, :, 0]
    cams, frames = S.mip_camera_records(cam, S.orbit_poses(5), valid)
    runs = cams[0]["rows"]
    assert len(runs) == 30
    for row, (lo, hi) in zip(valid, runs):
        expect = np.zeros(40, bool)
        expect[lo:hi] = True
        np.testing.assert_array_equal(row, expect)
    assert [f["frame_index"] for f in frames] == list(range(5))
    assert cams[0]["params"][:2] == list(cam.focal)


def test_inference_tracer_rejects_unknown_modes():
    assert SHAPE_MODES == ("exact", "fused", "fused32", "fusedmix")
    with pytest.raises(ValueError):
        InferenceTracer({}, None, shape="float16")
    with pytest.raises(RuntimeError):
        InferenceTracer({"render": {"primitive_type": "trisurfel"}}, None)
