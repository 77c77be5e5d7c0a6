"""Host-side logic mirrored from the reference: tile-mask tokens, camera
factories, SplatRaster configuration, synthetic workloads."""

import hashlib
import json

import numpy as np
import pytest

from gofish_b200 import physical_tile_mask
from gofish_b200.camera import (EQUISOLID_KB4, ShutterType, fisheye_camera, fromOpenCVFisheyeCameraModelParameters,
                                fromOpenCVPinholeCameraModelParameters, monotone_branch_limit, radial_value)
from gofish_b200.scene import pack_particles, random_scene


def test_tile_token_matches_reference_construction():
    # physical_tile_mask.py:27-29 of the reference: sha256 of sorted compact JSON.
    payload = {"domain": "full-raster", "device": "cuda:0", "height": 320, "tile": 16, "width": 320}
    expect = hashlib.sha256(json.dumps(payload, sort_keys=True, separators=(",", ":")).encode()).hexdigest()
    got = physical_tile_mask._token(domain="full-raster", height=320, width=320, device="cuda:0")
    assert got == expect and len(got) == 64


def test_camera_factories_round_to_float32():
    cam = fromOpenCVFisheyeCameraModelParameters(np.array([640, 480], np.uint64), ShutterType.GLOBAL, [320.5, 240.25],
                                                 [200.1, 200.2], [0.1, 0.01, 0.001, 0.0001], 1.7)
    native = cam.native(640, 480)
    assert native.model == 1 and native.shutter == int(ShutterType.GLOBAL)
    assert native.focal_length[0] == np.float32(200.1)
    assert native.radial[3] == np.float32(0.0001) and native.radial[4] == 0.0
    pin = fromOpenCVPinholeCameraModelParameters([64, 48], ShutterType.GLOBAL, [32, 24], [50, 50], [0.0] * 6,
                                                 [0.0, 0.0], [0.0] * 4)
    assert pin.native(64, 48).model == 0
    with pytest.raises(ValueError):
        fromOpenCVFisheyeCameraModelParameters([64, 48], ShutterType.GLOBAL, [32, 24], [50, 50], [0.1] * 3, 1.0)


def test_equisolid_coefficients_follow_two_sin_half_theta():
    t = np.radians(102.5)
    assert abs(radial_value(t, EQUISOLID_KB4) - 2 * np.sin(t / 2)) < 1e-6 * 2 * np.sin(t / 2)
    assert monotone_branch_limit(EQUISOLID_KB4) > np.radians(102.5)


def test_fisheye_camera_maps_half_fov_to_inscribed_radius():
    cam = fisheye_camera(400, 300, 200.0, (0.01, -0.002, 0.0, 0.0))
    r = cam.focal[0] * radial_value(cam.max_angle, cam.coefficients)
    assert abs(r - 150.0) < 1e-3
    o, d, valid = cam.rays()
    assert o.shape == (1, 300, 400, 3) and valid.shape == (1, 300, 400, 1)
    np.testing.assert_allclose(np.linalg.norm(d, axis=-1), 1.0, atol=1e-6)
    assert not valid[0, 0, 0, 0] and valid[0, 150, 200, 0]


def test_packed_rows_hold_inverse_factors():
    sc = random_scene(200, 3, 0)
    rows = pack_particles(sc)
    B = rows[:, 12:21].reshape(-1, 3, 3).astype(np.float64)
    Binv = rows[:, 21:30].reshape(-1, 3, 3).astype(np.float64)
    np.testing.assert_allclose(B @ Binv, np.broadcast_to(np.eye(3), B.shape), atol=1e-5)
    np.testing.assert_array_equal(rows[:, 3], rows[:, 11])
    assert sc.features.shape == (200, 48)
