"""The oracle's indexed opacity field (a bounding-volume hierarchy over
conservative support spheres, used for the full-size mesh-query parity
tests) equals its brute-force field bit for bit: opacity bits, observed and
above, on sparse and dense scenes (saturated points exercise the early exit),
with masked and unmasked cameras and points behind the cameras."""

import math

import numpy as np
import pytest

import oracle
from gofish_b200.camera import fisheye_camera
from gofish_b200.mesh.cameras import fisheye_training_camera
from gofish_b200.mesh.shape import effective_shape
from gofish_b200.mesh.sites import generate_sites
from gofish_b200.scene import look_outward_pose, random_scene


@pytest.mark.parametrize("n,scale,masked", [(3000, 3.0, False), (12000, 8.0, True)])
def test_indexed_field_equals_brute_force(n, scale, masked):
    scene = random_scene(n, 0, 17 + n, r_min=1.0, r_max=3.0)
    shape = effective_shape(scene.positions, scene.scales * np.float32(scale), scene.rotations, scene.density)
    rng = np.random.default_rng(n)
    pts = generate_sites(shape).points
    pts = np.concatenate([pts[rng.choice(pts.shape[0], 2500, replace=False)],
                          rng.uniform(-4, 4, (500, 3)).astype(np.float32)])
    cam = fisheye_camera(64, 64, 200.0)
    ocam = oracle.camera(1, cam.width, cam.height, cam.principal, cam.focal, cam.coefficients, cam.max_angle)
    ray_o = np.zeros((64, 64, 3), np.float32)
    views = []
    for v in range(3):
        yaw = 2.0 * math.pi * v / 3 + 0.2
        pose = look_outward_pose(np.array([2.0 * math.cos(yaw), 2.0 * math.sin(yaw), 0.0]), yaw)
        mask = fisheye_training_camera(v, cam, pose, masked=True).physical_mask.numpy() if masked else None
        views.append((ocam, pose, ray_o, mask))
    packed = shape.packed_density()
    want = oracle.evaluate_field(views, packed, pts)
    with oracle.FieldIndex(packed, 20.0) as ix:
        got = ix.evaluate_field(views, pts)
    np.testing.assert_array_equal(got[0].view(np.uint32), want[0].view(np.uint32))
    np.testing.assert_array_equal(got[1], want[1])
    np.testing.assert_array_equal(got[2], want[2])
    observed = want[1] != 0
    assert 0 < observed.sum() < pts.shape[0]
    if scale >= 6.0:
        assert int((want[0][observed] == 1.0).sum()) >= 20  # saturated points (the early exit)
