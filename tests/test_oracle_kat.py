"""Known-answer tests that pin the CPU oracle (the reference ships no tests or
golden vectors for this path; these closed-form cases stand in for them)."""

import math

import numpy as np
import pytest

import oracle
from gofish_b200.scene import SH_C0, Scene, pack_particles
from gofish_b200.camera import fisheye_camera, first_branch_rays
from tests import harness

IDENTITY = np.array([0, 0, 0, 0, 0, 0, 1], dtype=np.float32)


def _scene(positions, scales, opacities, colors, rotations=None):
    n = len(positions)
    rot = np.tile(np.array([[1.0, 0, 0, 0]], dtype=np.float32), (n, 1)) if rotations is None else rotations
    feats = ((np.asarray(colors, dtype=np.float64) - 0.5) / SH_C0).astype(np.float32)
    return Scene(np.asarray(positions, dtype=np.float32), rot.astype(np.float32),
                 np.asarray(scales, dtype=np.float32), np.asarray(opacities, dtype=np.float32).reshape(n, 1), feats, 0)


def _odd_camera(size=65, fov=200.0):
    # Odd raster: the centre pixel's ray is exactly the optical axis.
    cam = fisheye_camera(size, size, fov)
    return cam


def test_equidistant_projection_identity():
    """r = f theta for an equidistant camera (k = 0), at the particle mean."""
    cam = fisheye_camera(321, 321, 200.0)
    f = cam.focal[0]
    rng = np.random.default_rng(0)
    thetas = rng.uniform(0.05, math.radians(95.0), 20)
    phis = rng.uniform(0, 2 * math.pi, 20)
    pos = np.stack([np.sin(thetas) * np.cos(phis), np.sin(thetas) * np.sin(phis), np.cos(thetas)], 1) * 3.0
    sc = _scene(pos, np.full((20, 3), 1e-4), np.full(20, 0.9), np.full((20, 3), 0.5))
    ocam = harness.oracle_camera(cam)
    pose = oracle.prepare_pose(IDENTITY)
    mask = np.ones(((321 + 15) // 16, (321 + 15) // 16), dtype=np.uint8)
    proj, _, counts = oracle.project(ocam, pose, pack_particles(sc), sc.features, 0, mask)
    expect = np.stack([f * thetas * np.cos(phis) + cam.principal[0], f * thetas * np.sin(phis) + cam.principal[1]], 1)
    np.testing.assert_allclose(proj[:, :2], expect, atol=2e-2)
    assert np.all(counts > 0)


def test_first_branch_rays_round_trip():
    """Rays from the Kannala-Brandt inverse project back onto their pixel centres."""
    rng = np.random.default_rng(1)
    k = (0.01, -0.005, 0.002, -0.0005)
    cam = fisheye_camera(128, 128, 200.0, k)
    r = 60.0 * np.sqrt(rng.random(200))
    a = rng.uniform(0, 2 * np.pi, 200)
    pts = np.stack([64.0 + r * np.cos(a), 64.0 + r * np.sin(a)], 1)
    rays, valid = first_branch_rays(pts, cam.focal, cam.principal, cam.coefficients, cam.max_angle)
    assert valid.all()
    theta = np.arctan2(np.linalg.norm(rays[:, :2], axis=1), rays[:, 2])
    y = theta * theta
    rho = theta * (1 + y * (k[0] + y * (k[1] + y * (k[2] + y * k[3]))))
    az = rays[:, :2] / np.linalg.norm(rays[:, :2], axis=1, keepdims=True)
    back = az * rho[:, None] * np.asarray(cam.focal) + np.asarray(cam.principal)
    np.testing.assert_allclose(back, pts, atol=1e-3)


def _render(sc, cam, k, key_mode):
    case = harness.make_case(sc, cam, IDENTITY)
    return case, harness.oracle_forward(case, k, key_mode)


@pytest.mark.parametrize("k", [0, 16])
def test_single_on_axis_gaussian(k):
    """Closed form: the axis ray meets the Gaussian at its centre (response 1)."""
    cam = _odd_camera()
    sc = _scene([[0.0, 0.0, 3.0]], [[0.1, 0.1, 0.1]], [0.8], [[0.2, 0.4, 0.6]])
    case, f = _render(sc, cam, k, 1)
    c = cam.width // 2
    np.testing.assert_allclose(f["rgba"][c, c], [0.8 * 0.2, 0.8 * 0.4, 0.8 * 0.6, 0.8], rtol=2e-6)
    np.testing.assert_allclose(f["hit_t"][c, c], 0.8 * 3.0, rtol=2e-6)
    assert f["hit_count"][c, c] == 1.0
    # global key = camera radial distance of the centre, exactly 3.0
    assert np.all((f["keys"] & np.uint64(0xFFFFFFFF)) == np.uint64(np.float32(3.0).view(np.uint32)))
    # far from the particle nothing is hit, and pixels outside the domain keep their initial values
    assert f["hit_count"][0, c] == 0.0
    outside = ~case.valid
    assert np.all(f["rgba"][outside] == 0.0)


@pytest.mark.parametrize("k", [0, 16])
@pytest.mark.parametrize("key_mode", [0, 1])
def test_two_gaussians_front_to_back(k, key_mode):
    cam = _odd_camera()
    # listed back-to-front: the sort must reorder them
    sc = _scene([[0.0, 0.0, 4.0], [0.0, 0.0, 2.0]], [[0.1] * 3, [0.05] * 3], [0.5, 0.5],
                [[0.0, 0.0, 1.0], [1.0, 0.0, 0.0]])
    _, f = _render(sc, cam, k, key_mode)
    c = cam.width // 2
    np.testing.assert_allclose(f["rgba"][c, c], [0.5, 0.0, 0.25, 0.75], rtol=2e-6, atol=1e-7)
    np.testing.assert_allclose(f["hit_t"][c, c], 0.5 * 2.0 + 0.25 * 4.0, rtol=2e-6)
    assert f["hit_count"][c, c] == 2.0


def test_kbuffer_reorders_hits_within_the_pixel():
    """With the global radial key, B (radial 3.02) sorts before A (radial 3.04),
    but on the axis ray A is hit first (tau 3.00 < 3.02).  K = 0 composites in
    key order, K = 16 in hit order."""
    cam = _odd_camera()
    sc = _scene([[0.5, 0.0, 3.0], [0.0, 0.0, 3.02]], [[0.6] * 3, [0.05] * 3], [0.5, 0.5],
                [[1.0, 0.0, 0.0], [0.0, 1.0, 0.0]])
    c = cam.width // 2
    _, f0 = _render(sc, cam, 0, 1)
    _, f16 = _render(sc, cam, 16, 1)
    # response of A on the axis: exp(-0.5 * (0.5/0.6)^2)
    alpha_a = 0.5 * math.exp(-0.5 * (0.5 / 0.6) ** 2)
    alpha_b = 0.5
    # K = 0: B then A
    np.testing.assert_allclose(f0["rgba"][c, c, :2], [(1 - alpha_b) * alpha_a, alpha_b], rtol=1e-5)
    # K = 16: A then B
    np.testing.assert_allclose(f16["rgba"][c, c, :2], [alpha_a, (1 - alpha_a) * alpha_b], rtol=1e-5)


def test_transmittance_cutoff_stops_compositing():
    """Opaque layers: compositing stops once T < 1e-4.  In float32
    1 - 0.99f = 0.00999999, so two layers give T = 9.99998e-5 < 1e-4 and the
    ray dies after the second hit."""
    cam = _odd_camera()
    sc = _scene([[0, 0, 2.0], [0, 0, 3.0], [0, 0, 4.0], [0, 0, 5.0]], [[0.1] * 3] * 4, [0.99] * 4,
                [[1.0, 1.0, 1.0]] * 4)
    _, f = _render(sc, cam, 16, 0)
    c = cam.width // 2
    assert f["hit_count"][c, c] == 2.0
    t = np.float32(1.0) - np.float32(0.99)
    np.testing.assert_allclose(f["rgba"][c, c, 3], np.float32(1.0) - t * t, rtol=1e-6)


def test_sort_order_and_ranges_cpu_scale():
    from gofish_b200.scene import workload_cpu_scale

    w = workload_cpu_scale()
    case = harness.make_case(w.scene, w.camera, w.poses[0])
    f = harness.oracle_forward(case, 16, 0)
    keys, ids, ranges = f["keys"], f["ids"], f["ranges"]
    assert keys.size == int(f["counts"].sum())
    assert np.all(keys[1:] >= keys[:-1])
    same = keys[1:] == keys[:-1]
    assert np.all(ids[1:][same] > ids[:-1][same])  # stable: equal keys keep particle order
    tiles = (keys >> np.uint64(32)).astype(np.int64)
    for t in np.unique(tiles):
        b, e = ranges[t]
        assert np.all(tiles[b:e] == t) and e - b == np.count_nonzero(tiles == t)
    empty = np.setdiff1d(np.arange(ranges.shape[0]), np.unique(tiles))
    assert np.all(ranges[empty] == 0)
    # emitted tiles are retained tiles
    assert np.all(case.tmask.reshape(-1)[np.unique(tiles)] == 1)
    # visibility follows the counts
    np.testing.assert_array_equal(f["visibility"], (f["counts"] > 0).astype(np.uint32))


def test_pinhole_axis_projects_to_principal_point():
    ocam = oracle.camera(0, 64, 48, (32.0, 24.0), (50.0, 50.0), [0.0] * 6)
    sc = _scene([[0.0, 0.0, 3.0]], [[1e-4] * 3], [0.9], [[0.5] * 3])
    pose = oracle.prepare_pose(IDENTITY)
    proj, _, counts = oracle.project(ocam, pose, pack_particles(sc), sc.features, 0, np.ones((3, 4), np.uint8))
    np.testing.assert_allclose(proj[0, :2], [32.0, 24.0], atol=1e-3)
    assert counts[0] > 0
