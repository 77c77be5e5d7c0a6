"""Host side of the mesh opacity query, without a GPU.

* the site generator, packed shape rows, signed field and bisection batch
  planner against golden vectors made from the reference's own Python
  modules (tests/golden/make_mesh_golden.py);
* the oracle's opacity field against closed forms (on-axis Gaussian,
  points behind the camera, the camera-min over views);
* the bisection driver (bracket / bisect) against a scalar restatement of
  the reference's update rules, with a fake raster on an analytic field.
"""

import math
from pathlib import Path

import numpy as np
import pytest
import torch

import oracle
from gofish_b200.camera import fisheye_camera
from gofish_b200.mesh import bisection, field, shape as shape_mod, sites
from gofish_b200.scene import IDENTITY_POSE

GOLDEN = Path(__file__).resolve().parent / "golden" / "mesh_golden.npz"


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def golden_shape(g):
    return shape_mod.EffectiveShape(positions=g["positions"], density=g["density"], factor=g["factor"],
                                    inverse_factor=g["inverse_factor"], sigma_max=g["sigma_max"],
                                    retained=g["retained"])


def test_sites_match_reference(golden):
    s = sites.generate_sites(golden_shape(golden))
    assert np.array_equal(s.points.view(np.uint32), golden["site_points"].view(np.uint32))
    assert np.array_equal(s.scale.view(np.uint32), golden["site_scale"].view(np.uint32))
    assert np.array_equal(s.owner, golden["site_owner"])
    r = sites.support_radius(golden["density"][golden["retained"], 0])
    assert np.array_equal(r, golden["radius"])


def test_packed_density_matches_reference(golden):
    assert np.array_equal(golden_shape(golden).packed_density(), golden["packed"])


def test_signed_field_matches_reference(golden):
    assert np.array_equal(field.signed_field(golden["minimum"], golden["observed"]), golden["signed"])


def test_batch_planner_matches_reference(golden):
    for (e, f, c), want in zip(golden["batch_cases"], golden["batch_sizes"]):
        assert bisection.batch_size(int(e), int(f), int(c)) == int(want)
    with pytest.raises(MemoryError):
        bisection.batch_size(5_000_000, 2 << 30, 1 << 29)
    pe, pv = bisection._padded_batch(golden["pad_ends"], golden["pad_vals"], 2, 7, 8)
    assert np.array_equal(pe, golden["padded_ends"]) and np.array_equal(pv, golden["padded_vals"])


def _one_gaussian(mu, sigma, density):
    row = np.zeros((1, 32), np.float32)
    row[0, 0:3] = mu
    row[0, 3] = density
    row[0, 12:21] = (np.eye(3) * sigma).reshape(-1)
    row[0, 21:30] = (np.eye(3) / sigma).reshape(-1)
    return row


def test_oracle_field_closed_forms():
    cam = fisheye_camera(64, 64, 200.0)
    ocam = oracle.camera(1, cam.width, cam.height, cam.principal, cam.focal, cam.coefficients, cam.max_angle)
    parts = _one_gaussian([0.0, 0.0, 3.0], 0.25, 0.8)
    ray_o = np.zeros((64, 64, 3), np.float32)
    pts = np.array([[0.0, 0.0, 5.0],     # through the centre: alpha = 0.8
                    [0.0, 0.0, 2.5],     # stops 2 sigma before the centre
                    [0.0, 0.0, -5.0],    # behind the 200 degree camera
                    [3.0, 0.0, 0.5]],    # in view, far from the Gaussian
                   np.float32)
    op, ob = oracle.field_camera(ocam, IDENTITY_POSE, parts, ray_o, pts)
    assert ob.tolist() == [1, 1, 0, 1]
    assert op[0] == np.float32(1.0) - (np.float32(1.0) - np.float32(0.8))
    assert op[1] == pytest.approx(0.8 * math.exp(-0.5 * 4.0), rel=1e-5)
    assert op[2] == 0.0 and op[3] == 0.0


def test_oracle_camera_min_and_round_classification():
    cam = fisheye_camera(64, 64, 200.0)
    ocam = oracle.camera(1, cam.width, cam.height, cam.principal, cam.focal, cam.coefficients, cam.max_angle)
    parts = _one_gaussian([0.0, 0.0, 3.0], 0.25, 0.5)
    ray_o = np.zeros((64, 64, 3), np.float32)
    # A second camera looking down -z from (0, 0, 6): the point (0,0,4.5) is
    # behind the Gaussian for the first camera and in front of it for the second.
    back = np.array([0.0, 0.0, 6.0, 1.0, 0.0, 0.0, 0.0], np.float32)  # R = diag(1,-1,-1), t = -R c
    views = [(ocam, IDENTITY_POSE, ray_o, None), (ocam, back, ray_o, None)]
    pts = np.array([[0.0, 0.0, 4.5], [0.0, 0.0, -4.0]], np.float32)
    a0, o0 = oracle.field_camera(ocam, IDENTITY_POSE, parts, ray_o, pts)
    a1, o1 = oracle.field_camera(ocam, back, parts, ray_o, pts)
    op, ob, ab = oracle.evaluate_field(views, parts, pts)
    assert ob.tolist() == [1, 1]
    assert op[0] == min(a0[0], a1[0]) and op[0] < 0.5 <= a0[0]
    above, observed, exact = oracle.bisection_round(views, parts, pts)
    assert above.tolist() == [int(op[0] >= 0.5), int(op[1] >= 0.5)]
    assert exact.tolist() == [int(op[0] == 0.5), int(op[1] == 0.5)]


class _AnalyticRaster:
    """Field O(x) = 1 if x.x < c else 0, unobserved where x.y > 5."""

    def __init__(self, c):
        self.c = c

    def evaluate_bisection_round(self, token, mid, r):
        x = mid.numpy()
        observed = (x[:, 1] <= 5.0).astype(np.uint8)
        o = np.where(x[:, 0] < self.c, np.float32(1.0), np.float32(0.0))
        o = np.where(x[:, 0] == self.c, np.float32(0.5), o)
        above = (observed != 0) & (o >= 0.5)
        exact = (observed != 0) & (o == np.float32(0.5))
        return (torch.from_numpy(above.astype(np.uint8)), torch.from_numpy(observed),
                torch.from_numpy(exact.astype(np.uint8)))


def _scalar_bisect(solid, free, raster):
    solid, free = solid.copy(), free.copy()
    for r in range(bisection.ROUNDS):
        mid = ((solid + free) * np.float32(0.5)).astype(np.float32)
        a, o, e = (t.numpy() for t in raster.evaluate_bisection_round(0, torch.from_numpy(mid[None]), r))
        above = bool(a[0]) or not bool(o[0])
        ex = bool(e[0]) and bool(o[0])
        if above:
            solid = mid
        if (not above) or ex:
            free = mid
    return ((solid + free) * np.float32(0.5)).astype(np.float32)


def test_bisection_driver_matches_scalar_rules():
    rng = np.random.default_rng(3)
    raster = _AnalyticRaster(0.3)
    e = 200
    a = np.stack([rng.uniform(-1, 0.3, e), rng.uniform(0, 6, e), rng.uniform(-1, 1, e)], 1).astype(np.float32)
    b = np.stack([rng.uniform(0.3, 1, e), rng.uniform(0, 6, e), rng.uniform(-1, 1, e)], 1).astype(np.float32)
    a[:5, 0] = 0.3 - 0.25
    b[:5, 0] = 0.3 + 0.25  # midpoint lands exactly on the tie after one round
    ends = np.stack([b, a], 1)  # endpoint 0 free, endpoint 1 solid: exercises the swap
    fields = np.stack([np.full(e, 0.5, np.float32), np.full(e, -0.5, np.float32)], 1)
    solid, free = bisection.bracket(torch.from_numpy(ends), torch.from_numpy(fields))
    got = bisection.bisect(raster, 0, solid, free).numpy()
    want = np.stack([_scalar_bisect(a[i], b[i], raster) for i in range(e)])
    assert np.array_equal(got, want)
    with pytest.raises(ValueError, match="sign crossings"):
        bisection.bracket(torch.from_numpy(ends), torch.from_numpy(np.abs(fields)))
