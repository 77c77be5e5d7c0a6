"""The oracle's per-pixel forward and backward against the reference's own
per-hit device functions (tests/golden/hit_golden.npz, made by
tests/golden/make_hit_golden.py from gaussianParticles.cuh processHitFwd
:611-686 and processHitBwd :736-1155 compiled for the host).

Each golden tile is one 16x16 tile whose rays composite the tile's particle
list in list order (K = 0).  The oracle renders it as a 16x16 camera with the
identity pose and the list as the tile's sorted range; its fused dot products
and its own exp differ from the reference's plain float arithmetic in the
last bits, so values are compared within a tolerance, and every branch (hit
or miss, alpha cap, transmittance cut-off, opacity thresholds, the 0.5
crossing) must agree exactly: hit counts are compared exactly and the
quantile depths are compared per entry.
"""

from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

import oracle

GOLDEN = Path(__file__).resolve().parent / "golden" / "hit_golden.npz"
IDENTITY_POSE = (0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 1.0)
# relative L2 error bounds per tile (float32 sums over a few hits, last-bit
# differences of exp and of the dot-product rounding; measured worst cases
# 1.3e-6 in the forward channels and 8e-6 in the gradients)
REL_L2 = 1e-5
REL_L2_GRAD = 5e-5
# the crossing rate -(T - 1/2)(2 AA t* + BB) cancels (2 AA t* + BB = -sqrt(disc)),
# so last-bit differences of AA and BB grow by |BB| / sqrt(disc) (worst 5.4e-4)
REL_L2_RATE = 5e-3


def rel_l2(a, b) -> float:
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / den) if den > 0 else float(np.linalg.norm(a))


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def tiles(g):
    start = 0
    for t, m in enumerate(g["counts"]):
        rows = g["rows"][start:start + m]
        colours = g["colours"][start:start + m]
        yield t, start, int(m), rows, colours
        start += int(m)


def render_tile(g, t, m, rows, colours):
    cam = oracle.camera(1, 16, 16, (8.0, 8.0), (10.0, 10.0), (0.0, 0.0, 0.0, 0.0), 3.0)
    pose = oracle.prepare_pose(IDENTITY_POSE)
    rays = g["rays"][t]
    ray_o = np.ascontiguousarray(rays[:, 0:3].reshape(16, 16, 3))
    ray_d = np.ascontiguousarray(rays[:, 3:6].reshape(16, 16, 3))
    mask = np.ones(1, np.uint8)
    ranges = np.array([[0, m]], np.uint32)
    ids = np.arange(m, dtype=np.uint32)
    return cam, pose, ray_o, ray_d, mask, ranges, ids


def golden_forward(g, t):
    """The reference's integrated channels of tile t in the oracle's output layout."""
    b = g["fwd_b"][t]
    quant = np.zeros((256, 10), np.float32)
    quant[:, 0:7] = b[:, 12:19]
    quant[:, 8] = b[:, 19]
    quant[:, 9] = b[:, 20]
    return dict(rgba=b[:, 0:4].reshape(16, 16, 4), hit_t=b[:, 4].reshape(16, 16),
                normal=b[:, 5:8].reshape(16, 16, 3), depth_var=b[:, 8].reshape(16, 16),
                extent=b[:, 9].reshape(16, 16), inv_depth=b[:, 10].reshape(16, 16),
                inv_depth2=b[:, 11].reshape(16, 16), quant=quant.reshape(16, 16, 10))


def test_golden_covers_the_branches(golden):
    a, b = golden["fwd_a"], golden["fwd_b"]
    assert golden["counts"].size >= 16 and a.shape[1] == 256
    assert (a[..., 5] == 0).any() and (a[..., 5] >= 8).any()          # rays without hits and with many
    assert (b[..., 3] > 1 - 1e-4).any()                                # rays cut at the minimum transmittance
    assert (b[..., 19] > 0).sum() > 1000                               # 0.5 crossings
    assert (golden["colours"] < 0).any()                               # clamped colours
    assert (golden["rows"][:, 3] > 0.95).any()                         # alpha cap reachable
    # the reference's backward writes no factor or intrinsic-density gradient
    assert not golden["grad"][:, 11:21].any()


def test_processhitfwd_matches_the_oracle_forward(golden):
    for t, _start, m, rows, colours in tiles(golden):
        cam, pose, ray_o, ray_d, mask, ranges, ids = render_tile(golden, t, m, rows, colours)
        rgba, hit_t, count = oracle.render_forward(cam, pose, rows, colours, ray_o, ray_d, mask, ranges, ids, 0)
        a = golden["fwd_a"][t]
        assert np.array_equal(count.reshape(-1), a[:, 5]), f"tile {t}: hit counts differ"
        assert rel_l2(rgba.reshape(-1, 4), a[:, 0:4]) < REL_L2, f"tile {t}"
        assert rel_l2(hit_t.reshape(-1), a[:, 4]) < REL_L2, f"tile {t}"


def test_training_channels_match_the_reference_forward(golden):
    for t, _start, m, rows, colours in tiles(golden):
        cam, pose, ray_o, ray_d, mask, ranges, ids = render_tile(golden, t, m, rows, colours)
        out = oracle.render_forward_geo(cam, pose, rows, colours, ray_o, ray_d, mask, ranges, ids, 0)
        ref = golden_forward(golden, t)
        for key in ("rgba", "hit_t", "normal", "depth_var", "extent", "inv_depth", "inv_depth2"):
            assert rel_l2(out[key], ref[key]) < REL_L2, f"tile {t}: {key}"
        # quantile depths: the same hit reaches each level (then the depths agree to rounding)
        q, rq = out["quant"][..., 0:7], ref["quant"][..., 0:7]
        assert np.array_equal(q == 0, rq == 0), f"tile {t}: quantile levels reached differ"
        np.testing.assert_allclose(q, rq, rtol=1e-5, atol=1e-6, err_msg=f"tile {t}: quantile depths")
        # the exact 0.5 crossing and its rate
        np.testing.assert_allclose(out["quant"][..., 8], ref["quant"][..., 8], rtol=1e-4, atol=1e-6,
                                   err_msg=f"tile {t}: crossing depth")
        assert rel_l2(out["quant"][..., 9], ref["quant"][..., 9]) < REL_L2_RATE, f"tile {t}: crossing rate"


def test_processhitbwd_matches_the_oracle_backward(golden):
    for t, start, m, rows, colours in tiles(golden):
        cam, pose, ray_o, ray_d, mask, ranges, ids = render_tile(golden, t, m, rows, colours)
        fwd = golden_forward(golden, t)
        gi = golden["grads"][t]
        quant_grad = np.zeros((256, 10), np.float32)
        quant_grad[:, 8] = gi[:, 12]
        grads = dict(rgba=gi[:, 0:4].reshape(16, 16, 4), hit_t=gi[:, 4].reshape(16, 16),
                     normal=gi[:, 5:8].reshape(16, 16, 3), depth_var=gi[:, 8].reshape(16, 16),
                     extent=gi[:, 9].reshape(16, 16), inv_depth=gi[:, 10].reshape(16, 16),
                     inv_depth2=gi[:, 11].reshape(16, 16), quant=quant_grad.reshape(16, 16, 10))
        rec, shape = oracle.render_backward_geo(cam, pose, rows, colours, ray_o, ray_d, mask, ranges, ids, 0, fwd,
                                                grads)
        ref = golden["grad"][start:start + m]
        ref_rgb = golden["grad_rgb"][start:start + m]
        for name, ours, theirs in (("position", rec[:, 0:3], ref[:, 0:3]), ("density", rec[:, 3], ref[:, 3]),
                                   ("inverse factor", rec[:, 4:13], ref[:, 21:30]),
                                   ("colour", rec[:, 13:16], ref_rgb),
                                   ("quaternion", shape[:, 0:4], ref[:, 4:8]),
                                   ("scale", shape[:, 4:7], ref[:, 8:11])):
            err = rel_l2(ours, theirs)
            assert err < REL_L2_GRAD, f"tile {t}: {name} gradient rel L2 {err:.2e}"


def test_sh_radiance_matches_the_reference(golden):
    """The projector's particle radiance (radianceFromSpH, gaussianParticles.cuh:188-220)
    against the oracle's, at SH degrees 0 to 3: particles on the unit sphere
    around the identity pose's centre, so their incident direction is their
    position; the oracle clamps at zero where the reference's renderer
    clamps at use (gutKBufferRenderer.cuh:404-405)."""
    cam = oracle.camera(0, 64, 64, (32.0, 32.0), (40.0, 40.0), (0.0,) * 6)
    pose = oracle.prepare_pose(IDENTITY_POSE)
    mask = np.ones(16, np.uint8)
    for degree in range(4):
        dirs = golden["sh_dirs"][degree]
        n = dirs.shape[0]
        rows = np.zeros((n, 32), np.float32)
        rows[:, 0:3] = dirs
        rows[:, 3] = 0.5
        rows[:, 4] = 1.0
        rows[:, 8:11] = 0.1
        rows[:, [12, 16, 20]] = 0.1
        rows[:, [21, 25, 29]] = 10.0
        _proj, rgb, _counts = oracle.project(cam, pose, rows, golden["sh_coeffs"][degree], degree, mask)
        ref = np.maximum(golden["sh_rgb"][degree], 0.0)
        np.testing.assert_allclose(rgb, ref, rtol=1e-5, atol=2e-6, err_msg=f"SH degree {degree}")


def test_world_abs_grad_matches_the_reference(golden):
    """The densification statistic (gutKBufferRenderer.cuh:290-294): per
    composited hit |g| of the hit's position gradient, summed per particle,
    against the reference's processHitBwd per hit; and the screen form with
    the map [[1,0,0],[0,1,0]] equals its first two components."""
    for t, start, m, rows, colours in tiles(golden):
        cam, pose, ray_o, ray_d, mask, ranges, ids = render_tile(golden, t, m, rows, colours)
        fwd = golden_forward(golden, t)
        gi = golden["grads"][t]
        quant_grad = np.zeros((256, 10), np.float32)
        quant_grad[:, 8] = gi[:, 12]
        grads = dict(rgba=gi[:, 0:4].reshape(16, 16, 4), hit_t=gi[:, 4].reshape(16, 16),
                     normal=gi[:, 5:8].reshape(16, 16, 3), depth_var=gi[:, 8].reshape(16, 16),
                     extent=gi[:, 9].reshape(16, 16), inv_depth=gi[:, 10].reshape(16, 16),
                     inv_depth2=gi[:, 11].reshape(16, 16), quant=quant_grad.reshape(16, 16, 10))
        with oracle.abs_grad(m, "world") as world:
            oracle.render_backward_geo(cam, pose, rows, colours, ray_o, ray_d, mask, ranges, ids, 0, fwd, grads)
        ref = golden["abs_world"][start:start + m]
        assert (ref >= 0).all()
        err = rel_l2(world.out, ref)
        assert err < REL_L2_GRAD, f"tile {t}: world abs-grad rel L2 {err:.2e}"
        mapping = np.zeros((m, 2, 3), np.float32)
        mapping[:, 0, 0] = 1.0
        mapping[:, 1, 1] = 1.0
        with oracle.abs_grad(m, "screen", mapping) as screen:
            oracle.render_backward_geo(cam, pose, rows, colours, ray_o, ray_d, mask, ranges, ids, 0, fwd, grads)
        np.testing.assert_array_equal(screen.out, world.out[:, 0:2])


def test_point_projection_matches_the_reference(golden):
    """The sensor-space projection of the UT's sigma points (projectPoint,
    cameraProjections.cuh:75-152, without raster bounds) against the oracle's,
    for three fisheye cameras (equidistant, Kannala-Brandt, equisolid 205 deg)
    and a distorted pinhole, over the whole sphere: validity exactly, pixel
    coordinates within 1e-5 relative + 1e-3 px (the oracle's atan2 is within
    2.5 ulp of the C library's)."""
    from tests.golden.make_hit_golden import PROJECTION_CAMERAS

    for c, (model, w, h, pp, f, k, tg, tp, max_angle) in enumerate(PROJECTION_CAMERAS):
        cam = oracle.camera(model, w, h, pp, f, k, max_angle, tangential=tg, thin_prism=tp)
        pts = golden["proj_points"][c]
        ref = golden["proj_out"][c]
        uv, valid = oracle.project_points(cam, pts)
        assert np.array_equal(valid, ref[:, 2] == 1.0), f"camera {c}: validity differs"
        assert valid.sum() > 1000 and (~valid).sum() > 100
        finite = np.isfinite(ref[:, :2]).all(axis=1)
        assert np.array_equal(finite, np.isfinite(uv).all(axis=1)), f"camera {c}"
        np.testing.assert_allclose(uv[finite], ref[finite, :2], rtol=1e-5, atol=1e-3, err_msg=f"camera {c}")


def test_kbuffer_order_matches_the_reference(golden):
    """The k-buffer's composite order (HitParticleKBufferT::insert fed as
    evalKBuffer feeds it, gutKBufferRenderer.cuh:118-166,676-699) against the
    oracle's KBuffer, exactly, for K = 4 ... 32 over sequences with ties,
    continuous, ascending, descending and constant distances.  The tracer's
    shared-memory ring is held to the same order by tests/test_kbuffer_model.py
    and the GPU parity tests."""
    off = golden["kb_offsets"]
    for s, k in enumerate(golden["kb_k"]):
        t = golden["kb_hit_t"][off[s]:off[s + 1]]
        ref = golden["kb_order"][off[s]:off[s + 1]]
        np.testing.assert_array_equal(oracle.kbuffer_order(int(k), t), ref.astype(np.uint32),
                                      err_msg=f"sequence {s}, K={k}")


def test_ut_projection_matches_the_reference(golden):
    """The 7-point UT projection of a particle (GUTProjector::
    unscentedParticleProjection, gutProjector.cuh:359-518, with its opacity
    gate, fisheye near radius, pinhole near plane and the projection of the
    sigma points) against the oracle's, around a random pose of three fisheye
    cameras and a distorted pinhole: validity exactly; the projected centre
    within 2e-3 px; the covariance within 1e-3 of its largest component (the
    covariance is a cancelling sum of sigma-point outer products)."""
    from tests.golden.make_hit_golden import PROJECTION_CAMERAS

    for c, (model, w, h, pp, f, k, tg, tp, max_angle) in enumerate(PROJECTION_CAMERAS):
        cam = oracle.camera(model, w, h, pp, f, k, max_angle, tangential=tg, thin_prism=tp)
        pose = oracle.prepare_pose(golden["ut_poses"][c])
        np.testing.assert_array_equal(np.array(pose.c, np.float32), golden["ut_centres"][c])
        out = oracle.ut_project(cam, pose, golden["ut_rows"][c])
        ref = golden["ut_out"][c]
        valid = ref[:, 5] == 1.0
        assert np.array_equal(out[:, 5] == 1.0, valid), f"camera {c}: UT validity differs"
        assert valid.sum() > 400 and (~valid).sum() > 400
        np.testing.assert_allclose(out[valid, :2], ref[valid, :2], rtol=0, atol=2e-3, err_msg=f"camera {c}")
        scale = np.abs(ref[valid, 2:5]).max(axis=1, keepdims=True)
        assert (np.abs(out[valid, 2:5] - ref[valid, 2:5]) <= 1e-3 * scale).all(), f"camera {c}: covariance"
