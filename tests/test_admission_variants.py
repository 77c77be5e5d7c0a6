"""The reference's two optional fast-admission variants (gutProjector.cuh):

* partial UT (render.gofish.fast_partial_ut_scale, :53-62 and :470-499): a
  particle whose projected mean is valid and whose every axis keeps one valid
  sigma point gets a footprint from its sigma points, each invalid one
  replaced by the reflection of its mirror about the projected mean, the
  covariance scaled by the scale's square;
* "cone_big" (render.gofish.fast_admission_fallback, :44-50 and :145-154):
  the cone fallback only for spheres that leave the camera centre outside and
  whose cap half-angle lies in [min, max].

CPU: the oracle's repaired footprints against a float64 restatement of the
repair, and its cone_big admission against the cap window.  GPU (marked):
projected state, keys, ids, ranges, counts and hit counts bit for bit against
the oracle with both variants on, images and gradients within tolerance."""

import math

import numpy as np
import pytest

import oracle
from tests import harness

SCALE = 1.5
UT_DELTA = math.sqrt(3.0)


def _kb_project(cam, p):
    """float64 KB projection of sensor-frame points [M,3] (cameraProjections.cuh:124-152):
    (uv [M,2], valid [M])."""
    rho = np.maximum(np.hypot(p[:, 0], p[:, 1]), np.finfo(np.float32).eps)
    theta_full = np.arctan2(rho, p[:, 2])
    theta = np.minimum(theta_full, cam.max_angle)
    t2 = theta * theta
    k = cam.coefficients
    poly = ((k[3] * t2 + k[2]) * t2 + k[1]) * t2 + k[0]
    delta = theta * (poly * t2 + 1.0) / rho
    uv = np.stack([cam.focal[0] * p[:, 0] * delta + cam.principal[0],
                   cam.focal[1] * p[:, 1] * delta + cam.principal[1]], axis=1)
    return uv, theta < cam.max_angle


def _repaired_ut(cam, row):
    """float64 partial UT of one packed row at the identity pose: (center,
    covariance) or None when the repair does not apply."""
    mu = row[0:3].astype(np.float64)
    B = row[12:21].astype(np.float64).reshape(3, 3)
    pts = [mu] + [mu + UT_DELTA * B[:, i] for i in range(3)] + [mu - UT_DELTA * B[:, i] for i in range(3)]
    uv, ok = _kb_project(cam, np.stack(pts))
    if ok.all() or not ok[0] or any(not ok[1 + i] and not ok[4 + i] for i in range(3)):
        return None
    for i in range(3):
        if not ok[1 + i]:
            uv[1 + i] = 2.0 * uv[0] - uv[4 + i]
        if not ok[4 + i]:
            uv[4 + i] = 2.0 * uv[0] - uv[1 + i]
    c = uv[1:].sum(axis=0) / 6.0
    d0 = uv[0] - c
    cov = 2.0 * np.outer(d0, d0) + sum(np.outer(d, d) for d in (uv[1:] - c)) / 6.0
    return c, cov * SCALE * SCALE


def _cov_from_conic(proj_row):
    """The 2x2 covariance behind a projected conic (conic = (cov + 0.3 I)^-1)."""
    c0, c1, c2 = (float(x) for x in proj_row[2:5])
    return np.linalg.inv(np.array([[c0, c1], [c1, c2]])) - 0.3 * np.eye(2)


@pytest.fixture(scope="module")
def horizon():
    return harness.horizon_case()


def _project(case, partial=0.0, cone_big=None):
    pose = oracle.prepare_pose(case.pose)
    with oracle.admission_variants(partial, cone_big):
        proj, _rgb, counts = oracle.project(case.ocam, pose, case.particles, case.features, case.scene.sh_degree,
                                            case.tmask, case.ray_d)
    return proj, counts


def test_partial_ut_repairs_rim_particles(horizon):
    case = horizon
    base, _ = _project(case)
    part, _ = _project(case, SCALE)
    valid_base = base[:, 6] > 0
    valid_part = part[:, 6] > 0
    # a particle whose full UT is valid is projected identically
    np.testing.assert_array_equal(part[valid_base].view(np.uint32), base[valid_base].view(np.uint32))
    repaired = np.flatnonzero(valid_part & ~valid_base)
    assert repaired.size >= 20, repaired.size
    for i in repaired[:200]:
        ref = _repaired_ut(case.camera, case.particles[i])
        assert ref is not None, i
        c, cov = ref
        np.testing.assert_allclose(part[i, 0:2], c, rtol=0, atol=1e-3 + 1e-5 * np.abs(c).max())
        got = _cov_from_conic(part[i])
        assert np.abs(got - cov).max() <= 2e-3 * np.abs(cov).max() + 1e-3, (i, got, cov)
    # and no particle that the float64 repair rejects gets a footprint from it
    rejected = [i for i in np.flatnonzero(~valid_base)[:400] if _repaired_ut(case.camera, case.particles[i]) is None]
    assert not valid_part[rejected].any()


def _cap_sine(row, pose_c=(0.0, 0.0, 0.0)):
    """float64 cap sine of the fallback's support sphere (Gershgorin bound), or
    None when the sphere holds the camera centre."""
    B = row[12:21].astype(np.float64).reshape(3, 3)
    M = B @ B.T
    lam = (np.abs(M).sum(axis=1)).max()
    rho = min(0.99, float(row[3]))
    canonical = min(2.994, math.sqrt(max(0.0, 2.0 * math.log(rho / (1.0 / 255.0)))))
    r = canonical * math.sqrt(lam) * 1.001
    D = float(np.linalg.norm(row[0:3].astype(np.float64) - np.asarray(pose_c)))
    if D <= r:
        return None
    return min(1.0, r / D * 1.0001)


@pytest.mark.parametrize("window_deg", [(0.0, 90.0), (5.0, 30.0)])
def test_cone_big_admits_only_its_window(horizon, window_deg):
    case = horizon
    window = tuple(math.radians(a) for a in window_deg)
    _, cone = _project(case)
    proj, big = _project(case, cone_big=window)
    fallback = np.flatnonzero(proj[:, 6] == 0)
    lo, hi = math.sin(window[0]), min(1.0, math.sin(window[1]))
    kept = dropped = 0
    for i in fallback:
        s = _cap_sine(case.particles[i])
        if s is None:
            assert big[i] == 0, i  # a sphere around the camera: never cone_big
            dropped += cone[i] > 0
            continue
        if abs(s - lo) < 1e-4 or abs(s - hi) < 1e-4:
            continue  # at the window's edge the float rounding decides
        if lo <= s <= hi:
            assert big[i] == cone[i], i
            kept += cone[i] > 0
        else:
            assert big[i] == 0, i
            dropped += cone[i] > 0
    assert kept > 0 and dropped > 0, (kept, dropped)


def test_admission_variant_config_is_validated():
    from gofish_b200.splat_raster import SplatRaster

    with pytest.raises(ValueError, match="cone_big"):
        SplatRaster({"render": {"gofish": {"fast_admission_fallback": "cone_huge"}}})
    with pytest.raises(ValueError, match="fast_partial_ut_scale"):
        SplatRaster({"render": {"gofish": {"fast_partial_ut_scale": 0.0}}})


@pytest.mark.gpu
@pytest.mark.parametrize("key_mode", [0, 1])
def test_gpu_admission_variants_match_oracle(cuda_device, horizon, key_mode):
    case = horizon
    window = (math.radians(2.0), math.radians(60.0))
    ref = harness.oracle_forward(case, 16, key_mode, partial_ut_scale=SCALE, cone_big=window)
    gofish = {"fast_partial_ut_scale": SCALE, "fast_admission_fallback": "cone_big",
              "fast_admission_fallback_min_angle_deg": 2.0, "fast_admission_fallback_max_angle_deg": 60.0}
    got = harness.GpuTracer(case, 16, key_mode, cuda_device, gofish=gofish).forward()
    harness.compare_forward(ref, got)
    rng = np.random.default_rng(3)
    g_rgba = rng.uniform(-1, 1, ref["rgba"].shape).astype(np.float32)
    g_hit = np.zeros(ref["hit_t"].shape, np.float32)
    gp_ref, gs_ref, _ = harness.oracle_backward(case, ref, 16, g_rgba, g_hit)
    gp, gs = harness.GpuTracer(case, 16, key_mode, cuda_device, gofish=gofish).backward_after_forward(g_rgba, g_hit)
    assert harness.rel_l2(gp, gp_ref) <= 1e-3 and harness.rel_l2(gs, gs_ref) <= 1e-3
