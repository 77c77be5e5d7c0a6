"""The sm_100a opacity field and bisection rounds against the oracle, through
the mesh SplatRaster (C ABI gf_field_*).  The field is integer-exact work on
fp32: opacity, observed and above must match the oracle bit for bit."""

import numpy as np
import pytest
import torch

from gofish_b200.mesh import SplatRaster
from gofish_b200.mesh.bisection import bisect, bracket, refine_crossings
from gofish_b200.mesh.field import camera_inputs, evaluate_field, signed_field

from tests.mesh_harness import field_case, oracle_field, oracle_round

pytestmark = pytest.mark.gpu


def gpu_field(raster, case, device, points=None):
    pts = case.points if points is None else points
    packed = torch.from_numpy(case.shape.packed_density()).to(device)
    sigma = torch.from_numpy(np.ascontiguousarray(case.shape.sigma_max)).to(device)
    query = torch.from_numpy(np.ascontiguousarray(pts)).to(device)
    token = raster.begin_opacity_field(packed, sigma, query)
    for cam in case.cameras:
        raster.integrate_opacity_field_camera(token, *camera_inputs(cam, device))
    opacity, observed, above = raster.finish_opacity_field(token)
    raster.release_opacity_field(token)
    torch.cuda.synchronize(device)
    return opacity.cpu().numpy(), observed.cpu().numpy(), above.cpu().numpy()


def assert_field_equal(got, want):
    op, ob, ab = got
    wop, wob, wab = want
    assert np.array_equal(ob, wob), f"observed differs at {np.flatnonzero(ob != wob)[:10]}"
    bad = np.flatnonzero(op.view(np.uint32) != wop.view(np.uint32))
    assert bad.size == 0, f"{bad.size} opacities differ, e.g. {bad[:5]}: {op[bad[:5]]} vs {wop[bad[:5]]}"
    assert np.array_equal(ab, wab)


@pytest.mark.parametrize("masked", [True, False])
def test_field_matches_oracle(cuda_device, masked):
    case = field_case(masked=masked)
    want = oracle_field(case)
    assert 0.05 < want[2].mean() < 0.95, "case must mix points above and below 1/2"
    assert want[1].mean() > 0.3
    got = gpu_field(SplatRaster(), case, cuda_device)
    assert_field_equal(got, want)


@pytest.mark.parametrize("n,boost", [(12000, 1.5), (40000, 4.0)])
def test_field_dense_scene(cuda_device, n, boost):
    # Many candidates per cell and per warp: larger Gaussians in a 1-2.5 m
    # shell; in the 40k case almost every observed point saturates (1 - T
    # rounds to 1 long before its last candidate).
    case = field_case(seed=5, n=n, size=128, num_views=3, site_gaussians=800, extra_points=4000,
                      scale_boost=boost, r_max=2.5, ring=1.5)
    want = oracle_field(case)
    if boost > 2.0:
        assert (want[0][want[1] != 0] == np.float32(1.0)).mean() > 0.5
    got = gpu_field(SplatRaster(), case, cuda_device)
    assert_field_equal(got, want)


def test_evaluate_field_api_and_determinism(cuda_device):
    case = field_case(seed=3, n=1500, num_views=3, site_gaussians=600, extra_points=1000)
    raster = SplatRaster()
    m1, o1 = evaluate_field(raster, case.shape, case.cameras, case.points, cuda_device)
    m2, o2 = evaluate_field(raster, case.shape, case.cameras, case.points, cuda_device)
    assert np.array_equal(m1.view(np.uint32), m2.view(np.uint32)) and np.array_equal(o1, o2)
    wop, wob, _ = oracle_field(case)
    assert np.array_equal(o1, wob) and np.array_equal(m1.view(np.uint32), wop.view(np.uint32))
    f = signed_field(m1, o1)
    assert np.all(f[o1 == 0] == np.float32(-0.5))


def test_unobserved_points(cuda_device):
    case = field_case(seed=4, n=500, num_views=1, site_gaussians=10, extra_points=10)
    # Points behind the single camera (outside its 200 degree field of view) and at its centre.
    pose = case.views[0][1]
    from gofish_b200.scene import quaternion_to_matrix
    x, y, z, w = (float(v) for v in pose[3:])
    R = quaternion_to_matrix(np.array([[w, x, y, z]]))[0]
    centre = -R.T @ pose[:3].astype(np.float64)
    back = centre - 3.0 * R[2]
    pts = np.array([back, centre], dtype=np.float32)
    op, ob, ab = gpu_field(SplatRaster(), case, cuda_device, points=pts)
    assert ob.tolist() == [0, 0] and op.tolist() == [0.0, 0.0] and ab.tolist() == [0, 0]


def test_bisection_rounds_match_oracle(cuda_device):
    case = field_case(seed=12, n=2500, num_views=3, site_gaussians=1000, extra_points=2000)
    rng = np.random.default_rng(0)
    q = case.points.shape[0]
    raster = SplatRaster()
    packed = torch.from_numpy(case.shape.packed_density()).to(cuda_device)
    sigma = torch.from_numpy(np.ascontiguousarray(case.shape.sigma_max)).to(cuda_device)
    token = raster.begin_bisection_table(packed, sigma, torch.from_numpy(case.points).to(cuda_device))
    for cam in case.cameras:
        raster.stage_bisection_camera(token, *camera_inputs(cam, cuda_device))
    raster.seal_bisection_table(token)
    for r in range(8):
        pts = case.points if r == 0 else (case.points + rng.normal(0, 0.02, (q, 3))).astype(np.float32)
        above, observed, exact = raster.evaluate_bisection_round(token, torch.from_numpy(pts).to(cuda_device), r)
        wa, wo, we = oracle_round(case, pts)
        assert np.array_equal(observed.cpu().numpy(), wo)
        assert np.array_equal(above.cpu().numpy(), wa)
        assert np.array_equal(exact.cpu().numpy(), we)
    with pytest.raises(RuntimeError, match="in order"):
        raster.evaluate_bisection_round(token, torch.from_numpy(case.points).to(cuda_device), 8)
    raster.reset_bisection_batch(token)
    above, observed, exact = raster.evaluate_bisection_round(token, torch.from_numpy(case.points).to(cuda_device), 0)
    wa, wo, we = oracle_round(case, case.points)
    assert np.array_equal(above.cpu().numpy(), wa)
    with pytest.raises(RuntimeError, match="after all eight rounds"):
        raster.release_bisection_table(token)
    for r in range(1, 8):
        raster.evaluate_bisection_round(token, torch.from_numpy(case.points).to(cuda_device), r)
    raster.release_bisection_table(token)


def test_exact_half_tie(cuda_device):
    # One isotropic Gaussian of density 1/2 straight ahead of the camera: a
    # point behind it on the optical axis sees alpha = 1/2 exactly.
    case = field_case(seed=2, n=1, num_views=1, site_gaussians=1, extra_points=1)
    pose = case.views[0][1]
    from gofish_b200.scene import quaternion_to_matrix
    x, y, z, w = (float(v) for v in pose[3:])
    R = quaternion_to_matrix(np.array([[w, x, y, z]]))[0]
    centre = -R.T @ pose[:3].astype(np.float64)
    mu = (centre + 2.0 * R[2]).astype(np.float32)
    shape = case.shape
    shape.positions[0] = mu
    shape.density[0] = 0.5
    shape.factor[0] = np.eye(3, dtype=np.float32) * 0.25
    shape.inverse_factor[0] = np.eye(3, dtype=np.float32) * 4.0
    pts = np.array([centre + 3.0 * R[2], centre + 1.0 * R[2]], dtype=np.float32)
    wop, wob, wab = oracle_field(case, pts)
    got = gpu_field(SplatRaster(), case, cuda_device, points=pts)
    assert_field_equal(got, (wop, wob, wab))
    wa, wo, we = oracle_round(case, pts)
    raster = SplatRaster()
    packed = torch.from_numpy(shape.packed_density()).to(cuda_device)
    sigma = torch.from_numpy(np.ascontiguousarray(shape.sigma_max)).to(cuda_device)
    tp = torch.from_numpy(pts).to(cuda_device)
    token = raster.begin_bisection_table(packed, sigma, tp)
    raster.stage_bisection_camera(token, *camera_inputs(case.cameras[0], cuda_device))
    raster.seal_bisection_table(token)
    above, observed, exact = raster.evaluate_bisection_round(token, tp, 0)
    assert np.array_equal(exact.cpu().numpy(), we) and np.array_equal(above.cpu().numpy(), wa)
    if wop[0] == np.float32(0.5):
        assert we[0] == 1
    for r in range(1, 8):
        raster.evaluate_bisection_round(token, tp, r)
    raster.release_bisection_table(token)


def test_refine_crossings_matches_oracle_driver(cuda_device):
    case = field_case(seed=21, n=2000, num_views=3, site_gaussians=800, extra_points=500)
    wop, wob, _ = oracle_field(case)
    f = signed_field(wop, wob)
    solid = np.flatnonzero(f <= 0)
    free = np.flatnonzero(f > 0)
    rng = np.random.default_rng(1)
    e = 3000
    fields = np.empty((e, 2), np.float32)
    sel_a = rng.choice(solid, e)
    sel_b = rng.choice(free, e)
    endpoints = np.stack([case.points[sel_a], case.points[sel_b]], axis=1).astype(np.float32)
    fields[:, 0] = f[sel_a]
    fields[:, 1] = f[sel_b]
    got = refine_crossings(SplatRaster(), case.shape, case.cameras, endpoints, fields, cuda_device)

    class OracleRaster:
        def evaluate_bisection_round(self, token, mid, r):
            wa, wo, we = oracle_round(case, mid.numpy())
            return torch.from_numpy(wa), torch.from_numpy(wo), torch.from_numpy(we)

    s, fr = bracket(torch.from_numpy(endpoints), torch.from_numpy(fields))
    want = bisect(OracleRaster(), 0, s, fr).numpy()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_state_errors(cuda_device):
    case = field_case(seed=9, n=300, num_views=2, site_gaussians=50, extra_points=50)
    raster = SplatRaster()
    packed = torch.from_numpy(case.shape.packed_density()).to(cuda_device)
    sigma = torch.from_numpy(np.ascontiguousarray(case.shape.sigma_max)).to(cuda_device)
    query = torch.from_numpy(case.points).to(cuda_device)
    token = raster.begin_opacity_field(packed, sigma, query)
    with pytest.raises(RuntimeError, match="second opacity field"):
        raster.begin_opacity_field(packed, sigma, query)
    with pytest.raises(RuntimeError, match="no camera"):
        raster.finish_opacity_field(token)
    with pytest.raises(RuntimeError, match="stale"):
        raster.integrate_opacity_field_camera(token + 1, *camera_inputs(case.cameras[0], cuda_device))
    with pytest.raises(RuntimeError, match="before finish"):
        raster.release_opacity_field(token)
    with pytest.raises(RuntimeError, match="stage requires a bisection table"):
        raster.stage_bisection_camera(token, *camera_inputs(case.cameras[0], cuda_device))
    raster.integrate_opacity_field_camera(token, *camera_inputs(case.cameras[0], cuda_device))
    raster.finish_opacity_field(token)
    with pytest.raises(RuntimeError, match="after finish"):
        raster.integrate_opacity_field_camera(token, *camera_inputs(case.cameras[1], cuda_device))
    raster.release_opacity_field(token)
    # Per-pixel origins that differ are refused (one camera centre per view).
    args = list(camera_inputs(case.cameras[0], cuda_device))
    origin = args[1].clone()
    origin[0, 5, 7, 0] = 0.25
    args[1] = origin
    token = raster.begin_opacity_field(packed, sigma, query)
    with pytest.raises(RuntimeError, match="one camera center"):
        raster.integrate_opacity_field_camera(token, *args)
    raster.integrate_opacity_field_camera(token, *camera_inputs(case.cameras[0], cuda_device))
    raster.finish_opacity_field(token)
    raster.release_opacity_field(token)
    # Rolling shutter and differing poses are refused.
    args = list(camera_inputs(case.cameras[0], cuda_device))
    token = raster.begin_opacity_field(packed, sigma, query)
    moved = args[8].clone()
    moved[0] += 0.5
    with pytest.raises(RuntimeError, match="identical"):
        raster.integrate_opacity_field_camera(token, *args[:8], moved)
    raster.integrate_opacity_field_camera(token, *args)
    raster.finish_opacity_field(token)
    raster.release_opacity_field(token)
