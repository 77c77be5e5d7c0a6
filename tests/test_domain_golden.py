"""The per-pixel camera rays that feed every tracer, oracle and benchmark case
against golden vectors made by the reference's own Kannala-Brandt domain
(gofish/camera/domain.py:37-113; tests/golden/make_domain_golden.py).

Bit for bit: ``monotone_branch_limit`` (float64) over 28 polynomials
(equidistant, equisolid, the workloads' draws, folding ones), and the float32
unit rays and validity flags of ``first_branch_rays`` at sampled pixel
centres of the C0, C1, C3, C4 and ragged test cameras, both through
``first_branch_rays`` and through ``FisheyeCamera.rays()`` (the full ray
table the GPU and the oracle read).  The oracle's forward model is pinned to
the same rays: projecting a golden ray lands on its pixel centre.
"""

from pathlib import Path

import numpy as np
import pytest

from gofish_b200.camera import FisheyeCamera, first_branch_rays, monotone_branch_limit

GOLDEN = Path(__file__).resolve().parent / "golden" / "domain_golden.npz"


@pytest.fixture(scope="module")
def golden():
    return np.load(GOLDEN)


def _camera(golden, name) -> FisheyeCamera:
    c = golden[f"{name}/camera"]
    return FisheyeCamera(int(c[0]), int(c[1]), (float(c[2]), float(c[3])), (float(c[4]), float(c[5])),
                         tuple(float(v) for v in c[6:10]), float(c[10]))


def test_monotone_branch_limit_matches_reference(golden):
    coeffs = golden["limit_coefficients"]
    want = golden["limit_values"]
    got = np.asarray([monotone_branch_limit(tuple(k)) for k in coeffs], dtype=np.float64)
    np.testing.assert_array_equal(got.view(np.uint64), want.view(np.uint64))
    # the set holds folding polynomials as well as pi-limited ones
    assert (want < np.nextafter(np.pi, 0.0)).any() and (want == np.nextafter(np.pi, 0.0)).any()


@pytest.mark.parametrize("name", ["equidistant_200_320", "kb_200_1600", "equisolid_205_2560",
                                  "equidistant_200_800", "kb_200_250x170"])
def test_first_branch_rays_match_reference(golden, name):
    cam = _camera(golden, name)
    pix = golden[f"{name}/pixels"].astype(np.float64)
    rays, valid = first_branch_rays(pix + 0.5, cam.focal, cam.principal, cam.coefficients, cam.max_angle)
    np.testing.assert_array_equal(valid.astype(np.uint8), golden[f"{name}/valid"])
    np.testing.assert_array_equal(rays.view(np.uint32), golden[f"{name}/rays"].view(np.uint32))
    # both valid and invalid (forward placeholder) pixels are covered, except
    # on cameras whose raster lies entirely inside the image circle
    assert golden[f"{name}/valid"].any()


@pytest.mark.parametrize("name", ["equidistant_200_320", "kb_200_250x170"])
def test_ray_table_matches_reference(golden, name):
    """FisheyeCamera.rays() -- the [1,H,W,3] table given to the GPU and the
    oracle -- holds the reference's rays at every sampled pixel."""
    cam = _camera(golden, name)
    _o, d, valid = cam.rays()
    pix = golden[f"{name}/pixels"]
    got = d[0, pix[:, 1], pix[:, 0]]
    np.testing.assert_array_equal(got.view(np.uint32), golden[f"{name}/rays"].view(np.uint32))
    np.testing.assert_array_equal(valid[0, pix[:, 1], pix[:, 0], 0].astype(np.uint8), golden[f"{name}/valid"])


@pytest.mark.parametrize("name", ["equidistant_200_320", "kb_200_1600", "equisolid_205_2560"])
def test_oracle_projection_inverts_reference_rays(golden, name):
    """The oracle's fisheye projection (cameraProjections.cuh:124-152)
    maps each valid golden ray back onto its pixel centre."""
    import oracle

    cam = _camera(golden, name)
    ocam = oracle.camera(1, cam.width, cam.height, cam.principal, cam.focal, cam.coefficients, cam.max_angle)
    pose = oracle.prepare_pose(np.array([0, 0, 0, 0, 0, 0, 1], np.float32))
    valid = golden[f"{name}/valid"].astype(bool)
    rays = golden[f"{name}/rays"][valid]
    pix = golden[f"{name}/pixels"][valid].astype(np.float64) + 0.5
    # one particle per ray, 10 m out along it; the projected centre is proj[:, 0:2]
    n = rays.shape[0]
    parts = np.zeros((n, 32), np.float32)
    parts[:, 0:3] = rays * np.float32(10.0)
    parts[:, 3] = 0.9
    parts[:, 4] = 1.0
    parts[:, 8:11] = 1e-3
    eye = np.eye(3, dtype=np.float32).reshape(9) * np.float32(1e-3)
    parts[:, 12:21] = eye
    parts[:, 21:30] = np.eye(3, dtype=np.float32).reshape(9) * np.float32(1e3)
    sh = np.zeros((n, 3), np.float32)
    mask = np.ones(((cam.height + 15) // 16, (cam.width + 15) // 16), np.uint8)
    proj, _rgb, _counts = oracle.project(ocam, pose, parts, sh, 0, mask)
    # a particle whose sigma points cross the maximum angle has no projection
    ok = proj[:, 5] > 0
    assert ok.mean() > 0.9
    err = np.abs(proj[ok, 0:2].astype(np.float64) - pix[ok])
    assert float(err.max()) < 2e-3 * max(cam.width, cam.height) / 320.0
