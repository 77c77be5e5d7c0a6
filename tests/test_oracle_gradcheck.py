"""Finite-difference check of the oracle's backward (the restatement of the
reference's hand-written processHitBwd and SH backward).

A narrow equidistant camera looks at a few large Gaussians that cover every
pixel well inside their support (response > 0.0113, alpha < 0.99, T > 1e-4),
so the loss is smooth in every checked parameter and the tile binning does not
change under the perturbations.
"""

import numpy as np
import pytest

import oracle
import math

from gofish_b200.camera import FisheyeCamera
from gofish_b200.scene import Scene, pack_particles
from tests import harness

IDENTITY = np.array([0, 0, 0, 0, 0, 0, 1], dtype=np.float32)


def _scene(seed):
    rng = np.random.default_rng(seed)
    n = 5
    # Depths 1.5 m apart and near-isotropic shapes (scale ~ 0.25 depth): the
    # per-pixel hit order never changes inside the image, so the k-buffer
    # composite is smooth too.
    depth = 2.0 + 1.5 * rng.permutation(n)
    pos = np.stack([rng.uniform(-0.2, 0.2, n), rng.uniform(-0.2, 0.2, n), depth], 1)
    scales = 0.25 * depth[:, None] * rng.uniform(0.95, 1.05, (n, 3))
    q = rng.standard_normal((n, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    dens = rng.uniform(0.25, 0.55, (n, 1))
    feats = rng.normal(0, 0.3, (n, 3 * 4))
    feats[:, :3] = rng.uniform(-1.0, 1.0, (n, 3))
    return Scene(pos.astype(np.float32), q.astype(np.float32), scales.astype(np.float32), dens.astype(np.float32),
                 feats.astype(np.float32), 1)


def _loss(case, particles, feats, k, w_rgba, w_hit):
    c = harness.Case(case.scene, case.camera, case.pose, particles, feats, case.ray_o, case.ray_d, case.valid,
                     case.tmask)
    f = harness.oracle_forward(c, k, 0)
    return float(np.sum(f["rgba"].astype(np.float64) * w_rgba) + np.sum(f["hit_t"].astype(np.float64) * w_hit)), f


@pytest.mark.parametrize("k", [0, 16])
def test_backward_matches_finite_differences(k):
    # 33x33 raster over +-15 degrees of an equidistant lens whose calibrated
    # domain extends to 100 degrees, so the UT sigma points stay projectable.
    f = 16.5 / math.radians(15.0)
    cam = FisheyeCamera(33, 33, (f, f), (16.5, 16.5), (0.0, 0.0, 0.0, 0.0), float(np.float32(math.radians(100.0))))
    sc = _scene(4)
    case = harness.make_case(sc, cam, IDENTITY)
    rng = np.random.default_rng(9)
    w_rgba = rng.standard_normal((33, 33, 4))
    w_hit = 0.05 * rng.standard_normal((33, 33))
    base, fwd = _loss(case, case.particles, case.features, k, w_rgba, w_hit)
    assert np.all(fwd["hit_count"][case.valid] == sc.num)  # every ray hits every Gaussian
    gp, gs, _ = harness.oracle_backward(case, fwd, k, w_rgba.astype(np.float32), w_hit.astype(np.float32))

    def fd(arr_name, i, j, eps):
        parts = case.particles.copy()
        feats = case.features.copy()
        target = parts if arr_name == "p" else feats
        target[i, j] += eps
        lp, fp = _loss(case, parts, feats, k, w_rgba, w_hit)
        target[i, j] -= 2 * eps
        lm, fm = _loss(case, parts, feats, k, w_rgba, w_hit)
        assert np.array_equal(fp["counts"], fwd["counts"]) and np.array_equal(fm["counts"], fwd["counts"])
        return (lp - lm) / (2 * eps)

    analytic, numeric = [], []
    for i in range(sc.num):
        for j in list(range(0, 4)) + list(range(21, 30)):
            eps = 1e-3 if j < 4 else 2e-3 * max(1.0, abs(float(case.particles[i, j])))
            analytic.append(gp[i, j])
            numeric.append(fd("p", i, j, eps))
        for j in range(12):
            analytic.append(gs[i, j])
            numeric.append(fd("f", i, j, 1e-3))
    a = np.asarray(analytic, dtype=np.float64)
    n = np.asarray(numeric, dtype=np.float64)
    cos = float(a @ n / (np.linalg.norm(a) * np.linalg.norm(n)))
    assert cos > 0.999, cos
    big = np.abs(n) > 0.05 * np.abs(n).max()
    rel = np.abs(a[big] - n[big]) / np.abs(n[big])
    assert np.median(rel) < 1e-2 and rel.max() < 0.1, (np.median(rel), rel.max())
