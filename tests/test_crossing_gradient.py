"""Gradient of the exact 0.5-crossing depth t* (the quantile channel 8,
``pred_crossing``) by the implicit function theorem (gaussianParticles.cuh:
934-986, rayPayloadBackward.cuh:122-128): t* solves T_before (1 - alpha_k(t))
= 1/2 inside the crossing Gaussian k, so dL/dtheta = g dO/dtheta at t* with
g = -(dL/dt*) / Odot*.

CPU: the oracle's backward against central finite differences of the
oracle's own t* (the scene of the gradient check: every ray hits every
Gaussian, the binning and the crossing Gaussian do not change under the
perturbations).  GPU (marked): the CUDA backward against the oracle's."""

import math

import numpy as np
import pytest

import oracle
from gofish_b200.camera import FisheyeCamera
from tests import harness
from tests.test_oracle_gradcheck import IDENTITY, _scene

# packed-row slots whose gradient the render record carries: position,
# density, and B^-1 (record slots 4-12)
SLOTS = list(range(0, 4)) + list(range(21, 30))


def _case():
    f = 16.5 / math.radians(15.0)
    cam = FisheyeCamera(33, 33, (f, f), (16.5, 16.5), (0.0, 0.0, 0.0, 0.0), float(np.float32(math.radians(100.0))))
    sc = _scene(4)
    sc.density[:] = np.clip(sc.density * 1.6, 0.0, 0.9)  # crossings well inside the first hits
    return harness.make_case(sc, cam, IDENTITY)


def _geo(case, particles, fwd, k):
    return oracle.render_forward_geo(case.ocam, fwd["pose"], particles, fwd["rgb"], case.ray_o, case.ray_d,
                                     case.tmask, fwd["ranges"], fwd["ids"], k)


def _record_grad(case, fwd, geo, k, w):
    g_quant = np.zeros(geo["quant"].shape, np.float32)
    g_quant[..., 8] = w
    zeros = {"rgba": np.zeros(geo["rgba"].shape, np.float32), "hit_t": np.zeros(geo["hit_t"].shape, np.float32),
             "quant": g_quant}
    rec, _shape = oracle.render_backward_geo(case.ocam, fwd["pose"], case.particles, fwd["rgb"], case.ray_o,
                                             case.ray_d, case.tmask, fwd["ranges"], fwd["ids"], k, geo, zeros)
    return rec, g_quant


def _crossing_weights(geo, seed):
    valid = (np.abs(geo["quant"][..., 9]) > 1e-8) & (geo["quant"][..., 8] > 0)
    w = np.random.default_rng(seed).standard_normal(valid.shape) * valid
    return valid, w


@pytest.mark.parametrize("k", [0, 16])
def test_crossing_gradient_matches_finite_differences(k):
    case = _case()
    fwd = harness.oracle_forward(case, k, 0)
    geo = _geo(case, case.particles, fwd, k)
    valid, _ = _crossing_weights(geo, 5)
    assert valid.sum() > 200, valid.sum()

    def crossing(parts):
        g = _geo(case, parts, fwd, k)
        ok = (np.abs(g["quant"][..., 9]) > 1e-8) & (g["quant"][..., 8] > 0)
        return g["quant"][..., 8].astype(np.float64), ok

    # t* at +-eps for every checked slot; a pixel whose crossing flips to
    # another Gaussian (or loses it) under some perturbation is not smooth
    # there and is left out of the loss
    maps, stable = [], valid.copy()
    for i in range(case.particles.shape[0]):
        for j in SLOTS:
            eps = 1e-3 if j < 4 else 2e-3 * max(1.0, abs(float(case.particles[i, j])))
            p = case.particles.copy()
            p[i, j] += eps
            tp, okp = crossing(p)
            p[i, j] -= 2 * eps
            tm, okm = crossing(p)
            stable &= okp & okm
            maps.append((i, j, eps, tp, tm))
    t0 = geo["quant"][..., 8].astype(np.float64)
    for _, _, _, tp, tm in maps:  # a kink or jump shows as curvature against the slope
        stable &= np.abs(tp + tm - 2.0 * t0) <= 0.2 * np.abs(tp - tm) + 1e-5
    assert stable.sum() > 0.8 * valid.sum(), (stable.sum(), valid.sum())
    w = np.random.default_rng(5).standard_normal(valid.shape) * stable
    rec, _ = _record_grad(case, fwd, geo, k, w)
    # the record's slots: position 0-2, density 3, B^-1 4-12
    rec_slot = {0: 0, 1: 1, 2: 2, 3: 3, **{21 + j: 4 + j for j in range(9)}}
    analytic = np.asarray([rec[i, rec_slot[j]] for i, j, _, _, _ in maps], dtype=np.float64)
    numeric = np.asarray([np.sum((tp - tm) * w) / (2 * eps) for _, _, eps, tp, tm in maps], dtype=np.float64)
    cos = float(analytic @ numeric / (np.linalg.norm(analytic) * np.linalg.norm(numeric)))
    assert cos > 0.999, cos
    big = np.abs(numeric) > 0.05 * np.abs(numeric).max()
    rel = np.abs(analytic[big] - numeric[big]) / np.abs(numeric[big])
    assert np.median(rel) < 1e-2 and rel.max() < 0.1, (np.median(rel), rel.max())


def test_crossing_gradient_is_zero_without_its_channel():
    case = _case()
    fwd = harness.oracle_forward(case, 16, 0)
    geo = _geo(case, case.particles, fwd, 16)
    rec, _ = _record_grad(case, fwd, geo, 16, np.zeros(geo["hit_t"].shape))
    assert not rec.any()


@pytest.mark.gpu
@pytest.mark.parametrize("k,log_capacity", [(16, 0), (16, -1), (0, 0)])
def test_gpu_crossing_gradient_matches_oracle(cuda_device, k, log_capacity):
    """Through SplatRaster.trace_bwd (the log backward, the replay): the
    crossing depth's gradient reaches the position, density and B^-1 slots
    as the oracle's implicit-function backward says."""
    case = harness.small_case(seed=29, n=15_000, size=192)
    ref = harness.oracle_forward(case, k, 0)
    geo = _geo(case, case.particles, ref, k)
    gpu = harness.GpuTracer(case, k, 0, cuda_device, log_capacity=log_capacity, enable_normals=True)
    got = gpu.forward()
    np.testing.assert_array_equal(got["quant"], geo["quant"])
    valid, w = _crossing_weights(geo, 7)
    assert valid.sum() > 1000, valid.sum()
    rec, g_quant = _record_grad(case, ref, geo, k, w.astype(np.float32))
    gp_ref, _ = oracle.project_backward(ref["pose"], case.particles, case.features, case.scene.sh_degree,
                                        ref["counts"], rec)
    zero_rgba = np.zeros(geo["rgba"].shape, np.float32)
    zero_hit = np.zeros(geo["hit_t"].shape, np.float32)
    gp, _ = gpu.backward(zero_rgba, zero_hit, {"quant": g_quant})
    for cols, name in ((slice(0, 3), "position"), (slice(3, 4), "density"), (slice(21, 30), "inverse factor")):
        assert float(np.linalg.norm(gp_ref[:, cols])) > 0.0, name
        assert harness.rel_l2(gp[:, cols], gp_ref[:, cols]) <= 1e-3, name
