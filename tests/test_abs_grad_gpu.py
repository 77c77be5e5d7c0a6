"""The densification statistic of the backward (SplatRaster
set_exact_screen_absgrad_map / collect_abs_grad, splatRaster.cpp:515-531,
628-698; read by threedgrut/strategy/gs.py:88-96,306-313) against the
oracle: per composited hit, |M g| (screen, [N,2]) or |g| (world, [N,3]) of
the hit's position gradient g, summed per particle.  Relative L2 <= 1e-3,
the gradients' tolerance, on the composite-log backward, the k-buffer replay
and SOF's hierarchy."""

from __future__ import annotations

import numpy as np
import pytest

import oracle
from tests import harness

GRAD_RTOL_L2 = 1e-3


def _case_and_grads(seed: int):
    case = harness.small_case(seed=seed, n=20_000, size=256)
    rng = np.random.default_rng(seed + 1)
    h, w = case.ray_d.shape[:2]
    g_rgba = rng.standard_normal((h, w, 4)).astype(np.float32)
    g_hit = (0.1 * rng.standard_normal((h, w))).astype(np.float32)
    return case, g_rgba, g_hit


@pytest.mark.gpu
@pytest.mark.parametrize("k,log_capacity", [(16, 0), (16, -1), (oracle.SOF_HIERARCHY, 0)])
def test_screen_statistic_matches_the_oracle(cuda_device, k, log_capacity):
    import torch

    case, g_rgba, g_hit = _case_and_grads(41)
    n = case.particles.shape[0]
    mapping = np.random.default_rng(43).standard_normal((n, 2, 3)).astype(np.float32)
    gpu = harness.GpuTracer(case, k, 0, cuda_device, log_capacity=log_capacity)
    gpu.forward()
    gpu.raster.set_exact_screen_absgrad_map(torch.from_numpy(mapping).to(cuda_device))
    with pytest.raises(RuntimeError, match="armed twice"):
        gpu.raster.set_exact_screen_absgrad_map(torch.from_numpy(mapping).to(cuda_device))
    gpu.backward(g_rgba, g_hit)
    got = gpu.raster.collect_abs_grad().cpu().numpy()
    ref_fwd = harness.oracle_forward(case, k, 0)
    with oracle.abs_grad(n, "screen", mapping) as ref:
        harness.oracle_backward(case, ref_fwd, k, g_rgba, g_hit)
    assert got.shape == (n, 2) and (got >= 0).all()
    assert (ref.out > 0).sum() > 1000
    assert harness.rel_l2(got, ref.out) <= GRAD_RTOL_L2
    # the next backward was not armed: nothing to collect
    gpu.forward()
    gpu.backward(g_rgba, g_hit)
    with pytest.raises(RuntimeError, match="not armed"):
        gpu.raster.collect_abs_grad()


@pytest.mark.gpu
def test_world_statistic_matches_the_oracle(cuda_device):
    case, g_rgba, g_hit = _case_and_grads(47)
    n = case.particles.shape[0]
    gpu = harness.GpuTracer(case, 16, 0, cuda_device,
                            strategy={"densify": {"generic_camera_absgrad": False}})
    gpu.forward()
    gpu.backward(g_rgba, g_hit)
    got = gpu.raster.collect_abs_grad().cpu().numpy()
    ref_fwd = harness.oracle_forward(case, 16, 0)
    with oracle.abs_grad(n, "world") as ref:
        harness.oracle_backward(case, ref_fwd, 16, g_rgba, g_hit)
    assert got.shape == (n, 3)
    assert harness.rel_l2(got, ref.out) <= GRAD_RTOL_L2
    with pytest.raises(RuntimeError, match="generic_camera_absgrad"):
        gpu.raster.set_exact_screen_absgrad_map(gpu.particles.new_zeros((n, 2, 3)))
