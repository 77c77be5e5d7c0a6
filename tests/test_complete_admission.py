"""Complete admission (render.gofish.complete_admission): every particle of
density >= 1/255 is admitted by the conservative cone test of its support
sphere (the sphere of radius sigma_max sqrt(min(9, 2 ln(rho / alpha_min)))
around its mean holds every point its hit test can pass on), so no pixel's hit
is missed -- the property the reference's certified admission guarantees
(gutRenderer.cu:794-1521), here by an own construction rather than its
interval-certified route set.

CPU: the oracle's complete binning misses no brute-force hit on scenes where
the projected-footprint admission misses some, including particles beyond
the 180 deg horizon and holding the camera.  GPU (marked): keys, ids, ranges,
counts and hit counts bit for bit against the oracle in that mode."""

import numpy as np
import pytest

import oracle
from tests import harness

CASES = {
    "dense": lambda: harness.small_case(seed=5, n=3000, size=64),
    "horizon": lambda: harness.horizon_case(n=2000, big=150, size=64),
}


@pytest.mark.parametrize("name", sorted(CASES))
def test_oracle_complete_admission_misses_no_hit(name):
    case = CASES[name]()
    pose = oracle.prepare_pose(case.pose)
    fast = harness.oracle_forward(case, 16, 0)
    complete = harness.oracle_forward(case, 16, 0, complete=True)
    missed_fast, _ = oracle.admission_misses(case.ocam, pose, case.particles, case.ray_o, case.ray_d, case.tmask,
                                             fast["ranges"], fast["ids"])
    missed, examples = oracle.admission_misses(case.ocam, pose, case.particles, case.ray_o, case.ray_d, case.tmask,
                                               complete["ranges"], complete["ids"])
    assert missed_fast > 0  # the projected footprint is not complete
    assert missed == 0, examples
    # the complete list holds every pixel hit, so compositing it cannot composite less
    assert complete["hit_count"].sum() >= fast["hit_count"].sum()


@pytest.mark.gpu
@pytest.mark.parametrize("name", sorted(CASES))
@pytest.mark.parametrize("key_mode", [0, 1])
def test_gpu_complete_admission_matches_oracle(cuda_device, name, key_mode):
    case = CASES[name]()
    ref = harness.oracle_forward(case, 16, key_mode, complete=True)
    got = harness.GpuTracer(case, 16, key_mode, cuda_device, complete=True).forward()
    harness.compare_forward(ref, got)
    rng = np.random.default_rng(2)
    g_rgba = rng.uniform(-1, 1, ref["rgba"].shape).astype(np.float32)
    g_hit = np.zeros(ref["hit_t"].shape, np.float32)
    gp_ref, gs_ref, _ = harness.oracle_backward(case, ref, 16, g_rgba, g_hit)
    gp, gs = harness.GpuTracer(case, 16, key_mode, cuda_device, complete=True).backward_after_forward(g_rgba, g_hit)
    assert harness.rel_l2(gp, gp_ref) <= 1e-3 and harness.rel_l2(gs, gs_ref) <= 1e-3
