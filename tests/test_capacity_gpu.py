"""Sizing of the tile-intersection keys without host synchronization.

The first forward of a tracer reads its intersection count after the count
scan; later forwards with the same particle count and raster reserve 1.5x the
largest count seen and leave the count on the device.  These tests check that
speculative forwards give the exact forward's results bit for bit, that a
forward whose count outgrows the reservation renders nothing and is reported
as a capacity error by the next call, and that the frame renders correctly
once it is traced again.
"""

import numpy as np
import pytest
import torch

from gofish_b200._native import NativeError
from tests import harness

pytestmark = pytest.mark.gpu


def _grow(particles: np.ndarray, factor: float) -> np.ndarray:
    """Rows with every support scaled by ``factor`` (B * f, B^-1 / f)."""
    rows = particles.copy()
    rows[:, 12:21] *= np.float32(factor)
    rows[:, 21:30] /= np.float32(factor)
    return rows


def test_speculative_forwards_match_the_exact_one(cuda_device):
    case = harness.small_case(seed=5, n=20_000, size=256)
    ref = harness.oracle_forward(case, 16, 0)
    spec = harness.GpuTracer(case, 16, 0, cuda_device)
    for _ in range(3):  # the first forward reads its count, the others do not
        got = spec.forward()
        harness.compare_forward(ref, got)
    st = spec.raster.stats()
    assert st.total_forwards == 3 and st.total_intersections == 3 * ref["keys"].size
    rng = np.random.default_rng(3)
    g_rgba = rng.uniform(-1, 1, ref["rgba"].shape).astype(np.float32)
    g_hit = np.zeros(ref["hit_t"].shape, dtype=np.float32)
    gp_ref, gs_ref, _ = harness.oracle_backward(case, ref, 16, g_rgba, g_hit)
    gp, gs = spec.backward(g_rgba, g_hit)
    assert harness.rel_l2(gp, gp_ref) <= 1e-3 and harness.rel_l2(gs, gs_ref) <= 1e-3


def test_exact_mode_matches_speculative(cuda_device):
    case = harness.small_case(seed=6, n=10_000, size=192)
    spec = harness.GpuTracer(case, 16, 0, cuda_device)
    spec.forward()
    a = spec.forward()
    exact = harness.GpuTracer(case, 16, 0, cuda_device)
    from gofish_b200.splat_raster import SplatRaster

    exact.raster = SplatRaster({"render": {"splat": {"k_buffer_size": 16, "intersection_capacity": "exact"},
                                           "enable_hitcounts": True}})
    exact.raster.register_physical_tile_mask(torch.from_numpy(case.tmask).to(cuda_device), exact.token)
    b = exact.forward()
    for key in ("keys", "ids", "ranges", "rgba", "hit_t", "hit_count"):
        np.testing.assert_array_equal(a[key], b[key])


def test_overflow_is_reported_and_the_frame_renders_again(cuda_device):
    case = harness.small_case(seed=8, n=20_000, size=256)
    gpu = harness.GpuTracer(case, 16, 0, cuda_device)
    first = gpu.forward()
    n_small = first["keys"].size
    big = harness.make_case(case.scene, case.camera, case.pose)
    big.particles = _grow(case.particles, 6.0)
    ref = harness.oracle_forward(big, 16, 0)
    # beyond the reservation: 1.5x the largest count seen, at least 65,536
    assert ref["keys"].size > max(1.5 * n_small, 65_536) * 1.1
    gpu.particles.copy_(torch.from_numpy(big.particles).to(cuda_device))
    out = gpu.raster.trace(0, False, case.scene.sh_degree, gpu.particles, gpu.features, gpu.ray_o, gpu.ray_d, None,
                           gpu.sensor, 0, 1, gpu.pose, gpu.pose, gpu.token)
    torch.cuda.synchronize(cuda_device)
    # the overflowed forward composited nothing
    assert float(out[0].abs().max()) == 0.0
    assert float(out[2].abs().max()) == 0.0
    with pytest.raises(NativeError, match="render that frame again"):
        gpu.raster.stats()
    # the error is reported once; the capacity has grown and the frame traces correctly
    got = gpu.forward()
    harness.compare_forward(ref, got)
