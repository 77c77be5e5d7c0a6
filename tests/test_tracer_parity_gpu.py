"""Parity of the sm_100a tracer (through the C ABI) with the CPU oracle.

Bit-exact: projected state, per-particle tile counts, sorted (tile|depth)
keys and particle ids, per-tile ranges, per-pixel hit counts, visibility.
Tolerances: images max-abs <= 1e-3 (PSNR >= 60 dB), hit distance relative
<= 1e-3, gradients relative L2 <= 1e-3.
"""

import numpy as np
import pytest

from tests import harness

pytestmark = pytest.mark.gpu

IMAGE_ATOL = 1e-3
GRAD_RTOL_L2 = 1e-3


def _compare_forward(ref, got):
    np.testing.assert_array_equal(got["proj"].view(np.uint32), ref["proj"].view(np.uint32))
    np.testing.assert_array_equal(got["counts"].astype(np.uint32), ref["counts"])
    np.testing.assert_array_equal(got["keys"].view(np.uint64), ref["keys"])
    np.testing.assert_array_equal(got["ids"].view(np.uint32), ref["ids"])
    np.testing.assert_array_equal(got["ranges"].view(np.uint32), ref["ranges"])
    np.testing.assert_array_equal(got["hit_count"], ref["hit_count"])
    np.testing.assert_array_equal(got["visibility"], ref["visibility"])
    assert np.abs(got["rgba"] - ref["rgba"]).max() <= IMAGE_ATOL
    assert harness.psnr(got["rgba"], ref["rgba"]) >= 60.0
    np.testing.assert_allclose(got["hit_t"], ref["hit_t"], rtol=1e-3, atol=1e-4)


@pytest.mark.parametrize("k", [0, 16])
@pytest.mark.parametrize("key_mode", [0, 1])
def test_cpu_scale_workload_parity(cuda_device, k, key_mode):
    from gofish_b200.scene import workload_cpu_scale

    w = workload_cpu_scale()
    case = harness.make_case(w.scene, w.camera, w.poses[0])
    ref = harness.oracle_forward(case, k, key_mode)
    gpu = harness.GpuTracer(case, k, key_mode, cuda_device)
    got = gpu.forward()
    _compare_forward(ref, got)
    rng = np.random.default_rng(3)
    g_rgba = rng.standard_normal(ref["rgba"].shape).astype(np.float32)
    g_hit = (0.1 * rng.standard_normal(ref["hit_t"].shape)).astype(np.float32)
    gp_ref, gs_ref, _ = harness.oracle_backward(case, ref, k, g_rgba, g_hit)
    gp, gs = gpu.backward(g_rgba, g_hit)
    assert harness.rel_l2(gp, gp_ref) <= GRAD_RTOL_L2
    assert harness.rel_l2(gs, gs_ref) <= GRAD_RTOL_L2


@pytest.mark.parametrize("k", [0, 4, 12, 16, 32])
def test_single_view_sh3_parity(cuda_device, k):
    case = harness.small_case(seed=11, n=30_000, size=320)
    ref = harness.oracle_forward(case, k, 0)
    gpu = harness.GpuTracer(case, k, 0, cuda_device)
    got = gpu.forward()
    _compare_forward(ref, got)
    rng = np.random.default_rng(5)
    g_rgba = rng.uniform(-1, 1, ref["rgba"].shape).astype(np.float32)
    g_hit = np.zeros(ref["hit_t"].shape, dtype=np.float32)
    gp_ref, gs_ref, _ = harness.oracle_backward(case, ref, k, g_rgba, g_hit)
    gp, gs = gpu.backward(g_rgba, g_hit)
    assert harness.rel_l2(gp, gp_ref) <= GRAD_RTOL_L2
    assert harness.rel_l2(gs, gs_ref) <= GRAD_RTOL_L2
    # per-field: position, density, inverse factor
    for sl in (slice(0, 3), slice(3, 4), slice(21, 30)):
        assert harness.rel_l2(gp[:, sl], gp_ref[:, sl]) <= GRAD_RTOL_L2


def test_ragged_resolution_and_partial_mask(cuda_device):
    # 250x170 raster: partial edge tiles, and a tile mask with holes.
    case = harness.small_case(seed=21, n=8_000, size=170, width=250)
    rng = np.random.default_rng(0)
    holes = case.tmask.copy()
    holes[rng.random(holes.shape) < 0.3] = 0
    case = harness.make_case(case.scene, case.camera, case.pose, tmask_override=holes)
    ref = harness.oracle_forward(case, 16, 0)
    gpu = harness.GpuTracer(case, 16, 0, cuda_device)
    got = gpu.forward()
    _compare_forward(ref, got)
    # pixels of dropped tiles keep the initial values
    masked_px = np.kron(1 - holes, np.ones((16, 16), dtype=np.uint8))[:170, :250].astype(bool)
    assert np.all(got["rgba"][masked_px] == 0.0)
    assert np.all(got["hit_t"][masked_px] == 1e6)


@pytest.mark.parametrize("fallback", [False, True])
def test_particles_inside_the_near_radius(cuda_device, fallback):
    case = harness.small_case(seed=3, n=500, size=64, random_pose=False)
    # every particle inside the 0.2 m radial near gate: no valid projection.
    # Without a fallback nothing is admitted; the cone fallback admits them.
    scene = case.scene
    scene.positions[:] = np.array([0.05, 0.0, 0.05], dtype=np.float32)
    case = harness.make_case(scene, case.camera, case.pose)
    ref = harness.oracle_forward(case, 16, 0, fallback=fallback)
    gpu = harness.GpuTracer(case, 16, 0, cuda_device, fallback=fallback)
    got = gpu.forward()
    _compare_forward(ref, got)
    if fallback:
        # every particle is admitted (wide caps); those whose support sphere
        # holds the camera take every retained tile
        assert np.all(ref["counts"] > 0)
        assert int(ref["counts"].max()) == int(case.tmask.sum())
    else:
        assert got["keys"].size == 0 and ref["keys"].size == 0
        assert np.all(got["hit_count"] == 0)


def test_deterministic_repeat(cuda_device):
    case = harness.small_case(seed=5, n=20_000, size=256)
    gpu = harness.GpuTracer(case, 16, 0, cuda_device)
    a = gpu.forward()
    b = gpu.forward()
    for key in ("keys", "ids", "ranges", "rgba", "hit_t", "hit_count"):
        np.testing.assert_array_equal(a[key], b[key])


def test_zero_particles(cuda_device):
    import torch

    case = harness.small_case(seed=3, n=10, size=48, random_pose=False)
    gpu = harness.GpuTracer(case, 16, 0, cuda_device)
    gpu.particles = torch.zeros((0, 32), dtype=torch.float32, device=cuda_device)
    gpu.features = torch.zeros((0, 48), dtype=torch.float32, device=cuda_device)
    got = gpu.forward()
    assert got["keys"].size == 0
    inside = case.valid
    assert np.all(got["rgba"][inside] == 0.0)
    assert np.all(got["hit_t"][inside] == 0.0)
    assert np.all(got["hit_count"] == 0.0)


@pytest.mark.parametrize("k", [4, 16])
def test_kbuffer_exact_ties_from_duplicated_particles(cuda_device, k):
    """Three copies of every Gaussian (same geometry, different opacity and
    colour) meet each ray at exactly the same distance: the k-buffer's tie
    behaviour decides the compositing order and must match the reference
    network (the oracle) exactly."""
    from gofish_b200.scene import Scene

    base = harness.small_case(seed=31, n=4000, size=128)
    sc = base.scene
    rep = 3
    rng = np.random.default_rng(8)
    dens = np.clip(np.repeat(sc.density, rep, axis=0) * rng.uniform(0.5, 1.5, (sc.num * rep, 1)), 0.01, 0.98)
    feats = np.repeat(sc.features, rep, axis=0) + rng.normal(0, 0.5, (sc.num * rep, sc.features.shape[1]))
    dup = Scene(np.repeat(sc.positions, rep, axis=0), np.repeat(sc.rotations, rep, axis=0),
                np.repeat(sc.scales, rep, axis=0), dens.astype(np.float32), feats.astype(np.float32), sc.sh_degree)
    case = harness.make_case(dup, base.camera, base.pose)
    ref = harness.oracle_forward(case, k, 0)
    gpu = harness.GpuTracer(case, k, 0, cuda_device)
    got = gpu.forward()
    _compare_forward(ref, got)
    rng2 = np.random.default_rng(6)
    g_rgba = rng2.uniform(-1, 1, ref["rgba"].shape).astype(np.float32)
    g_hit = np.zeros(ref["hit_t"].shape, dtype=np.float32)
    gp_ref, gs_ref, _ = harness.oracle_backward(case, ref, k, g_rgba, g_hit)
    gp, gs = gpu.backward(g_rgba, g_hit)
    assert harness.rel_l2(gp, gp_ref) <= GRAD_RTOL_L2
    assert harness.rel_l2(gs, gs_ref) <= GRAD_RTOL_L2


@pytest.mark.parametrize("fallback", [True, False])
def test_horizon_particles_cone_fallback(cuda_device, fallback):
    """Large Gaussians around the camera (many straddle the 100 degree horizon
    or hold the camera centre) have no valid projection: the cone fallback
    admits them (single-thread walks and warp-cooperative ones), 'none' drops
    them; either way keys, ranges and hit counts match the oracle bit for bit."""
    case = harness.horizon_case()
    ref = harness.oracle_forward(case, 16, 0, fallback=fallback)
    gpu = harness.GpuTracer(case, 16, 0, cuda_device, fallback=fallback)
    got = gpu.forward()
    _compare_forward(ref, got)
    big = slice(case.scene.num - 300, case.scene.num)
    invalid = ref["proj"][big, 6] <= 1e-6
    assert invalid.sum() > 50
    admitted = ref["counts"][big][invalid]
    if fallback:
        assert (admitted > 0).mean() > 0.5
        assert admitted.max() == case.tmask.sum()  # spheres holding the camera admit every retained tile
    else:
        assert admitted.max() == 0
    rng = np.random.default_rng(8)
    g_rgba = rng.uniform(-1, 1, ref["rgba"].shape).astype(np.float32)
    g_hit = np.zeros(ref["hit_t"].shape, dtype=np.float32)
    gp_ref, gs_ref, _ = harness.oracle_backward(case, ref, 16, g_rgba, g_hit)
    gp, gs = gpu.backward(g_rgba, g_hit)
    assert harness.rel_l2(gp, gp_ref) <= GRAD_RTOL_L2
    assert harness.rel_l2(gs, gs_ref) <= GRAD_RTOL_L2


def _inside_cloud_case(size: int, seed: int = 61):
    """A camera inside the Gaussian shell (on a 2 m ring, looking outward) with
    extra large Gaussians within 0.6 m of it: many particles without a UT
    footprint, wide fallback caps and spheres holding the camera."""
    import math

    from gofish_b200.camera import fisheye_camera, random_kb_coefficients
    from gofish_b200.scene import Scene, look_outward_pose, random_scene

    base = random_scene(40_000, 3, seed)
    rng = np.random.default_rng(seed + 1)
    center = np.array([2.0, 0.0, 0.0])
    m = 400
    d = rng.standard_normal((m, 3))
    d /= np.linalg.norm(d, axis=1, keepdims=True)
    near = (center + d * (0.05 + 0.55 * rng.random((m, 1)))).astype(np.float32)
    scales = np.exp(rng.normal(math.log(0.08), 0.6, size=(m, 3))).astype(np.float32)
    q = rng.standard_normal((m, 4))
    scene = Scene(np.concatenate([base.positions, near]), np.concatenate([base.rotations,
                                                                           (q / np.linalg.norm(q, axis=1,
                                                                                               keepdims=True)).astype(
                                                                               np.float32)]),
                  np.concatenate([base.scales, scales]),
                  np.concatenate([base.density, rng.uniform(0.05, 0.95, (m, 1)).astype(np.float32)]),
                  np.concatenate([base.features, base.features[:m]]), 3)
    cam = fisheye_camera(size, size, 200.0, random_kb_coefficients(rng, 200.0))
    return harness.make_case(scene, cam, look_outward_pose(center, 0.3))


def test_camera_inside_the_cloud_parity(cuda_device):
    """400x400: a 4-level tile cone tree, full trace, forward and backward."""
    case = _inside_cloud_case(400)
    ref = harness.oracle_forward(case, 16, 0)
    no_footprint = (ref["proj"][:, 6] <= 0.0) & (ref["counts"] > 0)
    retained = int(case.tmask.sum())
    assert int(no_footprint.sum()) >= 50
    assert int((ref["counts"][no_footprint] >= retained).sum()) >= 1  # a sphere holding the camera
    assert int(((ref["counts"] > retained // 4) & (ref["counts"] < retained) & no_footprint).sum()) >= 1
    gpu = harness.GpuTracer(case, 16, 0, cuda_device)
    got = gpu.forward()
    _compare_forward(ref, got)
    rng = np.random.default_rng(8)
    g_rgba = rng.standard_normal(ref["rgba"].shape).astype(np.float32)
    g_hit = np.zeros(ref["hit_t"].shape, np.float32)
    gp_ref, gs_ref, _ = harness.oracle_backward(case, ref, 16, g_rgba, g_hit)
    gp, gs = gpu.backward(g_rgba, g_hit)
    assert harness.rel_l2(gp, gp_ref) <= GRAD_RTOL_L2
    assert harness.rel_l2(gs, gs_ref) <= GRAD_RTOL_L2


def test_camera_inside_the_cloud_binning_5_levels(cuda_device):
    """1040x1040: a 5-level tree (65x65 tiles); projection, keys, ids and ranges."""
    import oracle

    case = _inside_cloud_case(1040, seed=62)
    pose = oracle.prepare_pose(case.pose)
    proj, rgb, counts = oracle.project(case.ocam, pose, case.particles, case.features, 3, case.tmask, case.ray_d)
    tr = oracle.tile_rays(case.ocam, pose, case.ray_o, case.ray_d)
    keys, ids, ranges = oracle.bin(case.ocam, pose, case.particles, proj, counts, case.tmask, tr, 0, case.ray_d)
    gpu = harness.GpuTracer(case, 16, 0, cuda_device)
    got = gpu.forward()
    np.testing.assert_array_equal(got["counts"].astype(np.uint32), counts)
    np.testing.assert_array_equal(got["keys"].view(np.uint64), keys)
    np.testing.assert_array_equal(got["ids"].view(np.uint32), ids)
    np.testing.assert_array_equal(got["ranges"].view(np.uint32), ranges)
    assert int(((proj[:, 6] <= 0.0) & (counts > 0)).sum()) >= 50


@pytest.mark.parametrize("k", [0, 16])
@pytest.mark.parametrize("log_capacity", [-1, 6, 0])
def test_backward_paths_agree(cuda_device, k, log_capacity):
    """The backward from the composite log (default capacity), the k-buffer
    replay (no log) and their mix (a 6-entry log: most tiles overflow and are
    replayed) give the oracle's gradients; the forward is unchanged."""
    case = harness.small_case(seed=17, n=20_000, size=256)
    ref = harness.oracle_forward(case, k, 0)
    gpu = harness.GpuTracer(case, k, 0, cuda_device, log_capacity=log_capacity)
    got = gpu.forward()
    _compare_forward(ref, got)
    if log_capacity == 6:
        assert int((ref["hit_count"] > 6).sum()) > 0 and int((ref["hit_count"] <= 6).sum()) > 0
    # a pixel overflows the log only if it hit more particles than the log holds
    cap = 256 if log_capacity == 0 else log_capacity
    h, w = ref["hit_count"].shape
    deep = np.zeros((-(-h // 16) * 16, -(-w // 16) * 16), bool)
    deep[:h, :w] = ref["hit_count"] > cap
    deep_tiles = int(deep.reshape(deep.shape[0] // 16, 16, deep.shape[1] // 16, 16).any(axis=(1, 3)).sum())
    overflow = gpu.raster.log_overflow_tiles()
    if log_capacity < 0:
        assert overflow == 0
    else:
        assert overflow <= deep_tiles
    if log_capacity == 6:
        assert overflow > 0
    rng = np.random.default_rng(19)
    g_rgba = rng.standard_normal(ref["rgba"].shape).astype(np.float32)
    g_hit = (0.1 * rng.standard_normal(ref["hit_t"].shape)).astype(np.float32)
    gp_ref, gs_ref, _ = harness.oracle_backward(case, ref, k, g_rgba, g_hit)
    gp, gs = gpu.backward(g_rgba, g_hit)
    assert harness.rel_l2(gp, gp_ref) <= GRAD_RTOL_L2
    assert harness.rel_l2(gs, gs_ref) <= GRAD_RTOL_L2


@pytest.mark.parametrize("k", [0, 16])
def test_geometric_channels_forward(cuda_device, k):
    """enable_normals: normal sum, sum w t^2, extent, inverse-depth moments,
    quantile depths, max-weight depth and the exact 0.5 crossing equal the
    oracle's (the same hits in the same order with the same arithmetic); the
    colour outputs are unchanged."""
    import oracle

    case = harness.small_case(seed=23, n=20_000, size=256)
    ref = harness.oracle_forward(case, k, 0)
    geo = oracle.render_forward_geo(case.ocam, ref["pose"], case.particles, ref["rgb"], case.ray_o, case.ray_d,
                                    case.tmask, ref["ranges"], ref["ids"], k)
    gpu = harness.GpuTracer(case, k, 0, cuda_device, enable_normals=True)
    got = gpu.forward()
    _compare_forward(ref, got)
    np.testing.assert_array_equal(got["normal"], geo["normal"])
    for name in ("depth_var", "extent", "inv_depth", "inv_depth2"):
        np.testing.assert_array_equal(got[name][..., 0], geo[name], err_msg=name)
    np.testing.assert_array_equal(got["quant"], geo["quant"])
    assert not got["opacity_field"].any()
    valid = case.valid & (ref["rgba"][..., 3] > 0.6)
    assert valid.sum() > 100
    # sanity of the channels: normals are weighted unit vectors, every
    # threshold up to 0.5 and the 0.5 crossing are reached on opaque rays (the
    # quantile depths follow the composite order, which is the sorted tile
    # order, not each ray's own depth order)
    assert np.all(np.linalg.norm(got["normal"][valid], axis=-1) <= ref["rgba"][..., 3][valid] + 1e-4)
    q = got["quant"][valid]
    assert np.all((q[:, 8] > 0) & (q[:, :7] > 0).all(axis=1))
    assert np.count_nonzero(q[:, 9]) > 0


@pytest.mark.parametrize("k,log_capacity", [(16, 0), (16, -1), (16, 6), (0, 0)])
def test_geometric_channels_backward(cuda_device, k, log_capacity):
    """Gradients of the normal sum, sum w t^2, extent and inverse-depth
    moments (with colour and hit-distance gradients) match the oracle's
    restatement of processHitBwd's geometric terms, through the log backward,
    the replay and their mix; the extent's gradient reaches the rotation and
    scale slots of the row gradient."""
    import oracle

    case = harness.small_case(seed=29, n=15_000, size=192)
    ref = harness.oracle_forward(case, k, 0)
    fwd = oracle.render_forward_geo(case.ocam, ref["pose"], case.particles, ref["rgb"], case.ray_o, case.ray_d,
                                    case.tmask, ref["ranges"], ref["ids"], k)
    gpu = harness.GpuTracer(case, k, 0, cuda_device, log_capacity=log_capacity, enable_normals=True)
    got = gpu.forward()
    np.testing.assert_array_equal(got["normal"], fwd["normal"])
    rng = np.random.default_rng(31)
    h, w = case.camera.height, case.camera.width
    grads = {"rgba": rng.standard_normal((h, w, 4)).astype(np.float32),
             "hit_t": (0.1 * rng.standard_normal((h, w))).astype(np.float32),
             "normal": rng.standard_normal((h, w, 3)).astype(np.float32),
             "depth_var": (0.05 * rng.standard_normal((h, w))).astype(np.float32),
             "extent": rng.standard_normal((h, w)).astype(np.float32),
             "inv_depth": rng.standard_normal((h, w)).astype(np.float32),
             "inv_depth2": rng.standard_normal((h, w)).astype(np.float32)}
    rec, shape = oracle.render_backward_geo(case.ocam, ref["pose"], case.particles, ref["rgb"], case.ray_o,
                                            case.ray_d, case.tmask, ref["ranges"], ref["ids"], k, fwd, grads)
    gp_ref, gs_ref = oracle.project_backward(ref["pose"], case.particles, case.features, case.scene.sh_degree,
                                             ref["counts"], rec)
    gp_ref = gp_ref.copy()
    gp_ref[:, 4:8] += shape[:, 0:4]
    gp_ref[:, 8:11] += shape[:, 4:7]
    geometry = {name: grads[name] for name in ("normal", "depth_var", "extent", "inv_depth", "inv_depth2")}
    gp, gs = gpu.backward(grads["rgba"], grads["hit_t"], geometry)
    for cols, name in ((slice(0, 3), "position"), (slice(3, 4), "density"), (slice(4, 8), "rotation"),
                       (slice(8, 11), "scale"), (slice(21, 30), "inverse factor")):
        assert float(np.linalg.norm(gp_ref[:, cols])) > 0.0, name
        assert harness.rel_l2(gp[:, cols], gp_ref[:, cols]) <= GRAD_RTOL_L2, name
    assert harness.rel_l2(gs, gs_ref) <= GRAD_RTOL_L2


def _crowded_tile_case(n: int = 70_000, size: int = 32, seed: int = 23):
    """Opaque Gaussians clustered on the optical axis of a 32x32 fisheye, so
    that each of its four tiles holds more candidates than a 16-bit composite
    log entry can name; no pixel composites 1024 hits."""
    import dataclasses as dc

    from gofish_b200.camera import fisheye_camera, random_kb_coefficients
    from gofish_b200.scene import IDENTITY_POSE, random_scene

    rng = np.random.default_rng(seed)
    scene = random_scene(n, 1, seed)
    pos = np.stack([rng.uniform(-0.2, 0.2, n), rng.uniform(-0.2, 0.2, n), rng.uniform(2.5, 3.5, n)], 1)
    scene = dc.replace(scene, positions=pos.astype(np.float32),
                       scales=rng.uniform(0.25, 0.4, (n, 3)).astype(np.float32),
                       density=rng.uniform(0.9, 0.99, (n, 1)).astype(np.float32))
    cam = fisheye_camera(size, size, 200.0, random_kb_coefficients(rng, 200.0))
    return harness.make_case(scene, cam, IDENTITY_POSE.copy())


@pytest.mark.parametrize("k", [0, 16])
def test_tile_beyond_16bit_log_is_replayed(cuda_device, k):
    """A tile with more than 65,536 candidates cannot be named by the 16-bit
    composite log: the forward flags it for replay even though no pixel
    composited more hits than the (1024-entry) log holds, and the gradients
    are the oracle's."""
    case = _crowded_tile_case()
    ref = harness.oracle_forward(case, k, 0)
    per_tile = np.diff(ref["ranges"].reshape(-1, 2).astype(np.int64), axis=1)[:, 0]
    crowded = int((per_tile > 65_536).sum())
    assert crowded > 0 and int(ref["hit_count"].max()) <= 1024
    gpu = harness.GpuTracer(case, k, 0, cuda_device, log_capacity=1024)
    got = gpu.forward()
    _compare_forward(ref, got)
    assert gpu.raster.log_overflow_tiles() == crowded
    rng = np.random.default_rng(29)
    g_rgba = rng.standard_normal(ref["rgba"].shape).astype(np.float32)
    g_hit = (0.1 * rng.standard_normal(ref["hit_t"].shape)).astype(np.float32)
    gp_ref, gs_ref, _ = harness.oracle_backward(case, ref, k, g_rgba, g_hit)
    gp, gs = gpu.backward(g_rgba, g_hit)
    assert harness.rel_l2(gp, gp_ref) <= GRAD_RTOL_L2
    assert harness.rel_l2(gs, gs_ref) <= GRAD_RTOL_L2
