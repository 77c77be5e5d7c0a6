"""SOF's HEAD4 / MID8 / TAIL64 compositor on the GPU (k_render_fwd_sof,
the composite-log backward and the replay k_render_bwd_sof) against the
oracle's restatement (sofMid8Hierarchy.inl:161-598): hit counts bit for bit,
images max-abs <= 1e-3 and PSNR >= 60 dB, gradients within 1e-3 relative
L2, through the log, the full replay and their mix; with the geometric
channels; and the training entry point with render.splat.hierarchical_sort."""

import dataclasses

import numpy as np
import pytest

import oracle
from tests import harness

pytestmark = pytest.mark.gpu

SOF = oracle.SOF_HIERARCHY


def _dense(seed=9, n=12_000, size=128, grow=4.0):
    case = harness.small_case(seed=seed, n=n, size=size)
    scene = dataclasses.replace(case.scene, scales=case.scene.scales * np.float32(grow))
    return harness.make_case(scene, case.camera, case.pose)


@pytest.mark.parametrize("size,grow", [(128, 4.0), (200, 2.0)])
def test_sof_forward_matches_oracle(cuda_device, size, grow):
    case = _dense(size=size, grow=grow)
    ref = harness.oracle_forward(case, SOF, 0)
    got = harness.GpuTracer(case, SOF, 0, cuda_device).forward()
    harness.compare_forward(ref, got)
    flat = harness.oracle_forward(case, 4, 0)
    assert not np.array_equal(ref["rgba"], flat["rgba"])  # the hierarchy reorders this scene


@pytest.mark.parametrize("log_capacity", [0, -1, 6])
def test_sof_backward_matches_oracle(cuda_device, log_capacity):
    case = _dense(seed=12, size=96)
    ref = harness.oracle_forward(case, SOF, 0)
    gpu = harness.GpuTracer(case, SOF, 0, cuda_device, log_capacity=log_capacity)
    got = gpu.forward()
    harness.compare_forward(ref, got)
    rng = np.random.default_rng(4)
    g_rgba = rng.uniform(-1, 1, ref["rgba"].shape).astype(np.float32)
    g_hit = (0.05 * rng.standard_normal(ref["hit_t"].shape)).astype(np.float32)
    gp_ref, gs_ref, _ = harness.oracle_backward(case, ref, SOF, g_rgba, g_hit)
    gp, gs = gpu.backward(g_rgba, g_hit)
    assert harness.rel_l2(gp, gp_ref) <= 1e-3
    assert harness.rel_l2(gs, gs_ref) <= 1e-3
    if log_capacity == 6:
        assert gpu.raster.log_overflow_tiles() > 0  # most tiles replayed through the hierarchy


def test_sof_geometric_channels(cuda_device):
    case = _dense(seed=14, size=96)
    pose = oracle.prepare_pose(case.pose)
    ref = harness.oracle_forward(case, SOF, 0)
    geo = oracle.render_forward_geo(case.ocam, pose, case.particles, ref["rgb"], case.ray_o, case.ray_d, case.tmask,
                                    ref["ranges"], ref["ids"], SOF)
    gpu = harness.GpuTracer(case, SOF, 0, cuda_device, enable_normals=True)
    got = gpu.forward()
    np.testing.assert_array_equal(got["hit_count"], geo["hit_count"])
    for name in ("normal", "depth_var", "extent", "inv_depth", "inv_depth2"):
        want = geo[name]
        have = got[name].reshape(want.shape)
        assert np.abs(have - want).max() <= 1e-3 * max(1.0, float(np.abs(want).max())), name


def test_training_entry_point_renders_the_hierarchy(cuda_device):
    """Tracer.render with render.splat.hierarchical_sort equals SplatRaster.trace
    with the SOF compositor on the same rows."""
    import torch

    from gofish_b200 import scene as S
    from gofish_b200.batch import Batch
    from gofish_b200.camera import fisheye_camera, random_kb_coefficients
    from gofish_b200.tracer import SceneGaussians, Tracer

    scene = S.random_scene(8000, 3, 33)
    rng = np.random.default_rng(133)
    cam = fisheye_camera(112, 96, 200.0, random_kb_coefficients(rng, 200.0))
    pose = S.pose_world_to_sensor(rng.standard_normal(3) * 0.2, S.random_rotation_quaternion_xyzw(rng))
    o, d, valid = cam.rays()
    batch = Batch(torch.from_numpy(o).to(cuda_device), torch.from_numpy(d).to(cuda_device),
                  torch.from_numpy(S.pose_to_c2w(pose)[None]).float(),
                  intrinsics_OpenCVFisheyeCameraModelParameters=cam.intrinsics(),
                  physical_fov_mask=torch.from_numpy(valid).to(cuda_device), physical_fov_key="sof")
    conf = {"render": {"splat": {"hierarchical_sort": True}, "gofish": {"pixel_footprint_variance": 0.3}}}
    model = SceneGaussians.from_scene(scene, cuda_device, requires_grad=True)
    out = Tracer(conf).render(model, batch, train=True)
    with torch.no_grad():
        rows = harness.view_rows(model, batch, 0.3)
    case = harness.Case(scene, cam, np.asarray(pose, np.float32), rows.cpu().numpy(), scene.features, o[0], d[0],
                        valid[0, :, :, 0], harness.tile_mask(valid[0, :, :, 0]))
    ref = harness.oracle_forward(case, SOF, 0)
    got = torch.cat([out["pred_features"], out["pred_opacity"]], dim=-1)[0].detach().cpu().numpy()
    assert np.abs(got - ref["rgba"]).max() <= 1e-3
    loss = out["pred_features"].sum()
    loss.backward()
    assert model.positions.grad is not None and bool(torch.isfinite(model.positions.grad).all())


def test_sof_opacity_field_matches_oracle(cuda_device):
    """The SOF exact-crossing opacity field (gutRenderer.cuh:297-430) and its
    gradient to the intrinsic Gaussian against the oracle."""
    import torch

    case = _dense(seed=21, size=96)
    gpu = harness.GpuTracer(case, 16, 0, cuda_device, enable_normals=True)
    r = gpu.raster
    out = r.trace(0, True, case.scene.sh_degree, gpu.particles, gpu.features, gpu.ray_o, gpu.ray_d, None, gpu.sensor,
                  0, 1, gpu.pose, gpu.pose, gpu.token)
    field = out[8][..., 0].cpu().numpy()
    quant = out[6].cpu().numpy()
    pose = oracle.prepare_pose(case.pose)
    ref = harness.oracle_forward(case, 16, 0)
    geo = oracle.render_forward_geo(case.ocam, pose, case.particles, ref["rgb"], case.ray_o, case.ray_d, case.tmask,
                                    ref["ranges"], ref["ids"], 16)
    np.testing.assert_array_equal(quant.view(np.uint32), geo["quant"].view(np.uint32))
    want = oracle.sof_opacity(case.ocam, pose, case.particles, case.ray_o, case.ray_d, case.tmask, ref["ranges"],
                              ref["ids"], geo["quant"])
    np.testing.assert_array_equal(field.view(np.uint32), want.view(np.uint32))
    assert (want > 0.1).sum() > 500
    # gradient of sum(w * O) alone
    rng = np.random.default_rng(6)
    w = rng.uniform(-1, 1, field.shape).astype(np.float32)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(cuda_device)  # noqa: E731
    zeros = torch.zeros_like
    pairs = [out[5], None, out[7], None, out[8], dev(w)[..., None], out[6], None, out[4], None, out[9], None,
             out[10], None]
    gp, _gs = r.trace_bwd(0, True, case.scene.sh_degree, gpu.particles, gpu.features, gpu.ray_o, gpu.ray_d, None,
                          gpu.sensor, 0, 1, gpu.pose, gpu.pose, out[0], zeros(out[0]), out[1], zeros(out[1]), *pairs,
                          gpu.token)
    gp = gp.cpu().numpy()
    ref_g = oracle.sof_opacity_backward(case.ocam, pose, case.particles, case.ray_o, case.ray_d, case.tmask,
                                        ref["ranges"], ref["ids"], geo["quant"], want, w)
    for got, exp in ((gp[:, 0:3], ref_g[:, 0:3]), (gp[:, 4:8], ref_g[:, 4:8]), (gp[:, 8:11], ref_g[:, 8:11]),
                     (gp[:, 11], ref_g[:, 3])):
        assert harness.rel_l2(got, exp) <= 1e-3
    assert np.abs(ref_g[:, 3]).max() > 0
