"""Parity with the oracle at the benchmarked sizes.

* Single-view training view (1M Gaussians SH3, Kannala-Brandt 200 deg
  1600x1600, seed 1235, per-view full shape with gamma = 0.3, K = 16): the
  rows Tracer.render traces (product shape kernels) are given to the GPU
  tracer and to the oracle.  Over the whole frame, bit for bit: projected
  state, per-particle tile counts, (tile|depth) keys, particle ids, tile
  ranges, visibility and per-pixel hit counts -- including every particle
  admitted by the cone fallback.  Image max-abs <= 1e-3 and PSNR >= 60 dB,
  hit distance relative <= 1e-3; particle and SH gradients of a full-frame
  output gradient within 1e-3 relative L2.
* Mesh opacity query: 1M of the 27M sites of the 3M-Gaussian scene from 4
  of its 32 views: opacity bits, observed and above flags against the
  oracle's indexed field (itself equal to its brute force,
  tests/test_oracle_field_index.py).
* High-resolution inference orbit frame (6M Gaussians SH3, 5% large beside
  the camera path, equisolid 205 deg 2560x2560, K = 32, physical-mip filter
  from all 240 frames, per-frame full shape): binning bit for bit over the
  whole frame, the image on bands of tile rows through the centre and the
  rim.

Each case holds a few GB on the device (the 6M-Gaussian frame's 347M
intersections about 10 GB) and takes tens of seconds of host time for the
oracle.
"""

import numpy as np
import pytest
import torch

import oracle
from gofish_b200 import scene as S
from gofish_b200.batch import Batch
from gofish_b200.tracer import SceneGaussians
from oracle import full_shape as fs
from tests import harness

pytestmark = pytest.mark.gpu

GAMMA = 0.3
GRAD_RTOL_L2 = 1e-3


def _batch(cam, pose, rays, mask, key):
    c2w = torch.from_numpy(S.pose_to_c2w(pose)[None]).float()
    return Batch(rays[0], rays[1], c2w, intrinsics_OpenCVFisheyeCameraModelParameters=cam.intrinsics(),
                 physical_fov_mask=mask, physical_fov_key=key)


@pytest.fixture(scope="module")
def single_view(cuda_device):
    w = S.workload_single_view()
    cam, pose = w.camera, w.poses[0]
    o, d, valid = cam.rays()
    rays = (torch.from_numpy(o).to(cuda_device), torch.from_numpy(d).to(cuda_device))
    mask = torch.from_numpy(valid).to(cuda_device)
    model = SceneGaussians.from_scene(w.scene, cuda_device, requires_grad=False)
    batch = _batch(cam, pose, rays, mask, "kb-200-1600")
    with torch.no_grad():
        packed = harness.view_rows(model, batch, GAMMA)
    case = harness.Case(w.scene, cam, np.asarray(pose, np.float32), packed.cpu().numpy(), w.scene.features, o[0],
                        d[0], valid[0, :, :, 0], harness.tile_mask(valid[0, :, :, 0]))
    gpu = harness.GpuTracer(case, 16, 0, cuda_device)
    got = gpu.forward()
    ref = harness.oracle_forward(case, 16, 0)
    return dict(w=w, case=case, gpu=gpu, got=got, ref=ref, model=model, batch=batch)


def test_single_view_full_frame_forward(single_view):
    got, ref = single_view["got"], single_view["ref"]
    harness.compare_forward(ref, got)
    # the benchmarked view: millions of intersections, tens of thousands of
    # particles admitted only by the cone fallback, composited deep pixels
    assert ref["keys"].size > 3_000_000
    no_footprint = ref["proj"][:, 6] == 0.0
    fallback = np.flatnonzero(no_footprint & (ref["counts"] > 0))
    assert fallback.size > 10_000
    gpu_fallback = np.flatnonzero((got["proj"][:, 6] == 0.0) & (got["counts"] > 0))
    np.testing.assert_array_equal(gpu_fallback, fallback)
    assert float(ref["hit_count"].max()) > 100


def test_single_view_full_frame_backward(single_view):
    got, ref, case, gpu = single_view["got"], single_view["ref"], single_view["case"], single_view["gpu"]
    rng = np.random.default_rng(1235)
    target = rng.random(ref["rgba"].shape[:2] + (3,), dtype=np.float32)
    # the gradient of the benchmark's L1 loss on colour, plus a hit-distance term
    g_rgba = np.zeros_like(ref["rgba"])
    g_rgba[..., :3] = np.sign(ref["rgba"][..., :3] - target) * case.valid[..., None]
    g_hit = (1e-3 * rng.standard_normal(ref["hit_t"].shape)).astype(np.float32) * case.valid
    gp_ref, gs_ref, _ = harness.oracle_backward(case, ref, 16, g_rgba, g_hit)
    gp, gs = gpu.backward(g_rgba, g_hit)
    assert harness.rel_l2(gp, gp_ref) <= GRAD_RTOL_L2
    assert harness.rel_l2(gs, gs_ref) <= GRAD_RTOL_L2
    for sl in (slice(0, 3), slice(3, 4), slice(12, 21), slice(21, 30)):
        assert harness.rel_l2(gp[:, sl], gp_ref[:, sl]) <= GRAD_RTOL_L2
    del got


def test_single_view_shape_rows(single_view, cuda_device):
    """The traced rows against the float64 full-shape oracle on a 100k-row sample."""
    from gofish_b200 import view_observation_filter as vof

    w, model, batch = single_view["w"], single_view["model"], single_view["batch"]
    packed = single_view["case"].particles
    rows = np.sort(np.random.default_rng(5).choice(w.scene.num, 100_000, replace=False))
    with torch.no_grad():
        q6, jac, ob = vof.current_view_q6(model.positions, batch, GAMMA)
    q6, jac, ob = q6.cpu().numpy()[rows], jac.cpu().numpy()[rows], ob.cpu().numpy()[rows]
    cam = w.camera
    c2w = S.pose_to_c2w(w.poses[0])
    J, chart = fs.view_jacobian(w.scene.positions[rows], c2w, True, cam.focal, cam.coefficients, cam.max_angle)
    Q, want_ob = fs.minimum_norm_q(J, chart, GAMMA)
    assert np.array_equal(ob, want_ob) and want_ob.mean() > 0.3
    rel = np.abs(jac[ob] - J[ob]) / np.abs(J[ob]).max(axis=(1, 2))[:, None, None]
    assert rel.max() < 1e-5
    Qg = q6[:, [0, 1, 2, 1, 3, 4, 2, 4, 5]].reshape(-1, 3, 3)
    scale = model.get_scale().cpu().numpy()[rows]
    quat = model.get_rotation().cpu().numpy()[rows]
    dens = model.get_density().cpu().numpy()[rows, 0]
    _C, B, Bi, _m, d = fs.full_shape(scale, quat, dens, Qg, jac, ob, GAMMA, True, "exact")
    p = packed[rows].astype(np.float64)
    np.testing.assert_allclose(p[:, 3], d, rtol=2e-6)
    for got, want in ((p[:, 12:21].reshape(-1, 3, 3), B), (p[:, 21:30].reshape(-1, 3, 3), Bi)):
        assert (np.abs(got - want) / np.abs(want).max(axis=(1, 2))[:, None, None]).max() < 2e-6


# ----------------------------------------------------------------------------- inference orbit frame
@pytest.fixture(scope="module")
def orbit_frame(cuda_device):
    from gofish_b200.inference import FrozenGaussians, InferenceTracer
    from gofish_b200.physical_mip import compute_filter, pack_camera_table

    w = S.workload_inference()
    o, d, valid = w.camera.rays()
    cams, frames = S.mip_camera_records(w.camera, w.poses, valid[0, :, :, 0])
    table = pack_camera_table(cams, frames, cuda_device)
    filter_3d, _ = compute_filter(torch.from_numpy(w.scene.positions).to(cuda_device), table, 0.2)
    model = FrozenGaussians.from_scene(w.scene, cuda_device, filter_3d)
    rays = (torch.from_numpy(o).to(cuda_device), torch.from_numpy(d).to(cuda_device))
    mask = torch.from_numpy(valid).to(cuda_device)
    conf = {"render": {"splat": {"k_buffer_size": 32}, "gofish": {"pixel_footprint_variance": GAMMA}}}
    tracer = InferenceTracer(conf, model)
    frame = 0
    out = tracer.render(_batch(w.camera, w.poses[frame], rays, mask, "equisolid-205-2560"))
    inter = tracer.wrapper.copy_intermediates(cuda_device)
    torch.cuda.synchronize(cuda_device)
    got = {k: v.cpu().numpy() for k, v in inter.items()}
    del inter
    got["rgba"] = torch.cat([out["pred_features"], out["pred_opacity"]], dim=-1)[0].cpu().numpy()
    got["hit_t"] = out["pred_dist"][0, ..., 0].cpu().numpy()
    packed = tracer.packed.cpu().numpy()
    valid2 = valid[0, :, :, 0]
    tmask = harness.tile_mask(valid2)
    ocam = harness.oracle_camera(w.camera)
    pose = oracle.prepare_pose(w.poses[frame])
    proj, rgb, counts = oracle.project(ocam, pose, packed, w.scene.features, 3, tmask, d[0])
    tr = oracle.tile_rays(ocam, pose, o[0], d[0])
    keys, ids, ranges = oracle.bin(ocam, pose, packed, proj, counts, tmask, tr, 0, d[0])
    ref = dict(proj=proj, rgb=rgb, counts=counts, keys=keys, ids=ids, ranges=ranges, pose=pose)
    return dict(w=w, got=got, ref=ref, packed=packed, rays=(o[0], d[0]), tmask=tmask, ocam=ocam)


def test_orbit_frame_binning(orbit_frame):
    got, ref, w = orbit_frame["got"], orbit_frame["ref"], orbit_frame["w"]
    np.testing.assert_array_equal(got["proj"].view(np.uint32), ref["proj"].view(np.uint32))
    np.testing.assert_array_equal(got["rgb"].view(np.uint32), ref["rgb"].view(np.uint32))
    np.testing.assert_array_equal(got["counts"].astype(np.uint32), ref["counts"])
    assert got["keys"].size == ref["keys"].size > 100_000_000
    np.testing.assert_array_equal(got["keys"].view(np.uint64), ref["keys"])
    np.testing.assert_array_equal(got["ids"].view(np.uint32), ref["ids"])
    np.testing.assert_array_equal(got["ranges"].view(np.uint32), ref["ranges"])
    # the large Gaussians beside the camera path without a UT footprint are admitted by the cone fallback
    big = w.big_rows
    assert int(((ref["proj"][big, 6] == 0.0) & (ref["counts"][big] > 0)).sum()) > 1000


@pytest.mark.parametrize("band", ["centre", "rim"])
def test_orbit_frame_image_band(orbit_frame, band):
    got, ref, w = orbit_frame["got"], orbit_frame["ref"], orbit_frame["w"]
    ty, tx = orbit_frame["tmask"].shape
    r0 = ty // 2 - 1 if band == "centre" else ty // 10
    tiles = (r0 * tx, (r0 + 2) * tx)
    o, d = orbit_frame["rays"]
    rgba, hit_t, _ = oracle.render_forward(orbit_frame["ocam"], ref["pose"], orbit_frame["packed"], ref["rgb"], o, d,
                                           orbit_frame["tmask"], ref["ranges"], ref["ids"], 32, tiles)
    rows = slice(16 * r0, 16 * (r0 + 2))
    assert np.abs(got["rgba"][rows] - rgba[rows]).max() <= 1e-3
    assert harness.psnr(got["rgba"][rows], rgba[rows]) >= 60.0
    np.testing.assert_allclose(got["hit_t"][rows], hit_t[rows], rtol=1e-3, atol=1e-4)
    assert float(rgba[rows][..., 3].max()) > 0.5


# ----------------------------------------------------------------------------- mesh opacity query subset
@pytest.fixture(scope="module")
def mesh_subset(cuda_device):
    """The mesh-query scene (3M Gaussians, sites of every kept Gaussian), a
    seeded subset of 1M sites and 4 of its 32 equidistant 200 deg 800x800
    views (masked), evaluated by the GPU field and by the oracle's indexed
    field."""
    from gofish_b200.mesh import SplatRaster as FieldRaster
    from gofish_b200.mesh.cameras import fisheye_training_camera
    from gofish_b200.mesh.field import camera_inputs
    from gofish_b200.mesh.shape import effective_shape
    from gofish_b200.mesh.sites import generate_sites

    w = S.workload_mesh_query()
    shape = effective_shape(w.scene.positions, w.scene.scales, w.scene.rotations, w.scene.density)
    sites = generate_sites(shape).points
    rng = np.random.default_rng(1237)
    points = np.ascontiguousarray(sites[np.sort(rng.choice(sites.shape[0], 1_000_000, replace=False))])
    chosen = (0, 8, 16, 24)
    cameras = [fisheye_training_camera(v, w.camera, w.poses[v], masked=True) for v in chosen]
    raster = FieldRaster()
    packed = shape.packed_density()
    token = raster.begin_opacity_field(torch.from_numpy(packed).to(cuda_device),
                                       torch.from_numpy(np.ascontiguousarray(shape.sigma_max)).to(cuda_device),
                                       torch.from_numpy(points).to(cuda_device))
    for cam in cameras:
        raster.integrate_opacity_field_camera(token, *camera_inputs(cam, cuda_device))
    opacity, observed, above = (t.cpu().numpy() for t in raster.finish_opacity_field(token))
    raster.release_opacity_field(token)
    ocam = harness.oracle_camera(w.camera)
    ray_o = np.zeros((w.camera.height, w.camera.width, 3), np.float32)
    views = [(ocam, w.poses[v], ray_o, cam.physical_mask.numpy()) for v, cam in zip(chosen, cameras)]
    with oracle.FieldIndex(packed, 20.0) as index:
        ref = index.evaluate_field(views, points)
    return dict(got=(opacity, observed, above), ref=ref)


def test_mesh_query_subset_bit_exact(mesh_subset):
    (opacity, observed, above), (want_op, want_ob, want_ab) = mesh_subset["got"], mesh_subset["ref"]
    np.testing.assert_array_equal(observed, want_ob)
    np.testing.assert_array_equal(opacity.view(np.uint32), want_op.view(np.uint32))
    np.testing.assert_array_equal(above, want_ab)
    seen = want_ob != 0
    assert seen.mean() > 0.5
    # partial and saturated opacities both occur
    assert 0.05 < (want_op[seen] == 1.0).mean() < 0.95
    assert ((want_op[seen] > 0.0) & (want_op[seen] < 1.0)).sum() > 1000
