"""The training renderer ``Tracer(conf).render(gaussians, gpu_batch, train,
frame_id)`` (reference threedgut_tracer/tracer.py:142-525) on a small
Kannala-Brandt 200 deg view with the per-view footprint on (gamma = 0.3):

* the forward equals the hand-composed pipeline (Q_v, full shape, packed rows,
  ``SplatRaster.trace``) bit for bit, and matches the oracle traced on the
  same rows (max-abs <= 1e-3, PSNR >= 60 dB);
* autograd through ``Tracer._Autograd`` and the full-shape VJP gives the
  oracle's chain (oracle render backward, projection backward, then the
  numpy full-shape VJP) within 1e-3 relative L2 for the position, rotation,
  scale, opacity and SH gradients;
* the geometric channels are zeros, and configurations whose losses read them
  are refused.
"""

import numpy as np
import pytest
import torch

import oracle
from gofish_b200 import scene as S
from gofish_b200.batch import Batch, create_camera_parameters
from gofish_b200.camera import fisheye_camera, random_kb_coefficients
from gofish_b200.splat_raster import SplatRaster
from gofish_b200.tracer import SceneGaussians, Tracer
from gofish_b200.view_observation_filter import build_intrinsic_view_shape, current_view_q6
from oracle import full_shape as fs
from tests import harness

pytestmark = pytest.mark.gpu

GAMMA = 0.3
K = 16


def _conf():
    return {"render": {"splat": {"k_buffer_size": K}, "gofish": {"pixel_footprint_variance": GAMMA}}}


@pytest.fixture(scope="module")
def view(cuda_device):
    scene = S.random_scene(6000, 3, 31)
    rng = np.random.default_rng(131)
    cam = fisheye_camera(128, 112, 200.0, random_kb_coefficients(rng, 200.0))
    pose = S.pose_world_to_sensor(rng.standard_normal(3) * 0.2, S.random_rotation_quaternion_xyzw(rng))
    o, d, valid = cam.rays()
    c2w = torch.from_numpy(S.pose_to_c2w(pose)[None]).float()
    batch = Batch(torch.from_numpy(o).to(cuda_device), torch.from_numpy(d).to(cuda_device), c2w,
                  intrinsics_OpenCVFisheyeCameraModelParameters=cam.intrinsics(),
                  physical_fov_mask=torch.from_numpy(valid).to(cuda_device), physical_fov_key="kb-200")
    return scene, cam, batch, valid[0, :, :, 0]


def _packed(model, batch):
    n = model.num_gaussians
    shape = build_intrinsic_view_shape(model.get_scale(), model.get_rotation(), model.get_density(), model.positions,
                                       batch, pixel_footprint_variance=GAMMA)
    packed = torch.zeros((n, 32), dtype=torch.float32, device=model.positions.device)
    packed[:, 0:3] = model.positions
    packed[:, 3:4] = shape.density.reshape(n, 1)
    packed[:, 4:8] = model.get_rotation()
    packed[:, 8:11] = model.get_scale()
    packed[:, 11:12] = model.get_density()
    packed[:, 12:21] = shape.factor.reshape(n, 9)
    packed[:, 21:30] = shape.inverse_factor.reshape(n, 9)
    return packed


def test_forward_equals_composed_pipeline_and_oracle(view, cuda_device):
    scene, cam, batch, valid = view
    model = SceneGaussians.from_scene(scene, cuda_device, requires_grad=False)
    out = Tracer(_conf()).render(model, batch, train=True, frame_id=3)
    assert out["pred_features"].shape == (1, cam.height, cam.width, 3)
    assert out["pred_opacity"].shape == (1, cam.height, cam.width, 1)
    for key in ("pred_normals", "pred_depth_var", "pred_quant", "pred_extent", "pred_invd", "pred_invd2"):
        assert not bool(out[key].any())
    with torch.no_grad():
        packed = _packed(model, batch)
    raster = SplatRaster(_conf())
    tm = torch.from_numpy(harness.tile_mask(valid)).to(cuda_device)
    raster.register_physical_tile_mask(tm, "t")
    sensor, poses = create_camera_parameters(batch)
    ref = raster.trace(3, False, 3, packed, model.get_features(), batch.rays_ori, batch.rays_dir, None, sensor, 0, 1,
                       poses.T_world_sensors[0], poses.T_world_sensors[1], "t")
    image = torch.cat([out["pred_features"], out["pred_opacity"]], dim=-1)[0]
    assert torch.equal(image, ref[0])
    assert torch.equal(out["pred_dist"][0], ref[1])
    assert torch.equal(out["hits_count"][0], ref[2])
    want = oracle.trace(harness.oracle_camera(cam), poses.T_world_sensors[0], packed.cpu().numpy(), scene.features, 3,
                        batch.rays_ori[0].cpu().numpy(), batch.rays_dir[0].cpu().numpy(), harness.tile_mask(valid), K,
                        0)
    got = image.cpu().numpy()
    assert np.abs(got - want["rgba"]).max() <= 1e-3
    assert harness.psnr(got, want["rgba"]) >= 60.0
    assert np.array_equal(out["hits_count"][0, ..., 0].cpu().numpy(), want["hit_count"])
    assert float(want["rgba"][..., 3].max()) > 0.5


@pytest.mark.parametrize("geometry", [False, True])
def test_gradients_match_the_oracle_chain(view, cuda_device, geometry):
    """geometry: render.enable_normals with a loss on the normal, depth-moment,
    extent and inverse-depth channels besides the colour."""
    scene, cam, batch, valid = view
    model = SceneGaussians.from_scene(scene, cuda_device, requires_grad=True)
    conf = _conf()
    conf["render"]["enable_normals"] = geometry
    out = Tracer(conf).render(model, batch, train=True)
    rng = np.random.default_rng(5)
    g_rgba = rng.uniform(-1.0, 1.0, (cam.height, cam.width, 4)).astype(np.float32)
    g = torch.from_numpy(g_rgba).to(cuda_device)
    loss = (out["pred_features"][0] * g[..., :3]).sum() + (out["pred_opacity"][0] * g[..., 3:]).sum()
    h, w = cam.height, cam.width
    geo_grads = {"normal": rng.standard_normal((h, w, 3)).astype(np.float32),
                 "depth_var": (0.05 * rng.standard_normal((h, w))).astype(np.float32),
                 "extent": rng.standard_normal((h, w)).astype(np.float32),
                 "inv_depth": rng.standard_normal((h, w)).astype(np.float32),
                 "inv_depth2": rng.standard_normal((h, w)).astype(np.float32)}
    if geometry:
        keys = {"normal": "pred_normals", "depth_var": "pred_depth_var", "extent": "pred_extent",
                "inv_depth": "pred_invd", "inv_depth2": "pred_invd2"}
        for name, key in keys.items():
            gg = torch.from_numpy(geo_grads[name]).to(cuda_device).reshape(out[key].shape)
            loss = loss + (out[key] * gg).sum()
    loss.backward()

    # oracle chain on the same view: render + projection backward, then the full-shape VJP
    with torch.no_grad():
        packed = _packed(model, batch).cpu().numpy()
        q6, jac, obs = current_view_q6(model.positions, batch, GAMMA)
    _sensor, poses = create_camera_parameters(batch)
    ocam = harness.oracle_camera(cam)
    ro, rd, tm = batch.rays_ori[0].cpu().numpy(), batch.rays_dir[0].cpu().numpy(), harness.tile_mask(valid)
    fwd = oracle.trace(ocam, poses.T_world_sensors[0], packed, scene.features, 3, ro, rd, tm, K, 0)
    if geometry:
        geo_fwd = oracle.render_forward_geo(ocam, fwd["pose"], packed, fwd["rgb"], ro, rd, tm, fwd["ranges"],
                                            fwd["ids"], K)
        grads = dict(geo_grads, rgba=g_rgba, hit_t=np.zeros((h, w), np.float32))
        rec, shape = oracle.render_backward_geo(ocam, fwd["pose"], packed, fwd["rgb"], ro, rd, tm, fwd["ranges"],
                                                fwd["ids"], K, geo_fwd, grads)
        gp, gsh = oracle.project_backward(fwd["pose"], packed, scene.features, 3, fwd["counts"], rec)
        gp = gp.astype(np.float64)
        gp[:, 4:8] += shape[:, 0:4]
        gp[:, 8:11] += shape[:, 4:7]
    else:
        gp, gsh, _ = oracle.trace_backward(ocam, fwd, packed, scene.features, 3, ro, rd, tm, K, g_rgba,
                                           np.zeros((cam.height, cam.width), np.float32))
        gp = gp.astype(np.float64)
    q = q6.cpu().numpy()
    Q = np.stack([q[:, 0], q[:, 1], q[:, 2], q[:, 1], q[:, 3], q[:, 4], q[:, 2], q[:, 4], q[:, 5]], 1).reshape(-1, 3, 3)
    n = scene.num
    gs, gq, go = fs.full_shape_vjp(scene.scales, scene.rotations, scene.density, Q, jac.cpu().numpy(),
                                   obs.cpu().numpy(), GAMMA, np.zeros((n, 3, 3)), gp[:, 12:21].reshape(n, 3, 3),
                                   gp[:, 21:30].reshape(n, 3, 3), np.zeros(n), gp[:, 3])
    want = {
        "positions": gp[:, 0:3],
        "rotation": gq + gp[:, 4:8],
        "scale": gs + gp[:, 8:11],
        "density": go[:, None] + gp[:, 11:12],
        "features": gsh,
    }
    for name, w in want.items():
        got = getattr(model, name).grad
        assert got is not None, name
        assert float(np.linalg.norm(w)) > 0.0, name
        assert harness.rel_l2(got.cpu().numpy(), w) <= 1e-3, name


def test_opacity_field_loss_needs_the_geometric_channels():
    with pytest.raises(ValueError, match="lambda_opa"):
        Tracer({"render": {"enable_normals": False}, "loss": {"lambda_opa": 0.004}})


def test_shape_failure_is_raised_by_render(view, cuda_device):
    """A row whose full shape is not positive definite raises
    FootprintNumericalError with its global row: from the render call once
    its status words have reached the host, or at the latest from
    check_shapes() (render does not wait for them)."""
    from gofish_b200.footprint_shape_operator import FootprintNumericalError

    scene, cam, batch, valid = view
    model = SceneGaussians.from_scene(scene, cuda_device, requires_grad=False)
    _q6, _jac, obs = current_view_q6(model.positions, batch, GAMMA)
    row = int(torch.nonzero(obs).reshape(-1)[11])
    model.scale[row] = 0.0  # C = Q_v has rank 2
    tracer = Tracer(_conf())
    with pytest.raises(FootprintNumericalError) as err:
        tracer.render(model, batch, train=True)
        tracer.check_shapes()
    assert err.value.global_row == row


def test_shape_failure_surfaces_within_the_unchecked_window(view, cuda_device):
    """Without check_shapes(), the failure raises from one of the next
    renders: at most MAX_UNCHECKED_SHAPES views stay unchecked."""
    from gofish_b200.footprint_shape_operator import FootprintNumericalError
    from gofish_b200.tracer import MAX_UNCHECKED_SHAPES

    scene, cam, batch, valid = view
    bad = SceneGaussians.from_scene(scene, cuda_device, requires_grad=False)
    good = SceneGaussians.from_scene(scene, cuda_device, requires_grad=False)
    _q6, _jac, obs = current_view_q6(bad.positions, batch, GAMMA)
    bad.scale[int(torch.nonzero(obs).reshape(-1)[5])] = 0.0
    tracer = Tracer(_conf())
    with pytest.raises(FootprintNumericalError):
        tracer.render(bad, batch, train=True)
        for _ in range(MAX_UNCHECKED_SHAPES + 1):
            tracer.render(good, batch, train=True)
