"""The forward-only inference renderer (InferenceTracer, reference
threedgut_tracer/inference.py:77-235) on a small high-resolution-orbit scene:
equisolid 205 deg fisheye, k = 32, physical-mip 3-D filter on, large
Gaussians beside the camera path straddling the 90 deg horizon.

* ``render`` equals the hand-composed pipeline (Q_v, full shape, packed rows,
  ``trace_inference``) bit for bit;
* its image and hit distance match the oracle traced on the same packed rows
  (max-abs <= 1e-3, PSNR >= 60 dB; hit distance relative <= 1e-3);
* the fused (Cholesky) shape renders the same scene within 40 dB of the exact
  one; with gamma = 0 the shape is computed once and reused.
"""

import numpy as np
import pytest
import torch

import oracle
from gofish_b200 import scene as S
from gofish_b200.batch import Batch, create_camera_parameters
from gofish_b200.footprint_shape_operator import build_full_shape
from gofish_b200.inference import FrozenGaussians, InferenceTracer
from gofish_b200.physical_mip import compute_filter, pack_camera_table
from gofish_b200.splat_raster import SplatRaster
from gofish_b200.view_observation_filter import current_view_q6
from tests import harness

pytestmark = pytest.mark.gpu

GAMMA = 0.3


@pytest.fixture(scope="module")
def orbit(cuda_device):
    w = S.workload_inference(seed=41, n=20_000, frames=8, size=256)
    o, d, valid = w.camera.rays()
    cams, frames = S.mip_camera_records(w.camera, w.poses, valid[0, :, :, 0])
    table = pack_camera_table(cams, frames, cuda_device)
    pos = torch.from_numpy(w.scene.positions).to(cuda_device)
    filter_3d, _ = compute_filter(pos, table, 0.2)
    model = FrozenGaussians.from_scene(w.scene, cuda_device, filter_3d)
    rays = (torch.from_numpy(o).to(cuda_device), torch.from_numpy(d).to(cuda_device))
    mask = torch.from_numpy(valid).to(cuda_device)
    return w, model, rays, mask, valid[0, :, :, 0]


def _batch(w, rays, mask, frame):
    c2w = torch.from_numpy(S.pose_to_c2w(w.poses[frame])[None]).float()
    return Batch(rays[0], rays[1], c2w, intrinsics_OpenCVFisheyeCameraModelParameters=w.camera.intrinsics(),
                 physical_fov_mask=mask, physical_fov_key="equisolid-205")


def _conf(gamma=GAMMA):
    return {"render": {"splat": {"k_buffer_size": 32}, "gofish": {"pixel_footprint_variance": gamma}}}


def _image(out):
    return torch.cat([out["pred_features"], out["pred_opacity"]], dim=-1)[0].cpu().numpy()


def test_render_equals_the_composed_pipeline(orbit):
    w, model, rays, mask, _valid = orbit
    tracer = InferenceTracer(_conf(), model)
    batch = _batch(w, rays, mask, 3)
    out = tracer.render(batch)
    # the same steps by hand
    n = w.scene.num
    scale = model.get_scale_with_3D_filter()
    q6, jac, obs = current_view_q6(model.positions, batch, GAMMA)
    shape = build_full_shape(scale, model.get_rotation(), model.get_density(), q6, jac, obs, mass_preserving=True,
                             pixel_variance=GAMMA)
    packed = torch.zeros((n, 32), dtype=torch.float32, device=model.positions.device)
    packed[:, 0:3] = model.positions
    packed[:, 3:4] = shape.density.reshape(n, 1)
    packed[:, 4:8] = model.get_rotation()
    packed[:, 8:11] = scale
    packed[:, 11:12] = model.get_density()
    packed[:, 12:21] = shape.factor.reshape(n, 9)
    packed[:, 21:30] = shape.inverse_factor.reshape(n, 9)
    assert torch.equal(packed, tracer.packed)
    raster = SplatRaster(_conf())
    tm = torch.from_numpy(harness.tile_mask(mask[0, :, :, 0].cpu().numpy())).to(packed.device)
    raster.register_physical_tile_mask(tm, "t")
    sensor, poses = create_camera_parameters(batch)
    rgba, hit = raster.trace_inference(3, packed, model.get_features(), rays[0], rays[1], sensor, 0, 1,
                                       poses.T_world_sensors[0], poses.T_world_sensors[1], "t")
    assert torch.equal(torch.cat([out["pred_features"], out["pred_opacity"]], dim=-1)[0], rgba)
    assert torch.equal(out["pred_dist"][0], hit)


@pytest.mark.parametrize("frame", [0, 5])
def test_render_matches_the_oracle(orbit, frame):
    w, model, rays, mask, valid = orbit
    tracer = InferenceTracer(_conf(), model)
    batch = _batch(w, rays, mask, frame)
    out = tracer.render(batch)
    _sensor, poses = create_camera_parameters(batch)
    ref = oracle.trace(harness.oracle_camera(w.camera), poses.T_world_sensors[0], tracer.packed.cpu().numpy(),
                       w.scene.features, 3, rays[0][0].cpu().numpy(), rays[1][0].cpu().numpy(),
                       harness.tile_mask(valid), 32, 0)
    got = _image(out)
    assert np.abs(got - ref["rgba"]).max() <= 1e-3
    assert harness.psnr(got, ref["rgba"]) >= 60.0
    np.testing.assert_allclose(out["pred_dist"][0, ..., 0].cpu().numpy(), ref["hit_t"], rtol=1e-3, atol=1e-4)
    # the scene exercises the cone fallback: large Gaussians without a UT footprint are admitted
    big = w.big_rows
    no_footprint = ref["proj"][big, 6] <= 1e-6
    assert int((no_footprint & (ref["counts"][big] > 0)).sum()) >= 10
    assert float(ref["rgba"][..., 3].max()) > 0.5


def test_fused_shape_renders_close_to_exact(orbit):
    w, model, rays, mask, _valid = orbit
    batch = _batch(w, rays, mask, 2)
    exact = _image(InferenceTracer(_conf(), model).render(batch))
    fused_tracer = InferenceTracer(_conf(), model, shape="fused")
    fused = _image(fused_tracer.render(batch))
    assert fused_tracer.shape_status() == 0
    assert harness.psnr(fused, exact) >= 40.0


def test_zero_footprint_shape_is_computed_once(orbit):
    w, model, rays, mask, _valid = orbit
    tracer = InferenceTracer(_conf(0.0), model)
    first = _image(tracer.render(_batch(w, rays, mask, 1)))
    shape = tracer.static_shape
    assert shape is not None
    packed = tracer.packed.clone()
    second = _image(tracer.render(_batch(w, rays, mask, 6)))
    assert tracer.static_shape is shape
    assert torch.equal(tracer.packed, packed)  # the cached rows are not rewritten
    # C = R S^2 R^T for every view; only the factor of rows unobserved in the
    # caching frame (R S instead of the symmetric root) differs from a fresh shape
    fresh = InferenceTracer(_conf(0.0), model)
    assert harness.psnr(second, _image(fresh.render(_batch(w, rays, mask, 6)))) >= 60.0
    assert not np.array_equal(first, second)
