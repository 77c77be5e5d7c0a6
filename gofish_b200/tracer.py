"""Training renderer: ``Tracer(conf).render(gaussians, gpu_batch, train, frame_id)``
(reference threedgut_tracer/tracer.py:142-525).

One render of one view:

1. the physical tile mask of the camera is registered once per (domain,
   device, raster) under its token (tracer.py:380-404);
2. the per-view full shape is built from the model's intrinsic shape:
   Q_v of the active camera, C = R S^2 R^T + Q_v, its factor B = C^(1/2) R,
   B^-1 and the mass-preserving density m * o (``build_intrinsic_view_shape``,
   tracer.py:406-433), all differentiable;
3. ``Tracer._Autograd`` packs the reference's [N,32] particle rows and calls
   the native ``SplatRaster.trace``; its backward calls ``trace_bwd`` and
   splits the [N,32] row gradient into the per-slot gradients in the
   reference's order (tracer.py:142-353), so autograd carries them back
   through the full-shape VJP to the scale, rotation and opacity.

With ``render.enable_normals`` the geometric training channels are rendered
(normal sum, sum w t^2, quantile and exact 0.5-crossing depths, intrinsic
extent, inverse-depth moments) and the normal, depth-moment, extent,
inverse-depth and exact-crossing-depth channels carry gradients (the
crossing depth by the implicit function theorem); without it they are zeros,
as the reference's buffers are with its normal channel compiled out.  The
CoMe colour confidence (``loss.color_confidence``) is refused.
"""

from __future__ import annotations

from typing import Any

import torch

from . import _native
from .batch import create_camera_parameters
from .physical_mip import scale_with_3d_filter
from .physical_tile_mask import build_physical_tile_binding
from .splat_raster import SplatRaster, _select
from .view_observation_filter import build_intrinsic_view_shape, pixel_footprint_variance

# Row layout of the packed particle ABI (gaussianParticles.cuh:33-46) and the
# gradient split of tracer.py:334-343.
PACKED_SPLIT = (3, 1, 4, 3, 1, 9, 9, 2)

# Losses on the geometric training channels (they need render.enable_normals;
# loss.lambda_opa, on the SOF opacity field, as well), and those refused here
# (none).
GEOMETRIC_LOSSES = ("lambda_distortion", "lambda_dnc", "lambda_esmooth", "lambda_extent", "lambda_normal_variance")
UNSUPPORTED_LOSSES: tuple = ()


def _conf_value(conf, path: str, default):
    if isinstance(conf, dict) or conf is None:
        return _select(conf, path, default)
    node: Any = conf
    for part in path.split("."):
        node = getattr(node, part, None) if not isinstance(node, dict) else node.get(part)
        if node is None:
            return default
    return node


# views whose full-shape status may still be in flight when render returns
MAX_UNCHECKED_SHAPES = 8


class Tracer:
    """Differentiable fisheye renderer of a Gaussian scene (reference ``Tracer``)."""

    class _Autograd(torch.autograd.Function):
        """Argument order of tracer.py:144-164; gradients in the same order."""

        @staticmethod
        def forward(ctx, tracer_wrapper, physical_tile_token, frame_id, sof_exact_opacity_active, n_active_features,
                    ray_ori, ray_dir, mog_pos, mog_rot, mog_scl, mog_dns, mog_intrinsic_dns, mog_factor,
                    mog_inverse_factor, mog_sph, sensor_params, sensor_poses, mog_confidence):
            n = mog_pos.shape[0]
            if mog_confidence.numel() != 0:
                raise NotImplementedError("CoMe colour confidence is not rendered by this tracer")
            if mog_factor.shape != (n, 3, 3) or mog_inverse_factor.shape != mog_factor.shape:
                raise ValueError("full-shape factor tensors must have shape [N,3,3]")
            particle_density = _pack_rows(mog_pos, mog_dns, mog_rot, mog_scl, mog_intrinsic_dns, mog_factor,
                                          mog_inverse_factor)
            particle_features = mog_sph.float().contiguous()
            t0, t1 = sensor_poses.timestamps_us[0], sensor_poses.timestamps_us[1]
            p0, p1 = sensor_poses.T_world_sensors[0], sensor_poses.T_world_sensors[1]
            outs = tracer_wrapper.trace(frame_id, sof_exact_opacity_active, n_active_features, particle_density,
                                        particle_features, ray_ori, ray_dir, None, sensor_params, t0, t1, p0, p1,
                                        physical_tile_token)
            rgba, hit_distance = outs[0], outs[1]
            # forward values of the geometric channels (normal ... inverse depth squared) for the backward
            ctx.save_for_backward(ray_ori, ray_dir, rgba, hit_distance, particle_density, particle_features,
                                  *outs[4:])
            ctx.frame_id = frame_id
            ctx.sof_exact_opacity_active = bool(sof_exact_opacity_active)
            ctx.n_active_features = n_active_features
            ctx.sensor_params = sensor_params
            ctx.sensor_poses = sensor_poses
            ctx.tracer_wrapper = tracer_wrapper
            ctx.physical_tile_token = physical_tile_token
            ctx.set_materialize_grads(False)
            ctx.mark_non_differentiable(outs[2], outs[3])
            return outs

        @staticmethod
        def backward(ctx, ray_features_density_grd, ray_hit_distance_grd, _count_grd, _visibility_grd, normal_grd,
                     depth_var_grd, quant_grd, extent_grd, opacity_field_grd, invd_grd, invd2_grd):
            (ray_ori, ray_dir, rgba, hit_distance, particle_density, particle_features, normal, depth_var, quant,
             extent, opacity_field, invd, invd2) = ctx.saved_tensors
            geometric = (normal_grd, depth_var_grd, quant_grd, extent_grd, opacity_field_grd, invd_grd, invd2_grd)
            if ray_features_density_grd is None and ray_hit_distance_grd is None and all(
                    g is None for g in geometric):
                return (None,) * 18
            if ray_features_density_grd is None:
                ray_features_density_grd = torch.zeros_like(rgba)
            poses = ctx.sensor_poses
            grad_density, grad_features = ctx.tracer_wrapper.trace_bwd(
                ctx.frame_id, ctx.sof_exact_opacity_active, ctx.n_active_features, particle_density,
                particle_features, ray_ori, ray_dir, None, ctx.sensor_params, poses.timestamps_us[0],
                poses.timestamps_us[1], poses.T_world_sensors[0], poses.T_world_sensors[1], rgba,
                ray_features_density_grd, hit_distance, ray_hit_distance_grd, depth_var, depth_var_grd, extent,
                extent_grd, opacity_field, opacity_field_grd, quant, quant_grd, normal, normal_grd, invd, invd_grd,
                invd2, invd2_grd, ctx.physical_tile_token)
            g_pos, g_dns, g_rot, g_scl, g_intrinsic, g_factor, g_inverse = _unpack_rows(grad_density)
            return (None, None, None, None, None, None, None, g_pos, g_rot, g_scl, g_dns, g_intrinsic, g_factor,
                    g_inverse, grad_features.contiguous(), None, None, None)

    def __init__(self, conf):
        self.device = "cuda"
        self.conf = conf
        if _conf_value(conf, "render.primitive_type", "instances") == "trisurfel":
            raise RuntimeError("GOFish renders volumetric Gaussians only")
        def active(names):
            return [name for name in names if float(_conf_value(conf, f"loss.{name}", 0.0) or 0.0) > 0.0]

        if active(UNSUPPORTED_LOSSES):
            raise NotImplementedError("unsupported losses: " + ", ".join(active(UNSUPPORTED_LOSSES)))
        geometric = active(GEOMETRIC_LOSSES + ("lambda_opa",))
        if geometric and not bool(_conf_value(conf, "render.enable_normals", False)):
            raise ValueError("losses on the geometric channels (" + ", ".join(geometric) +
                             ") need render.enable_normals")
        if bool(_conf_value(conf, "loss.color_confidence", False)):
            raise NotImplementedError("CoMe colour confidence (loss.color_confidence) is not rendered by this tracer")
        self._view_observation_filter = True
        self._pixel_footprint_variance = pixel_footprint_variance(conf)
        self.tracer_wrapper = SplatRaster(_plain(conf))
        self._physical_tile_binding_cache: dict = {}
        self._physical_tile_registration_cache: set = set()
        self._pending_shape = None
        self._unchecked_shapes: list = []

    def _check_shapes(self, keep: int) -> None:
        """Checks, in order, the per-view shapes whose status words have reached
        the host, waiting only for those beyond the newest ``keep``."""
        while self._unchecked_shapes:
            shape = self._unchecked_shapes[0]
            if len(self._unchecked_shapes) <= keep and not shape.ready():
                return
            self._unchecked_shapes.pop(0)
            shape.check()

    def check_shapes(self) -> None:
        """Waits for every rendered view's shape status and raises
        FootprintNumericalError for the first failed row."""
        self._check_shapes(0)

    def _physical_tile_token(self, wrapper, gpu_batch, rays) -> str:
        """The tile mask of the batch's calibrated domain, registered once per camera."""
        mask = getattr(gpu_batch, "physical_fov_mask", None)
        domain = getattr(gpu_batch, "physical_fov_key", None)
        if domain is None:
            domain = "full-raster" if mask is None else f"mask:{id(mask)}"
        key = (str(domain), str(rays.device), int(rays.shape[1]), int(rays.shape[2]))
        binding = self._physical_tile_binding_cache.get(key)
        if binding is None:
            binding = build_physical_tile_binding(gpu_batch, rays, str(domain))
            self._physical_tile_binding_cache[key] = binding
        registration = (id(wrapper), binding.token)
        if registration not in self._physical_tile_registration_cache:
            wrapper.register_physical_tile_mask(binding.mask, binding.token)
            self._physical_tile_registration_cache.add(registration)
        return binding.token

    def _density_shape_inputs(self, gaussians, gpu_batch=None, detach=False, frame_id=None):
        """(rotation, intrinsic scale, view density m*o, intrinsic density, B, B^-1) of this view."""
        if gpu_batch is None:
            raise RuntimeError("the per-view footprint requires the active camera batch")
        rotation = gaussians.get_rotation()
        raw_density = gaussians.get_density()
        physical_scale = (gaussians.get_scale_with_3D_filter()
                          if bool(getattr(gaussians, "_use_physical_mip3d_filter", False)) else gaussians.get_scale())
        if detach:
            rotation, raw_density, physical_scale = rotation.detach(), raw_density.detach(), physical_scale.detach()
        shape = build_intrinsic_view_shape(physical_scale, rotation, raw_density, gaussians.positions.detach(),
                                           gpu_batch, pixel_footprint_variance=self._pixel_footprint_variance,
                                           frame_id=frame_id, defer_check=True)
        self._pending_shape = shape
        return rotation, physical_scale, shape.density, raw_density, shape.factor, shape.inverse_factor

    @property
    def timings(self):
        return self.tracer_wrapper.collect_times()

    def build_acc(self, gaussians, rebuild=True):
        """No acceleration structure for a rasterised tracer (tracer.py:443-444)."""

    def _sof_opacity_active(self, train: bool, frame_id: int) -> bool:
        """tracer.py:433-448: the SOF opacity field is traced for training
        frames with loss.lambda_opa > 0 from loss.opa_warmup (default
        loss.geom_warmup, 15,000) until the distillation steps."""
        lam = float(_conf_value(self.conf, "loss.lambda_opa", 0.0) or 0.0)
        warm = _conf_value(self.conf, "loss.opa_warmup", None)
        if warm is None:
            warm = _conf_value(self.conf, "loss.geom_warmup", 15_000)
        total = int(_conf_value(self.conf, "n_iterations", 0) or 0)
        distill = int(_conf_value(self.conf, "post_processing.n_distillation_steps", 0) or 0)
        return bool(train and lam > 0.0 and int(warm or 0) <= int(frame_id) < total - distill)

    def render(self, gaussians, gpu_batch, train=False, frame_id=0) -> dict[str, Any]:
        rays_o = gpu_batch.rays_ori
        rays_d = gpu_batch.rays_dir
        token = self._physical_tile_token(self.tracer_wrapper, gpu_batch, rays_d)
        sensor, poses = create_camera_parameters(gpu_batch)
        sof_active = self._sof_opacity_active(train, frame_id)
        rot, scale, dens, intrinsic_dens, factor, inverse_factor = self._density_shape_inputs(
            gaussians, gpu_batch, detach=False, frame_id=frame_id)
        confidence = gaussians.positions.new_empty((0, 1))
        (features_alpha, pred_dist, hits_count, visibility, normal, depth_var, quant, extent, opacity_field, invd,
         invd2) = Tracer._Autograd.apply(
            self.tracer_wrapper, token, frame_id, sof_active, gaussians.n_active_features, rays_o.contiguous(),
            rays_d.contiguous(), gaussians.positions.contiguous(), rot.contiguous(), scale.contiguous(),
            dens.contiguous(), intrinsic_dens.contiguous(), factor.contiguous(), inverse_factor.contiguous(),
            gaussians.get_features().contiguous(), sensor, poses, confidence)
        # The shape's status words reach the host asynchronously: views are
        # checked once their copy has landed (without waiting), and only the
        # MAX_UNCHECKED_SHAPES views before this one may stay unchecked, so a
        # numerical failure raises within a few calls without a per-view wait.
        shape, self._pending_shape = self._pending_shape, None
        self._unchecked_shapes.append(shape)
        self._check_shapes(MAX_UNCHECKED_SHAPES)
        f = gaussians.ray_feature_dim
        timings = self.tracer_wrapper.collect_times()
        return {
            "pred_features": features_alpha[..., :f].unsqueeze(0).contiguous(),
            "pred_opacity": features_alpha[..., f:].unsqueeze(0).contiguous(),
            "pred_dist": pred_dist.unsqueeze(0).contiguous(),
            "pred_normals": normal.unsqueeze(0).contiguous(),
            "pred_depth_var": depth_var.unsqueeze(0).contiguous(),
            "pred_quant": quant.unsqueeze(0).contiguous(),
            "pred_crossing": quant[..., 8:9].unsqueeze(0).contiguous(),
            "pred_crossing_rate": quant[..., 9:10].unsqueeze(0).contiguous(),
            "pred_extent": extent.unsqueeze(0).contiguous(),
            "pred_opacity_field": opacity_field.unsqueeze(0).contiguous(),
            "pred_invd": invd.unsqueeze(0).contiguous(),
            "pred_invd2": invd2.unsqueeze(0).contiguous(),
            "hits_count": hits_count.unsqueeze(0).contiguous(),
            "frame_time_ms": timings.get("forward_render", 0.0),
            "mog_visibility": visibility,
        }


class SceneGaussians:
    """A Gaussian scene with the accessors the tracer reads (the reference
    model's ``positions``, ``get_rotation``, ``get_scale``,
    ``get_scale_with_3D_filter``, ``get_density``, ``get_features``), holding
    activated values.  Tensors that require grad receive the render's
    gradients."""

    def __init__(self, positions, rotations, scales, density, features, sh_degree: int, filter_3d=None):
        self.positions = positions
        self.rotation = rotations
        self.scale = scales
        self.density = density
        self.features = features
        self.n_active_features = int(sh_degree)
        self.ray_feature_dim = 3
        self.filter_3d = filter_3d
        self._use_physical_mip3d_filter = filter_3d is not None

    @classmethod
    def from_scene(cls, scene, device, requires_grad: bool = True, filter_3d=None) -> "SceneGaussians":
        def t(a, shape=None):
            v = torch.as_tensor(a, dtype=torch.float32).to(device)
            v = (v.reshape(shape) if shape is not None else v).contiguous()
            return v.requires_grad_(requires_grad)

        n = scene.num
        return cls(t(scene.positions), t(scene.rotations), t(scene.scales), t(scene.density, (n, 1)),
                   t(scene.features), scene.sh_degree, filter_3d)

    @property
    def num_gaussians(self) -> int:
        return int(self.positions.shape[0])

    def parameters(self) -> list[torch.Tensor]:
        return [self.positions, self.rotation, self.scale, self.density, self.features]

    def get_rotation(self):
        return self.rotation

    def get_scale(self):
        return self.scale

    def get_scale_with_3D_filter(self):
        return scale_with_3d_filter(self.scale, self.filter_3d)

    def get_density(self):
        return self.density

    def get_features(self):
        return self.features


def _pack_rows(pos, dns, rot, scl, idns, factor, inverse):
    """The [N,32] particle rows (reference tracer.py:171-179): one sm_100a
    kernel for CUDA tensors, a concatenation for host tensors."""
    n = pos.shape[0]
    parts = [t.detach().float().contiguous() for t in (pos, dns, rot, scl, idns, factor, inverse)]
    if not pos.is_cuda:
        return torch.cat([parts[0], parts[1].reshape(n, 1), parts[2], parts[3], parts[4].reshape(n, 1),
                          parts[5].reshape(n, 9), parts[6].reshape(n, 9), pos.new_zeros((n, 2))], dim=1)
    rows = torch.empty((n, 32), dtype=torch.float32, device=pos.device)
    _native.check(_native.load().gf_pack_particle_rows(*(t.data_ptr() for t in parts), n, rows.data_ptr(),
                                                       torch.cuda.current_stream(pos.device).cuda_stream),
                  "pack particle rows")
    return rows


def _unpack_rows(grad):
    """Per-slot gradients of the [N,32] row gradient (reference tracer.py:334-343):
    position [N,3], view density [N,1], rotation [N,4], scale [N,3],
    intrinsic density [N,1], factor [N,3,3], inverse factor [N,3,3]."""
    n = grad.shape[0]
    if not grad.is_cuda:
        g_pos, g_dns, g_rot, g_scl, g_idns, g_factor, g_inverse, _pad = torch.split(grad, list(PACKED_SPLIT), dim=1)
        return (g_pos.contiguous(), g_dns.contiguous(), g_rot.contiguous(), g_scl.contiguous(), g_idns.contiguous(),
                g_factor.reshape(-1, 3, 3), g_inverse.reshape(-1, 3, 3))
    out = [grad.new_empty(shape) for shape in ((n, 3), (n, 1), (n, 4), (n, 3), (n, 1), (n, 3, 3), (n, 3, 3))]
    _native.check(_native.load().gf_unpack_particle_rows(grad.contiguous().data_ptr(), n,
                                                         *(t.data_ptr() for t in out),
                                                         torch.cuda.current_stream(grad.device).cuda_stream),
                  "unpack particle rows")
    return tuple(out)


def _plain(conf):
    """A nested dict view of ``conf`` for the native renderer's settings."""
    if conf is None or isinstance(conf, dict):
        return conf
    to_container = getattr(type(conf), "to_container", None)
    if to_container is not None:
        return to_container(conf)
    out = {}
    for section in ("render", "loss"):
        node = getattr(conf, section, None)
        if node is not None:
            out[section] = node if isinstance(node, dict) else dict(vars(node))
    return out


__all__ = ["PACKED_SPLIT", "SceneGaussians", "Tracer"]
