"""Forward-only renderer of a frozen scene (reference
threedgut_tracer/inference.py:77-235, same constructor, ``freeze``,
``view_shape`` and ``render``).

Per scene, ``freeze`` packs the fixed slots of the [N,32] particle rows once:
position, rotation, the intrinsic scale (with the physical-mip 3-D filter in
quadrature when the model has it on) and the intrinsic density.  Per frame
only the view-dependent slots are rewritten: the pixel-footprint covariance
Q_v of the frame's camera, the full shape C = R S^2 R^T + Q_v with its factor
B = C^(1/2) (or the Cholesky factor), B^-1 and the mass-preserving density
m * o, followed by one forward trace.

Shape modes:

* ``"exact"``: the reference operators — ``current_view_q6`` and
  ``build_full_shape`` (float64 Jacobi symmetric square root);
* ``"fused"``, ``"fused32"``, ``"fusedmix"``: one fused kernel per frame that
  writes Q_v, the Cholesky factor and m straight into the packed rows
  (reference fast_shape.cu:136-197, the real-time renderer's path).  The
  reference's float32 variants are served by the same float64 kernel.

With a zero pixel footprint (gamma = 0) the factors do not depend on the view
and are computed once per scene (``cache_static_shape``).
"""

from __future__ import annotations

import ctypes
from typing import Any

import torch

from . import _native
from .batch import create_camera_parameters
from .physical_mip import scale_with_3d_filter
from .physical_tile_mask import build_physical_tile_binding
from .scene import PACKED_WIDTH, SLOTS
from .splat_raster import SplatRaster, _select
from .view_observation_filter import current_view_q6, pixel_footprint_variance, shape_camera

# frames whose full-shape status may still be in flight when render returns
MAX_UNCHECKED_SHAPES = 8

SHAPE_MODES = ("exact", "fused", "fused32", "fusedmix")


class FrozenGaussians:
    """A trained scene with the accessors the inference renderer reads (the
    reference model's ``get_rotation``, ``get_density``, ``get_scale``,
    ``get_scale_with_3D_filter`` and ``get_features``), as device tensors of
    already-activated values.  ``filter_3d`` [N,1] switches the physical-mip
    3-D filter on."""

    def __init__(self, positions, rotations, scales, density, features, sh_degree: int, filter_3d=None):
        self.positions = positions.contiguous()
        self._rotation = rotations.contiguous()
        self._scale = scales.contiguous()
        self._density = density.reshape(-1, 1).contiguous()
        self._features = features.contiguous()
        self.n_active_features = int(sh_degree)
        self.ray_feature_dim = 3
        self.filter_3d = filter_3d
        self._use_physical_mip3d_filter = filter_3d is not None

    @classmethod
    def from_scene(cls, scene, device, filter_3d=None) -> "FrozenGaussians":
        def t(a):
            return torch.as_tensor(a, dtype=torch.float32).to(device).contiguous()

        return cls(t(scene.positions), t(scene.rotations), t(scene.scales), t(scene.density), t(scene.features),
                   scene.sh_degree, filter_3d)

    def get_rotation(self):
        return self._rotation

    def get_density(self):
        return self._density

    def get_scale(self):
        return self._scale

    def get_scale_with_3D_filter(self):
        return scale_with_3d_filter(self._scale, self.filter_3d)

    def get_features(self):
        return self._features


class InferenceTracer:
    """Forward-only renderer bound to one frozen scene."""

    def __init__(self, conf, model, cache_static_shape: bool = True, shape: str = "exact"):
        if _select(conf, "render.primitive_type", "instances") == "trisurfel":
            raise RuntimeError("GOFish renders volumetric Gaussians only")
        if shape not in SHAPE_MODES:
            raise ValueError(f"unknown shape mode {shape!r}")
        self.conf = conf
        self.wrapper = SplatRaster(conf)
        self.gamma = pixel_footprint_variance(conf)
        self._tile_tokens: dict = {}
        self._registered: set = set()
        self.cache_static_shape = bool(cache_static_shape)
        self.static_shape = None
        self._unchecked_shapes: list = []
        self.shape_mode = shape
        self._status = None
        self.freeze(model)

    @torch.no_grad()
    def freeze(self, model) -> None:
        """Pack the per-scene fixed data of ``model``."""
        self.positions = model.positions.detach().contiguous()
        self.rotation = model.get_rotation().detach().contiguous()
        self.raw_density = model.get_density().detach().contiguous()
        scale = (model.get_scale_with_3D_filter()
                 if bool(getattr(model, "_use_physical_mip3d_filter", False)) else model.get_scale())
        self.physical_scale = scale.detach().contiguous()
        self.features = model.get_features().detach().contiguous()
        self.n_active_features = int(model.n_active_features)
        self.ray_feature_dim = int(model.ray_feature_dim)
        n = int(self.positions.shape[0])
        for name, value in (("positions", self.positions), ("rotation", self.rotation),
                            ("density", self.raw_density), ("scale", self.physical_scale)):
            if value.dtype != torch.float32:
                raise RuntimeError(f"inference renderer expects float32 {name}")
            if not value.is_cuda:
                raise RuntimeError(f"inference renderer expects CUDA {name}")
        packed = torch.zeros((n, PACKED_WIDTH), dtype=torch.float32, device=self.positions.device)
        packed[:, slice(*SLOTS["position"])] = self.positions
        packed[:, slice(*SLOTS["rotation"])] = self.rotation
        packed[:, slice(*SLOTS["scale"])] = self.physical_scale
        packed[:, slice(*SLOTS["intrinsic_density"])] = self.raw_density.reshape(n, 1)
        self.packed = packed
        self.num_gaussians = n
        self.static_shape = None
        self._packed_shape = None

    def _tile_token(self, gpu_batch, rays) -> str:
        mask = getattr(gpu_batch, "physical_fov_mask", None)
        domain = getattr(gpu_batch, "physical_fov_key", None)
        if domain is None:
            domain = "full-raster" if mask is None else f"mask:{id(mask)}"
        key = (str(domain), str(rays.device), int(rays.shape[1]), int(rays.shape[2]))
        binding = self._tile_tokens.get(key)
        if binding is None:
            tile = int(_select(self.conf, "render.gofish.fast_tile_size", 16) or 16)
            binding = build_physical_tile_binding(gpu_batch, rays, str(domain), tile=tile)
            self._tile_tokens[key] = binding
        if binding.token not in self._registered:
            self.wrapper.register_physical_tile_mask(binding.mask, binding.token)
            self._registered.add(binding.token)
        return binding.token

    def view_shape(self, gpu_batch):
        """C = Sigma + Q_v and the mass-preserving density (reference operators);
        computed once per scene when gamma = 0."""
        from .footprint_shape_operator import build_full_shape

        if self.static_shape is not None:
            return self.static_shape
        q6, jacobian, observed = current_view_q6(self.positions, gpu_batch, self.gamma, host_sync_free=True)
        shape = build_full_shape(self.physical_scale, self.rotation, self.raw_density, q6, jacobian, observed,
                                 mass_preserving=True, pixel_variance=self.gamma, defer_check=True)
        # the status words are checked once they reach the host (at most
        # MAX_UNCHECKED_SHAPES frames later, or by check_shapes())
        self._unchecked_shapes.append(shape)
        self._check_shapes(MAX_UNCHECKED_SHAPES)
        if self.gamma == 0.0 and self.cache_static_shape:
            self.static_shape = shape
        return shape

    def _check_shapes(self, keep: int) -> None:
        while self._unchecked_shapes:
            shape = self._unchecked_shapes[0]
            if len(self._unchecked_shapes) <= keep and not shape.ready():
                return
            self._unchecked_shapes.pop(0)
            shape.check()

    def check_shapes(self) -> None:
        """Waits for every rendered frame's shape status and raises
        FootprintNumericalError for the first failed row."""
        self._check_shapes(0)

    def _fused_shape(self, gpu_batch) -> None:
        """Q_v, the Cholesky factor and m of every row written into the packed rows."""
        if self._status is None:
            self._status = torch.zeros(4, dtype=torch.int32, device=self.positions.device)
        cam = shape_camera(gpu_batch)
        stream = torch.cuda.current_stream(self.positions.device).cuda_stream
        _native.check(_native.load().gf_view_shape_packed(
            self.positions.data_ptr(), self.rotation.data_ptr(), self.physical_scale.data_ptr(),
            self.raw_density.data_ptr(), self.num_gaussians, ctypes.byref(cam), float(self.gamma), 1,
            self.packed.data_ptr(), self._status.data_ptr(), stream), "fused view shape")

    def shape_status(self) -> int:
        """Failure flags of the last fused shape pass (0: every row factorised)."""
        return 0 if self._status is None else int(self._status[0])

    @torch.no_grad()
    def render(self, gpu_batch) -> dict[str, Any]:
        rays_o = gpu_batch.rays_ori.contiguous()
        rays_d = gpu_batch.rays_dir.contiguous()
        token = self._tile_token(gpu_batch, rays_d)
        sensor, poses = create_camera_parameters(gpu_batch)
        if self.shape_mode != "exact":
            self._fused_shape(gpu_batch)
            shape = self._packed_shape = None
        else:
            shape = self.view_shape(gpu_batch)
        if shape is not None and shape is not self._packed_shape:  # a cached static shape is packed once
            n = self.num_gaussians
            self.packed[:, slice(*SLOTS["density"])] = shape.density.reshape(n, 1)
            self.packed[:, slice(*SLOTS["factor"])] = shape.factor.reshape(n, 9)
            self.packed[:, slice(*SLOTS["inverse_factor"])] = shape.inverse_factor.reshape(n, 9)
            self._packed_shape = shape
        features_alpha, hit_distance = self.wrapper.trace_inference(
            self.n_active_features, self.packed, self.features, rays_o, rays_d, sensor, poses.timestamps_us[0],
            poses.timestamps_us[1], poses.T_world_sensors[0], poses.T_world_sensors[1], token)
        f = self.ray_feature_dim
        return {
            "pred_features": features_alpha[..., :f].unsqueeze(0).contiguous(),
            "pred_opacity": features_alpha[..., f:].unsqueeze(0).contiguous(),
            "pred_dist": hit_distance.unsqueeze(0).contiguous(),
        }


__all__ = ["FrozenGaussians", "InferenceTracer", "SHAPE_MODES"]
