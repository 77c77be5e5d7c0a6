"""``SplatRaster``: the reference's native renderer object, over the C ABI.

Method names, argument order and outputs follow the reference's pybind module
(threedgut_tracer/bindings.cpp:106-124, src/splatRaster.cpp): ``trace``,
``trace_bwd``, ``trace_inference``, ``register_physical_tile_mask``,
``collect_times``, and the densification statistic's
``set_exact_screen_absgrad_map`` and ``collect_abs_grad``.  Tensors stay on the device of the rays; every call is
enqueued on the current CUDA stream of that device.
"""

from __future__ import annotations

import ctypes
import math
from typing import Any, Mapping

import torch

from . import _native
from ._native import (GfTraceGrads, GfTraceInputs, GfTraceOutputs, GfTracerConfig, GfTraceStats, check)
from .camera import CameraModelParameters

# Channels of the reference's trace() outputs that are produced by the SOF
# geometric losses of training (normals, distortion moments, quantile and
# exact-crossing depth, extent, opacity field, inverse-depth moments).
QUANT_CHANNELS = 10


def _select(conf: Mapping[str, Any] | None, path: str, default):
    node: Any = conf
    for part in path.split("."):
        if not isinstance(node, Mapping) or part not in node:
            return default
        node = node[part]
    return default if node is None else node


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _pose7(pose) -> list[float]:
    values = torch.as_tensor(pose, dtype=torch.float32).reshape(-1).cpu().tolist()
    if len(values) != 7:
        raise ValueError("sensor pose must have 7 values [tx, ty, tz, qx, qy, qz, qw]")
    return values


class SplatRaster:
    """Renderer state of one scene/configuration (reference SplatRaster)."""

    def __init__(self, conf: Mapping[str, Any] | None = None):
        self._lib = _native.load()
        cfg = GfTracerConfig()
        cfg.k_buffer_size = int(_select(conf, "render.splat.k_buffer_size", 16))
        cfg.sort_key = (_native.GF_KEY_GLOBAL_DEPTH if bool(_select(conf, "render.gofish.fast_global_depth_key", False))
                        else _native.GF_KEY_PER_TILE_DEPTH)
        cfg.enable_hit_counts = 1 if bool(_select(conf, "render.enable_hitcounts", True)) else 0
        # particles without a valid projection (setup_3dgut.py:232-239): dropped, the cone test, or the cone
        # test restricted to spheres away from the camera whose cap half-angle lies in a window (degrees)
        fallback = str(_select(conf, "render.gofish.fast_admission_fallback", "cone"))
        modes = {"none": _native.GF_FALLBACK_NONE, "cone": _native.GF_FALLBACK_CONE,
                 "cone_big": _native.GF_FALLBACK_CONE_BIG}
        if fallback not in modes:
            raise ValueError("render.gofish.fast_admission_fallback must be 'none', 'cone' or 'cone_big' "
                             f"(got {fallback!r})")
        cfg.admission_fallback = modes[fallback]
        cfg.fallback_min_angle = math.radians(float(_select(conf, "render.gofish.fast_admission_fallback_min_angle_deg",
                                                            0.0)))
        cfg.fallback_max_angle = math.radians(float(_select(conf, "render.gofish.fast_admission_fallback_max_angle_deg",
                                                            90.0)))
        # partial UT (gutProjector.cuh:53-62): None = off, else the covariance scale of repaired projections
        partial = _select(conf, "render.gofish.fast_partial_ut_scale", None)
        cfg.partial_ut_scale = 0.0 if partial is None else float(partial)
        if partial is not None and not cfg.partial_ut_scale > 0.0:
            raise ValueError(f"render.gofish.fast_partial_ut_scale must be positive (got {partial!r})")
        # entries per pixel of the composite log the backward reads (0: default, < 0: replay every tile)
        cfg.composite_log_capacity = int(_select(conf, "render.splat.composite_log_capacity", 0))
        # the geometric training channels (normals, depth moments, quantile depths, extent, inverse depth)
        cfg.enable_normals = 1 if bool(_select(conf, "render.enable_normals", False)) else 0
        # tile-intersection keys: "speculative" (no host synchronization; an overflowed forward renders nothing
        # and the next call raises) or "exact" (one synchronization per forward reads the count)
        capacity = str(_select(conf, "render.splat.intersection_capacity", "speculative"))
        if capacity not in ("speculative", "exact"):
            raise ValueError(f"render.splat.intersection_capacity must be 'speculative' or 'exact' (got {capacity!r})")
        cfg.intersection_capacity = (_native.GF_CAPACITY_EXACT if capacity == "exact"
                                     else _native.GF_CAPACITY_SPECULATIVE)
        # SOF's HEAD4 / MID8 / TAIL64 hierarchy instead of the flat k-buffer
        hierarchical = bool(_select(conf, "render.splat.hierarchical_sort", False))
        if hierarchical and not bool(_select(conf, "render.splat.sof_mid8_hierarchy", True)):
            raise NotImplementedError("render.splat.hierarchical_sort renders with SOF's MID8 hierarchy only")
        if hierarchical and (int(_select(conf, "render.splat.head_size", 4)) != 4
                             or int(_select(conf, "render.splat.mid_size", 8)) != 8
                             or int(_select(conf, "render.splat.tail_size", 64)) != 64):
            raise ValueError("SOF's hierarchy uses HEAD4, MID8 and TAIL64")
        cfg.compositor = _native.GF_COMPOSITOR_SOF if hierarchical else _native.GF_COMPOSITOR_KBUFFER
        # every particle admitted by the conservative cone test (complete: no pixel's hit is missed)
        cfg.complete_admission = 1 if bool(_select(conf, "render.gofish.complete_admission", False)) else 0
        handle = self._lib.gf_tracer_create(ctypes.byref(cfg))
        if not handle:
            raise _native.NativeError("gf_tracer_create failed: " + self._lib.gf_last_error().decode())
        self._handle = ctypes.c_void_p(handle)
        self.config = cfg
        self._masks: dict[str, torch.Tensor] = {}
        self._times: dict[str, float] = {}
        self._events: list[tuple[str, torch.cuda.Event, torch.cuda.Event]] = []
        self.enable_kernel_timings = bool(_select(conf, "render.enable_kernel_timings", False))
        # densification statistic (setup_3dgut.py:135,182): per-hit |map g| with a caller-armed map, or per-hit
        # |g| in world space
        self._abs_grad_screen = bool(_select(conf, "strategy.densify.generic_camera_absgrad", True))
        self._abs_workspace: torch.Tensor | None = None
        self._last_abs_grad: torch.Tensor | None = None

    def __del__(self):
        handle = getattr(self, "_handle", None)
        if handle is not None and handle.value:
            self._lib.gf_tracer_destroy(handle)
            self._handle = None

    # ------------------------------------------------------------------ registry
    def register_physical_tile_mask(self, mask: torch.Tensor, token: str) -> None:
        """splatRaster.cpp:229-248: keep the uint8 [Ty,Tx] tile mask under ``token``."""
        if mask.dtype != torch.uint8 or mask.ndim != 2 or not mask.is_cuda:
            raise RuntimeError("physical tile mask must be a CUDA uint8 [Ty,Tx] tensor")
        mask = mask.contiguous()
        with torch.cuda.device(mask.device):
            check(self._lib.gf_tracer_register_tile_mask(self._handle, mask.data_ptr(), mask.shape[0], mask.shape[1],
                                                         token.encode(), _stream(mask.device)),
                  "register_physical_tile_mask")
        self._masks[token] = mask

    # ------------------------------------------------------------------ helpers
    def _inputs(self, frame, n_active_features, particle_density, particle_radiance, ray_ori, ray_dir,
                sensor: CameraModelParameters, t0, t1, pose0, pose1, token) -> GfTraceInputs:
        for name, t in (("particle_density", particle_density), ("particle_radiance", particle_radiance),
                        ("ray_ori", ray_ori), ("ray_dir", ray_dir)):
            if not t.is_cuda or t.dtype != torch.float32 or not t.is_contiguous():
                raise RuntimeError(f"{name} must be a contiguous CUDA float32 tensor")
        if particle_density.ndim != 2 or particle_density.shape[1] != 32:
            raise RuntimeError("particle_density must be [N,32]")
        n = particle_density.shape[0]
        if particle_radiance.shape[0] != n or particle_radiance.numel() % (3 * max(n, 1)) != 0:
            raise RuntimeError("particle_radiance must be [N, 3*C]")
        if ray_ori.ndim != 4 or ray_ori.shape[0] != 1 or ray_ori.shape[-1] != 3 or ray_dir.shape != ray_ori.shape:
            raise RuntimeError("rays must be [1,H,W,3]")
        height, width = int(ray_ori.shape[1]), int(ray_ori.shape[2])
        inp = GfTraceInputs()
        inp.frame = int(frame)
        inp.sh_degree = int(n_active_features)
        inp.num_particles = n
        inp.sh_coeffs = particle_radiance.numel() // (3 * n) if n > 0 else 1
        inp.particles = particle_density.data_ptr()
        inp.features = particle_radiance.data_ptr()
        inp.ray_origin = ray_ori.data_ptr()
        inp.ray_direction = ray_dir.data_ptr()
        inp.camera = sensor.native(width, height)
        inp.pose_start[:] = _pose7(pose0)
        inp.pose_end[:] = _pose7(pose1)
        inp.timestamp_start = int(t0)
        inp.timestamp_end = int(t1)
        inp.tile_token = token.encode()
        return inp

    def _timed(self, name: str, device):
        if not self.enable_kernel_timings:
            return None
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record(torch.cuda.current_stream(device))
        self._events.append((name, start, end))
        return end

    # ------------------------------------------------------------------ trace
    def trace(self, frame_id, sof_exact_opacity_active, n_active_features, particle_density, particle_radiance,
              ray_ori, ray_dir, ray_time, sensor, t0, t1, pose0, pose1, token):
        """splatRaster.cpp:259-380.  Returns the reference's 11 tensors:
        radiance+opacity [H,W,4], hit distance [H,W,1], hit count [H,W,1],
        visibility [N,1], and the seven training geometric channels."""
        if sof_exact_opacity_active and not self.config.enable_normals:
            raise ValueError("the SOF opacity field needs render.enable_normals (its exact crossing depth)")
        device = ray_ori.device
        height, width = int(ray_ori.shape[1]), int(ray_ori.shape[2])
        n = particle_density.shape[0]
        f32 = dict(dtype=torch.float32, device=device)
        rgba = torch.empty((height, width, 4), **f32)
        hit_distance = torch.empty((height, width, 1), **f32)
        hit_count = torch.zeros((height, width, 1), **f32)
        visibility = torch.zeros((n, 1), **f32)
        inp = self._inputs(frame_id, n_active_features, particle_density, particle_radiance, ray_ori, ray_dir,
                           sensor, t0, t1, pose0, pose1, token)
        out = GfTraceOutputs()
        out.rgba = rgba.data_ptr()
        out.hit_distance = hit_distance.data_ptr()
        out.hit_count = hit_count.data_ptr()
        out.visibility = visibility.data_ptr() if n > 0 else None
        zeros = lambda c: torch.zeros((height, width, c), **f32)  # noqa: E731
        # normal, depth var, quantiles, extent, opacity field, inverse depth, inverse depth squared
        geo = [zeros(3), zeros(1), zeros(QUANT_CHANNELS), zeros(1), zeros(1), zeros(1), zeros(1)]
        if self.config.enable_normals:
            out.normal, out.depth_var, out.quant, out.extent = (t.data_ptr() for t in geo[:4])
            out.inv_depth, out.inv_depth2 = geo[5].data_ptr(), geo[6].data_ptr()
        if sof_exact_opacity_active:
            inp.sof_opacity_active = 1
            out.opacity_field = geo[4].data_ptr()
        with torch.cuda.device(device):
            end = self._timed("forward_render", device)
            check(self._lib.gf_tracer_trace(self._handle, ctypes.byref(inp), ctypes.byref(out), _stream(device)),
                  "trace")
            if end is not None:
                end.record(torch.cuda.current_stream(device))
        return (rgba, hit_distance, hit_count, visibility, *geo)

    def trace_inference(self, n_active_features, particle_density, particle_radiance, ray_ori, ray_dir, sensor, t0,
                        t1, pose0, pose1, token):
        """splatRaster.cpp:383-466: radiance+opacity [H,W,4], hit distance [H,W,1]."""
        device = ray_ori.device
        height, width = int(ray_ori.shape[1]), int(ray_ori.shape[2])
        f32 = dict(dtype=torch.float32, device=device)
        rgba = torch.empty((height, width, 4), **f32)
        hit_distance = torch.empty((height, width, 1), **f32)
        inp = self._inputs(0, n_active_features, particle_density, particle_radiance, ray_ori, ray_dir, sensor, t0,
                           t1, pose0, pose1, token)
        with torch.cuda.device(device):
            check(self._lib.gf_tracer_trace_inference(self._handle, ctypes.byref(inp), rgba.data_ptr(),
                                                      hit_distance.data_ptr(), _stream(device)), "trace_inference")
        return rgba, hit_distance

    def trace_bwd(self, frame_id, sof_exact_opacity_active, n_active_features, particle_density, particle_radiance,
                  ray_ori, ray_dir, ray_time, sensor, t0, t1, pose0, pose1, ray_features_density,
                  ray_features_density_grd, ray_hit_distance, ray_hit_distance_grd, *geometry_and_token):
        """splatRaster.cpp:469-640.  ``geometry_and_token`` holds the seven
        (value, gradient) pairs of the geometric channels followed by the tile
        token, as in the reference's argument list.  Returns the [N,32]
        particle gradient and the [N, 3*C] SH gradient."""
        *geometry, token = geometry_and_token
        if len(geometry) not in (0, 14):
            raise TypeError("trace_bwd expects the seven (value, gradient) geometric channel pairs and the token")
        device = ray_ori.device
        n = particle_density.shape[0]
        grad_particles = torch.empty((n, 32), dtype=torch.float32, device=device)
        grad_features = torch.empty_like(particle_radiance)
        inp = self._inputs(frame_id, n_active_features, particle_density, particle_radiance, ray_ori, ray_dir,
                           sensor, t0, t1, pose0, pose1, token)
        g = GfTraceGrads()
        rgba = ray_features_density.float().contiguous()
        grad_rgba = ray_features_density_grd.float().contiguous()
        hd = ray_hit_distance.contiguous()
        ghd = (ray_hit_distance_grd if ray_hit_distance_grd is not None else torch.zeros_like(hd)).contiguous()
        g.rgba = rgba.data_ptr()
        g.hit_distance = hd.data_ptr()
        g.grad_rgba = grad_rgba.data_ptr()
        g.grad_hit_distance = ghd.data_ptr()
        g.grad_particles = grad_particles.data_ptr()
        g.grad_features = grad_features.data_ptr()
        keep = self._geometry_grads(g, geometry, int(ray_ori.shape[1]), int(ray_ori.shape[2]))
        abs_grad = self._abs_grad_buffer(n, device)
        if abs_grad is not None:
            g.position_abs_grad = abs_grad.data_ptr()
            g.position_abs_grad_mode = _native.GF_ABS_GRAD_SCREEN if self._abs_grad_screen else _native.GF_ABS_GRAD_WORLD
        with torch.cuda.device(device):
            end = self._timed("backward_render", device)
            check(self._lib.gf_tracer_trace_bwd(self._handle, ctypes.byref(inp), ctypes.byref(g), _stream(device)),
                  "trace_bwd")
            if end is not None:
                end.record(torch.cuda.current_stream(device))
        # splatRaster.cpp:628-637: the statistic of this backward
        if self._abs_grad_screen:
            self._last_abs_grad = None if abs_grad is None else abs_grad[:, 6:8].contiguous()
            self._abs_workspace = None
        else:
            self._last_abs_grad = abs_grad
        return grad_particles, grad_features

    # ------------------------------------------------------------------ densification statistic
    def _abs_grad_buffer(self, n: int, device) -> torch.Tensor | None:
        """The statistic's buffer for a backward over n particles
        (splatRaster.cpp:515-531): the armed [N,8] map workspace in screen
        mode (None when unarmed), a zeroed [N,3] in world mode."""
        if not self._abs_grad_screen:
            return torch.zeros((n, 3), dtype=torch.float32, device=device)
        w = self._abs_workspace
        if w is None:
            return None
        if w.device != device or w.dim() != 2 or w.shape[0] != n or w.shape[1] != 8:
            raise RuntimeError("exact screen AbsGrad workspace differs")
        return w

    def set_exact_screen_absgrad_map(self, mapping: torch.Tensor) -> None:
        """splatRaster.cpp:688-698: arms the next backward with the per-particle
        2x3 map M (float32 [N,2,3] on the device); that backward adds, for every
        composited hit, |M g| of the hit's position gradient g to the
        particle's two sums, which collect_abs_grad() then returns."""
        if not self._abs_grad_screen:
            raise RuntimeError("set_exact_screen_absgrad_map needs strategy.densify.generic_camera_absgrad")
        if not (torch.is_tensor(mapping) and mapping.is_cuda and mapping.dtype == torch.float32
                and mapping.is_contiguous() and mapping.dim() == 3 and mapping.shape[1] == 2 and mapping.shape[2] == 3):
            raise RuntimeError("exact screen AbsGrad map must be contiguous CUDA float32 [N,2,3]")
        if self._abs_workspace is not None:
            raise RuntimeError("exact screen AbsGrad map was armed twice before backward")
        w = torch.zeros((mapping.shape[0], 8), dtype=torch.float32, device=mapping.device)
        w[:, 0:6].copy_(mapping.reshape(mapping.shape[0], 6))
        self._abs_workspace = w

    def collect_abs_grad(self) -> torch.Tensor | None:
        """splatRaster.cpp:642-650: the statistic of the last backward, [N,2]
        in screen mode (raises if that backward was not armed), [N,3] in
        world mode."""
        last = self._last_abs_grad
        if self._abs_grad_screen and (last is None or last.dim() != 2 or last.shape[1] != 2):
            raise RuntimeError("exact screen AbsGrad was not armed for the last backward")
        return last

    # (value, gradient) pairs of trace_bwd in the reference's order (splatRaster.cpp:469-500) and their
    # channel widths; of the quantile channels only the exact crossing depth (channel 8) carries a
    # gradient, and the forward values also feed the opacity field's gradient
    GEOMETRY_PAIRS = (("depth_var", 1), ("extent", 1), ("opacity_field", 1), ("quant", QUANT_CHANNELS),
                      ("normal", 3), ("inv_depth", 1), ("inv_depth2", 1))

    def _geometry_grads(self, g: GfTraceGrads, geometry, height: int, width: int) -> list:
        """Fills the geometric channel pairs of ``g`` (enable_normals); returns the
        tensors that must outlive the call."""
        keep = []
        if not geometry or not self.config.enable_normals:
            return keep
        for i, (name, channels) in enumerate(self.GEOMETRY_PAIRS):
            value, grad = geometry[2 * i], geometry[2 * i + 1]
            if name == "quant":
                # the forward's crossing depths (read by the opacity field's gradient) and the crossing
                # depth's gradient (implicit-function backward through the hits up to the crossing)
                if value is not None and value.numel() == height * width * channels:
                    q = value.float().contiguous()
                    keep.append(q)
                    g.quant = q.data_ptr()
                    if grad is not None and grad.numel() == height * width * channels:
                        gq = grad.float().contiguous()
                        keep.append(gq)
                        g.grad_quant = gq.data_ptr()
                continue
            if grad is None or value is None or grad.numel() != height * width * channels:
                continue
            if name == "opacity_field":
                v, gv = value.float().contiguous(), grad.float().contiguous()
                keep += [v, gv]
                g.opacity_field, g.grad_opacity_field = v.data_ptr(), gv.data_ptr()
                continue
            v = value.float().contiguous()
            d = grad.float().contiguous()
            keep += [v, d]
            setattr(g, name, v.data_ptr())
            setattr(g, "grad_" + name, d.data_ptr())
        return keep

    # ------------------------------------------------------------------ introspection
    def collect_times(self) -> dict[str, float]:
        """splatRaster.cpp:702-732: milliseconds of the timed calls since the last collection."""
        times: dict[str, float] = {}
        for name, start, end in self._events:
            end.synchronize()
            times[name] = times.get(name, 0.0) + start.elapsed_time(end)
        self._events.clear()
        return times

    def enable_stage_timing(self, enable: bool = True) -> None:
        check(self._lib.gf_tracer_enable_timing(self._handle, 1 if enable else 0), "enable_timing")

    def collect_stage_times(self) -> dict[str, tuple[float, int]]:
        """Milliseconds and launch count per native stage since the last collection."""
        ms = (ctypes.c_float * len(_native.STAGES))()
        launches = (ctypes.c_uint32 * len(_native.STAGES))()
        check(self._lib.gf_tracer_collect_times(self._handle, ms, launches), "collect_times")
        return {name: (float(ms[i]), int(launches[i])) for i, name in enumerate(_native.STAGES)}

    def stats(self) -> GfTraceStats:
        st = GfTraceStats()
        check(self._lib.gf_tracer_stats(self._handle, ctypes.byref(st)), "stats")
        return st

    def log_overflow_tiles(self) -> int:
        """Tiles of the last training forward replayed by the backward because a
        pixel composited more hits than the composite log holds (waits for
        that forward's render)."""
        tiles = ctypes.c_uint32(0)
        check(self._lib.gf_tracer_log_overflow_tiles(self._handle, ctypes.byref(tiles)), "log_overflow_tiles")
        return int(tiles.value)

    def copy_intermediates(self, device) -> dict[str, torch.Tensor]:
        """Projected state, radiance, counts, sorted keys/ids and tile ranges of the last forward."""
        st = self.stats()
        n, t, i = st.num_particles, st.num_tiles, st.num_intersections
        dev = torch.device(device)
        proj = torch.empty((n, 8), dtype=torch.float32, device=dev)
        rgb = torch.empty((n, 3), dtype=torch.float32, device=dev)
        counts = torch.empty((n,), dtype=torch.int32, device=dev)
        keys = torch.empty((max(i, 1),), dtype=torch.int64, device=dev)
        ids = torch.empty((max(i, 1),), dtype=torch.int32, device=dev)
        ranges = torch.empty((t, 2), dtype=torch.int32, device=dev)
        with torch.cuda.device(dev):
            check(self._lib.gf_tracer_copy_intermediates(self._handle, proj.data_ptr(), rgb.data_ptr(),
                                                         counts.data_ptr(), keys.data_ptr(), ids.data_ptr(), max(i, 1),
                                                         ranges.data_ptr(), _stream(dev)), "copy_intermediates")
        return dict(proj=proj, rgb=rgb, counts=counts, keys=keys[:i], ids=ids[:i], ranges=ranges)
