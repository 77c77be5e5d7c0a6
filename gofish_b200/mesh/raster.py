"""The mesh SplatRaster methods over the C ABI (gf_field_*).

Mirrors the pybind class of gofish/mesh/native/bindings.cpp:82-114: the
same method names, argument order, tensor contracts and error messages
(opacityFieldBinding.inl:78-545).  Work runs on the current CUDA stream of
the query points' device; every call of one context must use that stream.
"""

from __future__ import annotations

import ctypes

import torch

from .. import _native
from .._native import FIELD_STAGES, GfFieldCamera, GfFieldStats


def _stream(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def _require(tensor: torch.Tensor, name: str, device: torch.device, dtype: torch.dtype) -> None:
    if not isinstance(tensor, torch.Tensor) or not tensor.is_cuda or not tensor.is_contiguous():
        raise RuntimeError(f"{name} must be a contiguous CUDA tensor")
    if tensor.device != device:
        raise RuntimeError(f"{name} is on the wrong CUDA device")
    if tensor.dtype != dtype:
        raise RuntimeError(f"{name} has the wrong dtype")


def _pose7(pose, name: str, device: torch.device) -> list[float]:
    if not isinstance(pose, torch.Tensor) or not pose.is_contiguous() or pose.dtype != torch.float32 \
            or pose.numel() != 7:
        raise RuntimeError(f"{name} must be contiguous float32 [7]")
    if pose.is_cuda and pose.device != device:
        raise RuntimeError(f"{name} is on the wrong CUDA device")
    return pose.detach().reshape(-1).cpu().tolist()


class SplatRaster:
    """Opacity-field state (one context at a time, as in the reference)."""

    def __init__(self, conf=None):
        self._lib = _native.load()
        handle = self._lib.gf_field_create()
        if not handle:
            raise _native.NativeError("gf_field_create failed")
        self._handle = ctypes.c_void_p(handle)
        self._device: torch.device | None = None
        self._queries = 0

    def __del__(self):
        handle = getattr(self, "_handle", None)
        if handle is not None and handle.value:
            self._lib.gf_field_destroy(handle)
            self._handle = None

    # ------------------------------------------------------------------ helpers
    def _begin(self, fn, what, particle_density, particle_sigma_max, query_points) -> int:
        if not isinstance(query_points, torch.Tensor) or not query_points.is_cuda:
            raise RuntimeError("query points must be CUDA")
        device = query_points.device
        if torch.cuda.current_device() != device.index:
            raise RuntimeError(f"{what}: expected cuda:{device.index}, current cuda:{torch.cuda.current_device()}")
        _require(query_points, "query points", device, torch.float32)
        _require(particle_density, "particle density", device, torch.float32)
        _require(particle_sigma_max, "particle sigma_max", device, torch.float32)
        if query_points.dim() != 2 or query_points.shape[1] != 3 or not 0 < query_points.shape[0] <= 2**31 - 1:
            raise RuntimeError("query points must be nonempty float32 [Q,3]")
        if particle_density.dim() != 2 or particle_density.shape[1] != 32 or \
                not 0 < particle_density.shape[0] <= 2**32 - 1:
            raise RuntimeError("particle density must be float32 [N,32]")
        n = particle_density.shape[0]
        if not ((particle_sigma_max.dim() == 1 or (particle_sigma_max.dim() == 2 and particle_sigma_max.shape[1] == 1))
                and particle_sigma_max.numel() == n):
            raise RuntimeError("particle sigma_max must be float32 [N] or [N,1]")
        token = ctypes.c_int64(0)
        _native.check(fn(self._handle, particle_density.data_ptr(), particle_sigma_max.data_ptr(), n,
                         query_points.data_ptr(), query_points.shape[0], ctypes.byref(token), _stream(device)), what)
        self._device = device
        self._queries = int(query_points.shape[0])
        return int(token.value)

    def _camera(self, frame_number, ray_origin, ray_direction, physical_mask, sensor_model, start_timestamp,
                end_timestamp, sensors_start_pose, sensors_end_pose) -> GfFieldCamera:
        device = self._device
        if device is None:
            raise RuntimeError("missing or stale opacity-field context")
        _require(ray_origin, "ray origin", device, torch.float32)
        _require(ray_direction, "ray direction", device, torch.float32)
        if ray_origin.shape != ray_direction.shape or ray_origin.dim() != 4 or ray_origin.shape[0] != 1 or \
                ray_origin.shape[3] != 3 or ray_origin.shape[1] <= 0 or ray_origin.shape[2] <= 0:
            raise RuntimeError("rays must be nonempty [1,H,W,3]")
        height, width = int(ray_origin.shape[1]), int(ray_origin.shape[2])
        if not torch.equal(ray_origin, ray_origin[:, :1, :1, :].expand_as(ray_origin)):
            raise RuntimeError("the opacity field requires one camera center per view")
        mask_ptr = None
        if physical_mask is not None and physical_mask.numel() != 0:
            _require(physical_mask, "physical mask", device, torch.uint8)
            if physical_mask.dim() != 2 or tuple(physical_mask.shape) != (height, width):
                raise RuntimeError("physical mask must be contiguous uint8 [H,W]")
            mask_ptr = physical_mask.data_ptr()
        cam = GfFieldCamera()
        cam.frame_number = int(frame_number)
        cam.camera = sensor_model.native(width, height)
        cam.ray_origin = ray_origin.data_ptr()
        cam.pixel_mask = mask_ptr
        cam.timestamp_start = int(start_timestamp)
        cam.timestamp_end = int(end_timestamp)
        cam.pose_start[:] = _pose7(sensors_start_pose, "camera start pose", device)
        cam.pose_end[:] = _pose7(sensors_end_pose, "camera end pose", device)
        return cam

    def _stream(self) -> int:
        if self._device is None:
            raise RuntimeError("missing or stale opacity-field context")
        return _stream(self._device)

    # ------------------------------------------------------------------ field
    def begin_opacity_field(self, particle_density, particle_sigma_max, query_points) -> int:
        """opacityFieldBinding.inl:203-268."""
        return self._begin(self._lib.gf_field_begin, "begin opacity field", particle_density, particle_sigma_max,
                           query_points)

    def integrate_opacity_field_camera(self, context_token, frame_number, ray_origin, ray_direction, physical_mask,
                                       sensor_model, start_timestamp, end_timestamp, sensors_start_pose,
                                       sensors_end_pose) -> None:
        """opacityFieldBinding.inl:270-316."""
        cam = self._camera(frame_number, ray_origin, ray_direction, physical_mask, sensor_model, start_timestamp,
                           end_timestamp, sensors_start_pose, sensors_end_pose)
        _native.check(self._lib.gf_field_integrate_camera(self._handle, int(context_token), ctypes.byref(cam),
                                                          self._stream()), "integrate opacity-field camera")

    def finish_opacity_field(self, context_token):
        """opacityFieldBinding.inl:318-338: (opacity f32[Q], observed u8[Q], above u8[Q])."""
        device = self._device
        if device is None:
            raise RuntimeError("missing or stale opacity-field context")
        q = self._queries
        opacity = torch.empty(q, dtype=torch.float32, device=device)
        observed = torch.empty(q, dtype=torch.uint8, device=device)
        above = torch.empty(q, dtype=torch.uint8, device=device)
        _native.check(self._lib.gf_field_finish(self._handle, int(context_token), opacity.data_ptr(),
                                                observed.data_ptr(), above.data_ptr(), self._stream()),
                      "finish opacity field")
        return opacity, observed, above

    def release_opacity_field(self, context_token) -> None:
        """opacityFieldBinding.inl:340-347."""
        _native.check(self._lib.gf_field_release(self._handle, int(context_token), self._stream()),
                      "release opacity field")

    # ------------------------------------------------------------------ bisection table
    def begin_bisection_table(self, particle_density, particle_sigma_max, probe_query_points) -> int:
        """opacityFieldBinding.inl:349-368."""
        return self._begin(self._lib.gf_field_begin_table, "begin bisection table", particle_density,
                           particle_sigma_max, probe_query_points)

    def stage_bisection_camera(self, context_token, frame_number, ray_origin, ray_direction, physical_mask,
                               sensor_model, start_timestamp, end_timestamp, sensors_start_pose,
                               sensors_end_pose) -> None:
        """opacityFieldBinding.inl:370-431."""
        cam = self._camera(frame_number, ray_origin, ray_direction, physical_mask, sensor_model, start_timestamp,
                           end_timestamp, sensors_start_pose, sensors_end_pose)
        _native.check(self._lib.gf_field_stage_camera(self._handle, int(context_token), ctypes.byref(cam),
                                                      self._stream()), "stage bisection camera")

    def seal_bisection_table(self, context_token) -> None:
        """opacityFieldBinding.inl:433-478."""
        _native.check(self._lib.gf_field_seal_table(self._handle, int(context_token), self._stream()),
                      "seal bisection table")

    def evaluate_bisection_round(self, context_token, query_points, round_ordinal):
        """opacityFieldBinding.inl:480-521: (above, observed, exact) u8[Q]."""
        device = self._device
        if device is None:
            raise RuntimeError("missing or stale opacity-field context")
        _require(query_points, "round query points", device, torch.float32)
        if query_points.dim() != 2 or query_points.shape[1] != 3 or query_points.shape[0] != self._queries:
            raise RuntimeError("round query shape differs from the table capacity")
        q = self._queries
        above = torch.empty(q, dtype=torch.uint8, device=device)
        observed = torch.empty(q, dtype=torch.uint8, device=device)
        exact = torch.empty(q, dtype=torch.uint8, device=device)
        _native.check(self._lib.gf_field_evaluate_round(self._handle, int(context_token), query_points.data_ptr(), q,
                                                        int(round_ordinal), above.data_ptr(), observed.data_ptr(),
                                                        exact.data_ptr(), self._stream()),
                      "evaluate bisection round")
        return above, observed, exact

    def reset_bisection_batch(self, context_token) -> None:
        """opacityFieldBinding.inl:523-531."""
        _native.check(self._lib.gf_field_reset_batch(self._handle, int(context_token), self._stream()),
                      "reset bisection batch")

    def release_bisection_table(self, context_token) -> None:
        """opacityFieldBinding.inl:533-545."""
        _native.check(self._lib.gf_field_release_table(self._handle, int(context_token), self._stream()),
                      "release bisection table")

    def stats(self) -> GfFieldStats:
        out = GfFieldStats()
        _native.check(self._lib.gf_field_get_stats(self._handle, ctypes.byref(out)), "field stats")
        return out

    def enable_stage_timing(self, enable: bool = True) -> None:
        """CUDA-event timing of every stage of later camera passes."""
        _native.check(self._lib.gf_field_enable_timing(self._handle, 1 if enable else 0), "field timing")

    def collect_stage_times(self) -> dict[str, tuple[float, int]]:
        """{stage: (milliseconds, kernel launches)} since the last collect."""
        ms = (ctypes.c_float * len(FIELD_STAGES))()
        launches = (ctypes.c_uint32 * len(FIELD_STAGES))()
        _native.check(self._lib.gf_field_collect_times(self._handle, ms, launches), "field timing")
        return {name: (float(ms[i]), int(launches[i])) for i, name in enumerate(FIELD_STAGES)}
