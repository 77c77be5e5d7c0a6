"""ctypes binding of the C ABI declared in include/gofish_b200.h.

Loading fails loudly: there is no CPU fallback for any entry point.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

from .build import LIBRARY

GF_OK = 0
GF_CAMERA_OPENCV_PINHOLE = 0
GF_CAMERA_OPENCV_FISHEYE = 1
GF_KEY_PER_TILE_DEPTH = 0
GF_KEY_GLOBAL_DEPTH = 1
GF_FALLBACK_NONE = 0
GF_CAPACITY_SPECULATIVE = 0
GF_CAPACITY_EXACT = 1
GF_COMPOSITOR_KBUFFER = 0
GF_COMPOSITOR_SOF = 1
GF_FALLBACK_CONE = 1
GF_FALLBACK_CONE_BIG = 5
GF_ABS_GRAD_SCREEN = 1
GF_ABS_GRAD_WORLD = 2
ABI_VERSION = 7  # GF_ABI_VERSION of include/gofish_b200.h
STAGES = ("tile_rays", "project", "scan", "emit", "sort", "ranges", "render_fwd", "render_bwd", "project_bwd")


class GfCamera(ctypes.Structure):
    _fields_ = [
        ("model", ctypes.c_int32),
        ("width", ctypes.c_int32),
        ("height", ctypes.c_int32),
        ("shutter", ctypes.c_int32),
        ("principal_point", ctypes.c_float * 2),
        ("focal_length", ctypes.c_float * 2),
        ("radial", ctypes.c_float * 6),
        ("tangential", ctypes.c_float * 2),
        ("thin_prism", ctypes.c_float * 4),
        ("max_angle", ctypes.c_float),
        ("reserved", ctypes.c_float),
    ]


class GfTracerConfig(ctypes.Structure):
    _fields_ = [
        ("k_buffer_size", ctypes.c_int32),
        ("sort_key", ctypes.c_int32),
        ("enable_hit_counts", ctypes.c_int32),
        ("admission_fallback", ctypes.c_int32),
        ("composite_log_capacity", ctypes.c_int32),
        ("enable_normals", ctypes.c_int32),
        ("intersection_capacity", ctypes.c_int32),
        ("compositor", ctypes.c_int32),
        ("complete_admission", ctypes.c_int32),
        ("fallback_min_angle", ctypes.c_float),
        ("fallback_max_angle", ctypes.c_float),
        ("partial_ut_scale", ctypes.c_float),
    ]


class GfTraceInputs(ctypes.Structure):
    _fields_ = [
        ("frame", ctypes.c_uint32),
        ("sh_degree", ctypes.c_int32),
        ("num_particles", ctypes.c_uint32),
        ("sh_coeffs", ctypes.c_uint32),
        ("particles", ctypes.c_void_p),
        ("features", ctypes.c_void_p),
        ("ray_origin", ctypes.c_void_p),
        ("ray_direction", ctypes.c_void_p),
        ("camera", GfCamera),
        ("pose_start", ctypes.c_float * 7),
        ("pose_end", ctypes.c_float * 7),
        ("timestamp_start", ctypes.c_int64),
        ("timestamp_end", ctypes.c_int64),
        ("tile_token", ctypes.c_char_p),
        ("sof_opacity_active", ctypes.c_int32),
    ]


class GfTraceOutputs(ctypes.Structure):
    _fields_ = [
        ("rgba", ctypes.c_void_p),
        ("hit_distance", ctypes.c_void_p),
        ("hit_count", ctypes.c_void_p),
        ("visibility", ctypes.c_void_p),
        ("normal", ctypes.c_void_p),
        ("depth_var", ctypes.c_void_p),
        ("quant", ctypes.c_void_p),
        ("extent", ctypes.c_void_p),
        ("inv_depth", ctypes.c_void_p),
        ("inv_depth2", ctypes.c_void_p),
        ("opacity_field", ctypes.c_void_p),
    ]


class GfTraceGrads(ctypes.Structure):
    _fields_ = [
        ("rgba", ctypes.c_void_p),
        ("hit_distance", ctypes.c_void_p),
        ("grad_rgba", ctypes.c_void_p),
        ("grad_hit_distance", ctypes.c_void_p),
        ("grad_particles", ctypes.c_void_p),
        ("grad_features", ctypes.c_void_p),
        ("normal", ctypes.c_void_p),
        ("grad_normal", ctypes.c_void_p),
        ("depth_var", ctypes.c_void_p),
        ("grad_depth_var", ctypes.c_void_p),
        ("extent", ctypes.c_void_p),
        ("grad_extent", ctypes.c_void_p),
        ("inv_depth", ctypes.c_void_p),
        ("grad_inv_depth", ctypes.c_void_p),
        ("inv_depth2", ctypes.c_void_p),
        ("grad_inv_depth2", ctypes.c_void_p),
        ("quant", ctypes.c_void_p),
        ("opacity_field", ctypes.c_void_p),
        ("grad_opacity_field", ctypes.c_void_p),
        ("grad_quant", ctypes.c_void_p),
        ("position_abs_grad", ctypes.c_void_p),
        ("position_abs_grad_mode", ctypes.c_int32),
    ]


class GfTraceStats(ctypes.Structure):
    _fields_ = [
        ("num_intersections", ctypes.c_uint64),
        ("num_tiles", ctypes.c_uint32),
        ("num_particles", ctypes.c_uint32),
        ("kernel_launches", ctypes.c_uint32),
        ("fallback_particles", ctypes.c_uint32),
        ("total_kernel_launches", ctypes.c_uint64),
        ("total_forwards", ctypes.c_uint64),
        ("total_intersections", ctypes.c_uint64),
        ("total_fallback_particles", ctypes.c_uint64),
        ("total_host_wait_us", ctypes.c_uint64),
    ]


class GfFieldCamera(ctypes.Structure):
    _fields_ = [
        ("frame_number", ctypes.c_uint32),
        ("reserved0", ctypes.c_uint32),
        ("camera", GfCamera),
        ("ray_origin", ctypes.c_void_p),
        ("pixel_mask", ctypes.c_void_p),
        ("timestamp_start", ctypes.c_int64),
        ("timestamp_end", ctypes.c_int64),
        ("pose_start", ctypes.c_float * 7),
        ("pose_end", ctypes.c_float * 7),
    ]


class GfFieldStats(ctypes.Structure):
    _fields_ = [
        ("evaluations", ctypes.c_uint64),
        ("pairs", ctypes.c_uint64),
        ("cameras", ctypes.c_uint64),
        ("kernel_launches", ctypes.c_uint64),
        ("candidate_loads", ctypes.c_uint64),
        ("hit_tests", ctypes.c_uint64),
        ("hits", ctypes.c_uint64),
        ("warp_iterations", ctypes.c_uint64),
    ]


FIELD_STAGES = ("points", "cones", "candidates", "sort", "integrate", "finish")


class GfShapeCamera(ctypes.Structure):
    _fields_ = [
        ("c2w", ctypes.c_float * 16),
        ("fisheye", ctypes.c_int32),
        ("reserved0", ctypes.c_int32),
        ("focal_length", ctypes.c_float * 2),
        ("radial", ctypes.c_float * 4),
        ("max_angle", ctypes.c_float),
        ("reserved1", ctypes.c_float),
    ]


_vp, _u32, _i64p = ctypes.c_void_p, ctypes.c_uint32, ctypes.POINTER(ctypes.c_int64)

# (name, restype, argtypes) of every exported symbol of include/gofish_b200.h.
_SIGNATURES = [
    ("gf_abi_version", ctypes.c_int, []),
    ("gf_last_error", ctypes.c_char_p, []),
    ("gf_tracer_create", ctypes.c_void_p, [ctypes.POINTER(GfTracerConfig)]),
    ("gf_tracer_destroy", None, [ctypes.c_void_p]),
    ("gf_tracer_register_tile_mask", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_char_p, ctypes.c_void_p]),
    ("gf_tracer_trace", ctypes.c_int,
     [ctypes.c_void_p, ctypes.POINTER(GfTraceInputs), ctypes.POINTER(GfTraceOutputs), ctypes.c_void_p]),
    ("gf_tracer_trace_bwd", ctypes.c_int,
     [ctypes.c_void_p, ctypes.POINTER(GfTraceInputs), ctypes.POINTER(GfTraceGrads), ctypes.c_void_p]),
    ("gf_tracer_trace_inference", ctypes.c_int,
     [ctypes.c_void_p, ctypes.POINTER(GfTraceInputs), ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    ("gf_tracer_enable_timing", ctypes.c_int, [ctypes.c_void_p, ctypes.c_int]),
    ("gf_tracer_collect_times", ctypes.c_int, [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]),
    ("gf_tracer_stats", ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(GfTraceStats)]),
    ("gf_tracer_log_overflow_tiles", ctypes.c_int, [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]),
    ("gf_tracer_copy_intermediates", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p,
      ctypes.c_uint64, ctypes.c_void_p, ctypes.c_void_p]),
    ("gf_sort_tile_keys_static", ctypes.c_int,
     [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_uint32, ctypes.c_int,
      ctypes.c_void_p]),
    ("gf_field_create", _vp, []),
    ("gf_field_destroy", None, [_vp]),
    ("gf_field_begin", ctypes.c_int, [_vp, _vp, _vp, _u32, _vp, _u32, _i64p, _vp]),
    ("gf_field_integrate_camera", ctypes.c_int, [_vp, ctypes.c_int64, ctypes.POINTER(GfFieldCamera), _vp]),
    ("gf_field_finish", ctypes.c_int, [_vp, ctypes.c_int64, _vp, _vp, _vp, _vp]),
    ("gf_field_release", ctypes.c_int, [_vp, ctypes.c_int64, _vp]),
    ("gf_field_begin_table", ctypes.c_int, [_vp, _vp, _vp, _u32, _vp, _u32, _i64p, _vp]),
    ("gf_field_stage_camera", ctypes.c_int, [_vp, ctypes.c_int64, ctypes.POINTER(GfFieldCamera), _vp]),
    ("gf_field_seal_table", ctypes.c_int, [_vp, ctypes.c_int64, _vp]),
    ("gf_field_evaluate_round", ctypes.c_int, [_vp, ctypes.c_int64, _vp, _u32, _u32, _vp, _vp, _vp, _vp]),
    ("gf_field_reset_batch", ctypes.c_int, [_vp, ctypes.c_int64, _vp]),
    ("gf_field_release_table", ctypes.c_int, [_vp, ctypes.c_int64, _vp]),
    ("gf_field_get_stats", ctypes.c_int, [_vp, ctypes.POINTER(GfFieldStats)]),
    ("gf_field_enable_timing", ctypes.c_int, [_vp, ctypes.c_int]),
    ("gf_view_q6", ctypes.c_int, [_vp, ctypes.c_int64, ctypes.POINTER(GfShapeCamera), ctypes.c_double, _vp, _vp, _vp,
                                  _vp]),
    ("gf_full_shape", ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_int64, ctypes.c_double, ctypes.c_int,
                                     ctypes.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    ("gf_full_shape_bwd", ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_int64, ctypes.c_double, ctypes.c_int,
                                         _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    ("gf_view_shape_packed", ctypes.c_int, [_vp, _vp, _vp, _vp, ctypes.c_int64, ctypes.POINTER(GfShapeCamera),
                                            ctypes.c_double, ctypes.c_int, _vp, _vp, _vp]),
    ("gf_pack_particle_rows", ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, ctypes.c_int64, _vp, _vp]),
    ("gf_unpack_particle_rows", ctypes.c_int, [_vp, ctypes.c_int64, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    ("gf_mip_best_rate", ctypes.c_int,
     [_vp, ctypes.c_int64, _vp, _vp, _vp, _vp, _vp, ctypes.c_int64, _vp, _vp, _vp, _vp, _vp, ctypes.c_int32, _vp, _vp,
      ctypes.c_int64, _vp, _vp, _vp, _vp, _vp]),
    ("gf_field_collect_times", ctypes.c_int, [_vp, _vp, _vp]),
    ("gf_mesh_sites", ctypes.c_int, [_vp, _vp, _vp, _vp, _u32, _vp, _vp, _vp, _vp, _vp, _vp]),
    ("gf_mesh_mt_create", _vp, []),
    ("gf_mesh_mt_destroy", None, [_vp]),
    ("gf_mesh_mt_run", ctypes.c_int, [_vp, _vp, ctypes.c_uint64, _vp, ctypes.c_uint64, _vp, _vp, ctypes.c_uint64,
                                      ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64), _vp]),
    ("gf_mesh_mt_outputs", ctypes.c_int, [_vp, _vp, _vp, _vp, _vp, _vp, _vp]),
    ("gf_mesh_sof_vertex_filter", ctypes.c_int, [_vp, _vp, _vp, ctypes.c_uint64, _vp, _vp]),
    ("gf_mesh_gof_cell_filter", ctypes.c_int, [_vp, ctypes.c_uint64, _vp, _vp, _vp, _vp, _vp]),
]

STATIC_SORT_MAX_PAIRS = 262144

EXPORTED_SYMBOLS = [name for name, _, _ in _SIGNATURES]

_lib = None


class NativeError(RuntimeError):
    """A gofish_b200 entry point returned an error code."""


def load(path: Path | None = None):
    """Load libgofish_b200.so (raises if it is missing: there is no fallback)."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    target = Path(path) if path is not None else LIBRARY
    if not target.exists():
        raise RuntimeError(
            f"gofish_b200 native library not found at {target}; build it with `python -m gofish_b200.build` "
            "(the tracer has no CPU fallback)")
    lib = ctypes.CDLL(str(target))
    for name, restype, argtypes in _SIGNATURES:
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    if lib.gf_abi_version() != ABI_VERSION:
        raise RuntimeError("gofish_b200 native library ABI version mismatch")
    if path is None:
        _lib = lib
    return lib


def check(code: int, what: str) -> None:
    if code != GF_OK:
        message = load().gf_last_error().decode(errors="replace")
        raise NativeError(f"{what} failed ({code}): {message}")
