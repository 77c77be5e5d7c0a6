"""CPU oracle of the GOFish fisheye tracer -- TEST INFRASTRUCTURE ONLY.

A scalar C++ restatement (gofish_oracle.cpp) of the reference renderer's
equations, each function citing the reference file:line it follows.  Only
tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg use it, as
the checker or as the timed CPU baseline; the product never imports it.

Parity status: the reference's CUDA extension cannot be built or run in this
environment as a whole (empty tiny-cuda-nn submodule, no slangc) and the
reference ships no tests or golden vectors for this path.  Its header-only
per-hit device code is compiled for the host from the reference checkout
(oracle/ref_device, ``make -C oracle ref REF=...``), and the hit test,
compositing, training channels, backward and SH radiance of this oracle are
checked against its outputs (tests/test_hit_golden.py); the camera rays are
checked against the reference's Python domain module
(tests/test_domain_golden.py).  The projection, admission, binning, sort and
k-buffer order are pinned by analytic known-answer tests and
finite-difference gradient checks (tests/test_oracle_kat.py,
tests/test_oracle_gradcheck.py).
"""

from __future__ import annotations

import ctypes
import math
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIBRARY = HERE / "liboracle.so"

_lib = None


def build(force: bool = False) -> Path:
    """Compile liboracle.so with the Makefile beside this file."""
    src = [HERE / "gofish_oracle.cpp", HERE.parent / "gofish_b200" / "csrc" / "gf_elementary.h"]
    if force or not LIBRARY.exists() or any(p.stat().st_mtime > LIBRARY.stat().st_mtime for p in src):
        subprocess.run(["make", "-s", "-B", "-C", str(HERE), "liboracle.so"], check=True)
    return LIBRARY


class OracleCamera(ctypes.Structure):
    _fields_ = [
        ("model", ctypes.c_int32),
        ("width", ctypes.c_int32),
        ("height", ctypes.c_int32),
        ("pad0", ctypes.c_int32),
        ("principal", ctypes.c_float * 2),
        ("focal", ctypes.c_float * 2),
        ("radial", ctypes.c_float * 6),
        ("tangential", ctypes.c_float * 2),
        ("thin_prism", ctypes.c_float * 4),
        ("max_angle", ctypes.c_float),
        ("pad1", ctypes.c_float),
    ]


class OraclePose(ctypes.Structure):
    _fields_ = [("R", ctypes.c_float * 9), ("t", ctypes.c_float * 3), ("Rinv", ctypes.c_float * 9),
                ("c", ctypes.c_float * 3)]


def _p(a: np.ndarray):
    return a.ctypes.data_as(ctypes.c_void_p)


def _opt(a):
    """Contiguous float32 copy of optional ray directions (held by the caller for the call)."""
    return None if a is None else np.ascontiguousarray(a, dtype=np.float32)


def _po(a):
    return None if a is None else _p(a)


def _tiles(tiles, total):
    """(tile index array or None, (t0, t1)) of a render call's ``tiles``."""
    if tiles is None:
        return None, (0, total)
    if isinstance(tiles, tuple) and len(tiles) == 2:
        return None, (int(tiles[0]), int(tiles[1]))
    arr = np.ascontiguousarray(np.asarray(tiles, dtype=np.int32).reshape(-1))
    if arr.size and (arr.min() < 0 or arr.max() >= total):
        raise ValueError("tile index out of range")
    return arr, (0, int(arr.size))


class _tile_list:
    """Context that sets the oracle's tile list for one render call."""

    def __init__(self, lib, arr):
        self.lib, self.arr = lib, arr

    def __enter__(self):
        if self.arr is not None:
            self.lib.oracle_set_tile_list(_p(self.arr), int(self.arr.size))

    def __exit__(self, *exc):
        if self.arr is not None:
            self.lib.oracle_set_tile_list(None, 0)
        return False


def load():
    global _lib
    if _lib is not None:
        return _lib
    build()
    lib = ctypes.CDLL(str(LIBRARY))
    vp, i32, i64, f32 = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float
    cam_p, pose_p = ctypes.POINTER(OracleCamera), ctypes.POINTER(OraclePose)
    sig = {
        "oracle_prepare_pose": (None, [vp, pose_p]),
        "oracle_project": (i32, [cam_p, pose_p, i32, vp, vp, i32, i32, vp, vp, vp, vp, vp]),
        "oracle_tile_rays": (i32, [cam_p, pose_p, vp, vp, vp]),
        "oracle_bin": (i64, [cam_p, pose_p, i32, vp, vp, vp, vp, vp, vp, i32, vp, vp, i64, vp]),
        "oracle_render_forward": (i32, [cam_p, pose_p, i32, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, vp, vp, vp]),
        "oracle_render_forward_geo": (i32, [cam_p, pose_p, i32, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp,
                                            vp, vp, vp, vp, vp, vp, vp, vp]),
        "oracle_render_backward_geo": (i32, [cam_p, pose_p, i32, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, i32, vp,
                                             vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
        "oracle_render_backward": (i32, [cam_p, pose_p, i32, vp, vp, vp, vp, vp, vp, vp, i32, i32, i32, vp, vp, vp, vp,
                                         vp]),
        "oracle_project_backward": (i32, [pose_p, i32, vp, vp, i32, i32, vp, vp, vp, vp]),
        "oracle_visibility": (i32, [i32, vp, vp]),
        "oracle_field_camera": (i32, [cam_p, pose_p, i32, vp, vp, vp, i32, vp, vp, vp]),
        "oracle_mip_best_rate": (i32, [vp, i64, vp, vp, vp, vp, vp, i64, vp, vp, vp, vp, vp, vp, vp, i64, vp, vp, vp,
                                       vp]),
        "oracle_atan2d": (ctypes.c_double, [ctypes.c_double, ctypes.c_double]),
        "oracle_set_tile_list": (None, [vp, i32]),
        "oracle_set_complete_admission": (None, [i32]),
        "oracle_set_abs_grad": (None, [vp, vp, i32]),
        "oracle_project_points": (i32, [cam_p, i32, vp, vp, vp]),
        "oracle_kbuffer_order": (i32, [i32, i32, vp, vp]),
        "oracle_ut_project": (i32, [cam_p, pose_p, i32, vp, vp]),
        "oracle_set_admission_variants": (None, [ctypes.c_float, i32, ctypes.c_float, ctypes.c_float]),
        "oracle_admission_misses": (i64, [cam_p, pose_p, i32, vp, vp, vp, vp, vp, vp, i64, vp, vp]),
        "oracle_sof_feeds": (i64, [cam_p, pose_p, i32, vp, vp, vp, vp, vp, i32, vp, vp, i64]),
        "oracle_sof_opacity_forward": (i32, [cam_p, pose_p, vp, vp, vp, vp, vp, vp, vp, vp]),
        "oracle_sof_opacity_backward": (i32, [cam_p, pose_p, i32, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp]),
        "oracle_field_index_build": (vp, [i32, vp, ctypes.c_double]),
        "oracle_field_index_free": (None, [vp]),
        "oracle_field_camera_indexed": (i32, [vp, cam_p, pose_p, vp, vp, i32, vp, vp, vp]),
        "oracle_num_threads": (i32, []),
        "oracle_expf": (f32, [f32]),
        "oracle_logf": (f32, [f32]),
        "oracle_atan2f": (f32, [f32, f32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


def camera(model: int, width: int, height: int, principal, focal, radial, max_angle: float = 0.0,
           tangential=(0.0, 0.0), thin_prism=(0.0, 0.0, 0.0, 0.0)) -> OracleCamera:
    cam = OracleCamera()
    cam.model = int(model)
    cam.width = int(width)
    cam.height = int(height)
    cam.principal[:] = [float(np.float32(v)) for v in principal]
    cam.focal[:] = [float(np.float32(v)) for v in focal]
    r = [float(np.float32(v)) for v in radial] + [0.0] * (6 - len(radial))
    cam.radial[:] = r[:6]
    cam.tangential[:] = [float(np.float32(v)) for v in tangential]
    cam.thin_prism[:] = [float(np.float32(v)) for v in thin_prism]
    cam.max_angle = float(np.float32(max_angle))
    return cam


def prepare_pose(pose7) -> OraclePose:
    p = np.ascontiguousarray(np.asarray(pose7, dtype=np.float32).reshape(7))
    out = OraclePose()
    load().oracle_prepare_pose(_p(p), ctypes.byref(out))
    return out


def num_threads() -> int:
    return int(load().oracle_num_threads())


def tile_grid(cam: OracleCamera) -> tuple[int, int]:
    return (cam.width + 15) // 16, (cam.height + 15) // 16


def project(cam, pose, particles, sh, sh_degree, mask, ray_d=None):
    """UT projection, radiance and tile counts; with ``ray_d`` ([H,W,3] sensor
    ray directions) particles without a valid projection use the cone
    fallback admission."""
    lib = load()
    particles = np.ascontiguousarray(particles, dtype=np.float32)
    sh = np.ascontiguousarray(sh, dtype=np.float32)
    mask = np.ascontiguousarray(mask, dtype=np.uint8)
    ray_d = _opt(ray_d)
    n = particles.shape[0]
    proj = np.zeros((n, 8), dtype=np.float32)
    rgb = np.zeros((n, 3), dtype=np.float32)
    counts = np.zeros(n, dtype=np.uint32)
    lib.oracle_project(ctypes.byref(cam), ctypes.byref(pose), n, _p(particles), _p(sh), sh.shape[1] // 3,
                       int(sh_degree), _p(mask), _po(ray_d), _p(proj), _p(rgb), _p(counts))
    return proj, rgb, counts


def ut_project(cam, pose, particles) -> np.ndarray:
    """The UT projection of packed rows alone: [n,6] = centre u, v,
    covariance xx, xy, yy, valid (0/1)."""
    rows = np.ascontiguousarray(particles, dtype=np.float32)
    out = np.zeros((rows.shape[0], 6), np.float32)
    load().oracle_ut_project(ctypes.byref(cam), ctypes.byref(pose), rows.shape[0], _p(rows), _p(out))
    return out


def kbuffer_order(k: int, hit_t) -> np.ndarray:
    """Composite order (hit indices) of a K-entry k-buffer fed the hit
    distances ``hit_t`` in sequence."""
    t = np.ascontiguousarray(hit_t, dtype=np.float32)
    order = np.zeros(t.size, np.uint32)
    if load().oracle_kbuffer_order(int(k), int(t.size), _p(t), _p(order)) != 0:
        raise ValueError("k-buffer size must be 1..64")
    return order


def project_points(cam, points):
    """Sensor-space projection of [n,3] points without raster bounds:
    (uv [n,2] float32, valid [n] bool)."""
    pts = np.ascontiguousarray(points, dtype=np.float32).reshape(-1, 3)
    uv = np.zeros((pts.shape[0], 2), np.float32)
    valid = np.zeros(pts.shape[0], np.uint8)
    load().oracle_project_points(ctypes.byref(cam), pts.shape[0], _p(pts), _p(uv), _p(valid))
    return uv, valid.astype(bool)


def tile_rays(cam, pose, ray_o, ray_d):
    gx, gy = tile_grid(cam)
    out = np.zeros((gx * gy, 8), dtype=np.float32)
    ray_o = np.ascontiguousarray(ray_o, dtype=np.float32)
    ray_d = np.ascontiguousarray(ray_d, dtype=np.float32)
    load().oracle_tile_rays(ctypes.byref(cam), ctypes.byref(pose), _p(ray_o), _p(ray_d), _p(out))
    return out


def bin(cam, pose, particles, proj, counts, mask, tile_ray_table, key_mode, ray_d=None):
    ray_d = _opt(ray_d)
    lib = load()
    gx, gy = tile_grid(cam)
    total = int(counts.astype(np.uint64).sum())
    keys = np.zeros(max(total, 1), dtype=np.uint64)
    ids = np.zeros(max(total, 1), dtype=np.uint32)
    ranges = np.zeros((gx * gy, 2), dtype=np.uint32)
    particles = np.ascontiguousarray(particles, dtype=np.float32)
    got = lib.oracle_bin(ctypes.byref(cam), ctypes.byref(pose), particles.shape[0], _p(particles),
                         _p(np.ascontiguousarray(proj)), _p(np.ascontiguousarray(counts)),
                         _p(np.ascontiguousarray(mask, dtype=np.uint8)), _p(np.ascontiguousarray(tile_ray_table)),
                         _po(ray_d), int(key_mode), _p(keys), _p(ids), total, _p(ranges))
    if got != total:
        raise RuntimeError("oracle_bin capacity mismatch")
    return keys[:total], ids[:total], ranges


def render_forward(cam, pose, particles, rgb, ray_o, ray_d, mask, ranges, sorted_ids, k, tiles=None, out=None):
    """Forward compositing of the tiles ``tiles``: a range (t0, t1), an array
    of tile indices, or None for all tiles.  ``out``: (rgba, hit_t, count)
    arrays to write instead of new ones (pixels of other tiles keep their
    contents)."""
    lib = load()
    h, w = cam.height, cam.width
    gx, gy = tile_grid(cam)
    tile_list, (t0, t1) = _tiles(tiles, gx * gy)
    if out is None:
        rgba = np.zeros((h, w, 4), dtype=np.float32)
        hit_t = np.full((h, w), 1e6, dtype=np.float32)
        count = np.zeros((h, w), dtype=np.float32)
    else:
        rgba, hit_t, count = out
    particles = np.ascontiguousarray(particles, dtype=np.float32)
    ids = np.ascontiguousarray(sorted_ids, dtype=np.uint32)
    if ids.size == 0:
        ids = np.zeros(1, dtype=np.uint32)
    with _tile_list(lib, tile_list):
        lib.oracle_render_forward(ctypes.byref(cam), ctypes.byref(pose), particles.shape[0], _p(particles),
                                  _p(np.ascontiguousarray(rgb, dtype=np.float32)),
                                  _p(np.ascontiguousarray(ray_o, dtype=np.float32)),
                                  _p(np.ascontiguousarray(ray_d, dtype=np.float32)),
                                  _p(np.ascontiguousarray(mask, dtype=np.uint8)), _p(np.ascontiguousarray(ranges)),
                                  _p(ids), int(k), int(t0), int(t1), _p(rgba), _p(hit_t), _p(count))
    return rgba, hit_t, count


def render_forward_geo(cam, pose, particles, rgb, ray_o, ray_d, mask, ranges, sorted_ids, k, tiles=None,
                       pinhole=False):
    """render_forward plus the geometric training channels: a dict with rgba,
    hit_t, hit_count, normal [H,W,3], depth_var, quant [H,W,10], extent,
    inv_depth, inv_depth2 (zeros outside retained tiles and for invalid rays)."""
    lib = load()
    h, w = cam.height, cam.width
    gx, gy = tile_grid(cam)
    t0, t1 = (0, gx * gy) if tiles is None else tiles
    out = dict(rgba=np.zeros((h, w, 4), np.float32), hit_t=np.full((h, w), 1e6, np.float32),
               hit_count=np.zeros((h, w), np.float32), normal=np.zeros((h, w, 3), np.float32),
               depth_var=np.zeros((h, w), np.float32), quant=np.zeros((h, w, 10), np.float32),
               extent=np.zeros((h, w), np.float32), inv_depth=np.zeros((h, w), np.float32),
               inv_depth2=np.zeros((h, w), np.float32))
    particles = np.ascontiguousarray(particles, dtype=np.float32)
    ids = np.ascontiguousarray(sorted_ids, dtype=np.uint32)
    if ids.size == 0:
        ids = np.zeros(1, dtype=np.uint32)
    lib.oracle_render_forward_geo(ctypes.byref(cam), ctypes.byref(pose), particles.shape[0], _p(particles),
                                  _p(np.ascontiguousarray(rgb, dtype=np.float32)),
                                  _p(np.ascontiguousarray(ray_o, dtype=np.float32)),
                                  _p(np.ascontiguousarray(ray_d, dtype=np.float32)),
                                  _p(np.ascontiguousarray(mask, dtype=np.uint8)), _p(np.ascontiguousarray(ranges)),
                                  _p(ids), int(k), int(t0), int(t1), int(bool(pinhole)),
                                  *(_p(out[k_]) for k_ in ("rgba", "hit_t", "hit_count", "normal", "depth_var",
                                                           "quant", "extent", "inv_depth", "inv_depth2")))
    return out


def render_backward(cam, pose, particles, rgb, ray_o, ray_d, mask, ranges, sorted_ids, k, rgba, hit_t, grad_rgba,
                    grad_hit_t, tiles=None, out=None):
    """Gradient records [N,16] of the tiles ``tiles`` (a range (t0, t1), an
    array of tile indices, or None for all tiles); ``out``: an array to
    overwrite instead of a new one."""
    lib = load()
    gx, gy = tile_grid(cam)
    tile_list, (t0, t1) = _tiles(tiles, gx * gy)
    n = particles.shape[0]
    grad = np.zeros((n, 16), dtype=np.float32) if out is None else out
    ids = np.ascontiguousarray(sorted_ids, dtype=np.uint32)
    if ids.size == 0:
        ids = np.zeros(1, dtype=np.uint32)
    with _tile_list(lib, tile_list):
        lib.oracle_render_backward(ctypes.byref(cam), ctypes.byref(pose), n,
                                   _p(np.ascontiguousarray(particles, dtype=np.float32)),
                                   _p(np.ascontiguousarray(rgb, dtype=np.float32)),
                                   _p(np.ascontiguousarray(ray_o, dtype=np.float32)),
                                   _p(np.ascontiguousarray(ray_d, dtype=np.float32)),
                                   _p(np.ascontiguousarray(mask, dtype=np.uint8)), _p(np.ascontiguousarray(ranges)),
                                   _p(ids), int(k), int(t0), int(t1),
                                   _p(np.ascontiguousarray(rgba, dtype=np.float32)),
                                   _p(np.ascontiguousarray(hit_t, dtype=np.float32)),
                                   _p(np.ascontiguousarray(grad_rgba, dtype=np.float32)),
                                   _p(np.ascontiguousarray(grad_hit_t, dtype=np.float32)), _p(grad))
    return grad


def render_backward_geo(cam, pose, particles, rgb, ray_o, ray_d, mask, ranges, sorted_ids, k, fwd, grads,
                        tiles=None, pinhole=False):
    """render_backward with the geometric channels.  fwd: render_forward_geo's
    dict; grads: dict of output gradients (rgba, hit_t, and any of normal,
    depth_var, extent, inv_depth, inv_depth2, and quant: only its crossing
    depth channel 8 is read).  Returns (grad record [N,16],
    shape gradient [N,8]: quaternion w,x,y,z | scale xyz, 0)."""
    lib = load()
    gx, gy = tile_grid(cam)
    t0, t1 = (0, gx * gy) if tiles is None else tiles
    n = particles.shape[0]
    grad = np.zeros((n, 16), dtype=np.float32)
    gshape = np.zeros((n, 8), dtype=np.float32)
    ids = np.ascontiguousarray(sorted_ids, dtype=np.uint32)
    if ids.size == 0:
        ids = np.zeros(1, dtype=np.uint32)

    def opt(d, key):
        return None if d.get(key) is None else _p(np.ascontiguousarray(d[key], dtype=np.float32))

    keep = {key: np.ascontiguousarray(fwd[key], dtype=np.float32) for key in ("rgba", "hit_t", "normal", "depth_var")}
    if grads.get("quant") is not None:
        keep["quant"] = np.ascontiguousarray(fwd["quant"], dtype=np.float32)
    lib.oracle_render_backward_geo(ctypes.byref(cam), ctypes.byref(pose), n,
                                   _p(np.ascontiguousarray(particles, dtype=np.float32)),
                                   _p(np.ascontiguousarray(rgb, dtype=np.float32)),
                                   _p(np.ascontiguousarray(ray_o, dtype=np.float32)),
                                   _p(np.ascontiguousarray(ray_d, dtype=np.float32)),
                                   _p(np.ascontiguousarray(mask, dtype=np.uint8)), _p(np.ascontiguousarray(ranges)),
                                   _p(ids), int(k), int(t0), int(t1), int(bool(pinhole)), _p(keep["rgba"]),
                                   _p(keep["hit_t"]), opt(grads, "rgba"), opt(grads, "hit_t"),
                                   _p(keep["normal"]) if grads.get("normal") is not None else None,
                                   opt(grads, "normal"),
                                   _p(keep["depth_var"]) if grads.get("depth_var") is not None else None,
                                   opt(grads, "depth_var"), opt(grads, "extent"), opt(grads, "inv_depth"),
                                   opt(grads, "inv_depth2"),
                                   _p(keep["quant"]) if grads.get("quant") is not None else None,
                                   opt(grads, "quant"), _p(grad), _p(gshape))
    return grad, gshape


def project_backward(pose, particles, sh, sh_degree, counts, grad_record):
    lib = load()
    n = particles.shape[0]
    sh = np.ascontiguousarray(sh, dtype=np.float32)
    gp = np.zeros((n, 32), dtype=np.float32)
    gs = np.zeros_like(sh)
    lib.oracle_project_backward(ctypes.byref(pose), n, _p(np.ascontiguousarray(particles, dtype=np.float32)), _p(sh),
                                sh.shape[1] // 3, int(sh_degree), _p(np.ascontiguousarray(counts)),
                                _p(np.ascontiguousarray(grad_record, dtype=np.float32)), _p(gp), _p(gs))
    return gp, gs


class complete_admission:
    """Context in which project / bin admit every particle (density >= 1/255)
    by the conservative cone test of its support sphere (the tracer's
    render.gofish.complete_admission)."""

    def __init__(self, on: bool = True):
        self.on = bool(on)

    def __enter__(self):
        load().oracle_set_complete_admission(1 if self.on else 0)

    def __exit__(self, *exc):
        load().oracle_set_complete_admission(0)
        return False


class abs_grad:
    """Context in which render_backward / render_backward_geo accumulate the
    densification statistic (gutKBufferRenderer.cuh:54-60,283-296): for every
    composited hit, |M g| of its position gradient g with the per-particle
    map M ([N,2,3], mode "screen", sums [N,2]) or |g| (mode "world", [N,3]).
    The sums are in ``.out`` after the block."""

    def __init__(self, n: int, mode: str, mapping=None):
        if mode not in ("screen", "world"):
            raise ValueError("abs_grad mode must be 'screen' or 'world'")
        self.mode = 1 if mode == "screen" else 2
        self.map = None if mapping is None else np.ascontiguousarray(np.asarray(mapping, np.float32).reshape(n, 6))
        if self.mode == 1 and self.map is None:
            raise ValueError("screen mode needs the [N,2,3] map")
        self.out = np.zeros((n, 2 if self.mode == 1 else 3), np.float32)

    def __enter__(self):
        load().oracle_set_abs_grad(_po(self.map), _p(self.out), self.mode)
        return self

    def __exit__(self, *exc):
        load().oracle_set_abs_grad(None, None, 0)
        return False


def cap_sine(angle: float) -> np.float32:
    """Sine bound of a cone_big half-angle bound (the tracer's cap_sine): 1
    from pi/2 up, else sin(max(angle, 0)) in double rounded to float32."""
    a = np.float32(angle)
    if not a < np.float32(math.pi / 2):
        return np.float32(1.0)
    return np.float32(math.sin(float(max(a, np.float32(0.0)))))


class admission_variants:
    """Context of project / bin with the reference's fast-admission variants:
    the partial UT (render.gofish.fast_partial_ut_scale; 0 = off) and the
    "cone_big" fallback window (min, max) half-angle in radians (None: the
    plain cone fallback)."""

    def __init__(self, partial_ut_scale: float = 0.0, cone_big=None):
        s = np.float32(partial_ut_scale)
        self.scale2 = float(s * s) if s > 0 else 0.0
        self.cone_big = cone_big

    def __enter__(self):
        lo, hi = (cap_sine(self.cone_big[0]), cap_sine(self.cone_big[1])) if self.cone_big is not None else (0.0, 1.0)
        load().oracle_set_admission_variants(self.scale2, 1 if self.cone_big is not None else 0, float(lo), float(hi))

    def __exit__(self, *exc):
        load().oracle_set_admission_variants(0.0, 0, 0.0, 1.0)
        return False


def admission_misses(cam, pose, particles, ray_o, ray_d, mask, ranges, sorted_ids, max_misses=64):
    """(count, [(pixel, particle)...]) of brute-force hits on valid rays of
    retained tiles whose particle is missing from the tile's candidate list."""
    lib = load()
    ids = np.ascontiguousarray(sorted_ids, dtype=np.uint32)
    if ids.size == 0:
        ids = np.zeros(1, dtype=np.uint32)
    pix = np.zeros(max_misses, np.int64)
    part = np.zeros(max_misses, np.uint32)
    particles = np.ascontiguousarray(particles, dtype=np.float32)
    n = lib.oracle_admission_misses(ctypes.byref(cam), ctypes.byref(pose), particles.shape[0], _p(particles),
                                    _p(np.ascontiguousarray(ray_o, dtype=np.float32)),
                                    _p(np.ascontiguousarray(ray_d, dtype=np.float32)),
                                    _p(np.ascontiguousarray(mask, dtype=np.uint8)),
                                    _p(np.ascontiguousarray(ranges, dtype=np.uint32)), _p(ids), max_misses, _p(pix),
                                    _p(part))
    k = min(int(n), max_misses)
    return int(n), list(zip(pix[:k].tolist(), part[:k].tolist()))


def trace(cam, pose7, particles, sh, sh_degree, ray_o, ray_d, mask, k, key_mode, tiles=None, fallback=True,
          complete=False, partial_ut_scale=0.0, cone_big=None):
    """Full forward pass; returns a dict of every intermediate and output.
    ``fallback`` admits particles without a valid projection by the cone test
    (render.gofish.fast_admission_fallback = "cone"; ``cone_big`` = (min, max)
    radians restricts it to that cap window); ``complete`` admits every
    particle that way (render.gofish.complete_admission);
    ``partial_ut_scale`` > 0 repairs partially valid projections."""
    pose = prepare_pose(pose7)
    rd = ray_d if (fallback or complete) else None
    with complete_admission(complete), admission_variants(partial_ut_scale, cone_big):
        proj, rgb, counts = project(cam, pose, particles, sh, sh_degree, mask, rd)
        tr = tile_rays(cam, pose, ray_o, ray_d)
        keys, ids, ranges = bin(cam, pose, particles, proj, counts, mask, tr, key_mode, rd)
    rgba, hit_t, count = render_forward(cam, pose, particles, rgb, ray_o, ray_d, mask, ranges, ids, k, tiles)
    vis = (counts > 0).astype(np.uint32)
    return dict(pose=pose, proj=proj, rgb=rgb, counts=counts, tile_rays=tr, keys=keys, ids=ids, ranges=ranges,
                rgba=rgba, hit_t=hit_t, hit_count=count, visibility=vis)


def trace_backward(cam, fwd, particles, sh, sh_degree, ray_o, ray_d, mask, k, grad_rgba, grad_hit_t, tiles=None):
    rec = render_backward(cam, fwd["pose"], particles, fwd["rgb"], ray_o, ray_d, mask, fwd["ranges"], fwd["ids"], k,
                          fwd["rgba"], fwd["hit_t"], grad_rgba, grad_hit_t, tiles)
    gp, gs = project_backward(fwd["pose"], particles, sh, sh_degree, fwd["counts"], rec)
    return gp, gs, rec


SOF_HIERARCHY = -1  # the k argument of the render calls that selects SOF's HEAD4 / MID8 / TAIL64 hierarchy


def sof_feeds(cam, pose, particles, ray_o, ray_d, ranges, sorted_ids, tile):
    """The SOF hierarchy's feed sequence (sorted positions, in order) of every
    pixel of one tile: a list of 256 arrays, row-major within the tile."""
    lib = load()
    particles = np.ascontiguousarray(particles, dtype=np.float32)
    ids = np.ascontiguousarray(sorted_ids, dtype=np.uint32)
    if ids.size == 0:
        ids = np.zeros(1, dtype=np.uint32)
    r = np.ascontiguousarray(ranges, dtype=np.uint32)
    count = int(r.reshape(-1, 2)[tile, 1] - r.reshape(-1, 2)[tile, 0])
    offset = np.zeros(257, dtype=np.uint32)
    feed = np.zeros(max(1, 256 * count), dtype=np.uint32)
    total = lib.oracle_sof_feeds(ctypes.byref(cam), ctypes.byref(pose), particles.shape[0], _p(particles),
                                 _p(np.ascontiguousarray(ray_o, dtype=np.float32)),
                                 _p(np.ascontiguousarray(ray_d, dtype=np.float32)), _p(r), _p(ids), int(tile),
                                 _p(offset), _p(feed), feed.size)
    if total < 0:
        raise RuntimeError("oracle_sof_feeds capacity")
    return [feed[offset[p]:offset[p + 1]].copy() for p in range(256)]


def sof_opacity(cam, pose, particles, ray_o, ray_d, mask, ranges, sorted_ids, quant):
    """SOF opacity field [H,W] (zero for invalid rays and dropped tiles) from
    the forward's quantile channel [H,W,10]."""
    c = lambda a, dt: np.ascontiguousarray(a, dtype=dt)  # noqa: E731
    ids = c(sorted_ids, np.uint32)
    if ids.size == 0:
        ids = np.zeros(1, dtype=np.uint32)
    out = np.zeros((cam.height, cam.width), np.float32)
    load().oracle_sof_opacity_forward(ctypes.byref(cam), ctypes.byref(pose), _p(c(particles, np.float32)),
                                      _p(c(ray_o, np.float32)), _p(c(ray_d, np.float32)), _p(c(mask, np.uint8)),
                                      _p(c(ranges, np.uint32)), _p(ids), _p(c(quant, np.float32)), _p(out))
    return out


def sof_opacity_backward(cam, pose, particles, ray_o, ray_d, mask, ranges, sorted_ids, quant, opacity, grad):
    """Gradient [N,16] of the SOF opacity field: position xyz, intrinsic
    density | quaternion wxyz | scale xyz, 0 | 0."""
    c = lambda a, dt: np.ascontiguousarray(a, dtype=dt)  # noqa: E731
    particles = c(particles, np.float32)
    ids = c(sorted_ids, np.uint32)
    if ids.size == 0:
        ids = np.zeros(1, dtype=np.uint32)
    out = np.zeros((particles.shape[0], 16), np.float32)
    load().oracle_sof_opacity_backward(ctypes.byref(cam), ctypes.byref(pose), particles.shape[0], _p(particles),
                                       _p(c(ray_o, np.float32)), _p(c(ray_d, np.float32)), _p(c(mask, np.uint8)),
                                       _p(c(ranges, np.uint32)), _p(ids), _p(c(quant, np.float32)),
                                       _p(c(opacity, np.float32)), _p(c(grad, np.float32)), _p(out))
    return out


def field_camera(cam, pose7, particles, ray_o, points, pixel_mask=None):
    """One camera of the opacity field: (opacity [Q] float32, observed [Q] uint8)."""
    lib = load()
    pose = prepare_pose(pose7)
    points = np.ascontiguousarray(points, dtype=np.float32).reshape(-1, 3)
    q = points.shape[0]
    opacity = np.zeros(q, dtype=np.float32)
    observed = np.zeros(q, dtype=np.uint8)
    mask = None if pixel_mask is None else np.ascontiguousarray(pixel_mask, dtype=np.uint8)
    particles = np.ascontiguousarray(particles, dtype=np.float32)
    ray_o = np.ascontiguousarray(ray_o, dtype=np.float32)
    lib.oracle_field_camera(ctypes.byref(cam), ctypes.byref(pose), particles.shape[0], _p(particles), _p(ray_o),
                            None if mask is None else _p(mask), q, _p(points), _p(opacity), _p(observed))
    return opacity, observed


def evaluate_field(views, particles, points):
    """Camera-min field over views, each (cam, pose7, ray_o, pixel_mask or None).

    Returns (opacity [Q] with 0 where unobserved, observed [Q], above [Q]):
    the outputs of the reference's finish_opacity_field
    (opacityFieldBinding.inl:318-338)."""
    q = np.asarray(points).reshape(-1, 3).shape[0]
    minimum = np.ones(q, dtype=np.float32)
    observed = np.zeros(q, dtype=np.uint8)
    for cam, pose7, ray_o, mask in views:
        op, ob = field_camera(cam, pose7, particles, ray_o, points, mask)
        first = (ob != 0) & (observed == 0)
        both = (ob != 0) & (observed != 0)
        minimum[first] = op[first]
        minimum[both] = np.minimum(minimum[both], op[both])
        observed |= ob
    opacity = np.where(observed != 0, minimum, np.float32(0.0)).astype(np.float32)
    above = ((observed != 0) & (opacity >= np.float32(0.5))).astype(np.uint8)
    return opacity, observed, above


class FieldIndex:
    """Spatial index of oracle_field_camera_indexed over packed [N,32] rows
    (the rows are kept alive by this object).  ``scene_bound`` must bound
    every distance from a camera origin to a particle mean and every query
    segment's length."""

    def __init__(self, particles, scene_bound: float):
        self.particles = np.ascontiguousarray(particles, dtype=np.float32)
        self.handle = load().oracle_field_index_build(self.particles.shape[0], _p(self.particles), float(scene_bound))

    def close(self):
        if self.handle:
            load().oracle_field_index_free(self.handle)
            self.handle = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()
        return False

    def field_camera(self, cam, pose7, ray_o, points, pixel_mask=None):
        """oracle field of one camera (field_camera) over the index."""
        pose = prepare_pose(pose7)
        points = np.ascontiguousarray(points, dtype=np.float32).reshape(-1, 3)
        q = points.shape[0]
        opacity = np.zeros(q, dtype=np.float32)
        observed = np.zeros(q, dtype=np.uint8)
        mask = None if pixel_mask is None else np.ascontiguousarray(pixel_mask, dtype=np.uint8)
        ray_o = np.ascontiguousarray(ray_o, dtype=np.float32)
        load().oracle_field_camera_indexed(self.handle, ctypes.byref(cam), ctypes.byref(pose), _p(ray_o),
                                           None if mask is None else _p(mask), q, _p(points), _p(opacity),
                                           _p(observed))
        return opacity, observed

    def evaluate_field(self, views, points):
        """evaluate_field over the index: (opacity, observed, above)."""
        return _camera_min(views, points, self.field_camera)


def _camera_min(views, points, camera_fn):
    q = np.asarray(points).reshape(-1, 3).shape[0]
    minimum = np.ones(q, dtype=np.float32)
    observed = np.zeros(q, dtype=np.uint8)
    for cam, pose7, ray_o, mask in views:
        op, ob = camera_fn(cam, pose7, ray_o, points, mask)
        first = (ob != 0) & (observed == 0)
        both = (ob != 0) & (observed != 0)
        minimum[first] = op[first]
        minimum[both] = np.minimum(minimum[both], op[both])
        observed |= ob
    opacity = np.where(observed != 0, minimum, np.float32(0.0)).astype(np.float32)
    above = ((observed != 0) & (opacity >= np.float32(0.5))).astype(np.uint8)
    return opacity, observed, above


def bisection_round(views, particles, points):
    """One bisection round's (above, observed, exact) vectors.

    The reference's tie-aware round (bisectionTableImpl.inl:222-357) stops a
    camera once its opacity is strictly above 1/2 and then classifies; since
    T only decreases, that equals: above = observed and min >= 1/2, exact =
    observed and min == 1/2, with min the camera-min field."""
    opacity, observed, above = evaluate_field(views, particles, points)
    exact = ((observed != 0) & (opacity == np.float32(0.5))).astype(np.uint8)
    return above, observed, exact


def mip_best_rate(points, rotations, centers, frame_camera, frame_index, frame_rank, camera_model, camera_width,
                  camera_height, camera_params, camera_max_angle, row_lo, row_hi):
    """The physical-mip search on numpy arrays: (best [N] f64, owner [N] i32,
    observed [N] u8, direction [N,3] f64)."""
    lib = load()
    c = lambda a, dt: np.ascontiguousarray(a, dtype=dt)  # noqa: E731
    pts = c(points, np.float64).reshape(-1, 3)
    n = pts.shape[0]
    rot = c(rotations, np.float64)
    f = rot.shape[0]
    lo = c(row_lo, np.int32)
    args = [c(centers, np.float64), c(frame_camera, np.int32), c(frame_index, np.int32), c(frame_rank, np.int64)]
    cam = [c(camera_model, np.int32), c(camera_width, np.int32), c(camera_height, np.int32),
           c(camera_params, np.float64), c(camera_max_angle, np.float64)]
    hi = c(row_hi, np.int32)
    best = np.zeros(n, np.float64)
    owner = np.full(n, -1, np.int32)
    observed = np.zeros(n, np.uint8)
    direction = np.zeros((n, 3), np.float64)
    lib.oracle_mip_best_rate(_p(pts), n, _p(rot), *(_p(a) for a in args), f, *(_p(a) for a in cam), _p(lo), _p(hi),
                             lo.shape[1], _p(best), _p(owner), _p(observed), _p(direction))
    return best, owner, observed, direction


def atan2d(y: float, x: float) -> float:
    return float(load().oracle_atan2d(float(y), float(x)))
