"""Shared inputs for the parity tests: one workload rendered by the oracle and
by the sm_100a tracer (through SplatRaster, i.e. the C ABI)."""

from __future__ import annotations

import dataclasses
import math

import numpy as np

import oracle
from gofish_b200.camera import FisheyeCamera, fisheye_camera, random_kb_coefficients
from gofish_b200.scene import (IDENTITY_POSE, Scene, pack_particles, pose_world_to_sensor, random_rotation_quaternion_xyzw,
                               random_scene)


def tile_mask(valid_px: np.ndarray) -> np.ndarray:
    """uint8 [Ty,Tx] mask of tiles holding at least one valid pixel ([H,W] bool input)."""
    h, w = valid_px.shape
    ty, tx = (h + 15) // 16, (w + 15) // 16
    pad = np.zeros((ty * 16, tx * 16), dtype=bool)
    pad[:h, :w] = valid_px
    return pad.reshape(ty, 16, tx, 16).any(axis=(1, 3)).astype(np.uint8)


def oracle_camera(cam: FisheyeCamera) -> oracle.OracleCamera:
    return oracle.camera(1, cam.width, cam.height, cam.principal, cam.focal, cam.coefficients, cam.max_angle)


@dataclasses.dataclass
class Case:
    scene: Scene
    camera: FisheyeCamera
    pose: np.ndarray
    particles: np.ndarray
    features: np.ndarray
    ray_o: np.ndarray      # [H,W,3]
    ray_d: np.ndarray      # [H,W,3]
    valid: np.ndarray      # [H,W] bool
    tmask: np.ndarray      # [Ty,Tx] uint8

    @property
    def ocam(self):
        return oracle_camera(self.camera)


def make_case(scene: Scene, camera: FisheyeCamera, pose, tmask_override=None) -> Case:
    o, d, valid = camera.rays()
    valid2 = valid[0, :, :, 0]
    tm = tile_mask(valid2) if tmask_override is None else tmask_override
    return Case(scene, camera, np.asarray(pose, dtype=np.float32), pack_particles(scene), scene.features, o[0], d[0],
                valid2, tm)


def small_case(seed: int = 7, n: int = 20_000, size: int = 256, sh_degree: int = 3, fov: float = 200.0,
               random_pose: bool = True, width: int | None = None) -> Case:
    scene = random_scene(n, sh_degree, seed)
    rng = np.random.default_rng(seed + 99)
    k = random_kb_coefficients(rng, fov)
    cam = fisheye_camera(width or size, size, fov, k)
    if random_pose:
        c = rng.standard_normal(3)
        c = c / np.linalg.norm(c) * 0.5 * np.cbrt(rng.random())
        pose = pose_world_to_sensor(c, random_rotation_quaternion_xyzw(rng))
    else:
        pose = IDENTITY_POSE.copy()
    return make_case(scene, cam, pose)


def oracle_forward(case: Case, k: int, key_mode: int, tiles=None, fallback: bool = True, complete: bool = False,
                   partial_ut_scale: float = 0.0, cone_big=None):
    return oracle.trace(case.ocam, case.pose, case.particles, case.features, case.scene.sh_degree, case.ray_o,
                        case.ray_d, case.tmask, k, key_mode, tiles, fallback, complete, partial_ut_scale, cone_big)


def oracle_backward(case: Case, fwd, k: int, grad_rgba, grad_hit, tiles=None):
    return oracle.trace_backward(case.ocam, fwd, case.particles, case.features, case.scene.sh_degree, case.ray_o,
                                 case.ray_d, case.tmask, k, grad_rgba, grad_hit, tiles)


class GpuTracer:
    """The product path: SplatRaster over the C ABI on one CUDA device."""

    def __init__(self, case: Case, k: int, key_mode: int, device, fallback: bool = True, log_capacity: int = 0,
                 enable_normals: bool = False, complete: bool = False, gofish: dict | None = None,
                 strategy: dict | None = None):
        """k: k-buffer size, or oracle.SOF_HIERARCHY for SOF's hierarchy;
        ``gofish``: further render.gofish keys; ``strategy``: the configuration's
        strategy section."""
        import torch

        from gofish_b200.splat_raster import SplatRaster

        self.torch = torch
        self.case = case
        self.device = device
        sof = k == oracle.SOF_HIERARCHY
        conf = {"render": {"splat": {"k_buffer_size": 16 if sof else k, "composite_log_capacity": log_capacity,
                                     "hierarchical_sort": sof},
                           "gofish": {"fast_global_depth_key": key_mode == 1,
                                      "fast_admission_fallback": "cone" if fallback else "none",
                                      "complete_admission": complete, **(gofish or {})},
                           "enable_hitcounts": True, "enable_normals": enable_normals},
                "strategy": strategy or {}}
        self.raster = SplatRaster(conf)
        self.token = "test-token"
        self.raster.register_physical_tile_mask(torch.from_numpy(case.tmask).to(device), self.token)
        self.particles = torch.from_numpy(case.particles).to(device)
        self.features = torch.from_numpy(np.ascontiguousarray(case.features)).to(device)
        self.ray_o = torch.from_numpy(case.ray_o[None].copy()).to(device)
        self.ray_d = torch.from_numpy(case.ray_d[None].copy()).to(device)
        self.sensor = case.camera.model()
        self.pose = torch.from_numpy(case.pose.copy())

    def forward(self):
        torch = self.torch
        out = self.raster.trace(0, False, self.case.scene.sh_degree, self.particles, self.features, self.ray_o,
                                self.ray_d, None, self.sensor, 0, 1, self.pose, self.pose, self.token)
        self.out = out
        inter = self.raster.copy_intermediates(self.device)
        torch.cuda.synchronize(self.device)
        res = {k: v.cpu().numpy() for k, v in inter.items()}
        res["rgba"] = out[0].cpu().numpy()
        res["hit_t"] = out[1][..., 0].cpu().numpy()
        res["hit_count"] = out[2][..., 0].cpu().numpy()
        res["visibility"] = out[3][:, 0].cpu().numpy().view(np.uint32)
        for name, t in zip(("normal", "depth_var", "quant", "extent", "opacity_field", "inv_depth", "inv_depth2"),
                           out[4:]):
            res[name] = t.cpu().numpy()
        return res

    def backward_after_forward(self, grad_rgba: np.ndarray, grad_hit: np.ndarray):
        """forward() then backward()."""
        self.forward()
        return self.backward(grad_rgba, grad_hit)

    def backward(self, grad_rgba: np.ndarray, grad_hit: np.ndarray, geometry: dict | None = None):
        """geometry: output gradients of the geometric channels by name (normal,
        depth_var, extent, inv_depth, inv_depth2), [H,W] or [H,W,3] arrays."""
        torch = self.torch
        g_rgba = torch.from_numpy(grad_rgba).to(self.device)
        g_hit = torch.from_numpy(grad_hit[..., None].copy()).to(self.device)
        pairs = [torch.zeros(1, device=self.device)] * 14
        if geometry:
            names = ("depth_var", "extent", "opacity_field", "quant", "normal", "inv_depth", "inv_depth2")
            index = {"depth_var": 5, "extent": 7, "opacity_field": 8, "quant": 6, "normal": 4, "inv_depth": 9,
                     "inv_depth2": 10}
            pairs = []
            for name in names:
                value = self.out[index[name]]
                grad = geometry.get(name)
                pairs += [value, None if grad is None else
                          torch.from_numpy(np.ascontiguousarray(grad, np.float32)).to(self.device).reshape(value.shape)]
        gp, gs = self.raster.trace_bwd(0, False, self.case.scene.sh_degree, self.particles, self.features, self.ray_o,
                                       self.ray_d, None, self.sensor, 0, 1, self.pose, self.pose, self.out[0], g_rgba,
                                       self.out[1], g_hit, *pairs, self.token)
        torch.cuda.synchronize(self.device)
        return gp.cpu().numpy(), gs.cpu().numpy()


def rel_l2(a: np.ndarray, b: np.ndarray) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    denom = max(np.linalg.norm(b), 1e-30)
    return float(np.linalg.norm(a - b) / denom)


def psnr(a: np.ndarray, b: np.ndarray) -> float:
    mse = float(np.mean((np.asarray(a, np.float64) - np.asarray(b, np.float64)) ** 2))
    return math.inf if mse == 0 else 10 * math.log10(1.0 / mse)


def horizon_case(seed: int = 31, n: int = 6000, big: int = 300, size: int = 192) -> Case:
    """A scene with large Gaussians (scale 0.5-2 m) within 1 m of the camera,
    many straddling the 100 degree horizon of a 200 degree fisheye or holding
    the camera centre: their unscented projection is invalid, so only the cone
    fallback admits them."""
    import dataclasses as dc

    scene = random_scene(n, 1, seed)
    rng = np.random.default_rng(seed + 1)
    u = rng.standard_normal((big, 3))
    u /= np.linalg.norm(u, axis=1, keepdims=True)
    u[: big // 2, 2] = rng.uniform(-0.25, 0.1, big // 2)  # near the horizon of a +z camera
    u /= np.linalg.norm(u, axis=1, keepdims=True)
    pos = (u * rng.uniform(0.05, 3.0, (big, 1))).astype(np.float32)
    scales = rng.uniform(0.5, 2.0, (big, 3)).astype(np.float32) * np.float32(0.12)
    positions = np.concatenate([scene.positions, pos]).astype(np.float32)
    sc = np.concatenate([scene.scales, scales]).astype(np.float32)
    q = rng.standard_normal((big, 4))
    rot = np.concatenate([scene.rotations, (q / np.linalg.norm(q, axis=1, keepdims=True)).astype(np.float32)])
    dens = np.concatenate([scene.density, rng.uniform(0.05, 0.6, (big, 1)).astype(np.float32)])
    feats = np.concatenate([scene.features, (rng.standard_normal((big, scene.features.shape[1])) * 0.2)
                            .astype(np.float32)])
    scene = dc.replace(scene, positions=positions, scales=sc, rotations=rot, density=dens, features=feats)
    cam = fisheye_camera(size, size, 200.0, random_kb_coefficients(rng, 200.0))
    return make_case(scene, cam, IDENTITY_POSE.copy())

def view_rows(model, batch, gamma: float):
    """The packed [N,32] rows Tracer.render traces for one view: the per-view
    full shape (Q_v with pixel variance ``gamma``, C = R S^2 R^T + Q_v, B =
    C^(1/2) R, B^-1, density m*o) through the product's shape kernels."""
    import torch

    from gofish_b200.view_observation_filter import build_intrinsic_view_shape

    n = model.num_gaussians
    shape = build_intrinsic_view_shape(model.get_scale(), model.get_rotation(), model.get_density(), model.positions,
                                       batch, pixel_footprint_variance=gamma)
    packed = torch.zeros((n, 32), dtype=torch.float32, device=model.positions.device)
    packed[:, 0:3] = model.positions
    packed[:, 3:4] = shape.density.reshape(n, 1)
    packed[:, 4:8] = model.get_rotation()
    packed[:, 8:11] = model.get_scale()
    packed[:, 11:12] = model.get_density()
    packed[:, 12:21] = shape.factor.reshape(n, 9)
    packed[:, 21:30] = shape.inverse_factor.reshape(n, 9)
    return packed


def compare_forward(ref, got, image_atol: float = 1e-3, tiles=None):
    """Bit-exact projected state, counts, keys, ids, ranges and visibility;
    hit counts bit-exact, images max-abs <= ``image_atol`` with PSNR >= 60
    dB and hit distance relative <= 1e-3, over the pixels of ``tiles``
    ([t0, t1) tile range, row-major) or the whole frame."""
    np.testing.assert_array_equal(got["proj"].view(np.uint32), ref["proj"].view(np.uint32))
    np.testing.assert_array_equal(got["counts"].astype(np.uint32), ref["counts"])
    np.testing.assert_array_equal(got["keys"].view(np.uint64), ref["keys"])
    np.testing.assert_array_equal(got["ids"].view(np.uint32), ref["ids"])
    np.testing.assert_array_equal(got["ranges"].view(np.uint32), ref["ranges"])
    np.testing.assert_array_equal(got["visibility"], ref["visibility"])
    h, w = ref["hit_count"].shape
    if tiles is None:
        sel = (slice(None), slice(None))
    else:
        tx = (w + 15) // 16
        r0, r1 = tiles[0] // tx, (tiles[1] + tx - 1) // tx
        assert tiles[0] % tx == 0 and tiles[1] % tx == 0, "tile bands are whole tile rows"
        sel = (slice(16 * r0, min(h, 16 * r1)), slice(None))
    np.testing.assert_array_equal(got["hit_count"][sel], ref["hit_count"][sel])
    assert np.abs(got["rgba"][sel] - ref["rgba"][sel]).max() <= image_atol
    assert psnr(got["rgba"][sel], ref["rgba"][sel]) >= 60.0
    np.testing.assert_allclose(got["hit_t"][sel], ref["hit_t"][sel], rtol=1e-3, atol=1e-4)
