"""Seeded synthetic scenes and cameras of the five benchmark workloads.

The reference measures on public datasets (FIORD, FullCircle, ScanNet++,
Tanks and Temples) that are not available here; these generators stand in
for them with the workload shapes and value distributions:

* means uniform in the spherical shell 1-5 m around the origin,
* log-scales N(ln 0.02, 0.5^2) per axis, uniform unit quaternions,
* opacity sigmoid(N(0, 1.5^2)),
* SH DC chosen so the base colour is U[0,1] (c0 = (rgb - 0.5) / 0.2820948),
  higher SH coefficients N(0, 0.1^2).

``pack_particles`` builds the reference's packed [N,32] particle rows
(threedgut_tracer/tracer.py:171-179): position, density, rotation (w,x,y,z),
scale, intrinsic density, factor B = R diag(s) and its inverse, padding.
"""

from __future__ import annotations

import dataclasses
import math

import numpy as np

from .camera import EQUISOLID_KB4, FisheyeCamera, fisheye_camera, random_kb_coefficients

SH_C0 = 0.28209479177387814
PACKED_WIDTH = 32
SLOTS = {"position": (0, 3), "density": (3, 4), "rotation": (4, 8), "scale": (8, 11),
         "intrinsic_density": (11, 12), "factor": (12, 21), "inverse_factor": (21, 30), "padding": (30, 32)}


@dataclasses.dataclass
class Scene:
    positions: np.ndarray   # [N,3] float32
    rotations: np.ndarray   # [N,4] float32 unit quaternions (w, x, y, z)
    scales: np.ndarray      # [N,3] float32
    density: np.ndarray     # [N,1] float32 opacity in (0, 1)
    features: np.ndarray    # [N, 3*C] float32, coefficient k of channel c at [3k + c]
    sh_degree: int

    @property
    def num(self) -> int:
        return int(self.positions.shape[0])

    @property
    def sh_coeffs(self) -> int:
        return int(self.features.shape[1] // 3)


def quaternion_to_matrix(q: np.ndarray) -> np.ndarray:
    """Rotation matrices [N,3,3] of unit quaternions (w, x, y, z)."""
    q = np.asarray(q, dtype=np.float64)
    w, x, y, z = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    R = np.empty((q.shape[0], 3, 3), dtype=np.float64)
    R[:, 0, 0] = 1 - 2 * (y * y + z * z)
    R[:, 0, 1] = 2 * (x * y - w * z)
    R[:, 0, 2] = 2 * (x * z + w * y)
    R[:, 1, 0] = 2 * (x * y + w * z)
    R[:, 1, 1] = 1 - 2 * (x * x + z * z)
    R[:, 1, 2] = 2 * (y * z - w * x)
    R[:, 2, 0] = 2 * (x * z - w * y)
    R[:, 2, 1] = 2 * (y * z + w * x)
    R[:, 2, 2] = 1 - 2 * (x * x + y * y)
    return R


def pack_particles(scene: Scene, chunk: int = 1 << 20) -> np.ndarray:
    """[N,32] float32 packed rows with B = R diag(s), B^-1 = diag(1/s) R^T."""
    n = scene.num
    out = np.zeros((n, PACKED_WIDTH), dtype=np.float32)
    for b in range(0, n, chunk):
        e = min(n, b + chunk)
        R = quaternion_to_matrix(scene.rotations[b:e])
        s = scene.scales[b:e].astype(np.float64)
        B = R * s[:, None, :]
        Binv = np.transpose(R, (0, 2, 1)) / s[:, :, None]
        rows = out[b:e]
        rows[:, 0:3] = scene.positions[b:e]
        rows[:, 3:4] = scene.density[b:e]
        rows[:, 4:8] = scene.rotations[b:e]
        rows[:, 8:11] = scene.scales[b:e]
        rows[:, 11:12] = scene.density[b:e]
        rows[:, 12:21] = B.reshape(-1, 9).astype(np.float32)
        rows[:, 21:30] = Binv.reshape(-1, 9).astype(np.float32)
    return out


def _uniform_directions(rng: np.random.Generator, n: int) -> np.ndarray:
    v = rng.standard_normal((n, 3))
    return v / np.linalg.norm(v, axis=1, keepdims=True)


def random_scene(n: int, sh_degree: int, seed: int, r_min: float = 1.0, r_max: float = 5.0) -> Scene:
    rng = np.random.default_rng(seed)
    u = rng.random(n)
    radius = np.cbrt(u * (r_max ** 3 - r_min ** 3) + r_min ** 3)
    positions = (_uniform_directions(rng, n) * radius[:, None]).astype(np.float32)
    scales = np.exp(rng.normal(math.log(0.02), 0.5, size=(n, 3))).astype(np.float32)
    q = rng.standard_normal((n, 4))
    rotations = (q / np.linalg.norm(q, axis=1, keepdims=True)).astype(np.float32)
    density = (1.0 / (1.0 + np.exp(-rng.normal(0.0, 1.5, size=(n, 1))))).astype(np.float32)
    coeffs = (sh_degree + 1) ** 2
    features = np.empty((n, 3 * coeffs), dtype=np.float32)
    rgb = rng.random((n, 3))
    features[:, 0:3] = ((rgb - 0.5) / SH_C0).astype(np.float32)
    if coeffs > 1:
        features[:, 3:] = rng.normal(0.0, 0.1, size=(n, 3 * (coeffs - 1))).astype(np.float32)
    return Scene(positions, rotations, scales, density, features, sh_degree)


def random_rotation_quaternion_xyzw(rng: np.random.Generator) -> np.ndarray:
    q = rng.standard_normal(4)
    q /= np.linalg.norm(q)
    return q.astype(np.float64)  # (x, y, z, w)


def pose_world_to_sensor(center: np.ndarray, quat_xyzw: np.ndarray) -> np.ndarray:
    """7-float world->sensor pose [t, q(x,y,z,w)] of a camera at ``center``
    whose world->sensor rotation is ``quat_xyzw`` (t = -R c)."""
    x, y, z, w = (float(v) for v in quat_xyzw)
    R = quaternion_to_matrix(np.array([[w, x, y, z]]))[0]
    t = -R @ np.asarray(center, dtype=np.float64)
    return np.concatenate([t, [x, y, z, w]]).astype(np.float32)


def look_outward_pose(center: np.ndarray, yaw: float) -> np.ndarray:
    """World->sensor pose of a camera at ``center`` whose optical axis (+z)
    points horizontally outward at azimuth ``yaw`` (world z up)."""
    forward = np.array([math.cos(yaw), math.sin(yaw), 0.0])
    up = np.array([0.0, 0.0, 1.0])
    right = np.cross(forward, up)
    right /= np.linalg.norm(right)
    down = np.cross(forward, right)
    # Sensor axes (x right, y down, z forward) expressed in world coordinates are
    # the rows of the world->sensor rotation.
    R = np.stack([right, down, forward], axis=0)
    # quaternion (x, y, z, w) of R
    tr = np.trace(R)
    if tr > 0:
        s = math.sqrt(tr + 1.0) * 2
        w = 0.25 * s
        x = (R[2, 1] - R[1, 2]) / s
        y = (R[0, 2] - R[2, 0]) / s
        z = (R[1, 0] - R[0, 1]) / s
    elif R[0, 0] > R[1, 1] and R[0, 0] > R[2, 2]:
        s = math.sqrt(1.0 + R[0, 0] - R[1, 1] - R[2, 2]) * 2
        w = (R[2, 1] - R[1, 2]) / s
        x = 0.25 * s
        y = (R[0, 1] + R[1, 0]) / s
        z = (R[0, 2] + R[2, 0]) / s
    elif R[1, 1] > R[2, 2]:
        s = math.sqrt(1.0 + R[1, 1] - R[0, 0] - R[2, 2]) * 2
        w = (R[0, 2] - R[2, 0]) / s
        x = (R[0, 1] + R[1, 0]) / s
        y = 0.25 * s
        z = (R[1, 2] + R[2, 1]) / s
    else:
        s = math.sqrt(1.0 + R[2, 2] - R[0, 0] - R[1, 1]) * 2
        w = (R[1, 0] - R[0, 1]) / s
        x = (R[0, 2] + R[2, 0]) / s
        y = (R[1, 2] + R[2, 1]) / s
        z = 0.25 * s
    q = np.array([x, y, z, w])
    q /= np.linalg.norm(q)
    return pose_world_to_sensor(center, q)


IDENTITY_POSE = np.array([0, 0, 0, 0, 0, 0, 1], dtype=np.float32)


@dataclasses.dataclass
class Workload:
    name: str
    scene: Scene
    camera: FisheyeCamera
    poses: list          # list of 7-float world->sensor poses
    k_buffer: int
    description: str
    big_rows: np.ndarray | None = None  # rows of the large Gaussians beside the camera path


def workload_cpu_scale(seed: int = 1234) -> Workload:
    """10,000 Gaussians, SH degree 0, equidistant 200 deg 320x320, identity pose, k = 16."""
    scene = random_scene(10_000, 0, seed)
    cam = fisheye_camera(320, 320, 200.0)
    return Workload("cpu_scale_fwd", scene, cam, [IDENTITY_POSE.copy()], 16,
                    "10k Gaussians SH0, equidistant 200deg 320x320, identity pose, K=16")


def workload_single_view(seed: int = 1235, n: int = 1_000_000, size: int = 1600) -> Workload:
    """1M Gaussians SH3, Kannala-Brandt 200 deg 1600x1600, random pose in r < 0.5 m, k = 16."""
    scene = random_scene(n, 3, seed)
    rng = np.random.default_rng(seed + 1000)
    k = random_kb_coefficients(rng, 200.0)
    cam = fisheye_camera(size, size, 200.0, k)
    center = _uniform_directions(rng, 1)[0] * 0.5 * np.cbrt(rng.random())
    pose = pose_world_to_sensor(center, random_rotation_quaternion_xyzw(rng))
    return Workload("single_view_fwd_bwd", scene, cam, [pose], 16,
                    f"{n} Gaussians SH3, KB 200deg {size}x{size}, random pose, K=16, L1 vs U[0,1] target")


def workload_multi_view(seed: int = 1236, n: int = 3_000_000, views: int = 64, size: int = 1600) -> Workload:
    """3M Gaussians SH3, 64 KB 200 deg 1600x1600 views on a 2 m ring."""
    scene = random_scene(n, 3, seed)
    rng = np.random.default_rng(seed + 1000)
    k = random_kb_coefficients(rng, 200.0)
    cam = fisheye_camera(size, size, 200.0, k)
    poses = []
    for v in range(views):
        yaw = rng.uniform(0.0, 2.0 * math.pi)
        center = np.array([2.0 * math.cos(yaw), 2.0 * math.sin(yaw), 0.0])
        poses.append(look_outward_pose(center, yaw))
    return Workload("multi_view_fwd_bwd", scene, cam, poses, 16,
                    f"{n} Gaussians SH3, {views} KB 200deg {size}x{size} views on a 2 m ring, K=16")


def workload_mesh_query(seed: int = 1237, n: int = 3_000_000, views: int = 32, size: int = 800) -> Workload:
    """GOF-style mesh opacity query: 3M Gaussians with the CPU-scale
    distributions (SH degree 0), queried at their sites (centre + 8 support-box
    corners, about 27M points) from 32 equidistant (k = 0) 200 deg fisheye
    views at 800x800, placed evenly on a 2 m ring and looking outward."""
    scene = random_scene(n, 0, seed)
    cam = fisheye_camera(size, size, 200.0)
    poses = []
    for v in range(views):
        yaw = 2.0 * math.pi * v / views
        centre = np.array([2.0 * math.cos(yaw), 2.0 * math.sin(yaw), 0.0])
        poses.append(look_outward_pose(centre, yaw))
    return Workload("mesh_opacity_query", scene, cam, poses, 0,
                    f"{n} Gaussians, sites (centre + 8 corners), {views} equidistant 200deg {size}x{size} views "
                    "on a 2 m ring")


def orbit_poses(frames: int, radius: float = 2.0) -> list:
    """World->sensor poses of ``frames`` cameras evenly spaced on a horizontal
    ring of ``radius`` metres around the origin, each looking outward."""
    poses = []
    for v in range(frames):
        yaw = 2.0 * math.pi * v / frames
        poses.append(look_outward_pose(np.array([radius * math.cos(yaw), radius * math.sin(yaw), 0.0]), yaw))
    return poses


def workload_inference(seed: int = 1238, n: int = 6_000_000, frames: int = 240, size: int = 2560,
                       big_fraction: float = 0.05, big_sigma=(0.05, 0.2), orbit_radius: float = 2.0) -> Workload:
    """High-resolution inference orbit: ``n`` Gaussians SH3 with the common
    distributions, of which ``big_fraction`` are large Gaussians beside the
    camera path (centres within 1 m of the orbit ring, in the plane
    perpendicular to the local outward optical axis, so that they straddle the
    theta = 90 deg horizon of the nearby frames; per-axis scale s * exp(N(0,
    0.2^2)), s ~ U(big_sigma)); equisolid (KB 4-term Taylor) 205 deg fisheye at
    size x size; ``frames`` outward-looking views on a ring of ``orbit_radius``
    metres; k = 32."""
    scene = random_scene(n, 3, seed)
    rng = np.random.default_rng(seed + 1000)
    nb = int(round(big_fraction * n))
    rows = np.zeros(0, dtype=np.int64)
    if nb > 0:
        rows = np.sort(rng.choice(n, size=nb, replace=False))
        phi = rng.uniform(0.0, 2.0 * math.pi, nb)
        rho = rng.uniform(0.2, 1.0, nb)
        psi = rng.uniform(0.0, 2.0 * math.pi, nb)
        ring = np.stack([orbit_radius * np.cos(phi), orbit_radius * np.sin(phi), np.zeros(nb)], axis=1)
        tangent = np.stack([-np.sin(phi), np.cos(phi), np.zeros(nb)], axis=1)
        outward = np.stack([np.cos(phi), np.sin(phi), np.zeros(nb)], axis=1)
        up = np.array([0.0, 0.0, 1.0])
        centre = (ring + rho[:, None] * (np.cos(psi)[:, None] * tangent + np.sin(psi)[:, None] * up)
                  + rng.uniform(-0.1, 0.1, nb)[:, None] * outward)
        s = rng.uniform(big_sigma[0], big_sigma[1], nb)
        scene.positions[rows] = centre.astype(np.float32)
        scene.scales[rows] = (s[:, None] * np.exp(rng.normal(0.0, 0.2, (nb, 3)))).astype(np.float32)
    cam = fisheye_camera(size, size, 205.0, EQUISOLID_KB4)
    return Workload("inference_orbit", scene, cam, orbit_poses(frames, orbit_radius), 32,
                    f"{n} Gaussians SH3 ({nb} large beside the camera path), equisolid 205deg {size}x{size}, "
                    f"{frames}-frame {orbit_radius:g} m orbit, K=32, physical-mip filter on", rows)


def pose_to_c2w(pose7) -> np.ndarray:
    """4x4 camera-to-world matrix of a world->sensor pose [t, q(x, y, z, w)]."""
    t = np.asarray(pose7[:3], dtype=np.float64)
    x, y, z, w = (float(v) for v in pose7[3:7])
    R = quaternion_to_matrix(np.array([[w, x, y, z]]))[0]
    c2w = np.eye(4)
    c2w[:3, :3] = R.T
    c2w[:3, 3] = -R.T @ t
    return c2w


def camera_valid_runs(valid: np.ndarray) -> list:
    """[lo, hi) column run of valid pixels per row of a convex [H,W] mask
    ([0, 0] for a row without one)."""
    runs = []
    for row in np.asarray(valid, dtype=bool):
        cols = np.flatnonzero(row)
        runs.append([int(cols[0]), int(cols[-1]) + 1] if cols.size else [0, 0])
    return runs


def mip_camera_records(camera: FisheyeCamera, poses: list, valid: np.ndarray, camera_id: int = 0):
    """Physical-mip camera and frame records (pack_camera_table format) of one
    fisheye camera seen from ``poses``; tie ranks follow the frame order."""
    cam = {"camera_id": camera_id, "model": "OPENCV_FISHEYE", "width": camera.width, "height": camera.height,
           "params": [*camera.focal, *camera.principal, *camera.coefficients], "max_angle": float(camera.max_angle),
           "rows": camera_valid_runs(valid)}
    frames = [{"frame_index": k, "camera_id": camera_id, "c2w": pose_to_c2w(p).reshape(-1).tolist(),
               "tie_break": f"{k:06d}"} for k, p in enumerate(poses)]
    return [cam], frames

