"""Random physical-mip camera tables for the oracle / GPU parity tests."""

from __future__ import annotations

import numpy as np

from gofish_b200.physical_mip import pack_camera_table


def _rotation(rng):
    q = rng.standard_normal(4)
    q /= np.linalg.norm(q)
    w, x, y, z = q
    return np.array([[1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)],
                     [2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)],
                     [2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)]])


def mip_records(seed: int = 3, frames_per_camera: int = 6):
    rng = np.random.default_rng(seed)
    fish_rows = [[max(0, 12 - abs(r - 24)), min(96, 84 + abs(r - 24) // 2)] if r % 17 else [0, 0] for r in range(48)]
    cameras = [
        {"camera_id": 1, "model": "OPENCV_FISHEYE", "width": 96, "height": 48,
         "params": [20.0, 21.0, 48.0, 24.0, 0.02, -0.003, 0.0004, -0.00002], "max_angle": 1.65, "rows": fish_rows},
        {"camera_id": 2, "model": "PINHOLE", "width": 64, "height": 48, "params": [50.0, 51.0, 32.0, 24.0],
         "max_angle": None, "rows": [[0, 64]] * 48},
        {"camera_id": 3, "model": "SIMPLE_RADIAL", "width": 40, "height": 30, "params": [35.0, 35.0, 20.0, 15.0, -0.05],
         "max_angle": None, "rows": [[1, 39]] * 30},
        {"camera_id": 4, "model": "RADIAL", "width": 40, "height": 30,
         "params": [35.0, 34.0, 20.0, 15.0, -0.05, 0.01], "max_angle": None, "rows": [[0, 40]] * 30},
        {"camera_id": 5, "model": "OPENCV", "width": 50, "height": 40,
         "params": [40.0, 41.0, 25.0, 20.0, -0.1, 0.02, 0.001, -0.002], "max_angle": None, "rows": [[0, 50]] * 40},
        {"camera_id": 6, "model": "FULL_OPENCV", "width": 50, "height": 40,
         "params": [40.0, 40.0, 25.0, 20.0, -0.1, 0.02, 0.001, -0.002, 0.001, 0.01, -0.002, 0.0003],
         "max_angle": None, "rows": [[0, 50]] * 40},
        {"camera_id": 8, "model": "SIMPLE_PINHOLE", "width": 30, "height": 30, "params": [25.0, 25.0, 15.0, 15.0],
         "max_angle": None, "rows": [[0, 30]] * 30},
    ]
    frames = []
    k = 0
    for cam in cameras:
        for j in range(frames_per_camera):
            m = np.eye(4)
            m[:3, :3] = _rotation(rng)
            m[:3, 3] = rng.uniform(-1.5, 1.5, 3)
            frames.append({"frame_index": k, "camera_id": cam["camera_id"], "c2w": m.reshape(-1).tolist(),
                           "tie_break": f"{(7 * k) % 11:03d}"})
            k += 1
    # Exact ties: copies of existing frames (same camera and pose), other ranks.
    for src in (0, 7, 13):
        dup = dict(frames[src])
        dup["frame_index"] = k
        dup["tie_break"] = "zz" + str(k) if src != 7 else "000"
        frames.append(dup)
        k += 1
    return cameras, frames


def mip_points(seed: int, n: int, frames) -> np.ndarray:
    rng = np.random.default_rng(seed)
    pts = rng.uniform(-4, 4, (n, 3))
    # a few points on camera optical axes (fisheye centre case) and at camera centres
    for j, f in enumerate(frames[:8]):
        m = np.asarray(f["c2w"]).reshape(4, 4)
        pts[j] = m[:3, 3] + 2.0 * m[:3, 2]
        pts[8 + j] = m[:3, 3]
    return pts


def table_numpy(table):
    return [t.cpu().numpy() for t in table.arguments()]


def cpu_table(seed: int = 3):
    cameras, frames = mip_records(seed)
    return cameras, frames, pack_camera_table(cameras, frames, "cpu")
