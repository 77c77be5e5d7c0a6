"""Generates tests/golden/mip_golden.npz from the reference's own
threedgrut/physical_mip.py (pack_camera_table and the frame tie-break key),
run in a container where the reference checkout is present.  The module is
loaded from its file with gofish.camera.pixel_chart (its only package
import) loaded from the checkout as well; no CUDA is involved.

    python tests/golden/make_mip_golden.py /path/to/reference
"""

from __future__ import annotations

import importlib.util
import sys
import types
from pathlib import Path

import numpy as np


def load(root: Path):
    for name in ("gofish", "gofish.camera"):
        mod = types.ModuleType(name)
        mod.__path__ = []
        sys.modules[name] = mod
    spec = importlib.util.spec_from_file_location("gofish.camera.pixel_chart",
                                                  root / "gofish" / "camera" / "pixel_chart.py")
    chart = importlib.util.module_from_spec(spec)
    sys.modules["gofish.camera.pixel_chart"] = chart
    spec.loader.exec_module(chart)
    spec = importlib.util.spec_from_file_location("ref_physical_mip", root / "threedgrut" / "physical_mip.py")
    mip = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mip)
    return mip


def records():
    """Three cameras (ids out of order, one fisheye with a support, one pinhole,
    one OpenCV) and seven frames with colliding tie-break strings."""
    cameras = [
        {"camera_id": 7, "model": "OPENCV_FISHEYE", "width": 40, "height": 30,
         "params": [12.0, 12.5, 20.0, 15.0, 0.01, -0.002, 0.0003, 0.0], "max_angle": 1.7,
         "rows": [[max(0, 10 - abs(r - 15)), min(40, 30 + abs(r - 15))] for r in range(30)]},
        {"camera_id": 2, "model": "PINHOLE", "width": 64, "height": 48, "params": [50.0, 51.0, 32.0, 24.0],
         "max_angle": None, "rows": [[0, 64]] * 48},
        {"camera_id": 4, "model": "OPENCV", "width": 32, "height": 20,
         "params": [30.0, 30.0, 16.0, 10.0, -0.1, 0.01, 0.001, -0.002], "max_angle": None,
         "rows": [[2, 30]] * 20},
    ]
    rng = np.random.default_rng(11)
    frames = []
    for k in range(7):
        m = np.eye(4)
        m[:3, 3] = rng.normal(size=3)
        frames.append({"frame_index": k, "camera_id": [7, 2, 4][k % 3], "c2w": m.reshape(-1).tolist(),
                       "tie_break": "t" + str((5 * k) % 4)})
    return cameras, frames


def main():
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} /path/to/reference")
    root = Path(sys.argv[1])
    mip = load(root)
    cameras, frames = records()
    table = mip.pack_camera_table(cameras, frames, "cpu")
    key = mip._tie_break_key("train:3:img/0003.png", 7, 3, "img/0003.png", [float(v) for v in range(16)])
    out = Path(__file__).resolve().parent / "mip_golden.npz"
    np.savez_compressed(out, key=np.array(key), **{name: getattr(table, name).numpy() for name in (
        "rotations", "centers", "frame_camera", "frame_index", "frame_rank", "camera_model", "camera_width",
        "camera_height", "camera_params", "camera_max_angle", "row_lo", "row_hi")})
    print("wrote", out)


if __name__ == "__main__":
    main()
