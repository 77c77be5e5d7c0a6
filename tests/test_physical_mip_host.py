"""Physical-mip 3-D filter, host side: the camera-table packing and tie-break
key against golden vectors made from the reference's own physical_mip.py
(tests/golden/make_mip_golden.py), the shared double atan2, and the oracle's
best-rate search on closed forms."""

import math
from pathlib import Path

import numpy as np
import pytest

import oracle
from gofish_b200 import physical_mip

GOLDEN = Path(__file__).resolve().parent / "golden" / "mip_golden.npz"


def _golden_records():
    import importlib.util
    spec = importlib.util.spec_from_file_location("make_mip_golden", Path(__file__).parent / "golden" /
                                                  "make_mip_golden.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod.records()


def test_pack_camera_table_matches_reference():
    g = np.load(GOLDEN)
    cameras, frames = _golden_records()
    table = physical_mip.pack_camera_table(cameras, frames, "cpu")
    for name in ("rotations", "centers", "frame_camera", "frame_index", "frame_rank", "camera_model", "camera_width",
                 "camera_height", "camera_params", "camera_max_angle", "row_lo", "row_hi"):
        got = getattr(table, name).numpy()
        assert got.dtype == g[name].dtype and np.array_equal(got, g[name]), name


def test_tie_break_key_matches_reference():
    g = np.load(GOLDEN)
    key = physical_mip.tie_break_key("train:3:img/0003.png", 7, 3, "img/0003.png", [float(v) for v in range(16)])
    assert key == str(g["key"])


def test_atan2d_accuracy():
    rng = np.random.default_rng(1)
    ys = np.concatenate([rng.normal(size=2000) * 10.0 ** rng.integers(-6, 6, 2000), [0.0, -0.0, 1.0, -1.0]])
    xs = np.concatenate([rng.normal(size=2000) * 10.0 ** rng.integers(-6, 6, 2000), [0.0, -1.0, 0.0, 1e-300]])
    worst = 0.0
    for y, x in zip(ys, xs):
        got, want = oracle.atan2d(y, x), math.atan2(y, x)
        if want != 0.0:
            worst = max(worst, abs(got - want) / math.ulp(want))
        else:
            assert got == want
    assert worst <= 2.0, worst


def test_best_rate_closed_forms():
    # 64x48 pinhole at the origin looking down +z (the reference's docstring example).
    cameras = [{"camera_id": 1, "model": "PINHOLE", "width": 64, "height": 48, "params": [50.0, 50.0, 32.0, 24.0],
                "max_angle": None, "rows": [[0, 64]] * 48}]
    frames = [{"frame_index": 0, "camera_id": 1, "tie_break": "f0", "c2w": [1, 0, 0, 0, 0, 1, 0, 0, 0, 0, 1, 0]}]
    table = physical_mip.pack_camera_table(cameras, frames, "cpu")
    pts = np.array([[0.0, 0.0, 2.0], [0.0, 0.0, -2.0], [0.0, 0.0, 0.1], [100.0, 0.0, 1.0]])
    best, owner, observed, direction = oracle.mip_best_rate(pts, *[t.numpy() for t in table.arguments()])
    assert best[0] == 25.0 and owner[0] == 0 and observed[0] == 1
    assert np.array_equal(direction[0], [0.0, 0.0, 1.0])
    assert observed[1:].tolist() == [0, 0, 0] and owner[1:].tolist() == [-1, -1, -1] and best[1] == 0.0
    # equidistant fisheye, point on the optical axis: J = diag(f/d) (centre case)
    cameras = [{"camera_id": 1, "model": "OPENCV_FISHEYE", "width": 64, "height": 64,
                "params": [20.0, 21.0, 32.0, 32.0, 0.0, 0.0, 0.0, 0.0], "max_angle": 1.7, "rows": [[0, 64]] * 64}]
    table = physical_mip.pack_camera_table(cameras, frames, "cpu")
    best, owner, observed, _ = oracle.mip_best_rate(np.array([[0.0, 0.0, 4.0], [0.0, 0.0, 0.15]]),
                                                    *[t.numpy() for t in table.arguments()])
    assert best[0] == 5.0 and observed.tolist() == [1, 0]


def test_best_rate_ties_go_to_smaller_rank():
    from tests.mip_harness import cpu_table, mip_points
    cameras, frames, table = cpu_table(3)
    pts = mip_points(4, 400, frames)
    best, owner, observed, _ = oracle.mip_best_rate(pts, *[t.numpy() for t in table.arguments()])
    assert observed.mean() > 0.2
    # Frames 42, 43, 44 copy frames 0, 7, 13 (same camera and pose).  The copy
    # of 7 sorts before it (tie_break "000", rank 1) and takes all its points;
    # the copies of 0 and 13 sort last and take none.
    assert (owner == 43).sum() > 0 and (owner == 7).sum() == 0
    assert (owner == 0).sum() > 0 and (owner == 42).sum() == 0
    assert (owner == 13).sum() > 0 and (owner == 44).sum() == 0
