"""Generates tests/golden/domain_golden.npz from the reference's own pure-Python
Kannala-Brandt camera domain (gofish/camera/domain.py:37-113 and
gofish/camera/pixel_chart.py), run in a container where the reference checkout
is present.

For a set of distortion polynomials it records the reference's
``monotone_branch_limit`` (float64), and for the cameras the parity tests and
benchmarks use (equidistant 200 deg 320x320, Kannala-Brandt 200 deg at
1600x1600 with the single-view workload's coefficients, the equisolid 205 deg
2560x2560 model, the mesh query's equidistant 800x800) it records the rays of
``FisheyeDomain.first_branch_rays`` (float32 unit rays and the validity flag)
at sampled pixel centres: whole pixel rows through the centre, the rim and
the corners, and seeded random pixels.  The ray generator of this library
(``gofish_b200.camera``), which feeds every tracer and oracle test, is
compared with these vectors bit for bit by tests/test_domain_golden.py.

    python tests/golden/make_domain_golden.py /path/to/reference
"""

from __future__ import annotations

import importlib.util
import math
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]


def load_reference(root: Path):
    """The reference's domain module, loaded from its file with the package
    path pointing at the reference checkout (its package inits are empty)."""
    gofish = types.ModuleType("gofish")
    gofish.__path__ = [str(root / "gofish")]
    camera = types.ModuleType("gofish.camera")
    camera.__path__ = [str(root / "gofish" / "camera")]
    sys.modules["gofish"] = gofish
    sys.modules["gofish.camera"] = camera
    for name in ("pixel_chart", "domain"):
        spec = importlib.util.spec_from_file_location(f"gofish.camera.{name}",
                                                      root / "gofish" / "camera" / f"{name}.py")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[f"gofish.camera.{name}"] = mod
        spec.loader.exec_module(mod)
    return sys.modules["gofish.camera.domain"]


def coefficient_sets():
    """Distortion polynomials: zero (equidistant), equisolid, the single-view
    and multi-view workloads' draws, and seeded U(-0.05, 0.05) / U(-0.3, 0.3)
    draws (the wider ones include folding polynomials)."""
    sys.path.insert(0, str(REPO))
    from gofish_b200.camera import EQUISOLID_KB4, random_kb_coefficients

    sets = [(0.0, 0.0, 0.0, 0.0), tuple(float(np.float32(c)) for c in EQUISOLID_KB4)]
    for seed in (1235, 1236):
        sets.append(random_kb_coefficients(np.random.default_rng(seed + 1000), 200.0))
    rng = np.random.default_rng(4242)
    for spread in (0.05, 0.3):
        for _ in range(12):
            sets.append(tuple(float(np.float32(v)) for v in rng.uniform(-spread, spread, 4)))
    return sets


def sample_pixels(width: int, height: int, seed: int, random: int = 4096) -> np.ndarray:
    """Integer pixel indices [M,2] (x, y): whole rows through the centre, near
    the rim and at the edges, the four corners' 8x8 blocks, and seeded random
    pixels."""
    picks = []
    for y in sorted({height // 2, height // 2 - 1, height // 8, height - 1 - height // 8, 0, height - 1}):
        xs = np.arange(width)
        picks.append(np.stack([xs, np.full_like(xs, y)], axis=1))
    for cx in (0, width - 8):
        for cy in (0, height - 8):
            yy, xx = np.meshgrid(np.arange(cy, cy + 8), np.arange(cx, cx + 8), indexing="ij")
            picks.append(np.stack([xx.reshape(-1), yy.reshape(-1)], axis=1))
    rng = np.random.default_rng(seed)
    picks.append(np.stack([rng.integers(0, width, random), rng.integers(0, height, random)], axis=1))
    return np.concatenate(picks).astype(np.int64)


def cameras():
    from gofish_b200.camera import EQUISOLID_KB4, fisheye_camera, random_kb_coefficients

    kb1 = random_kb_coefficients(np.random.default_rng(1235 + 1000), 200.0)
    return [
        ("equidistant_200_320", fisheye_camera(320, 320, 200.0)),
        ("kb_200_1600", fisheye_camera(1600, 1600, 200.0, kb1)),
        ("equisolid_205_2560", fisheye_camera(2560, 2560, 205.0, EQUISOLID_KB4)),
        ("equidistant_200_800", fisheye_camera(800, 800, 200.0)),
        ("kb_200_250x170", fisheye_camera(250, 170, 200.0,
                                          random_kb_coefficients(np.random.default_rng(21 + 99), 200.0))),
    ]


def main():
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} /path/to/reference")
    root = Path(sys.argv[1])
    domain = load_reference(root)
    import torch

    out = {}
    sets = coefficient_sets()
    out["limit_coefficients"] = np.asarray(sets, dtype=np.float64)
    out["limit_values"] = np.asarray([domain.monotone_branch_limit(k) for k in sets], dtype=np.float64)
    names = []
    for i, (name, cam) in enumerate(cameras()):
        names.append(name)
        native = (cam.focal[0], cam.focal[1], cam.principal[0], cam.principal[1], *cam.coefficients)
        dom = domain.FisheyeDomain(native_params=tuple(float(v) for v in native), max_angle_radians=cam.max_angle,
                                   active_ratio_x=1.0, active_ratio_y=1.0)
        pix = sample_pixels(cam.width, cam.height, seed=100 + i)
        # unproject_raster lifts integer raster indices to native pixel centres (pixel_chart.native_center)
        centres = torch.stack((torch.as_tensor(pix[:, 0], dtype=torch.float64) + 0.5,
                               torch.as_tensor(pix[:, 1], dtype=torch.float64) + 0.5), dim=1)
        rays, valid = dom.first_branch_rays(centres)
        out[f"{name}/pixels"] = pix.astype(np.int32)
        out[f"{name}/rays"] = rays.numpy().astype(np.float32)
        out[f"{name}/valid"] = valid.numpy().reshape(-1).astype(np.uint8)
        out[f"{name}/camera"] = np.asarray([cam.width, cam.height, *native, cam.max_angle], dtype=np.float64)
        assert math.isfinite(float(rays.abs().max()))
    out["camera_names"] = np.asarray(names)
    np.savez_compressed(HERE / "domain_golden.npz", **out)
    print(f"wrote {HERE / 'domain_golden.npz'}: {len(sets)} polynomials, {len(names)} cameras")


if __name__ == "__main__":
    main()
