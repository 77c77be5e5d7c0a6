"""Generates tests/golden/mesh_golden.npz from the reference's own pure-Python
mesh modules (gofish/mesh/sites.py, shape.py, field.py, bisection.py), run in
a container where the reference checkout is present.

The reference package's __init__ imports the whole extraction pipeline, and
its cameras module needs omegaconf, so the four modules are loaded from their
files into a stand-in package with a stub ``cameras`` module.  Inputs are
seeded; the outputs are the golden vectors the mesh host tests compare with.

    python tests/golden/make_mesh_golden.py /path/to/reference
"""

from __future__ import annotations

import importlib.util
import sys
import types
from pathlib import Path

import numpy as np


def load_reference(root: Path):
    pkg = types.ModuleType("refmesh")
    pkg.__path__ = [str(root / "gofish" / "mesh")]
    sys.modules["refmesh"] = pkg
    cameras = types.ModuleType("refmesh.cameras")

    class TrainingCamera:  # only used in type annotations
        pass

    cameras.TrainingCamera = TrainingCamera
    sys.modules["refmesh.cameras"] = cameras
    mods = {}
    for name in ("shape", "sites", "field", "bisection"):
        spec = importlib.util.spec_from_file_location(f"refmesh.{name}", root / "gofish" / "mesh" / f"{name}.py")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[f"refmesh.{name}"] = mod
        spec.loader.exec_module(mod)
        mods[name] = mod
    return mods


def random_shape(mods, n: int, seed: int):
    rng = np.random.default_rng(seed)
    positions = rng.uniform(-3, 3, (n, 3)).astype(np.float32)
    q = rng.standard_normal((n, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    w, x, y, z = q.T
    R = np.stack([
        np.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)], -1),
        np.stack([2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)], -1),
        np.stack([2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], -1),
    ], 1).astype(np.float32)
    s = np.exp(rng.normal(np.log(0.05), 0.5, (n, 3))).astype(np.float32)
    density = (1 / (1 + np.exp(-rng.normal(0, 2.0, (n, 1))))).astype(np.float32)
    density[:3] = np.float32(1.0 / 255.0) * np.float32(0.5)  # some dead Gaussians
    factor = (R * s[:, None, :]).astype(np.float32)
    inverse = (np.transpose(R, (0, 2, 1)) / s[:, :, None]).astype(np.float32)
    return mods["shape"].EffectiveShape(
        positions=positions, density=density, factor=factor, inverse_factor=inverse,
        sigma_max=s.max(axis=1, keepdims=True).astype(np.float32),
        retained=density[:, 0] > mods["shape"].DEAD_OPACITY)


def main():
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} /path/to/reference")
    root = Path(sys.argv[1])
    mods = load_reference(root)
    shape = random_shape(mods, 257, seed=31)
    sites = mods["sites"].generate_sites(shape)
    rng = np.random.default_rng(5)
    minimum = rng.random(1000).astype(np.float32)
    minimum[:10] = np.float32(0.5)
    observed = (rng.random(1000) < 0.8).astype(np.uint8)
    signed = mods["field"].signed_field(minimum, observed)
    cases = np.array([[10, 8 << 30, 1 << 20], [1 << 26, 40 << 30, 1 << 28], [1 << 30, 3 << 30, 0],
                      [5_000_000, 3 << 30, 1 << 29]], dtype=np.int64)
    sizes = np.array([mods["bisection"].batch_size(int(e), int(f), int(c)) for e, f, c in cases], dtype=np.int64)
    ends = rng.random((7, 2, 3)).astype(np.float32)
    vals = rng.random((7, 2)).astype(np.float32)
    pe, pv = mods["bisection"]._padded_batch(ends, vals, 2, 7, 8)
    out = Path(__file__).resolve().parent / "mesh_golden.npz"
    np.savez_compressed(
        out, positions=shape.positions, density=shape.density, factor=shape.factor,
        inverse_factor=shape.inverse_factor, sigma_max=shape.sigma_max, retained=shape.retained,
        packed=shape.packed_density(), site_points=sites.points, site_scale=sites.scale, site_owner=sites.owner,
        radius=mods["sites"].support_radius(shape.density[shape.retained, 0]),
        minimum=minimum, observed=observed, signed=signed, batch_cases=cases, batch_sizes=sizes,
        pad_ends=ends, pad_vals=vals, padded_ends=pe, padded_vals=pv)
    print("wrote", out)


if __name__ == "__main__":
    main()
