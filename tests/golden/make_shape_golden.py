"""Generates tests/golden/shape_golden.npz from the reference's own
threedgut_tracer/view_observation_filter.py (current_view_q6,
_minimum_norm_q6_from_float32_jacobian, footprint_covariance,
mass_preserving_factor), pure torch on the CPU, run in a container where the
reference checkout is present.  The module is loaded from its file; its one
package import (threedgrut.camera_local_validity) is loaded from the checkout
too.

    python tests/golden/make_shape_golden.py /path/to/reference
"""

from __future__ import annotations

import importlib.util
import math
import sys
import types
from pathlib import Path

import numpy as np
import torch


def load(root: Path):
    pkg = types.ModuleType("threedgrut")
    pkg.__path__ = []
    sys.modules["threedgrut"] = pkg
    spec = importlib.util.spec_from_file_location("threedgrut.camera_local_validity",
                                                  root / "threedgrut" / "camera_local_validity.py")
    mod = importlib.util.module_from_spec(spec)
    sys.modules["threedgrut.camera_local_validity"] = mod
    spec.loader.exec_module(mod)
    spec = importlib.util.spec_from_file_location("ref_vof", root / "threedgut_tracer" / "view_observation_filter.py")
    vof = importlib.util.module_from_spec(spec)
    sys.modules["ref_vof"] = vof
    spec.loader.exec_module(vof)
    return vof


def pose_c2w(rng):
    q = rng.standard_normal(4)
    q /= np.linalg.norm(q)
    w, x, y, z = q
    R = np.array([[1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)],
                  [2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)],
                  [2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)]])
    m = np.eye(4)
    m[:3, :3] = R
    m[:3, 3] = rng.uniform(-1, 1, 3)
    return m.astype(np.float32)


def points(rng, m, n):
    p = rng.uniform(-4, 4, (n, 3))
    c, R = m[:3, 3].astype(np.float64), m[:3, :3].astype(np.float64)
    p[:6] = c + np.array([[0, 0, 2.0], [0, 0, 0.1], [0, 0, -2.0], [0.5, 0, 0.0], [1e-14, 0, 3.0], [0, 0, 0.3]]) @ R.T
    return p.astype(np.float32)


def main():
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} /path/to/reference")
    root = Path(sys.argv[1])
    vof = load(root)
    rng = np.random.default_rng(8)
    out = {}
    # fisheye
    mf = pose_c2w(rng)
    pf = points(rng, mf, 1200)
    fish = {"focal_length": [310.0, 305.0], "radial_coeffs": [0.03, -0.004, 0.0005, -0.00003],
            "max_angle": 1.75}
    batch = types.SimpleNamespace(T_to_world=torch.from_numpy(mf)[None], T_to_world_end=None,
                                  rays_in_world_space=False, intrinsics_OpenCVFisheyeCameraModelParameters=fish)
    q6, jac, valid = vof.current_view_q6(torch.from_numpy(pf), batch, 0.3)
    out.update(fish_pose=mf, fish_points=pf, fish_q6=q6.numpy(), fish_jacobian=jac.numpy(),
               fish_valid=valid.numpy(), fish_focal=np.array(fish["focal_length"]),
               fish_k=np.array(fish["radial_coeffs"]), fish_max_angle=np.array(fish["max_angle"]))
    # ideal pinhole
    mp = pose_c2w(rng)
    pp = points(rng, mp, 800)
    pin = {"focal_length": [420.0, 415.0], "radial_coeffs": [0.0] * 6, "tangential_coeffs": [0.0, 0.0],
           "thin_prism_coeffs": [0.0] * 4}
    batch = types.SimpleNamespace(T_to_world=torch.from_numpy(mp)[None], T_to_world_end=None,
                                  rays_in_world_space=False, intrinsics_OpenCVPinholeCameraModelParameters=pin)
    q6, jac, valid = vof.current_view_q6(torch.from_numpy(pp), batch, 0.3)
    out.update(pin_pose=mp, pin_points=pp, pin_q6=q6.numpy(), pin_jacobian=jac.numpy(), pin_valid=valid.numpy(),
               pin_focal=np.array(pin["focal_length"]))
    # mass-preserving factor and pseudo-inverse footprint on random full-rank J and SPD Sigma
    J = torch.from_numpy(rng.normal(size=(300, 2, 3)) * 50.0)
    A = torch.from_numpy(rng.normal(size=(300, 3, 3)) * 0.05)
    sigma = A @ A.transpose(1, 2) + 1e-4 * torch.eye(3, dtype=torch.float64)
    out.update(m_jacobian=J.numpy(), m_sigma=sigma.numpy(), m_value=vof.mass_preserving_factor(sigma, J, 0.3).numpy(),
               q_value=vof.footprint_covariance(J, 0.3).numpy())
    path = Path(__file__).resolve().parent / "shape_golden.npz"
    np.savez_compressed(path, **out)
    print("wrote", path, {k: v.shape for k, v in out.items() if hasattr(v, "shape")})


if __name__ == "__main__":
    main()
