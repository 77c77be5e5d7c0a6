"""Effective (Mip-filtered) Gaussian shape used by the opacity field.

Follows gofish/mesh/shape.py:23-126: the scale is combined with the
training-camera Mip 3-D filter, S' = sqrt(S^2 + f^2), the rotation is kept,
B = R S' and B^-1 = S'^-1 R^T; no per-view footprint is applied.  The
checkpoint reader of the reference is replaced by ``effective_shape``, which
takes the activated arrays directly.
"""

from __future__ import annotations

from dataclasses import dataclass

import numpy as np

from ..scene import quaternion_to_matrix

DEAD_OPACITY = 1.0 / 255.0


@dataclass
class EffectiveShape:
    positions: np.ndarray  # [N, 3] float32
    density: np.ndarray  # [N, 1] float32, activated opacity
    factor: np.ndarray  # [N, 3, 3] float32, B = R S'
    inverse_factor: np.ndarray  # [N, 3, 3] float32, B^-1 = S'^-1 R^T
    sigma_max: np.ndarray  # [N, 1] float32, largest filtered scale
    retained: np.ndarray  # [N] bool, opacity > 1/255

    @property
    def count(self) -> int:
        return int(self.positions.shape[0])

    def packed_density(self) -> np.ndarray:
        """[N, 32] float32 rows in the tracer's packed layout (shape.py:34-48):
        position 0-2, density 3, identity quaternion 4-7, unit scale 8-10,
        zero 11, B 12-20, B^-1 21-29, zero 30-31."""
        n = self.count
        packed = np.zeros((n, 32), dtype=np.float32)
        packed[:, 0:3] = self.positions
        packed[:, 3:4] = self.density
        packed[:, 4] = 1.0
        packed[:, 8:11] = 1.0
        packed[:, 12:21] = self.factor.reshape(n, 9)
        packed[:, 21:30] = self.inverse_factor.reshape(n, 9)
        return packed


def effective_shape(positions: np.ndarray, scales: np.ndarray, rotations_wxyz: np.ndarray, opacity: np.ndarray,
                    mip_filter: np.ndarray | None = None) -> EffectiveShape:
    """Filtered shape from activated scales [N,3], unit quaternions (w,x,y,z)
    [N,4], opacities [N] or [N,1] and an optional Mip filter [N,1]
    (shape.py:76-126 after activation)."""
    positions = np.ascontiguousarray(positions, dtype=np.float32)
    n = positions.shape[0]
    scales = np.asarray(scales, dtype=np.float32).reshape(n, 3)
    filt = np.zeros((n, 1), np.float32) if mip_filter is None else np.asarray(mip_filter, np.float32).reshape(n, 1)
    alpha = np.asarray(opacity, dtype=np.float32).reshape(n, 1)
    scales_eff = np.sqrt(scales * scales + filt * filt).astype(np.float32)
    rot = quaternion_to_matrix(np.asarray(rotations_wxyz, dtype=np.float32)).astype(np.float32)
    factor = (rot * scales_eff[:, None, :]).astype(np.float32)
    inverse = (np.transpose(rot, (0, 2, 1)) / scales_eff[:, :, None]).astype(np.float32)
    if not (np.isfinite(factor).all() and np.isfinite(inverse).all()):
        raise ValueError("the filtered Gaussian shape is not finite")
    return EffectiveShape(
        positions=positions,
        density=np.ascontiguousarray(alpha),
        factor=np.ascontiguousarray(factor),
        inverse_factor=np.ascontiguousarray(inverse),
        sigma_max=np.ascontiguousarray(scales_eff.max(axis=1, keepdims=True)),
        retained=alpha[:, 0] > DEAD_OPACITY,
    )
