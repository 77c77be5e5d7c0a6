"""Calibrated Mip filtering, view-independent part: the 3-D filter
(threedgrut/physical_mip.py:1-266 and its CUDA extension).

Each Gaussian gets an isotropic 3-D low-pass filter from the finest pixel
sampling rate at which any training frame observes its centre: over the
frames whose calibrated support holds the projected centre, the rate is the
smallest singular value of the 2x3 world pixel Jacobian, and
filter_3D = sqrt(variance) / best_rate; unobserved Gaussians get the largest
observed filter.  The search runs in float64 on the GPU (gf_mip_best_rate);
equal rates go to the frame with the smaller tie-break rank.
"""

from __future__ import annotations

import hashlib
import json
import math
import struct
from dataclasses import dataclass
from typing import Any

import torch

from . import _native

MODEL_IDS = {
    "SIMPLE_PINHOLE": 0,
    "PINHOLE": 1,
    "OPENCV_FISHEYE": 2,
    "SIMPLE_RADIAL": 3,
    "RADIAL": 4,
    "OPENCV": 5,
    "FULL_OPENCV": 6,
}
PACKED_PARAMETER_COUNT = 12
MAX_CAMERAS = 64


@dataclass(frozen=True)
class CameraTable:
    """Training-camera table consumed by the GPU search (physical_mip.py:76-99)."""

    rotations: torch.Tensor  # [F, 3, 3] float64 camera-to-world rotation
    centers: torch.Tensor  # [F, 3] float64 camera centre
    frame_camera: torch.Tensor  # [F] int32 camera slot
    frame_index: torch.Tensor  # [F] int32 training frame index
    frame_rank: torch.Tensor  # [F] int64 tie-break rank
    camera_model: torch.Tensor  # [C] int32
    camera_width: torch.Tensor  # [C] int32
    camera_height: torch.Tensor  # [C] int32
    camera_params: torch.Tensor  # [C, 12] float64, [fx, fy, cx, cy, distortion...]
    camera_max_angle: torch.Tensor  # [C] float64, -1 for none
    row_lo: torch.Tensor  # [C, Hmax] int32 valid column runs [lo, hi) per row
    row_hi: torch.Tensor

    def arguments(self) -> tuple[torch.Tensor, ...]:
        return (self.rotations, self.centers, self.frame_camera, self.frame_index, self.frame_rank,
                self.camera_model, self.camera_width, self.camera_height, self.camera_params,
                self.camera_max_angle, self.row_lo, self.row_hi)


def _canonical_json_sha256(value: Any) -> str:
    payload = json.dumps(value, sort_keys=True, separators=(",", ":"), allow_nan=False) + "\n"
    return hashlib.sha256(payload.encode("utf-8")).hexdigest()


def tie_break_key(frame_id: str, camera_id: int, source_index: int, relative_path: str, pose_values) -> str:
    """Deterministic tie-break string of a training frame (physical_mip.py:102-110)."""
    pose = hashlib.sha256(struct.pack("<16f", *pose_values)).hexdigest()
    return _canonical_json_sha256({"frame_id": frame_id, "camera_id": int(camera_id),
                                   "source_frame_index": int(source_index), "relative_image_path": relative_path,
                                   "pose_sha256": pose})


def pack_camera_table(cameras: list[dict], frames: list[dict], device) -> CameraTable:
    """Pack camera and frame records (format of physical_mip.py:172-224).

    ``cameras``: ``{"camera_id", "model", "width", "height", "params" (at the
    active raster), "max_angle" (None for none), "rows" ([lo, hi) per row)}``.
    ``frames``: ``{"frame_index", "camera_id", "c2w" (3x4 or 4x4 row-major),
    "tie_break"}``.  Cameras are slotted by ascending id; frames are ordered by
    (camera slot, tie rank), the rank being the position in (tie_break,
    frame_index) order.
    """
    cams = sorted(cameras, key=lambda c: c["camera_id"])
    if not 0 < len(cams) <= MAX_CAMERAS:
        raise ValueError(f"between 1 and {MAX_CAMERAS} cameras are supported")
    slot = {c["camera_id"]: k for k, c in enumerate(cams)}
    rank_of = {f["frame_index"]: r for r, f in enumerate(sorted(frames, key=lambda f: (f["tie_break"],
                                                                                       f["frame_index"])))}
    ordered = sorted(frames, key=lambda f: (f["camera_id"], rank_of[f["frame_index"]]))
    rot, cen, fcam, fidx, frank = [], [], [], [], []
    for f in ordered:
        m = f["c2w"]
        rot.append([[m[4 * r + c] for c in range(3)] for r in range(3)])
        cen.append([m[3], m[7], m[11]])
        fcam.append(slot[f["camera_id"]])
        fidx.append(f["frame_index"])
        frank.append(rank_of[f["frame_index"]])
    hmax = max(c["height"] for c in cams)
    model, width, height, params, cap, lo, hi = [], [], [], [], [], [], []
    for c in cams:
        runs = list(c["rows"]) + [[0, 0]] * (hmax - c["height"])
        model.append(MODEL_IDS[c["model"]])
        width.append(c["width"])
        height.append(c["height"])
        params.append(list(c["params"]) + [0.0] * (PACKED_PARAMETER_COUNT - len(c["params"])))
        cap.append(-1.0 if c["max_angle"] is None else float(c["max_angle"]))
        lo.append([r[0] for r in runs])
        hi.append([r[1] for r in runs])

    def t(v, dtype):
        return torch.as_tensor(v, dtype=dtype, device=device).contiguous()

    return CameraTable(t(rot, torch.float64), t(cen, torch.float64), t(fcam, torch.int32), t(fidx, torch.int32),
                       t(frank, torch.int64), t(model, torch.int32), t(width, torch.int32), t(height, torch.int32),
                       t(params, torch.float64), t(cap, torch.float64), t(lo, torch.int32), t(hi, torch.int32))


def _check(value: torch.Tensor, name: str, device, dtype, dim: int | None = None) -> None:
    if not isinstance(value, torch.Tensor) or not value.is_cuda or not value.is_contiguous():
        raise RuntimeError(f"{name} must be a contiguous CUDA tensor")
    if value.device != device:
        raise RuntimeError(f"{name} must be on the positions device")
    if value.dtype != dtype or (dim is not None and value.dim() != dim):
        raise RuntimeError(f"{name} has the wrong dtype or rank")


def best_rate(positions, rotations, centers, frame_camera, frame_index, frame_rank, camera_model, camera_width,
              camera_height, camera_params, camera_max_angle, row_lo, row_hi, canonical_pixel_chart: bool = True):
    """The extension's best_rate (bindings.cpp:34-101): (best float64 [N],
    owner int32 [N], observed uint8 [N], direction float64 [N,3])."""
    if not canonical_pixel_chart:
        raise RuntimeError("physical Mip requires the COLMAP corner-coordinate pixel chart")
    device = positions.device
    _check(positions, "positions", device, torch.float64, 2)
    if positions.shape[1] != 3 or positions.shape[0] == 0:
        raise RuntimeError("positions must be contiguous CUDA float64 [N,3]")
    _check(rotations, "rotations", device, torch.float64, 3)
    _check(centers, "centers", device, torch.float64, 2)
    f = rotations.shape[0]
    if f == 0 or tuple(rotations.shape[1:]) != (3, 3) or tuple(centers.shape) != (f, 3):
        raise RuntimeError("rotations must be float64 [F,3,3] and centers [F,3]")
    for t, n, dt in ((frame_camera, "frame_camera", torch.int32), (frame_index, "frame_index", torch.int32),
                     (frame_rank, "frame_rank", torch.int64)):
        _check(t, n, device, dt, 1)
        if t.numel() != f:
            raise RuntimeError("frame arrays differ")
    _check(camera_params, "camera_params", device, torch.float64, 2)
    c = camera_params.shape[0]
    if camera_params.shape[1] != PACKED_PARAMETER_COUNT:
        raise RuntimeError("camera_params must be float64 [C,12]")
    for t, n, dt in ((camera_model, "camera_model", torch.int32), (camera_width, "camera_width", torch.int32),
                     (camera_height, "camera_height", torch.int32),
                     (camera_max_angle, "camera_max_angle", torch.float64)):
        _check(t, n, device, dt, 1)
        if t.numel() != c:
            raise RuntimeError("camera arrays differ")
    _check(row_lo, "row_lo", device, torch.int32, 2)
    _check(row_hi, "row_hi", device, torch.int32, 2)
    if row_lo.shape != row_hi.shape or row_lo.shape[0] != c or row_lo.shape[1] == 0:
        raise RuntimeError("row runs must be matching int32 [C,Hmax]")
    if int(camera_height.max().item()) > row_lo.shape[1]:
        raise RuntimeError("row runs must cover every camera row")
    fc = frame_camera
    if bool(((fc < 0) | (fc >= c)).any().item()):
        raise RuntimeError("frame_camera holds a slot outside the camera table")
    n = positions.shape[0]
    best = torch.zeros(n, dtype=torch.float64, device=device)
    owner = torch.full((n,), -1, dtype=torch.int32, device=device)
    observed = torch.zeros(n, dtype=torch.uint8, device=device)
    direction = torch.zeros((n, 3), dtype=torch.float64, device=device)
    lib = _native.load()
    _native.check(lib.gf_mip_best_rate(
        positions.data_ptr(), n, rotations.data_ptr(), centers.data_ptr(), frame_camera.data_ptr(),
        frame_index.data_ptr(), frame_rank.data_ptr(), f, camera_model.data_ptr(), camera_width.data_ptr(),
        camera_height.data_ptr(), camera_params.data_ptr(), camera_max_angle.data_ptr(), c, row_lo.data_ptr(),
        row_hi.data_ptr(), row_lo.shape[1], best.data_ptr(), owner.data_ptr(), observed.data_ptr(),
        direction.data_ptr(), torch.cuda.current_stream(device).cuda_stream), "best_rate")
    return best, owner, observed, direction


class _Extension:
    """What load_extension() returns: the object with best_rate."""

    best_rate = staticmethod(best_rate)


def load_extension(verbose: bool = False):
    """The GPU search (the library is prebuilt; there is no JIT step)."""
    _native.load()
    return _Extension


@torch.no_grad()
def compute_filter(positions: torch.Tensor, table: CameraTable, variance: float):
    """(filter_3D [N,1], filter_dir [N,3]) in the dtype of ``positions``
    (physical_mip.py:226-245)."""
    points64 = positions.detach().to(dtype=torch.float64).contiguous()
    best, _owner, observed_u8, direction64 = load_extension().best_rate(points64, *table.arguments(), True)
    observed = observed_u8.to(torch.bool)
    if not bool(observed.any()):
        raise RuntimeError("no Gaussian is observed by a training camera")
    scalar64 = torch.empty_like(best)
    scalar64[observed] = math.sqrt(variance) / best[observed]
    scalar64[~observed] = torch.max(scalar64[observed])
    return scalar64.to(positions.dtype)[:, None].contiguous(), direction64.to(positions.dtype).contiguous()


def scale_with_3d_filter(scale: torch.Tensor, filter_3d: torch.Tensor) -> torch.Tensor:
    """sqrt(s^2 + f^2) (threedgrut/model/model.py:80-93)."""
    return torch.sqrt(scale * scale + filter_3d * filter_3d)
