"""Mesh filters on the GPU: SOF's vertex filter and GOF's tetrahedron cell
filter (reference gofish/mesh/filters.py:15-96, same names, arguments and
results).  The per-edge and per-cell distance tests run in sm_100a kernels
(gf_mesh_sof_vertex_filter, gf_mesh_gof_cell_filter); the index bookkeeping
of the filtered meshes is host numpy, as in the reference.
"""

from __future__ import annotations

import numpy as np
import torch

from .. import _native
from .marching_tetrahedra import marching_tetrahedra


def _stream(device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def sof_vertex_filter(points: torch.Tensor, scale: torch.Tensor, edges: np.ndarray,
                      device: torch.device) -> np.ndarray:
    """Keep mask [E] (bool): a crossing vertex survives when its edge is no
    longer than the sum of the two endpoint sites' scales."""
    device = torch.device(device)
    if device.type != "cuda":
        raise RuntimeError("sof_vertex_filter runs on a CUDA device only")
    pts = points.detach().to(device=device, dtype=torch.float32).contiguous()
    sc = scale.detach().to(device=device, dtype=torch.float32).reshape(-1).contiguous()
    edge = torch.as_tensor(np.ascontiguousarray(edges, dtype=np.int64)).to(device).reshape(-1, 2).contiguous()
    keep = torch.empty(edge.shape[0], dtype=torch.uint8, device=device)
    with torch.cuda.device(device):
        _native.check(_native.load().gf_mesh_sof_vertex_filter(pts.data_ptr(), sc.data_ptr(), edge.data_ptr(),
                                                               edge.shape[0], keep.data_ptr(), _stream(device)),
                      "SOF vertex filter")
    return keep.cpu().numpy().astype(bool)


def apply_vertex_filter(vertices: np.ndarray, faces: np.ndarray, keep_vertex: np.ndarray):
    """(kept vertices float32, faces int32 over them): the faces whose three
    vertices all survive, renumbered."""
    keep_vertex = np.asarray(keep_vertex, dtype=bool)
    faces = np.asarray(faces)
    new_index = np.cumsum(keep_vertex, dtype=np.int64) - 1
    face_kept = keep_vertex[faces].all(axis=1)
    return (np.ascontiguousarray(np.asarray(vertices)[keep_vertex], dtype="<f4"),
            np.ascontiguousarray(new_index[faces[face_kept]], dtype="<i4"))


def gof_cell_filter(cells: torch.Tensor, points: torch.Tensor, scale: torch.Tensor,
                    owner: torch.Tensor, device: torch.device | None = None) -> torch.Tensor:
    """The cells [K, 4] without an edge joining two different owners farther
    apart than the sum of their scales (on ``device``, CUDA; the kept cells
    come back on the cells' device)."""
    device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    c = cells.detach().to(device=device, dtype=torch.int64).contiguous()
    pts = points.detach().to(device=device, dtype=torch.float32).contiguous()
    sc = scale.detach().to(device=device, dtype=torch.float32).reshape(-1).contiguous()
    own = owner.detach().to(device=device, dtype=torch.int64).contiguous()
    keep = torch.empty(c.shape[0], dtype=torch.uint8, device=device)
    with torch.cuda.device(device):
        _native.check(_native.load().gf_mesh_gof_cell_filter(c.data_ptr(), c.shape[0], pts.data_ptr(), sc.data_ptr(),
                                                             own.data_ptr(), keep.data_ptr(), _stream(device)),
                      "GOF cell filter")
    return c[keep.bool()].to(cells.device)


def cell_filtered_mesh(points: torch.Tensor, kept_cells: torch.Tensor, values: torch.Tensor,
                       scale: torch.Tensor, raw_edges: np.ndarray, raw_vertices: np.ndarray,
                       keep_vertex: np.ndarray, device: torch.device):
    """Marching tetrahedra over the kept cells, reusing each crossing edge's
    refined vertex and vertex-filter decision from the full extraction (every
    crossing edge of a cell subset is one of the full set, so nothing is
    evaluated again).  Returns (vertices float32, faces int32)."""
    device = torch.device(device)
    n = int(points.shape[0])
    pscale = scale.float().reshape(-1)
    _, _, faces_t, edges_t = marching_tetrahedra(points[None].to(device), kept_cells.to(device),
                                                 values[None].to(device), pscale[None, :, None].to(device))
    edges = edges_t[0].cpu().numpy().astype(np.int64)
    faces = faces_t[0].cpu().numpy().astype(np.int64)
    # each subset edge's row in the full set: join on the (a * n + b) key
    full_keys = np.asarray(raw_edges, dtype=np.int64)[:, 0] * n + np.asarray(raw_edges, dtype=np.int64)[:, 1]
    by_key = np.argsort(full_keys, kind="stable")
    keys = edges[:, 0] * n + edges[:, 1]
    at = np.searchsorted(full_keys[by_key], keys)
    if not (np.all(at < full_keys.size) and np.array_equal(full_keys[by_key][np.minimum(at, full_keys.size - 1)],
                                                            keys)):
        raise RuntimeError("a cell-filtered crossing edge is not a crossing edge of the full set")
    rows = by_key[at]
    return apply_vertex_filter(np.asarray(raw_vertices)[rows], faces, np.asarray(keep_vertex, dtype=bool)[rows])
