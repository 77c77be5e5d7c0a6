"""Marching tetrahedra of the mesh extraction on the GPU (reference
gofish/mesh/marching_tetrahedra.py:141-162, GOF's variant of Kaolin's
marching tetrahedra: each crossing edge's endpoints are returned instead of an
interpolated vertex, and the caller places the vertex by bisection).

``marching_tetrahedra`` keeps the reference's signature and outputs; the work
runs in the sm_100a kernels of gf_mesh_mt_run / gf_mesh_mt_outputs (CUDA
tensors only: there is no CPU path).
"""

from __future__ import annotations

import ctypes

import torch

from .. import _native

__all__ = ["marching_tetrahedra"]

# tetrahedra per chunk of the reference, which fixes the order of the faces of larger grids
CHUNK_TETS = 32 * 1024 * 1024


def _one_grid(vertices: torch.Tensor, tets: torch.Tensor, sdf: torch.Tensor, scales: torch.Tensor,
              chunk_tets: int):
    device = vertices.device
    if device.type != "cuda":
        raise RuntimeError("marching_tetrahedra runs on CUDA tensors only")
    v = vertices.detach().to(torch.float32).contiguous()
    t = tets.detach().to(device=device, dtype=torch.int64).contiguous()
    f = sdf.detach().to(device=device, dtype=torch.float32).reshape(-1).contiguous()
    s = scales.detach().to(device=device, dtype=torch.float32).reshape(-1).contiguous()
    if f.numel() != v.shape[0] or s.numel() != v.shape[0]:
        raise ValueError("sdf and scales need one value per vertex")
    lib = _native.load()
    handle = lib.gf_mesh_mt_create()
    try:
        with torch.cuda.device(device):
            stream = torch.cuda.current_stream(device).cuda_stream
            ne, nf = ctypes.c_uint64(0), ctypes.c_uint64(0)
            _native.check(lib.gf_mesh_mt_run(handle, v.data_ptr(), v.shape[0], t.data_ptr(), t.shape[0], f.data_ptr(),
                                             s.data_ptr(), int(chunk_tets), ctypes.byref(ne), ctypes.byref(nf),
                                             stream), "marching tetrahedra")
            e, n = int(ne.value), int(nf.value)
            endpoints = torch.empty((e, 2, 3), dtype=torch.float32, device=device)
            fields = torch.empty((e, 2, 1), dtype=torch.float32, device=device)
            vscales = torch.empty((e, 2, 1), dtype=torch.float32, device=device)
            faces = torch.empty((n, 3), dtype=torch.int64, device=device)
            edges = torch.empty((e, 2), dtype=torch.int64, device=device)
            _native.check(lib.gf_mesh_mt_outputs(handle, endpoints.data_ptr(), fields.data_ptr(), vscales.data_ptr(),
                                                 faces.data_ptr(), edges.data_ptr(), stream), "marching tetrahedra")
            torch.cuda.current_stream(device).synchronize()  # the inputs may be released after the return
    finally:
        lib.gf_mesh_mt_destroy(handle)
    return (endpoints, fields), vscales, faces, edges


def marching_tetrahedra(vertices, tets, sdf, scales, chunk_tets: int = CHUNK_TETS):
    """Crossing edges and triangles of the zero level set of ``sdf``.

    Args: ``vertices`` [B, V, 3], ``tets`` [T, 4] shared by the batch, ``sdf``
    [B, V] (inside: sdf > 0) and ``scales`` [B, V] or [B, V, 1].  Returns, as
    tuples over the batch: ``(endpoints [E, 2, 3], endpoint sdf [E, 2, 1])``,
    endpoint scales [E, 2, 1], faces [F, 3] indexing the crossing edges, and
    the edges' vertex ids [E, 2] -- the reference's outputs in its order."""
    outs = [_one_grid(vertices[b], tets, sdf[b], scales[b], chunk_tets) for b in range(vertices.shape[0])]
    verts, vscales, faces, edges = zip(*outs)
    return verts, vscales, faces, edges
