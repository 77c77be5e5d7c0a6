"""Numpy restatement of the mesh extraction's marching tetrahedra and mesh
filters -- TEST INFRASTRUCTURE ONLY (the checker of gofish_b200's
gf_marching_tets / gf_mesh_* kernels).

Follows gofish/mesh/marching_tetrahedra.py:47-140 (GOF's variant of Kaolin's
marching tetrahedra, which returns each crossing edge's endpoints instead of
an interpolated vertex) and gofish/mesh/filters.py:15-58 (SOF's vertex filter,
GOF's cell filter).  Semantics restated here:

* a vertex is inside when sdf > 0; a tetrahedron is active when 1 to 3 of its
  vertices are inside; its code is sum(inside_k << k);
* the edges of active tetrahedra, (min, max) oriented, deduplicated and
  sorted lexicographically; the crossing edges are those with exactly one
  inside endpoint, numbered in that order;
* faces: one or two triangles per active tetrahedron from the fixed
  16-case table over its six edges (0-1, 0-2, 0-3, 1-2, 1-3, 2-3); all
  one-triangle tetrahedra first (in tetrahedron order), then the
  two-triangle ones (two consecutive faces each), per chunk of
  ceil(T / n) tetrahedra with n = T // chunk + 1 chunks when T exceeds the
  chunk size (the reference processes large grids chunk by chunk and
  concatenates their faces).

Pinned by golden vectors of the reference's own functions
(tests/golden/make_mt_golden.py, tests/test_mesh_ops_host.py).
"""

from __future__ import annotations

import numpy as np

# Triangles of the 16 inside/outside cases as local edge indices (-1: none);
# the case table of marching tetrahedra, which fixes face order and winding.
TRIANGLE_TABLE = np.array([
    [-1, -1, -1, -1, -1, -1], [1, 0, 2, -1, -1, -1], [4, 0, 3, -1, -1, -1], [1, 4, 2, 1, 3, 4],
    [3, 1, 5, -1, -1, -1], [2, 3, 0, 2, 5, 3], [1, 4, 0, 1, 5, 4], [4, 2, 5, -1, -1, -1],
    [4, 5, 2, -1, -1, -1], [4, 1, 0, 4, 5, 1], [3, 2, 0, 3, 5, 2], [1, 3, 5, -1, -1, -1],
    [4, 1, 2, 4, 3, 1], [3, 0, 4, -1, -1, -1], [2, 0, 1, -1, -1, -1], [-1, -1, -1, -1, -1, -1]], dtype=np.int64)
TRIANGLE_COUNT = np.array([0, 1, 1, 2, 1, 2, 2, 1, 1, 2, 2, 1, 2, 1, 1, 0], dtype=np.int64)
TET_EDGES = np.array([[0, 1], [0, 2], [0, 3], [1, 2], [1, 3], [2, 3]], dtype=np.int64)
REFERENCE_CHUNK_TETS = 32 * 1024 * 1024


def marching_tetrahedra(vertices, tets, sdf, scales, chunk_tets: int = REFERENCE_CHUNK_TETS):
    """(endpoints [E,2,3], endpoint sdf [E,2,1], endpoint scales [E,2,1],
    faces [F,3] int64, edges [E,2] int64) of one grid."""
    vertices = np.asarray(vertices, dtype=np.float32).reshape(-1, 3)
    tets = np.asarray(tets, dtype=np.int64).reshape(-1, 4)
    sdf = np.asarray(sdf, dtype=np.float32).reshape(-1)
    scales = np.asarray(scales, dtype=np.float32).reshape(-1)
    inside = sdf > 0
    occ = inside[tets]                                   # [T,4]
    count = occ.sum(axis=1)
    active = (count > 0) & (count < 4)
    code = (occ * (1 << np.arange(4))).sum(axis=1)
    act = np.flatnonzero(active)
    ends = tets[act][:, TET_EDGES]                       # [A,6,2]
    lo, hi = np.minimum(ends[..., 0], ends[..., 1]), np.maximum(ends[..., 0], ends[..., 1])
    pairs = np.stack([lo.reshape(-1), hi.reshape(-1)], axis=1)
    unique, inverse = np.unique(pairs, axis=0, return_inverse=True)
    inverse = inverse.reshape(-1)
    crossing = inside[unique[:, 0]] != inside[unique[:, 1]]
    number = np.full(unique.shape[0], -1, dtype=np.int64)
    number[crossing] = np.arange(int(crossing.sum()))
    slot = number[inverse].reshape(-1, 6)                # crossing-edge number of each active tet's edges
    edges = unique[crossing]
    # faces, chunk by chunk, one-triangle tets before two-triangle tets
    t = tets.shape[0]
    size = t if t <= chunk_tets else -(-t // (t // chunk_tets + 1))
    ntri = TRIANGLE_COUNT[code[act]]
    chunk = act // max(size, 1)
    faces = []
    for c in np.unique(chunk):
        for k in (1, 2):
            rows = np.flatnonzero((chunk == c) & (ntri == k))
            if rows.size == 0:
                continue
            local = TRIANGLE_TABLE[code[act[rows]]][:, :3 * k]
            faces.append(np.take_along_axis(slot[rows], local, axis=1).reshape(-1, 3))
    faces = np.concatenate(faces, axis=0) if faces else np.zeros((0, 3), np.int64)
    endpoints = vertices[edges.reshape(-1)].reshape(-1, 2, 3)
    fields = sdf[edges.reshape(-1)].reshape(-1, 2, 1)
    escales = scales[edges.reshape(-1)].reshape(-1, 2, 1)
    return endpoints, fields, escales, faces.astype(np.int64), edges.astype(np.int64)


def sof_vertex_filter(points, scale, edges) -> np.ndarray:
    """Keep a crossing vertex when |p_a - p_b| <= scale_a + scale_b (float32
    norm of the float32 difference)."""
    p = np.asarray(points, dtype=np.float32)
    s = np.asarray(scale, dtype=np.float32).reshape(-1)
    e = np.asarray(edges, dtype=np.int64)
    d = p[e[:, 0]] - p[e[:, 1]]
    dist = np.sqrt((d.astype(np.float32) ** 2).sum(axis=1, dtype=np.float32))
    return dist <= s[e[:, 0]] + s[e[:, 1]]


def gof_cell_filter(cells, points, scale, owner) -> np.ndarray:
    """Cells without an edge joining two different owners farther apart
    than the sum of their scales."""
    c = np.asarray(cells, dtype=np.int64)
    p = np.asarray(points, dtype=np.float32)
    s = np.asarray(scale, dtype=np.float32).reshape(-1)
    o = np.asarray(owner, dtype=np.int64)
    keep = np.ones(c.shape[0], dtype=bool)
    for a, b in TET_EDGES:
        d = p[c[:, a]] - p[c[:, b]]
        dist = np.sqrt((d ** 2).sum(axis=1, dtype=np.float32))
        keep &= ~((o[c[:, a]] != o[c[:, b]]) & (dist > s[c[:, a]] + s[c[:, b]]))
    return c[keep]
