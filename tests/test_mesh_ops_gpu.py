"""Marching tetrahedra and the mesh filters on the GPU against golden vectors
of the reference's own functions (gofish/mesh/marching_tetrahedra.py,
filters.py; tests/golden/make_mt_golden.py) and against the oracle's
restatement (oracle/mesh_ops.py) on a larger grid and with chunked face
order: edges, endpoints, endpoint fields and scales, faces, keep masks and
filtered meshes, exactly."""

from pathlib import Path

import numpy as np
import pytest
import torch

from gofish_b200.mesh import filters
from gofish_b200.mesh.marching_tetrahedra import marching_tetrahedra
from oracle import mesh_ops

pytestmark = pytest.mark.gpu
G = np.load(Path(__file__).resolve().parent / "golden" / "mt_golden.npz")


def _run(points, cells, field, scale, device, chunk_tets=None):
    kw = {} if chunk_tets is None else {"chunk_tets": chunk_tets}
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(device)  # noqa: E731
    (verts,), (vs,), (faces,), (edges,) = marching_tetrahedra(t(points)[None], t(cells), t(field)[None],
                                                              t(scale).reshape(1, -1, 1), **kw)
    return (verts[0].cpu().numpy(), verts[1].cpu().numpy(), vs.cpu().numpy(), faces.cpu().numpy(),
            edges.cpu().numpy())


def _same(got, want):
    ends, fields, scales, faces, edges = got
    np.testing.assert_array_equal(edges, want[4])
    np.testing.assert_array_equal(faces, want[3])
    np.testing.assert_array_equal(ends.view(np.uint32), want[0].view(np.uint32))
    np.testing.assert_array_equal(fields.view(np.uint32), want[1].view(np.uint32))
    np.testing.assert_array_equal(scales.view(np.uint32), want[2].view(np.uint32))


def test_marching_tetrahedra_matches_reference(cuda_device):
    got = _run(G["points"], G["cells"], G["field"], G["scale"], cuda_device)
    _same(got, (G["mt_endpoints"], G["mt_endpoint_fields"], G["mt_scales"], G["mt_faces"], G["mt_edges"]))


def test_chunked_face_order_matches_oracle(cuda_device):
    got = _run(G["points"], G["cells"], G["field"], G["scale"], cuda_device, chunk_tets=5000)
    _same(got, mesh_ops.marching_tetrahedra(G["points"], G["cells"], G["field"], G["scale"], chunk_tets=5000))


def test_large_grid_matches_oracle(cuda_device):
    from scipy.spatial import Delaunay

    rng = np.random.default_rng(11)
    points = rng.uniform(-1, 1, (150_000, 3)).astype(np.float32)
    cells = Delaunay(points.astype(np.float64)).simplices.astype(np.int64)
    field = (np.float32(0.5) - np.abs(points).max(axis=1)).astype(np.float32)
    field[rng.choice(points.shape[0], 500, replace=False)] = 0.0
    scale = rng.uniform(0.01, 0.05, points.shape[0]).astype(np.float32)
    assert cells.shape[0] > 800_000
    got = _run(points, cells, field, scale, cuda_device)
    _same(got, mesh_ops.marching_tetrahedra(points, cells, field, scale))


def test_empty_level_set(cuda_device):
    field = np.ones(G["points"].shape[0], np.float32)
    ends, fields, scales, faces, edges = _run(G["points"], G["cells"], field, G["scale"], cuda_device)
    assert edges.shape == (0, 2) and faces.shape == (0, 3) and ends.shape == (0, 2, 3)


def test_filters_match_reference(cuda_device):
    pts, scale = torch.from_numpy(G["points"]), torch.from_numpy(G["scale"])
    keep = filters.sof_vertex_filter(pts, scale, G["mt_edges"], cuda_device)
    np.testing.assert_array_equal(keep, G["sof_keep"])
    v, f = filters.apply_vertex_filter(G["raw_vertices"], G["mt_faces"], keep)
    np.testing.assert_array_equal(v.view(np.uint32), G["sof_vertices"].view(np.uint32))
    np.testing.assert_array_equal(f, G["sof_faces"])
    kept = filters.gof_cell_filter(torch.from_numpy(G["cells"]), pts, scale, torch.from_numpy(G["owner"]),
                                   cuda_device)
    np.testing.assert_array_equal(kept.numpy(), G["gof_kept_cells"])
    cv, cf = filters.cell_filtered_mesh(pts, kept, torch.from_numpy(G["field"]), scale, G["mt_edges"],
                                        G["raw_vertices"], keep, cuda_device)
    np.testing.assert_array_equal(cv.view(np.uint32), G["cell_vertices"].view(np.uint32))
    np.testing.assert_array_equal(cf, G["cell_faces"])
