"""The oracle's marching tetrahedra and mesh filters (oracle/mesh_ops.py)
against golden vectors of the reference's own functions
(gofish/mesh/marching_tetrahedra.py, filters.py;
tests/golden/make_mt_golden.py): crossing edges, endpoints, endpoint fields
and scales, faces, SOF's vertex filter and GOF's cell filter, exactly."""

from pathlib import Path

import numpy as np

from oracle import mesh_ops

G = np.load(Path(__file__).resolve().parent / "golden" / "mt_golden.npz")


def test_marching_tetrahedra_matches_reference():
    ends, fields, scales, faces, edges = mesh_ops.marching_tetrahedra(G["points"], G["cells"], G["field"], G["scale"])
    np.testing.assert_array_equal(edges, G["mt_edges"])
    np.testing.assert_array_equal(faces, G["mt_faces"])
    np.testing.assert_array_equal(ends.view(np.uint32), G["mt_endpoints"].view(np.uint32))
    np.testing.assert_array_equal(fields.view(np.uint32), G["mt_endpoint_fields"].view(np.uint32))
    np.testing.assert_array_equal(scales.view(np.uint32), G["mt_scales"].view(np.uint32))
    assert edges.shape[0] > 1000 and faces.shape[0] > 2000


def test_chunked_face_order_is_per_chunk():
    """With chunks, the same edges come out and each chunk's faces keep the
    one-triangle-then-two-triangle order (the reference's chunked merge)."""
    full = mesh_ops.marching_tetrahedra(G["points"], G["cells"], G["field"], G["scale"])
    chunked = mesh_ops.marching_tetrahedra(G["points"], G["cells"], G["field"], G["scale"], chunk_tets=5000)
    np.testing.assert_array_equal(chunked[4], full[4])
    assert chunked[3].shape == full[3].shape
    assert not np.array_equal(chunked[3], full[3])
    np.testing.assert_array_equal(np.sort(chunked[3], axis=0), np.sort(full[3], axis=0))


def test_filters_match_reference():
    keep = mesh_ops.sof_vertex_filter(G["points"], G["scale"], G["mt_edges"])
    np.testing.assert_array_equal(keep, G["sof_keep"])
    assert 0 < keep.sum() < keep.size
    kept = mesh_ops.gof_cell_filter(G["cells"], G["points"], G["scale"], G["owner"])
    np.testing.assert_array_equal(kept, G["gof_kept_cells"])
