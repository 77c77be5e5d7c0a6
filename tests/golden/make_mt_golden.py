"""Generates tests/golden/mt_golden.npz from the reference's own marching
tetrahedra and mesh filters (gofish/mesh/marching_tetrahedra.py,
gofish/mesh/filters.py), run on the CPU in a container where the reference
checkout is present.

Inputs are seeded: sites of 400 synthetic Gaussians (centre + 8 box
corners), their Delaunay tetrahedra (scipy; the reference uses CGAL, which
only supplies the cells), a signed field that is positive inside a sphere
with exact zeros on some sites, per-site scales and owners.  Outputs: the
crossing edges, endpoints, endpoint fields and scales, and faces of
marching_tetrahedra; SOF's vertex filter and its application; GOF's cell
filter and the cell-filtered mesh.

    python tests/golden/make_mt_golden.py /path/to/reference
"""

from __future__ import annotations

import importlib.util
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent


def load_reference(root: Path):
    pkg = types.ModuleType("refmt")
    pkg.__path__ = [str(root / "gofish" / "mesh")]
    sys.modules["refmt"] = pkg
    mods = {}
    for name in ("marching_tetrahedra", "filters"):
        spec = importlib.util.spec_from_file_location(f"refmt.{name}", root / "gofish" / "mesh" / f"{name}.py")
        mod = importlib.util.module_from_spec(spec)
        sys.modules[f"refmt.{name}"] = mod
        spec.loader.exec_module(mod)
        mods[name] = mod
    return mods


def make_inputs(seed: int = 2026, gaussians: int = 400):
    """Sites, Delaunay cells, field, scales and owners of a synthetic scene."""
    from scipy.spatial import Delaunay

    rng = np.random.default_rng(seed)
    centre = rng.uniform(-1.0, 1.0, (gaussians, 3))
    half = rng.uniform(0.02, 0.12, (gaussians, 3))
    signs = np.array([[x, y, z] for x in (-1.0, 1.0) for y in (-1.0, 1.0) for z in (-1.0, 1.0)])
    corners = centre[:, None, :] + signs[None] * half[:, None, :]
    points = np.concatenate([centre[:, None, :], corners], axis=1).reshape(-1, 3).astype(np.float32)
    owner = np.repeat(np.arange(gaussians, dtype=np.int64), 9)
    scale = np.repeat(np.linalg.norm(half, axis=1), 9).astype(np.float32).reshape(-1, 1)
    cells = Delaunay(points.astype(np.float64)).simplices.astype(np.int64)
    field = (np.float32(0.6) - np.linalg.norm(points, axis=1)).astype(np.float32)
    field[rng.choice(points.shape[0], 40, replace=False)] = 0.0  # ties on the inside/outside cut (sdf > 0)
    return points, cells, field, scale, owner


def main():
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {sys.argv[0]} /path/to/reference")
    mods = load_reference(Path(sys.argv[1]))
    import torch

    mt, filters = mods["marching_tetrahedra"], mods["filters"]
    points, cells, field, scale, owner = make_inputs()
    pts_t = torch.from_numpy(points)
    cells_t = torch.from_numpy(cells)
    field_t = torch.from_numpy(field)
    scale_t = torch.from_numpy(scale)
    verts, vscales, faces, edges = mt.marching_tetrahedra(pts_t[None], cells_t, field_t[None], scale_t[None])
    endpoints, endpoint_fields = verts[0]
    out = dict(points=points, cells=cells, field=field, scale=scale, owner=owner,
               mt_endpoints=endpoints.numpy(), mt_endpoint_fields=endpoint_fields.numpy(),
               mt_scales=vscales[0].numpy(), mt_faces=faces[0].numpy(), mt_edges=edges[0].numpy())
    edges_np = edges[0].numpy().astype(np.int64)
    keep = filters.sof_vertex_filter(pts_t, scale_t, edges_np, torch.device("cpu"))
    rng = np.random.default_rng(7)
    raw_vertices = (endpoints.numpy().mean(axis=1) + rng.normal(0, 1e-3, (edges_np.shape[0], 3))).astype(np.float32)
    sof_v, sof_f = filters.apply_vertex_filter(raw_vertices, faces[0].numpy(), keep)
    kept_cells = filters.gof_cell_filter(cells_t, pts_t, scale_t, torch.from_numpy(owner))
    cell_v, cell_f = filters.cell_filtered_mesh(pts_t, kept_cells, field_t, scale_t, edges_np, raw_vertices, keep,
                                                torch.device("cpu"))
    out.update(sof_keep=keep, raw_vertices=raw_vertices, sof_vertices=sof_v, sof_faces=sof_f,
               gof_kept_cells=kept_cells.numpy(), cell_vertices=cell_v, cell_faces=cell_f)
    np.savez_compressed(HERE / "mt_golden.npz", **out)
    print(f"wrote {HERE / 'mt_golden.npz'}: {cells.shape[0]} cells, {edges_np.shape[0]} crossing edges, "
          f"{faces[0].shape[0]} faces, {int(keep.sum())} kept vertices, {kept_cells.shape[0]} kept cells")


if __name__ == "__main__":
    main()
