"""Tetrahedralization sites on the GPU (gf_mesh_sites) against the golden
vectors made by the reference's own gofish/mesh/sites.py
(tests/golden/make_mesh_golden.py) and against the host restatement on a
large scene, bit for bit: points, scales and owners."""

from pathlib import Path

import numpy as np
import pytest

from gofish_b200.mesh import sites
from gofish_b200.mesh.shape import EffectiveShape, effective_shape

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).resolve().parent / "golden" / "mesh_golden.npz"


def _check(got, want):
    np.testing.assert_array_equal(got.points.cpu().numpy().view(np.uint32), want.points.view(np.uint32))
    np.testing.assert_array_equal(got.scale.cpu().numpy().view(np.uint32), want.scale.view(np.uint32))
    np.testing.assert_array_equal(got.owner.cpu().numpy(), want.owner)


def test_sites_match_reference_golden(cuda_device):
    g = np.load(GOLDEN)
    shape = EffectiveShape(positions=g["positions"], density=g["density"], factor=g["factor"],
                           inverse_factor=g["inverse_factor"], sigma_max=g["sigma_max"], retained=g["retained"])
    got = sites.generate_sites_cuda(shape, cuda_device)
    want = sites.Sites(points=g["site_points"], scale=g["site_scale"], owner=g["site_owner"])
    _check(got, want)


def test_sites_match_host_on_a_large_scene(cuda_device):
    from gofish_b200.scene import random_scene

    scene = random_scene(300_000, 0, 1237)
    shape = effective_shape(scene.positions, scene.scales * np.float32(3.0), scene.rotations, scene.density)
    want = sites.generate_sites(shape)
    assert want.count > 8 * 250_000  # most Gaussians are kept; some are below 1/255
    _check(sites.generate_sites_cuda(shape, cuda_device), want)


def test_no_kept_gaussian_raises(cuda_device):
    g = np.load(GOLDEN)
    n = g["positions"].shape[0]
    dead = np.full((n, 1), 0.5 / 255.0, np.float32)
    shape = EffectiveShape(positions=g["positions"], density=dead, factor=g["factor"],
                           inverse_factor=g["inverse_factor"], sigma_max=g["sigma_max"], retained=np.zeros(n, bool))
    with pytest.raises(ValueError, match="no Gaussian"):
        sites.generate_sites_cuda(shape, cuda_device)
