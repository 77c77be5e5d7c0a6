"""The sm_100a physical-mip search (gf_mip_best_rate) against the oracle:
best rate and direction as float64 bits, owner and observed exactly, over
all seven camera models, row-run supports with gaps, fisheye angular caps,
points at camera centres and on optical axes, and exact rate ties."""

import numpy as np
import pytest
import torch

import oracle
from gofish_b200 import physical_mip

from tests.mip_harness import mip_points, mip_records

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("seed", [3, 9])
def test_best_rate_matches_oracle(cuda_device, seed):
    cameras, frames = mip_records(seed, frames_per_camera=8 if seed == 9 else 6)
    table = physical_mip.pack_camera_table(cameras, frames, cuda_device)
    pts = mip_points(seed + 1, 20000, frames)
    want = oracle.mip_best_rate(pts, *[t.cpu().numpy() for t in table.arguments()])
    got = physical_mip.load_extension().best_rate(torch.from_numpy(pts).to(cuda_device), *table.arguments(), True)
    best, owner, observed, direction = (t.cpu().numpy() for t in got)
    assert want[2].mean() > 0.2
    assert np.array_equal(observed, want[2])
    assert np.array_equal(owner, want[1])
    assert np.array_equal(best.view(np.uint64), want[0].view(np.uint64))
    assert np.array_equal(direction.view(np.uint64), want[3].view(np.uint64))


def test_many_frames_span_chunks(cuda_device):
    # more frames than one shared-memory chunk (128)
    cameras, frames = mip_records(5, frames_per_camera=40)
    table = physical_mip.pack_camera_table(cameras, frames, cuda_device)
    pts = mip_points(6, 5000, frames)
    want = oracle.mip_best_rate(pts, *[t.cpu().numpy() for t in table.arguments()])
    got = physical_mip.best_rate(torch.from_numpy(pts).to(cuda_device), *table.arguments())
    assert np.array_equal(got[1].cpu().numpy(), want[1])
    assert np.array_equal(got[0].cpu().numpy().view(np.uint64), want[0].view(np.uint64))


def test_compute_filter(cuda_device):
    cameras, frames = mip_records(3)
    table = physical_mip.pack_camera_table(cameras, frames, cuda_device)
    pts = torch.from_numpy(mip_points(4, 3000, frames)).float().to(cuda_device)
    f3d, fdir = physical_mip.compute_filter(pts, table, 0.2)
    best, _, observed, _ = oracle.mip_best_rate(pts.double().cpu().numpy(),
                                                *[t.cpu().numpy() for t in table.arguments()])
    ob = observed != 0
    want = np.empty_like(best)
    want[ob] = np.sqrt(0.2) / best[ob]
    want[~ob] = want[ob].max()
    assert f3d.shape == (3000, 1) and fdir.shape == (3000, 3) and f3d.dtype == torch.float32
    assert np.array_equal(f3d[:, 0].cpu().numpy(), want.astype(np.float32))


def test_rejects_bad_tables(cuda_device):
    cameras, frames = mip_records(3)
    table = physical_mip.pack_camera_table(cameras, frames, cuda_device)
    pts = torch.zeros((4, 3), dtype=torch.float64, device=cuda_device)
    args = list(table.arguments())
    bad = args[2].clone()
    bad[0] = 99
    with pytest.raises(RuntimeError, match="slot"):
        physical_mip.best_rate(pts, *args[:2], bad, *args[3:])
    with pytest.raises(RuntimeError, match="dtype"):
        physical_mip.best_rate(pts.float(), *args)
