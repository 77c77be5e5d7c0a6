"""The sharded mesh opacity query on two CPU ranks (gloo): points and edges
are cut into contiguous slices, each rank evaluates its slice, and the final
all-gather gives every rank the single-rank result -- here the oracle's
opacity field over the unsharded points, bit for bit, and exact copies of
ragged arrays of several dtypes."""

import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from gofish_b200.mesh.sharded import gather_shards, shard_bounds


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _field_case():
    """A small scene, two fisheye views on a ring and its sites (host arrays)."""
    import math

    import oracle
    from gofish_b200.camera import fisheye_camera
    from gofish_b200.mesh.shape import effective_shape
    from gofish_b200.mesh.sites import generate_sites
    from gofish_b200.scene import look_outward_pose, random_scene

    scene = random_scene(600, 0, 91, r_min=1.0, r_max=3.0)
    shape = effective_shape(scene.positions, scene.scales * np.float32(3.0), scene.rotations, scene.density)
    points = generate_sites(shape).points[:1001]  # odd count: ragged shards
    cam = fisheye_camera(48, 48, 200.0)
    ocam = oracle.camera(1, cam.width, cam.height, cam.principal, cam.focal, cam.coefficients, cam.max_angle)
    ray_o = np.zeros((48, 48, 3), np.float32)
    views = []
    for v in range(2):
        yaw = math.pi * v + 0.3
        pose = look_outward_pose(np.array([2.0 * math.cos(yaw), 2.0 * math.sin(yaw), 0.0]), yaw)
        views.append((ocam, pose, ray_o, None))
    return views, shape.packed_density(), points


def _worker(rank, world, port, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import oracle

        views, packed, points = _field_case()
        q = points.shape[0]
        lo, hi = shard_bounds(q, rank, world)
        opacity, observed, _ = oracle.evaluate_field(views, packed, points[lo:hi])
        got = (gather_shards(opacity, q), gather_shards(observed, q))
        rng = np.random.default_rng(5)
        edges = rng.standard_normal((77, 3)).astype(np.float32)
        ids = np.arange(13, dtype=np.int64)
        a, b = shard_bounds(77, rank, world)
        c, d = shard_bounds(13, rank, world)
        out[rank] = (got[0], got[1], gather_shards(edges[a:b], 77), gather_shards(ids[c:d], 13))
    finally:
        dist.destroy_process_group()


def test_shard_bounds_cover_the_range():
    for total in (0, 1, 7, 1001):
        for world in (1, 2, 3, 8):
            cuts = [shard_bounds(total, r, world) for r in range(world)]
            assert cuts[0][0] == 0 and cuts[-1][1] == total
            assert all(cuts[r][1] == cuts[r + 1][0] for r in range(world - 1))
            sizes = [b - a for a, b in cuts]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


def test_two_rank_field_gather_matches_single_rank():
    import oracle

    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
        assert p.exitcode == 0
    views, packed, points = _field_case()
    want_op, want_ob, _ = oracle.evaluate_field(views, packed, points)
    assert 0 < int(want_ob.sum()) < points.shape[0]
    edges = np.random.default_rng(5).standard_normal((77, 3)).astype(np.float32)
    for r in range(world):
        op, ob, e, ids = out[r]
        np.testing.assert_array_equal(op.view(np.uint32), want_op.view(np.uint32))
        np.testing.assert_array_equal(ob, want_ob)
        np.testing.assert_array_equal(e, edges)
        np.testing.assert_array_equal(ids, np.arange(13))
