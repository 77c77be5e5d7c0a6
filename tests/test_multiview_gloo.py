"""Host-side multi-view data parallelism on two CPU ranks (gloo): view
sharding and the gradient all-reduce give every rank the gradient of the
whole batch, equal to the serial sum over all views."""

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gofish_b200.multiview import multiview_step, shard_views


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _fake_view_grads(v: int):
    g = torch.Generator().manual_seed(1000 + v)
    return torch.randn(37, 32, generator=g), torch.randn(37, 48, generator=g)


def _worker(rank, world, port, num_views, out):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        accum = [torch.empty(37, 32), torch.empty(37, 48)]
        multiview_step(_fake_view_grads, shard_views(num_views, rank, world), accum)
        out[rank] = [a.clone() for a in accum]
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("num_views", [5, 8])
def test_two_rank_gradient_allreduce_matches_serial_sum(num_views):
    world = 2
    port = _free_port()
    manager = mp.get_context("spawn").Manager()
    out = manager.dict()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, num_views, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    serial = [torch.zeros(37, 32), torch.zeros(37, 48)]
    for v in range(num_views):
        for s, g in zip(serial, _fake_view_grads(v)):
            s += g
    for r in range(world):
        for got, want in zip(out[r], serial):
            torch.testing.assert_close(got, want, rtol=1e-6, atol=1e-5)


def test_shard_views_partitions_the_batch():
    for world in (1, 2, 3, 8):
        views = sorted(v for r in range(world) for v in shard_views(64, r, world))
        assert views == list(range(64))
        sizes = [len(shard_views(64, r, world)) for r in range(world)]
        assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard_views(8, 2, 2)


def _bucket_worker(rank, world, port, out, early=False):
    from gofish_b200.multiview import GradientBucket

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        g = torch.Generator().manual_seed(7)
        pos = torch.randn(11, 3, generator=g).requires_grad_(True)
        sh = torch.randn(11, 48, generator=g).requires_grad_(True)
        bucket = GradientBucket([pos, sh], early=[sh] if early else ())
        if early:
            # the early parameter sits at the end of the flat buffer
            assert bucket.views[1].data_ptr() == bucket.flat[bucket.head_numel:].data_ptr()
        for step in range(2):
            bucket.attach()
            for v in range(2):  # two views per rank, accumulated in the bucket
                w = float(1 + rank * 2 + v + step)
                if early and v == 1:
                    bucket.arm()  # the tail's all-reduce starts inside this backward
                (w * (pos ** 2).sum() + w * sh.sum()).backward()
                if early:
                    assert (bucket._work is not None) == (v == 1)
            assert pos.grad.data_ptr() == bucket.views[0].data_ptr()
            bucket.allreduce()
        out[rank] = (pos.grad.clone(), sh.grad.clone(), pos.detach().clone())
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("early", [False, True])
def test_gradient_bucket_single_allreduce_matches_sum(early):
    """One all-reduce of the flat bucket, or (early) the SH tail reduced
    asynchronously from inside the last backward and the head after it."""
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    out = manager.dict()
    procs = [ctx.Process(target=_bucket_worker, args=(r, world, port, out, early)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    pos = out[0][2]
    # last step: weights (1 + 2r + v + 1) over ranks r and views v: 2+3+4+5 = 14
    for r in range(world):
        torch.testing.assert_close(out[r][0], 14.0 * 2.0 * pos)
        torch.testing.assert_close(out[r][1], torch.full((11, 48), 14.0))


def test_gradient_bucket_early_is_a_no_op_on_one_process():
    from gofish_b200.multiview import GradientBucket

    pos = torch.ones(4, 3, requires_grad=True)
    sh = torch.ones(4, 48, requires_grad=True)
    bucket = GradientBucket([pos, sh], early=[sh])
    bucket.attach()
    bucket.arm()
    (2.0 * pos.sum() + 3.0 * sh.sum()).backward()
    bucket.allreduce()
    assert torch.equal(pos.grad, torch.full((4, 3), 2.0)) and torch.equal(sh.grad, torch.full((4, 48), 3.0))
    with pytest.raises(ValueError):
        GradientBucket([pos], early=[sh])


def _second_producer_worker(rank, world, port, out):
    from gofish_b200.multiview import GradientBucket

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        pos = torch.ones(5, 3, requires_grad=True)
        sh = torch.ones(5, 48, requires_grad=True)
        bucket = GradientBucket([pos, sh], early=[sh])
        bucket.attach()
        bucket.arm()
        (pos.sum() + sh.sum()).backward()  # starts the tail's all-reduce
        raised = False
        try:
            (2.0 * sh.sum()).backward()  # a second producer of the early gradient
        except RuntimeError as exc:
            raised = "one gradient producer" in str(exc)
        bucket._work.wait()
        out[rank] = raised
    finally:
        dist.destroy_process_group()


def test_gradient_bucket_rejects_a_second_early_producer():
    """A gradient reaching an early parameter after its all-reduce started
    would be left out of the sum: the bucket raises instead."""
    world = 2
    port = _free_port()
    ctx = mp.get_context("spawn")
    out = ctx.Manager().dict()
    procs = [ctx.Process(target=_second_producer_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert out[0] and out[1]
