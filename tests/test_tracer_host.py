"""Host logic of the training renderer's autograd boundary
(reference threedgut_tracer/tracer.py:142-353), with a recording stand-in
for the native renderer: the packed [N,32] row layout sent to ``trace``, the
saved tensors handed to ``trace_bwd``, and the split of the [N,32] row
gradient back into the per-slot gradients in the reference's order."""

from types import SimpleNamespace

import pytest
import torch

from gofish_b200.tracer import PACKED_SPLIT, Tracer


class FakeRaster:
    def __init__(self, n, h=4, w=5):
        self.n, self.h, self.w = n, h, w
        self.calls = []

    def trace(self, frame_id, sof, n_active, density, features, ray_ori, ray_dir, ray_time, sensor, t0, t1, p0, p1,
              token):
        self.calls.append(("trace", density.clone(), features.clone(), token, frame_id, n_active))
        h, w = self.h, self.w
        rgba = torch.full((h, w, 4), 0.25)
        hit = torch.full((h, w, 1), 2.0)
        count = torch.ones((h, w, 1))
        vis = torch.ones((self.n, 1))
        z = lambda c: torch.zeros((h, w, c))  # noqa: E731
        return rgba, hit, count, vis, z(3), z(1), z(10), z(1), z(1), z(1), z(1)

    def trace_bwd(self, frame_id, sof, n_active, density, features, ray_ori, ray_dir, ray_time, sensor, t0, t1, p0, p1,
                  rgba, grad_rgba, hit, grad_hit, *geometry_and_token):
        *geometry, token = geometry_and_token
        assert len(geometry) == 14
        self.calls.append(("trace_bwd", grad_rgba.clone(), None if grad_hit is None else grad_hit.clone(), token,
                           geometry))
        # row gradient = slot index + 100 * row, so the split is visible
        slots = torch.arange(32, dtype=torch.float32)[None, :]
        rows = torch.arange(self.n, dtype=torch.float32)[:, None]
        return slots + 100.0 * rows, torch.full_like(features, 7.0)


def _inputs(n):
    g = torch.Generator().manual_seed(3)

    def r(*shape):
        return torch.randn(*shape, generator=g).requires_grad_(True)

    return dict(pos=r(n, 3), rot=r(n, 4), scl=r(n, 3), dns=r(n, 1), idns=r(n, 1), fac=r(n, 3, 3), inv=r(n, 3, 3),
                sph=r(n, 48))


def _apply(raster, x, n):
    poses = SimpleNamespace(timestamps_us=[0, 1], T_world_sensors=[torch.zeros(7), torch.zeros(7)])
    rays = torch.zeros((1, raster.h, raster.w, 3))
    return Tracer._Autograd.apply(raster, "tok", 9, False, 3, rays, rays, x["pos"], x["rot"], x["scl"], x["dns"],
                                  x["idns"], x["fac"], x["inv"], x["sph"], None, poses, torch.empty((0, 1)))


def test_packed_row_layout():
    n = 6
    raster = FakeRaster(n)
    x = _inputs(n)
    _apply(raster, x, n)
    kind, packed, features, token, frame, n_active = raster.calls[0]
    assert kind == "trace" and token == "tok" and frame == 9 and n_active == 3
    assert packed.shape == (n, 32)
    assert torch.equal(packed[:, 0:3], x["pos"].detach())
    assert torch.equal(packed[:, 3:4], x["dns"].detach())
    assert torch.equal(packed[:, 4:8], x["rot"].detach())
    assert torch.equal(packed[:, 8:11], x["scl"].detach())
    assert torch.equal(packed[:, 11:12], x["idns"].detach())
    assert torch.equal(packed[:, 12:21], x["fac"].detach().reshape(n, 9))
    assert torch.equal(packed[:, 21:30], x["inv"].detach().reshape(n, 9))
    assert not bool(packed[:, 30:32].any())
    assert torch.equal(features, x["sph"].detach())


def test_gradient_split_and_order():
    n = 5
    raster = FakeRaster(n)
    x = _inputs(n)
    outs = _apply(raster, x, n)
    assert len(outs) == 11
    g = torch.randn(raster.h, raster.w, 4)
    (outs[0] * g).sum().backward()
    kind, grad_rgba, grad_hit, _token, _geometry = raster.calls[1]
    assert kind == "trace_bwd"
    assert torch.equal(grad_rgba, g)
    assert grad_hit is None
    rows = 100.0 * torch.arange(n, dtype=torch.float32)[:, None]
    offsets = [0]
    for width in PACKED_SPLIT:
        offsets.append(offsets[-1] + width)
    slot = {name: torch.arange(offsets[i], offsets[i + 1], dtype=torch.float32)[None, :] + rows
            for i, name in enumerate(["pos", "dns", "rot", "scl", "idns", "fac", "inv", "pad"])}
    assert torch.equal(x["pos"].grad, slot["pos"])
    assert torch.equal(x["dns"].grad, slot["dns"])
    assert torch.equal(x["rot"].grad, slot["rot"])
    assert torch.equal(x["scl"].grad, slot["scl"])
    assert torch.equal(x["idns"].grad, slot["idns"])
    assert torch.equal(x["fac"].grad, slot["fac"].reshape(n, 3, 3))
    assert torch.equal(x["inv"].grad, slot["inv"].reshape(n, 3, 3))
    assert torch.equal(x["sph"].grad, torch.full((n, 48), 7.0))


def test_hit_distance_only_loss_sends_zero_colour_gradient():
    n = 3
    raster = FakeRaster(n)
    x = _inputs(n)
    outs = _apply(raster, x, n)
    outs[1].sum().backward()
    _kind, grad_rgba, grad_hit, _, _geometry = raster.calls[1]
    assert not bool(grad_rgba.any())
    assert torch.equal(grad_hit, torch.ones_like(grad_hit))


def test_confidence_is_refused():
    n = 2
    raster = FakeRaster(n)
    x = _inputs(n)
    poses = SimpleNamespace(timestamps_us=[0, 1], T_world_sensors=[torch.zeros(7), torch.zeros(7)])
    rays = torch.zeros((1, raster.h, raster.w, 3))
    with pytest.raises(NotImplementedError):
        Tracer._Autograd.apply(raster, "tok", 0, False, 3, rays, rays, x["pos"], x["rot"], x["scl"], x["dns"],
                               x["idns"], x["fac"], x["inv"], x["sph"], None, poses, torch.ones((n, 1)))


def test_opacity_field_loss_needs_the_geometric_channels():
    with pytest.raises(ValueError, match="lambda_opa"):
        Tracer({"render": {"enable_normals": False}, "loss": {"lambda_opa": 0.004}})


def test_opacity_field_activation_follows_the_reference():
    """tracer.py:433-448: active for training frames from opa_warmup (default
    geom_warmup) until the distillation steps, with lambda_opa > 0."""
    conf = {"render": {"enable_normals": True}, "loss": {"lambda_opa": 0.004, "geom_warmup": 100},
            "n_iterations": 1000, "post_processing": {"n_distillation_steps": 200}}
    t = Tracer(conf)
    assert not t._sof_opacity_active(True, 99)
    assert t._sof_opacity_active(True, 100) and t._sof_opacity_active(True, 799)
    assert not t._sof_opacity_active(True, 800)
    assert not t._sof_opacity_active(False, 500)
    conf["loss"]["opa_warmup"] = 10
    assert Tracer(conf)._sof_opacity_active(True, 10)
    conf["loss"]["lambda_opa"] = 0.0
    assert not Tracer(conf)._sof_opacity_active(True, 500)


@pytest.mark.parametrize("loss", ["lambda_distortion", "lambda_dnc", "lambda_esmooth", "lambda_extent",
                                  "lambda_normal_variance"])
def test_geometric_losses_need_normals(loss):
    with pytest.raises(ValueError, match=loss):
        Tracer({"render": {}, "loss": {loss: 0.01}})


def test_geometric_channel_gradients_reach_trace_bwd():
    n = 4
    raster = FakeRaster(n)
    x = _inputs(n)
    outs = _apply(raster, x, n)
    (outs[0].sum() + 2.0 * outs[4].sum() + 3.0 * outs[5].sum()).backward()
    geometry = raster.calls[1][4]
    # pairs in the reference's order: depth var, extent, opacity field, quant, normal, inv depth, inv depth^2
    assert torch.equal(geometry[1], torch.full((raster.h, raster.w, 1), 3.0))  # depth var gradient
    assert torch.equal(geometry[9], torch.full((raster.h, raster.w, 3), 2.0))  # normal gradient
    assert geometry[3] is None and geometry[5] is None and geometry[7] is None
