"""The sm_100a per-view full-shape kernels (gf_view_q6, gf_full_shape,
gf_full_shape_bwd, gf_view_shape_packed) against the float64 numpy oracle
(oracle/full_shape.py), and current_view_q6 against golden vectors of the
reference's own view_observation_filter."""

import types
from pathlib import Path

import numpy as np
import pytest
import torch

from gofish_b200 import footprint_shape_operator as fso
from gofish_b200 import view_observation_filter as vof
from oracle import full_shape as fs

pytestmark = pytest.mark.gpu
G = np.load(Path(__file__).resolve().parent / "golden" / "shape_golden.npz")


def fish_batch(pose, device, focal=(310.0, 305.0), k=(0.03, -0.004, 0.0005, -0.00003), max_angle=1.75):
    return types.SimpleNamespace(T_to_world=torch.from_numpy(np.asarray(pose, np.float32))[None].to(device),
                                 T_to_world_end=None, rays_in_world_space=False,
                                 intrinsics_OpenCVFisheyeCameraModelParameters={
                                     "focal_length": list(focal), "radial_coeffs": list(k), "max_angle": max_angle})


def pin_batch(pose, device, focal=(420.0, 415.0)):
    return types.SimpleNamespace(T_to_world=torch.from_numpy(np.asarray(pose, np.float32))[None].to(device),
                                 T_to_world_end=None, rays_in_world_space=False,
                                 intrinsics_OpenCVPinholeCameraModelParameters={
                                     "focal_length": list(focal), "radial_coeffs": [0.0] * 6,
                                     "tangential_coeffs": [0.0, 0.0], "thin_prism_coeffs": [0.0] * 4})


def q6_of(Q):
    return np.stack([Q[:, 0, 0], Q[:, 0, 1], Q[:, 0, 2], Q[:, 1, 1], Q[:, 1, 2], Q[:, 2, 2]], 1)


@pytest.mark.parametrize("kind", ["fish", "pin"])
def test_view_q6_matches_oracle_and_reference(cuda_device, kind):
    pose, pts = G[f"{kind}_pose"], G[f"{kind}_points"]
    batch = fish_batch(pose, cuda_device) if kind == "fish" else pin_batch(pose, cuda_device)
    q6, jac, ob = vof.current_view_q6(torch.from_numpy(pts).to(cuda_device), batch, 0.3)
    q6, jac, ob = q6.cpu().numpy(), jac.cpu().numpy(), ob.cpu().numpy()
    fisheye = kind == "fish"
    J, chart = fs.view_jacobian(pts, pose, fisheye, G[f"{kind}_focal"], G["fish_k"] if fisheye else (0, 0, 0, 0),
                                float(G["fish_max_angle"]) if fisheye else np.pi)
    Q, want_ob = fs.minimum_norm_q(J, chart, 0.3)
    assert np.array_equal(ob, want_ob)
    assert np.array_equal(ob, G[f"{kind}_valid"])
    # float32 J: identical up to the last bit of the double-precision atan2/hypot
    rel = np.abs(jac[ob] - J[ob]) / np.abs(J[ob]).max(axis=(1, 2))[:, None, None]
    assert rel.max() < 1e-6
    np.testing.assert_allclose(q6[ob], q6_of(Q)[ob], rtol=1e-5, atol=1e-12)
    np.testing.assert_allclose(q6[ob], G[f"{kind}_q6"][ob], rtol=1e-3, atol=1e-10)
    assert np.all(q6[~ob] == 0.0) and np.all(jac[~ob] == 0.0)


def random_rows(seed, n, device):
    rng = np.random.default_rng(seed)
    pose = np.eye(4, dtype=np.float32)
    pts = (rng.standard_normal((n, 3)) * 2.0).astype(np.float32)
    pts[:, 2] = np.abs(pts[:, 2]) + 0.5
    pts[::5, 2] = -pts[::5, 2]  # a fifth behind the camera (outside its 1.6 rad field of view)
    s = np.exp(rng.normal(np.log(0.04), 0.7, (n, 3))).astype(np.float32)
    q = rng.standard_normal((n, 4))
    q = (q / np.linalg.norm(q, axis=1, keepdims=True)).astype(np.float32)
    o = rng.uniform(0.02, 0.98, (n, 1)).astype(np.float32)
    batch = fish_batch(pose, device, focal=(200.0, 198.0), max_angle=1.6)
    return pts, s, q, o, batch


def oracle_inputs(pts, batch, gamma=0.3):
    J, chart = fs.view_jacobian(pts, np.eye(4), True, (200.0, 198.0), (0.03, -0.004, 0.0005, -0.00003), 1.6)
    Q, ob = fs.minimum_norm_q(J, chart, gamma)
    return J, Q, ob


@pytest.mark.parametrize("mode", ["exact", "cholesky"])
def test_full_shape_forward_matches_oracle(cuda_device, mode):
    pts, s, q, o, batch = random_rows(1, 20000, cuda_device)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device)  # noqa: E731
    q6, jac, ob = vof.current_view_q6(dev(pts), batch, 0.3)
    out = fso.build_full_shape(dev(s), dev(q), dev(o), q6, jac, ob, mode=mode)
    J, Q, want_ob = oracle_inputs(pts, batch)
    assert np.array_equal(ob.cpu().numpy(), want_ob) and 0.3 < want_ob.mean() < 1.0
    # the oracle consumes the same float32 J and float64 Q the kernel did
    C, B, Bi, m, d = fs.full_shape(s, q, o[:, 0], q6.cpu().numpy()[:, [0, 1, 2, 1, 3, 4, 2, 4, 5]].reshape(-1, 3, 3),
                                   jac.cpu().numpy(), want_ob, 0.3, True, "exact" if mode == "exact" else "chol")
    for got, want, name in ((out.covariance, C, "C"), (out.factor, B, "B"), (out.inverse_factor, Bi, "Bi")):
        g = got.cpu().numpy().astype(np.float64)
        scale = np.abs(want).max(axis=(1, 2))[:, None, None]
        assert (np.abs(g - want) / scale).max() < 2e-6, name
    np.testing.assert_allclose(out.compensation.cpu().numpy(), m, rtol=2e-6)
    np.testing.assert_allclose(out.density.cpu().numpy()[:, 0], d, rtol=2e-6)


def test_full_shape_vjp_matches_oracle(cuda_device):
    pts, s, q, o, batch = random_rows(2, 5000, cuda_device)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device)  # noqa: E731
    q6, jac, ob = vof.current_view_q6(dev(pts), batch, 0.3)
    st, qt, ot = dev(s).requires_grad_(), dev(q).requires_grad_(), dev(o).requires_grad_()
    out = fso.build_full_shape(st, qt, ot, q6, jac, ob)
    rng = np.random.default_rng(9)
    gC, gB, gBi = (rng.normal(size=(5000, 3, 3)).astype(np.float32) for _ in range(3))
    gm, gd = rng.normal(size=5000).astype(np.float32), rng.normal(size=(5000, 1)).astype(np.float32)
    loss = ((out.covariance * dev(gC)).sum() + (out.factor * dev(gB)).sum() + (out.inverse_factor * dev(gBi)).sum()
            + (out.compensation * dev(gm)).sum() + (out.density * dev(gd)).sum())
    loss.backward()
    Q = q6.cpu().numpy()[:, [0, 1, 2, 1, 3, 4, 2, 4, 5]].reshape(-1, 3, 3)
    ws, wq, wo = fs.full_shape_vjp(s, q, o[:, 0], Q, jac.cpu().numpy(), ob.cpu().numpy(), 0.3,
                                   gC.astype(np.float64), gB.astype(np.float64), gBi.astype(np.float64),
                                   gm.astype(np.float64), gd[:, 0].astype(np.float64))
    for got, want in ((st.grad, ws), (qt.grad, wq), (ot.grad[:, 0], wo)):
        g = got.cpu().numpy().astype(np.float64)
        assert np.linalg.norm(g - want) / np.linalg.norm(want) < 1e-5


@pytest.mark.parametrize("mode", [0, 1])
def test_packed_inference_shape(cuda_device, mode):
    import ctypes
    from gofish_b200 import _native
    pts, s, q, o, batch = random_rows(3, 8000, cuda_device)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device)  # noqa: E731
    packed = torch.zeros((8000, 32), dtype=torch.float32, device=cuda_device)
    status = torch.zeros(4, dtype=torch.int32, device=cuda_device)
    cam = vof.shape_camera(batch)
    inputs = [dev(pts), dev(q), dev(s), dev(o)]  # held until the kernel has run
    _native.check(_native.load().gf_view_shape_packed(*(t.data_ptr() for t in inputs), 8000, ctypes.byref(cam), 0.3,
                                                      mode, packed.data_ptr(), status.data_ptr(),
                                                      torch.cuda.current_stream().cuda_stream), "packed")
    torch.cuda.synchronize()
    assert int(status[0]) == 0
    J, Q, ob = oracle_inputs(pts, batch)
    C, B, Bi, m, d = fs.full_shape(s, q, o[:, 0], Q, J, ob, 0.3, True, "exact" if mode == 0 else "chol")
    p = packed.cpu().numpy().astype(np.float64)
    np.testing.assert_allclose(p[:, 3], d, rtol=2e-6)
    for got, want in ((p[:, 12:21].reshape(-1, 3, 3), B), (p[:, 21:30].reshape(-1, 3, 3), Bi)):
        scale = np.abs(want).max(axis=(1, 2))[:, None, None]
        assert (np.abs(got - want) / scale).max() < 2e-6


def test_numerical_failure_reports_row(cuda_device):
    pts, s, q, o, batch = random_rows(4, 1000, cuda_device)
    dev = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda_device)  # noqa: E731
    q6, jac, ob = vof.current_view_q6(dev(pts), batch, 0.3)
    row = int(np.flatnonzero(ob.cpu().numpy())[7])
    s = s.copy()
    s[row] = 0.0  # singular Sigma: C = Q has rank 2
    with pytest.raises(fso.FootprintNumericalError) as err:
        fso.build_full_shape(dev(s), dev(q), dev(o), q6, jac, ob)
    assert err.value.global_row == row
