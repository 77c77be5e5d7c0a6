"""The numpy restatement of the per-view full-shape operator (oracle/full_shape.py):
pixel Jacobian, footprint Q and compensation m against golden vectors made
from the reference's own view_observation_filter (tests/golden/
make_shape_golden.py); the factor identities; the VJP against central
finite differences."""

from pathlib import Path

import numpy as np
import pytest

from oracle import full_shape as fs

G = np.load(Path(__file__).resolve().parent / "golden" / "shape_golden.npz")


def q6_of(Q):
    return np.stack([Q[:, 0, 0], Q[:, 0, 1], Q[:, 0, 2], Q[:, 1, 1], Q[:, 1, 2], Q[:, 2, 2]], 1)


@pytest.mark.parametrize("kind", ["fish", "pin"])
def test_jacobian_and_validity_match_reference(kind):
    fisheye = kind == "fish"
    J, valid = fs.view_jacobian(G[f"{kind}_points"], G[f"{kind}_pose"], fisheye, G[f"{kind}_focal"],
                                G["fish_k"] if fisheye else (0, 0, 0, 0),
                                float(G["fish_max_angle"]) if fisheye else np.pi)
    Q, ob = fs.minimum_norm_q(J, valid, 0.3)
    want_valid = G[f"{kind}_valid"]
    assert np.array_equal(ob, want_valid)
    # the reference builds J with float32 torch operations, this restatement in float64
    Jw = G[f"{kind}_jacobian"]
    scale = np.abs(Jw[ob]).max(axis=(1, 2))[:, None, None]
    assert np.abs(J[ob] - Jw[ob]).max() <= 0 or (np.abs(J[ob] - Jw[ob]) / scale).max() < 2e-5


@pytest.mark.parametrize("kind", ["fish", "pin"])
def test_footprint_q_matches_reference(kind):
    Q, ob = fs.minimum_norm_q(G[f"{kind}_jacobian"], G[f"{kind}_valid"], 0.3)
    assert np.array_equal(ob, G[f"{kind}_valid"])
    np.testing.assert_allclose(q6_of(Q), G[f"{kind}_q6"], rtol=1e-12, atol=1e-300)


def test_q_equals_pseudo_inverse_form_and_m_matches_reference():
    J = G["m_jacobian"].astype(np.float32).astype(np.float64)
    Q, ob = fs.minimum_norm_q(G["m_jacobian"].astype(np.float32), np.ones(len(J), bool), 0.3)
    pinv = np.linalg.pinv(J)
    np.testing.assert_allclose(Q, 0.3 * pinv @ pinv.transpose(0, 2, 1), rtol=1e-9, atol=1e-18)
    Jg = G["m_jacobian"]
    S0 = Jg @ G["m_sigma"] @ Jg.transpose(0, 2, 1)
    m = np.sqrt(np.linalg.det(S0) / np.linalg.det(S0 + 0.3 * np.eye(2)))
    np.testing.assert_allclose(m, G["m_value"], rtol=1e-12)
    np.testing.assert_allclose(G["q_value"], 0.3 * np.linalg.pinv(Jg) @ np.linalg.pinv(Jg).transpose(0, 2, 1),
                               rtol=1e-10, atol=1e-18)


def _inputs(seed=0, n=64):
    rng = np.random.default_rng(seed)
    s = np.exp(rng.normal(np.log(0.05), 0.6, (n, 3)))
    q = rng.normal(size=(n, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    o = rng.uniform(0.05, 0.95, n)
    J = (rng.normal(size=(n, 2, 3)) * 300).astype(np.float32)
    Q, ob = fs.minimum_norm_q(J, rng.random(n) < 0.8, 0.3)
    return s, q, o, Q, J, ob


@pytest.mark.parametrize("mode", ["exact", "cholesky"])
def test_factor_identities(mode):
    s, q, o, Q, J, ob = _inputs(1)
    C, B, Bi, m, d = fs.full_shape(s, q, o, Q, J, ob, 0.3, True, mode)
    R = fs.rotation(q)
    np.testing.assert_allclose(B @ B.transpose(0, 2, 1), C, rtol=1e-10, atol=1e-14)
    np.testing.assert_allclose(Bi @ B, np.broadcast_to(np.eye(3), B.shape), atol=1e-9)
    if mode == "exact":
        root = B[ob] @ R[ob].transpose(0, 2, 1)
        np.testing.assert_allclose(root, root.transpose(0, 2, 1), atol=1e-12)
        assert (np.linalg.eigvalsh(root) > 0).all()
    else:
        assert np.allclose(np.triu(B[ob], 1), 0.0)
    u = ~ob
    np.testing.assert_allclose(B[u], R[u] * s[u][:, None, :], rtol=1e-14)
    assert np.all(m[u] == 1.0) and np.all((m[ob] > 0) & (m[ob] < 1))
    np.testing.assert_allclose(d, m * o)


def test_vjp_matches_finite_differences():
    s, q, o, Q, J, ob = _inputs(2, 24)
    rng = np.random.default_rng(5)
    gC, gB, gBi = (rng.normal(size=(24, 3, 3)) for _ in range(3))
    gm, gd = rng.normal(size=24), rng.normal(size=24)

    def loss(s_, q_, o_):
        C, B, Bi, m, d = fs.full_shape(s_, q_, o_, Q, J, ob, 0.3, True, "exact")
        return (gC * C).sum() + (gB * B).sum() + (gBi * Bi).sum() + (gm * m).sum() + (gd * d).sum()

    gs, gq, go = fs.full_shape_vjp(s, q, o, Q, J, ob, 0.3, gC, gB, gBi, gm, gd)
    for arr, grad, h in ((s, gs, 1e-7), (q, gq, 1e-7), (o, go, 1e-6)):
        flat = arr.reshape(-1)
        for idx in range(0, flat.size, 7):
            old = flat[idx]
            flat[idx] = old + h
            lp = loss(s, q, o)
            flat[idx] = old - h
            lm = loss(s, q, o)
            flat[idx] = old
            fd = (lp - lm) / (2 * h)
            g = grad.reshape(-1)[idx]
            assert abs(fd - g) <= 2e-5 * max(1.0, abs(fd)), (idx, fd, g)
