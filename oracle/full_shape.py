"""Float64 numpy restatement of the per-view full-shape operator -- TEST
INFRASTRUCTURE ONLY (the checker of gofish_b200's gf_shape kernels).

Follows threedgut_tracer/view_observation_filter.py:64-330 (pixel Jacobian of
the active camera, minimum-norm footprint Q_v = gamma J^+ J^+^T by pivoted
modified Gram-Schmidt, mass-preserving factor m) and the full-shape operator
(footprint_shape_operator.py; footprint_shape_operator_cuda.cu:709-825: the
symmetric root C^{1/2} of C = Sigma + Q_v, factor B = C^{1/2} R, B^-1 its
inverse, unobserved rows keep B = R S), plus the Cholesky variant of the fused
inference kernel (fast_shape.cu:136-197).  The symmetric root here comes from
numpy.linalg.eigh, independent of the sm_100a Jacobi solver it checks.

Pinned by golden vectors from the reference's own view_observation_filter
(tests/golden/make_shape_golden.py) for J, Q and m, and by finite differences
for the VJP (tests/test_shape_host.py).
"""

from __future__ import annotations

import math

import numpy as np

TINY = np.finfo(np.float64).tiny


def rotation(q: np.ndarray) -> np.ndarray:
    """Rotation of quaternions (w, x, y, z) [N,4], not normalized."""
    q = np.asarray(q, dtype=np.float64)
    w, x, y, z = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    R = np.empty((q.shape[0], 3, 3))
    R[:, 0, 0] = 1 - 2 * (y * y + z * z)
    R[:, 0, 1] = 2 * (x * y - z * w)
    R[:, 0, 2] = 2 * (x * z + y * w)
    R[:, 1, 0] = 2 * (x * y + z * w)
    R[:, 1, 1] = 1 - 2 * (x * x + z * z)
    R[:, 1, 2] = 2 * (y * z - x * w)
    R[:, 2, 0] = 2 * (x * z - y * w)
    R[:, 2, 1] = 2 * (y * z + x * w)
    R[:, 2, 2] = 1 - 2 * (x * x + y * y)
    return R


def view_jacobian(positions, c2w, fisheye: bool, focal, k=(0.0, 0.0, 0.0, 0.0), max_angle=math.pi):
    """World pixel Jacobian [N,2,3] rounded to float32 and the camera-chart
    validity (view_observation_filter.py:200-330)."""
    p = np.asarray(positions, dtype=np.float64)
    m = np.asarray(c2w, dtype=np.float64)
    Rc, c = m[:3, :3], m[:3, 3]
    cam = (p - c) @ Rc
    x, y, z = cam[:, 0], cam[:, 1], cam[:, 2]
    fx, fy = float(focal[0]), float(focal[1])
    Jc = np.zeros((p.shape[0], 2, 3))
    if fisheye:
        k1, k2, k3, k4 = (float(v) for v in k)
        dist = np.sqrt(x * x + y * y + z * z)
        rho = np.hypot(x, y)
        theta = np.arctan2(rho, z)
        t2 = theta * theta
        rt = theta * (1 + t2 * (k1 + t2 * (k2 + t2 * (k3 + t2 * k4))))
        rd = 1 + t2 * (3 * k1 + t2 * (5 * k2 + t2 * (7 * k3 + t2 * 9 * k4)))
        rs = np.maximum(rho, math.sqrt(TINY))
        d2 = np.maximum(dist * dist, TINY)
        cp, sp = x / rs, y / rs
        gt = np.stack([z * x / (rs * d2), z * y / (rs * d2), -rho / d2], 1)
        gp = np.stack([-y / (rs * rs), x / (rs * rs), np.zeros_like(x)], 1)
        Jc[:, 0] = fx * (rd[:, None] * cp[:, None] * gt - rt[:, None] * sp[:, None] * gp)
        Jc[:, 1] = fy * (rd[:, None] * sp[:, None] * gt + rt[:, None] * cp[:, None] * gp)
        axis = (rho <= 1e-12) & (z > 0)
        with np.errstate(divide="ignore", invalid="ignore"):
            Jc[axis] = 0.0
            Jc[axis, 0, 0] = fx / dist[axis]
            Jc[axis, 1, 1] = fy / dist[axis]
        valid = (dist > 0.2) & ((rho > 1e-12) | (z > 0)) & (theta < max_angle) & (rd > 0)
    else:
        valid = z > 0.2
        zs = np.where(valid, z, 1.0)
        Jc[:, 0, 0] = fx / zs
        Jc[:, 0, 2] = -fx * x / (zs * zs)
        Jc[:, 1, 1] = fy / zs
        Jc[:, 1, 2] = -fy * y / (zs * zs)
    with np.errstate(over="ignore", invalid="ignore"):
        Jw = np.einsum("nij,kj->nik", Jc, Rc).astype(np.float32)
    return Jw, valid


def minimum_norm_q(J32, chart_valid, gamma):
    """Q = gamma J^+ J^+^T from the float32 Jacobian by column-pivoted modified
    Gram-Schmidt of J^T with one reorthogonalization (view_observation_filter.py:
    90-163).  Returns (Q [N,3,3], observed [N])."""
    A = np.asarray(J32, dtype=np.float64).transpose(0, 2, 1)  # [N,3,2]
    a, b = A[:, :, 0], A[:, :, 1]
    swap = (b * b).sum(1) > (a * a).sum(1)
    lead = np.where(swap[:, None], b, a)
    trail = np.where(swap[:, None], a, b)
    p0 = np.linalg.norm(lead, axis=1)
    ok0 = np.isfinite(p0) & (p0 > 0)
    sp0 = np.where(ok0, p0, 1.0)
    u0 = lead / sp0[:, None]
    coef = (u0 * trail).sum(1)
    r = trail - coef[:, None] * u0
    corr = (u0 * r).sum(1)
    r = r - corr[:, None] * u0
    coef = coef + corr
    p1 = np.linalg.norm(r, axis=1)
    ok1 = np.isfinite(p1) & (p1 > 0)
    sp1 = np.where(ok1, p1, 1.0)
    u1 = r / sp1[:, None]
    c0 = u0 / sp0[:, None] + u1 * (-coef / (sp0 * sp1))[:, None]
    c1 = u1 / sp1[:, None]
    Q = gamma * (c0[:, :, None] * c0[:, None, :] + c1[:, :, None] * c1[:, None, :])
    valid = (np.asarray(chart_valid) & np.isfinite(J32).all((1, 2)) & ok0 & ok1 & np.isfinite(coef)
             & np.isfinite(u0).all(1) & np.isfinite(u1).all(1) & np.isfinite(Q).all((1, 2)))
    return np.where(valid[:, None, None], Q, 0.0), valid


def compensation(J32, R, s, gamma):
    """m = sqrt(det S0 / det(S0 + gamma I)), S0 = F F^T, F = J R S."""
    F = np.asarray(J32, np.float64) @ R * np.asarray(s, np.float64)[:, None, :]
    S0 = F @ F.transpose(0, 2, 1)
    det0 = np.linalg.det(S0)
    det1 = np.linalg.det(S0 + gamma * np.eye(2))
    return np.sqrt(det0 / det1), S0


def full_shape(scales, quats, density, Q, J32, observed, gamma, mass_preserving=True, mode="exact"):
    """(covariance, factor, inverse_factor, compensation, density') in float64."""
    s = np.asarray(scales, np.float64)
    R = rotation(quats)
    o = np.asarray(density, np.float64).reshape(-1)
    n = s.shape[0]
    sigma = R @ (s[:, :, None] ** 2 * R.transpose(0, 2, 1))
    C = sigma + Q
    B = R * s[:, None, :]
    Bi = (R / s[:, None, :]).transpose(0, 2, 1)
    m = np.ones(n)
    ob = np.asarray(observed, bool)
    if ob.any():
        if mode == "exact":
            lam, V = np.linalg.eigh(C[ob])
            root = V @ (np.sqrt(lam)[:, :, None] * V.transpose(0, 2, 1))
            iroot = V @ ((1.0 / np.sqrt(lam))[:, :, None] * V.transpose(0, 2, 1))
            B[ob] = root @ R[ob]
            Bi[ob] = R[ob].transpose(0, 2, 1) @ iroot
        else:
            L = np.linalg.cholesky(C[ob])
            B[ob] = L
            Bi[ob] = np.linalg.inv(L)
        m[ob] = compensation(J32[ob], R[ob], s[ob], gamma)[0]
    C = np.where(ob[:, None, None], C, sigma)
    dens = m * o if mass_preserving else o.copy()
    return C, B, Bi, m, dens


def full_shape_vjp(scales, quats, density, Q, J32, observed, gamma, gC, gB, gBi, gm, gd, mass_preserving=True):
    """Gradients (scales [N,3], quaternion [N,4], density [N]) of the exact
    operator for output gradients gC, gB, gBi [N,3,3], gm, gd [N]."""
    s = np.asarray(scales, np.float64)
    q = np.asarray(quats, np.float64)
    R = rotation(q)
    o = np.asarray(density, np.float64).reshape(-1)
    ob = np.asarray(observed, bool)
    n = s.shape[0]
    sym = lambda M: 0.5 * (M + M.transpose(0, 2, 1))  # noqa: E731
    gR = np.zeros((n, 3, 3))
    gs = np.zeros((n, 3))
    go = np.asarray(gd, np.float64).copy()
    gSigma = np.zeros((n, 3, 3))
    # unobserved rows: B = R S, B^-1 = S^-1 R^T, C = Sigma
    u = ~ob
    gR[u] += gB[u] * s[u][:, None, :]
    gs[u] += (gB[u] * R[u]).sum(1)
    gR[u] += (gBi[u] / s[u][:, :, None]).transpose(0, 2, 1)
    gs[u] -= (gBi[u] * R[u].transpose(0, 2, 1)).sum(2) / (s[u] ** 2)
    gSigma[u] += sym(gC[u])
    if ob.any():
        Ro, so = R[ob], s[ob]
        sigma = Ro @ (so[:, :, None] ** 2 * Ro.transpose(0, 2, 1))
        C = sigma + Q[ob]
        lam, V = np.linalg.eigh(C)
        r = np.sqrt(lam)
        root = V @ (r[:, :, None] * V.transpose(0, 2, 1))
        iroot = V @ ((1 / r)[:, :, None] * V.transpose(0, 2, 1))
        m, S0 = compensation(J32[ob], Ro, so, gamma)
        gmt = np.asarray(gm, np.float64)[ob] + (np.asarray(gd, np.float64)[ob] * o[ob] if mass_preserving else 0.0)
        if mass_preserving:
            go[ob] = np.asarray(gd, np.float64)[ob] * m
        G1 = gB[ob] @ Ro.transpose(0, 2, 1)          # dL/d root
        G2 = Ro @ gBi[ob]                             # dL/d C^{-1/2}
        gR[ob] += root @ gB[ob] + iroot @ gBi[ob].transpose(0, 2, 1)
        K1 = 1.0 / (r[:, :, None] + r[:, None, :])
        K2 = -K1 / (r[:, :, None] * r[:, None, :])
        Vt = V.transpose(0, 2, 1)
        gCo = sym(gC[ob]) + V @ ((Vt @ sym(G1) @ V) * K1 + (Vt @ sym(G2) @ V) * K2) @ Vt
        Jd = J32[ob].astype(np.float64)
        inner = np.linalg.inv(S0) - np.linalg.inv(S0 + gamma * np.eye(2))
        gSm = (gmt * m * 0.5)[:, None, None] * (Jd.transpose(0, 2, 1) @ inner @ Jd)
        gSigma[ob] += gCo + sym(gSm)
    # Sigma = R S^2 R^T
    gR += 2.0 * gSigma @ R * (s ** 2)[:, None, :]
    gs += 2.0 * s * np.einsum("nji,njk,nki->ni", R, gSigma, R)
    # R(q)
    w, x, y, z = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    G = gR
    gq = np.stack([
        2 * (-z * G[:, 0, 1] + y * G[:, 0, 2] + z * G[:, 1, 0] - x * G[:, 1, 2] - y * G[:, 2, 0] + x * G[:, 2, 1]),
        2 * (y * G[:, 0, 1] + z * G[:, 0, 2] + y * G[:, 1, 0] - 2 * x * G[:, 1, 1] - w * G[:, 1, 2] + z * G[:, 2, 0]
             + w * G[:, 2, 1] - 2 * x * G[:, 2, 2]),
        2 * (-2 * y * G[:, 0, 0] + x * G[:, 0, 1] + w * G[:, 0, 2] + x * G[:, 1, 0] + z * G[:, 1, 2] - w * G[:, 2, 0]
             + z * G[:, 2, 1] - 2 * y * G[:, 2, 2]),
        2 * (-2 * z * G[:, 0, 0] - w * G[:, 0, 1] + x * G[:, 0, 2] + w * G[:, 1, 0] - 2 * z * G[:, 1, 1]
             + y * G[:, 1, 2] + x * G[:, 2, 0] + y * G[:, 2, 1]),
    ], 1)
    return gs, gq, go
