"""Generates tests/golden/hit_golden.npz from the reference's own per-hit
device functions, compiled for the host cores and run in a container where
the reference checkout is present.

The reference's header-only per-hit code
(threedgut_tracer/include/3dgut/kernels/cuda/models/gaussianParticles.cuh:
processHitFwd :611-686, processHitBwd :736-1155,
particleExactDepthCrossingRaw :592-609, with gutHalfRayResponse.cuh,
finiteIntervalExactCrossing.cuh, alphaCapBackward.cuh, mathUtils.cuh,
cudaMath.cuh and sensorConstants.cuh) is built unmodified with g++ by
``make -C oracle ref REF=<reference>`` against oracle/ref_device/cuda_host_shim.h
into oracle/_ref/hit_pin_driver (see the driver's header for what it runs).

It also records the projector's particle radiance, radianceFromSpH
(gaussianParticles.cuh:188-220, unclamped as gutProjector.cuh:903 calls it),
at SH degrees 0 to 3, and the sensor-space point projection projectPoint
(cameraProjections.cuh:75-152, without raster bounds as the UT calls it) of
three fisheye cameras and a distorted pinhole, and the k-buffer's composite
order (HitParticleKBufferT, gutKBufferRenderer.cuh:118-166, compiled with its
renderer header) for every K the tracer supports, and the UT projection
(GUTProjector::unscentedParticleProjection, gutProjector.cuh:359-518) of
particles around each camera.

Inputs (seeded): tiles of 16x16 rays, each tile with its own ordered list
of 6 to 48 Gaussians (random rotation, log-normal scales, opacities up to 1
so the 0.99 alpha cap is reached, a few Gaussians behind the ray origins or
within the 0.2 m inverse-depth clip, colours in [-0.2, 1.2] so the zero clamp
is exercised) and per-ray output gradients.  Rays whose float64 evaluation
puts a hit, the minimum transmittance or an opacity threshold within a
relative 2e-3 of its decision boundary are redrawn, so that the float32
evaluations of the reference and of this library take the same branches.

    python tests/golden/make_hit_golden.py /path/to/reference
"""

from __future__ import annotations

import math
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
DRIVER = REPO / "oracle" / "_ref" / "hit_pin_driver"

TILES = 24
RAYS = 256
MIN_RESPONSE = 0.0113
MIN_ALPHA = 1.0 / 255.0
MAX_ALPHA = 0.99
MIN_TRANSMITTANCE = 1e-4
QUANTILES = (0.05, 0.10, 0.15, 0.20, 0.30, 0.40, 0.50)
MARGIN = 2e-3


def quaternion_matrix(q: np.ndarray) -> np.ndarray:
    """Rotation matrices of unit quaternions (w, x, y, z)."""
    w, x, y, z = q[:, 0], q[:, 1], q[:, 2], q[:, 3]
    return np.stack([
        np.stack([1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)], -1),
        np.stack([2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)], -1),
        np.stack([2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)], -1),
    ], -2)


def packed_rows(pos, quat, scale, density) -> np.ndarray:
    """[M,32] rows: position, density, quaternion (w,x,y,z), scale, intrinsic
    density, B = R diag(s) and B^-1 = diag(1/s) R^T row-major, two zeros."""
    m = pos.shape[0]
    R = quaternion_matrix(quat.astype(np.float64))
    s = scale.astype(np.float64)
    rows = np.zeros((m, 32), np.float32)
    rows[:, 0:3] = pos
    rows[:, 3] = density
    rows[:, 4:8] = quat
    rows[:, 8:11] = scale
    rows[:, 11] = density
    rows[:, 12:21] = (R * s[:, None, :]).reshape(m, 9)
    rows[:, 21:30] = (np.transpose(R, (0, 2, 1)) / s[:, :, None]).reshape(m, 9)
    return rows


def draw_tile(rng: np.random.Generator):
    m = int(rng.integers(6, 49))
    axis = rng.standard_normal(3)
    axis /= np.linalg.norm(axis)
    helper = np.array([1.0, 0.0, 0.0]) if abs(axis[0]) < 0.9 else np.array([0.0, 1.0, 0.0])
    u = np.cross(axis, helper)
    u /= np.linalg.norm(u)
    v = np.cross(axis, u)
    origin = rng.uniform(-0.5, 0.5, 3)
    depth = np.sort(rng.uniform(0.4, 6.0, m))
    depth[rng.random(m) < 0.08] = rng.uniform(-0.6, 0.15)          # behind the origins / inside the clip
    lateral = rng.uniform(-0.35, 0.35, (m, 2)) * np.maximum(depth, 0.3)[:, None]
    pos = origin + depth[:, None] * axis + lateral[:, :1] * u + lateral[:, 1:] * v
    q = rng.standard_normal((m, 4))
    q /= np.linalg.norm(q, axis=1, keepdims=True)
    scale = np.exp(rng.normal(np.log(0.12), 0.6, (m, 3)))
    density = np.where(rng.random(m) < 0.25, rng.uniform(0.9, 1.0, m), rng.uniform(0.02, 0.9, m))
    order = np.arange(m)
    swaps = rng.integers(0, max(1, m - 1), size=m // 4)               # the list need not be depth sorted
    for a in swaps:
        order[[a, a + 1]] = order[[a + 1, a]]
    rows = packed_rows(pos[order].astype(np.float32), q[order].astype(np.float32),
                       scale[order].astype(np.float32), density[order].astype(np.float32))
    colours = rng.uniform(-0.2, 1.2, (m, 3)).astype(np.float32)
    return rows, colours, origin, axis, u, v


def ray_is_clear(rows, o, d) -> bool:
    """No decision of the K = 0 walk lies near its boundary (float64)."""
    T = 1.0
    for r in rows.astype(np.float64):
        binv = r[21:30].reshape(3, 3)
        gro = binv @ (o - r[0:3])
        grdu = binv @ d
        den = grdu @ grdu
        tau_line = -(gro @ grdu) / den
        if abs(tau_line) < 1e-3:            # the closest point's interior flag flips at t_min = 0
            return False
        tau = max(tau_line, 0.0)
        p = gro + tau * grdu
        resp = np.exp(-0.5 * (p @ p))
        a_u = resp * r[3]
        for value, edge in ((resp, MIN_RESPONSE), (a_u, MIN_ALPHA), (a_u, MAX_ALPHA)):
            if abs(value - edge) <= MARGIN * edge:
                return False
        if resp > MIN_RESPONSE and min(a_u, MAX_ALPHA) > MIN_ALPHA:
            T_next = T * (1.0 - min(a_u, MAX_ALPHA))
            for level in QUANTILES:
                if abs((1.0 - T_next) - level) <= MARGIN * level:
                    return False
            if abs(T_next - MIN_TRANSMITTANCE) <= 0.05 * MIN_TRANSMITTANCE:
                return False
            T = T_next
            if T < MIN_TRANSMITTANCE:
                break
    return True


def aabb_exit(o: np.ndarray, d: np.ndarray) -> np.float32:
    """Far end of the +-1e6 scene box along the ray (float32 slab test of the
    renderer's ray set-up, bounding_box.h:89-133) for an origin inside it."""
    o32, d32 = o.astype(np.float32), d.astype(np.float32)
    far = np.float32(np.inf)
    for k in range(3):
        a = (np.float32(-1e6) - o32[k]) / d32[k]
        b = (np.float32(1e6) - o32[k]) / d32[k]
        far = min(far, max(a, b))
    return np.float32(far)


def sh_goldens(rng: np.random.Generator, items: int = 512):
    """The reference's unclamped particle radiance at SH degrees 0-3 for unit
    directions (seeded, plus the six axis directions) and N(0, 0.6)
    coefficients: arrays [4, items, 3], [4, items, 48], [4, items, 3]."""
    dirs = rng.standard_normal((4, items, 3))
    dirs[:, :6] = np.array([[1, 0, 0], [-1, 0, 0], [0, 1, 0], [0, -1, 0], [0, 0, 1], [0, 0, -1]], np.float64)
    dirs = (dirs / np.linalg.norm(dirs, axis=-1, keepdims=True)).astype(np.float32)
    coeffs = rng.normal(0.0, 0.6, (4, items, 48)).astype(np.float32)
    rgb = np.zeros((4, items, 3), np.float32)
    with tempfile.TemporaryDirectory() as tmp:
        for degree in range(4):
            src, dst = Path(tmp) / "sh.bin", Path(tmp) / "sh.out"
            with open(src, "wb") as f:
                f.write(np.array([items, degree], np.int32).tobytes())
                f.write(np.concatenate([dirs[degree], coeffs[degree]], axis=1).tobytes())
            subprocess.run([str(DRIVER), "sh", str(src), str(dst)], check=True)
            rgb[degree] = np.fromfile(dst, dtype=np.float32).reshape(items, 3)
    return dirs, coeffs, rgb


# Cameras of the projection goldens: model, width, height, principal, focal,
# radial[6], tangential[2], thin prism[4], max angle (rad): an equidistant and
# a Kannala-Brandt 200 deg fisheye, the equisolid 205 deg one (its 4-term
# Taylor series), and a distorted pinhole.
PROJECTION_CAMERAS = (
    (1, 320, 320, (160.0, 160.0), (91.67, 91.67), (0.0, 0.0, 0.0, 0.0, 0.0, 0.0), (0.0, 0.0), (0.0,) * 4,
     1.7453293),
    (1, 1600, 1600, (799.5, 800.5), (452.0, 455.0), (0.021, -0.012, 0.0031, -0.0004, 0.0, 0.0), (0.0, 0.0),
     (0.0,) * 4, 1.7453293),
    (1, 2560, 2560, (1280.0, 1280.0), (716.0, 716.0),
     (-1.0 / 24.0, 1.0 / 1920.0, -1.0 / 322560.0, 1.0 / 92897280.0, 0.0, 0.0), (0.0, 0.0), (0.0,) * 4, 1.7889625),
    (0, 640, 480, (321.5, 239.0), (500.0, 498.0), (0.11, -0.05, 0.012, 0.021, -0.011, 0.004), (0.0012, -0.0021),
     (1e-4, -2e-4, 3e-4, -1e-4), 3.1415927),
)


def projection_goldens(rng: np.random.Generator, points: int = 4096):
    """The reference's projectPoint for each camera of PROJECTION_CAMERAS at
    seeded points: directions over the whole sphere at 0.05-50 m, points on
    and near the optical axis and behind the camera; directions within 1e-4
    rad of the maximum angle are redrawn (the validity there depends on the
    last bit of atan2).  Returns ([C, P, 3] points, [C, P, 3] u, v, valid)."""
    all_pts, all_out = [], []
    with tempfile.TemporaryDirectory() as tmp:
        for model, w, h, pp, f, k, tg, tp, max_angle in PROJECTION_CAMERAS:
            pts = np.zeros((points, 3), np.float64)
            i = 0
            while i < points:
                d = rng.standard_normal(3)
                d /= np.linalg.norm(d)
                theta = math.atan2(math.hypot(d[0], d[1]), d[2])
                if abs(theta - max_angle) < 1e-4:
                    continue
                pts[i] = d * math.exp(rng.uniform(math.log(0.05), math.log(50.0)))
                i += 1
            pts[:8] = [[0, 0, 1], [0, 0, 3.5], [0, 0, -2], [1e-20, 0, 1], [0, -1e-20, 2], [1e-3, 2e-3, 1],
                       [0.5, -0.25, 1e-7], [3.0, 4.0, 0.0]]
            pts = pts.astype(np.float32)
            src, dst = Path(tmp) / "pr.bin", Path(tmp) / "pr.out"
            cam = np.array([*pp, *f, *k, *tg, *tp, max_angle, 0.1], np.float32)
            with open(src, "wb") as fh:
                fh.write(np.array([points, model, w, h], np.int32).tobytes())
                fh.write(cam.tobytes())
                fh.write(pts.tobytes())
            subprocess.run([str(DRIVER), "project", str(src), str(dst)], check=True)
            all_pts.append(pts)
            all_out.append(np.fromfile(dst, dtype=np.float32).reshape(points, 3))
    return np.stack(all_pts), np.stack(all_out)


def quaternion_xyzw_matrix(q) -> np.ndarray:
    """Rotation matrix of a unit quaternion (x, y, z, w), float64."""
    x, y, z, w = (float(v) for v in q)
    return np.array([[1 - 2 * (y * y + z * z), 2 * (x * y - w * z), 2 * (x * z + w * y)],
                     [2 * (x * y + w * z), 1 - 2 * (x * x + z * z), 2 * (y * z - w * x)],
                     [2 * (x * z - w * y), 2 * (y * z + w * x), 1 - 2 * (x * x + y * y)]])


def ut_goldens(rng: np.random.Generator, count: int = 3000):
    """The reference's UT projection (GUTProjector::unscentedParticleProjection)
    of seeded particles around a random global-shutter pose of each camera of
    PROJECTION_CAMERAS: means over the whole sphere at 0.1-20 m, log-normal
    scales up to metres (sigma points beyond the fisheye's limit angle), some
    opacities below 1/255.  Particles with the mean within 1e-3 m of the 0.2 m
    near radius, or a sigma point within 1e-4 rad of the limit angle or of the
    pinhole's z = 0, are redrawn.  Returns ([C,7] poses, [C,3] centres,
    [C,count,32] rows, [C,count,6] centre u, v, covariance xx, xy, yy, valid)."""
    poses, centres, all_rows, outs = [], [], [], []
    with tempfile.TemporaryDirectory() as tmp:
        for model, w, h, pp, f, k, tg, tp, max_angle in PROJECTION_CAMERAS:
            q = rng.standard_normal(4)
            q /= np.linalg.norm(q)
            pose = np.array([*rng.uniform(-1, 1, 3), *q], np.float32)
            R = quaternion_xyzw_matrix(pose[3:7].astype(np.float64))
            t = pose[0:3].astype(np.float64)
            centre = (-(R.T @ t)).astype(np.float32)
            rows = np.zeros((count, 32), np.float32)
            i = 0
            while i < count:
                d = rng.standard_normal(3)
                d /= np.linalg.norm(d)
                dist = math.exp(rng.uniform(math.log(0.1), math.log(20.0)))
                mean = centre.astype(np.float64) + d * dist
                if abs(dist - 0.2) < 1e-3:
                    continue
                qq = rng.standard_normal(4)
                qq /= np.linalg.norm(qq)
                scale = np.exp(rng.normal(math.log(0.05), 1.2, 3))
                opacity = rng.uniform(0.001, 1.0)
                row = packed_rows(mean[None].astype(np.float32), qq[None].astype(np.float32),
                                  scale[None].astype(np.float32), np.array([opacity], np.float32))[0]
                B = row[12:21].astype(np.float64).reshape(3, 3)
                near_edge = False
                for sgn in (1.0, -1.0):
                    for a in range(3):
                        p = R @ (row[0:3].astype(np.float64) + sgn * math.sqrt(3.0) * B[:, a]) + t
                        if model == 1:
                            th = math.atan2(math.hypot(p[0], p[1]), p[2])
                            near_edge |= abs(th - max_angle) < 1e-4
                        else:
                            near_edge |= abs(p[2]) < 1e-4
                if near_edge:
                    continue
                rows[i] = row
                i += 1
            src, dst = Path(tmp) / "ut.bin", Path(tmp) / "ut.out"
            cam = np.array([*pp, *f, *k, *tg, *tp, max_angle, 0.1], np.float32)
            with open(src, "wb") as fh:
                fh.write(np.array([count, model, w, h], np.int32).tobytes())
                fh.write(cam.tobytes())
                fh.write(pose.tobytes())
                fh.write(centre.tobytes())
                fh.write(rows.tobytes())
            subprocess.run([str(DRIVER), "ut", str(src), str(dst)], check=True)
            poses.append(pose)
            centres.append(centre)
            all_rows.append(rows)
            outs.append(np.fromfile(dst, dtype=np.float32).reshape(count, 6))
    return np.stack(poses), np.stack(centres), np.stack(all_rows), np.stack(outs)


KBUFFER_SIZES = (4, 8, 12, 16, 24, 32)


def kbuffer_goldens(rng: np.random.Generator, per_k: int = 64):
    """The reference k-buffer's composite order (HitParticleKBufferT::insert
    as evalKBuffer feeds it) for seeded hit-distance sequences of 1-300 hits
    per K of KBUFFER_SIZES: distances drawn from a few values (many ties, the
    case the compare-and-swap network orders by position), from a
    continuous range, and ascending, descending and constant runs.  Returns
    (k [S], offsets [S+1], hit distances [total], orders [total])."""
    ks, seqs = [], []
    for k in KBUFFER_SIZES:
        for j in range(per_k):
            n = int(rng.integers(1, 301))
            kind = j % 5
            if kind == 0:
                t = rng.integers(0, 4, n).astype(np.float32)
            elif kind == 1:
                t = rng.uniform(0.1, 10.0, n).astype(np.float32)
            elif kind == 2:
                t = np.sort(rng.uniform(0.1, 10.0, n)).astype(np.float32)
            elif kind == 3:
                t = np.sort(rng.uniform(0.1, 10.0, n))[::-1].astype(np.float32)
            else:
                t = np.full(n, 2.5, np.float32)
            ks.append(k)
            seqs.append(np.ascontiguousarray(t))
    with tempfile.TemporaryDirectory() as tmp:
        src, dst = Path(tmp) / "kb.bin", Path(tmp) / "kb.out"
        with open(src, "wb") as fh:
            fh.write(np.array([len(seqs)], np.int32).tobytes())
            for k, t in zip(ks, seqs):
                fh.write(np.array([k, t.size], np.int32).tobytes())
                fh.write(t.tobytes())
        subprocess.run([str(DRIVER), "kbuffer", str(src), str(dst)], check=True)
        orders = np.fromfile(dst, dtype=np.int32)
    offsets = np.concatenate([[0], np.cumsum([t.size for t in seqs])]).astype(np.int64)
    return np.array(ks, np.int32), offsets, np.concatenate(seqs), orders


def main(reference: Path) -> None:
    subprocess.run(["make", "-C", str(REPO / "oracle"), "ref", f"REF={reference}"], check=True)
    rng = np.random.default_rng(20261202)
    tiles = []
    for _ in range(TILES):
        rows, colours, origin, axis, u, v = draw_tile(rng)
        rays = np.zeros((RAYS, 8), np.float32)
        for i in range(RAYS):
            while True:
                o = origin + rng.uniform(-0.02, 0.02, 3)
                a, b = rng.uniform(-0.33, 0.33, 2)
                d = axis + a * u + b * v
                d /= np.linalg.norm(d)
                d32 = d.astype(np.float32)
                o32 = o.astype(np.float32)
                if ray_is_clear(rows, o32.astype(np.float64), d32.astype(np.float64)):
                    break
            rays[i, 0:3], rays[i, 3:6] = o32, d32
            rays[i, 6], rays[i, 7] = 0.0, aabb_exit(o32, d32)
        grads = rng.normal(0.0, 1.0, (RAYS, 13)).astype(np.float32)
        grads[:, 4] *= 0.2                       # hit distance
        grads[:, 8] *= 0.05                      # sum w t^2
        grads[:, 10:12] *= 0.1                   # inverse-depth moments
        grads[:, 12] *= 0.2                      # dL/dt*
        tiles.append((rows, colours, rays, grads))

    with tempfile.TemporaryDirectory() as tmp:
        src, dst = Path(tmp) / "in.bin", Path(tmp) / "out.bin"
        with open(src, "wb") as f:
            f.write(np.array([TILES, RAYS], np.int32).tobytes())
            for rows, colours, rays, grads in tiles:
                f.write(np.array([rows.shape[0]], np.int32).tobytes())
                f.write(rows.tobytes())
                f.write(colours.tobytes())
                f.write(np.concatenate([rays, grads], axis=1).astype(np.float32).tobytes())
        subprocess.run([str(DRIVER), str(src), str(dst)], check=True)
        out = np.fromfile(dst, dtype=np.float32)

    sh_dirs, sh_coeffs, sh_rgb = sh_goldens(rng)
    proj_points, proj_out = projection_goldens(rng)
    kb_k, kb_offsets, kb_hit_t, kb_order = kbuffer_goldens(rng)
    ut_poses, ut_centres, ut_rows, ut_out = ut_goldens(rng)
    counts = np.array([t[0].shape[0] for t in tiles], np.int32)
    fwd_a, fwd_b, grad, grad_rgb, abs_world = [], [], [], [], []
    at = 0
    for (rows, _c, _r, _g), m in zip(tiles, counts):
        per_ray = out[at:at + RAYS * 27].reshape(RAYS, 27)
        at += RAYS * 27
        fwd_a.append(per_ray[:, :6])
        fwd_b.append(per_ray[:, 6:])
        grad.append(out[at:at + m * 32].reshape(m, 32))
        at += m * 32
        grad_rgb.append(out[at:at + m * 3].reshape(m, 3))
        at += m * 3
        abs_world.append(out[at:at + m * 3].reshape(m, 3))
        at += m * 3
    assert at == out.size, (at, out.size)
    np.savez_compressed(
        HERE / "hit_golden.npz",
        counts=counts,
        rows=np.concatenate([t[0] for t in tiles]),
        colours=np.concatenate([t[1] for t in tiles]),
        rays=np.stack([t[2] for t in tiles]),
        grads=np.stack([t[3] for t in tiles]),
        fwd_a=np.stack(fwd_a),
        fwd_b=np.stack(fwd_b),
        grad=np.concatenate(grad),
        grad_rgb=np.concatenate(grad_rgb),
        abs_world=np.concatenate(abs_world),
        sh_dirs=sh_dirs,
        sh_coeffs=sh_coeffs,
        sh_rgb=sh_rgb,
        proj_points=proj_points,
        proj_out=proj_out,
        kb_k=kb_k,
        kb_offsets=kb_offsets,
        kb_hit_t=kb_hit_t,
        kb_order=kb_order,
        ut_poses=ut_poses,
        ut_centres=ut_centres,
        ut_rows=ut_rows,
        ut_out=ut_out,
    )
    print(f"{TILES} tiles x {RAYS} rays, {int(counts.sum())} Gaussians; "
          f"hits per ray {float(np.stack(fwd_a)[..., 5].mean()):.2f}, "
          f"crossings {int((np.stack(fwd_b)[..., 19] > 0).sum())}")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        sys.exit("usage: make_hit_golden.py REFERENCE_CHECKOUT")
    main(Path(sys.argv[1]).resolve())
