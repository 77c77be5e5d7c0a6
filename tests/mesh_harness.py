"""Shared inputs of the opacity-field tests: a small scene, fisheye training
cameras on a ring, query points (sites plus random points), and the same
views in the oracle's form."""

from __future__ import annotations

import dataclasses
import math

import numpy as np

import oracle
from gofish_b200.camera import fisheye_camera, random_kb_coefficients
from gofish_b200.mesh.cameras import TrainingCamera, fisheye_training_camera
from gofish_b200.mesh.shape import EffectiveShape, effective_shape
from gofish_b200.mesh.sites import generate_sites
from gofish_b200.scene import look_outward_pose, random_scene

from tests.harness import oracle_camera


@dataclasses.dataclass
class FieldCase:
    shape: EffectiveShape
    cameras: list[TrainingCamera]
    views: list          # oracle views: (camera, pose7, ray_o [H,W,3], mask [H,W] or None)
    points: np.ndarray   # [Q,3] float32


def field_case(seed: int = 11, n: int = 3000, size: int = 96, num_views: int = 4, site_gaussians: int = 1500,
               extra_points: int = 3000, masked: bool = True, scale_boost: float = 3.0, r_max: float = 3.0,
               ring: float = 2.0) -> FieldCase:
    scene = random_scene(n, 0, seed, r_min=1.0, r_max=r_max)
    scales = scene.scales * np.float32(scale_boost)
    shape = effective_shape(scene.positions, scales, scene.rotations, scene.density)
    rng = np.random.default_rng(seed + 7)
    cam = fisheye_camera(size, size, 200.0, random_kb_coefficients(rng, 200.0))
    cameras, views = [], []
    o, _d, _valid = cam.rays()
    for v in range(num_views):
        yaw = 2.0 * math.pi * v / num_views + 0.3
        centre = np.array([ring * math.cos(yaw), ring * math.sin(yaw), 0.1 * v])
        pose = look_outward_pose(centre, yaw)
        tc = fisheye_training_camera(v, cam, pose, masked=masked)
        cameras.append(tc)
        mask = None if tc.physical_mask is None else tc.physical_mask.numpy().copy()
        views.append((oracle_camera(cam), pose, np.ascontiguousarray(o[0], dtype=np.float32), mask))
    sub = dataclasses.replace(shape, positions=shape.positions[:site_gaussians],
                              density=shape.density[:site_gaussians], factor=shape.factor[:site_gaussians],
                              inverse_factor=shape.inverse_factor[:site_gaussians],
                              sigma_max=shape.sigma_max[:site_gaussians], retained=shape.retained[:site_gaussians])
    sites = generate_sites(sub).points
    u = rng.standard_normal((extra_points, 3))
    u /= np.linalg.norm(u, axis=1, keepdims=True)
    extra = (u * rng.uniform(0.2, r_max + 1.0, (extra_points, 1))).astype(np.float32)
    points = np.ascontiguousarray(np.concatenate([sites, extra]), dtype=np.float32)
    return FieldCase(shape, cameras, views, points)


def oracle_field(case: FieldCase, points: np.ndarray | None = None):
    pts = case.points if points is None else points
    return oracle.evaluate_field(case.views, case.shape.packed_density(), pts)


def oracle_round(case: FieldCase, points: np.ndarray):
    return oracle.bisection_round(case.views, case.shape.packed_density(), points)
