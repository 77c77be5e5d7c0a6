"""The oracle's restatement of SOF's HEAD4 / MID8 / TAIL64 compositor
(sofMid8Hierarchy.inl:161-598): every candidate of a tile reaches every
pixel's HEAD exactly once; a scene whose depth order agrees with the tile
order composites exactly as the flat k-buffer of 4; and a scene shuffled in
depth composites differently from it (the hierarchy reorders) but with the
same opacity coverage."""

import dataclasses

import numpy as np

import oracle
from gofish_b200.camera import fisheye_camera
from gofish_b200.scene import IDENTITY_POSE, random_scene
from tests import harness


def _depth_ordered_case(n=48, seed=3):
    rng = np.random.default_rng(seed)
    scene = random_scene(n, 0, seed)
    z = 1.0 + 0.3 * np.arange(n)
    xy = rng.uniform(-0.15, 0.15, (n, 2)) * z[:, None]
    scene = dataclasses.replace(scene, positions=np.column_stack([xy, z]).astype(np.float32),
                                scales=np.full((n, 3), 0.04, np.float32) * z[:, None].astype(np.float32),
                                density=np.full((n, 1), 0.35, np.float32))
    cam = fisheye_camera(64, 64, 200.0)
    return harness.make_case(scene, cam, IDENTITY_POSE.copy())


def _feeds_cover_every_candidate(case, ref):
    pose = oracle.prepare_pose(case.pose)
    ranges = ref["ranges"].reshape(-1, 2)
    checked = 0
    for tile in np.flatnonzero(ranges[:, 1] > ranges[:, 0]):
        feeds = oracle.sof_feeds(case.ocam, pose, case.particles, case.ray_o, case.ray_d, ref["ranges"], ref["ids"],
                                 int(tile))
        want = np.arange(ranges[tile, 0], ranges[tile, 1])
        ty, tx = divmod(int(tile), (case.camera.width + 15) // 16)
        for p, f in enumerate(feeds):
            py, px = ty * 16 + p // 16, tx * 16 + p % 16
            if py < case.camera.height and px < case.camera.width:
                np.testing.assert_array_equal(np.sort(f), want)
                checked += 1
    return checked


def test_every_candidate_is_fed_once():
    case = _dense_case()
    ref = harness.oracle_forward(case, 16, 0)
    assert _feeds_cover_every_candidate(case, ref) > 1000
    assert int(np.diff(ref["ranges"].reshape(-1, 2), axis=1).max()) > 64  # windows overflow and emit


def test_depth_ordered_scene_equals_flat_k4():
    case = _depth_ordered_case()
    flat = harness.oracle_forward(case, 4, 0)
    sof = harness.oracle_forward(case, oracle.SOF_HIERARCHY, 0)
    np.testing.assert_array_equal(sof["rgba"].view(np.uint32), flat["rgba"].view(np.uint32))
    np.testing.assert_array_equal(sof["hit_count"], flat["hit_count"])
    assert float(sof["rgba"][..., 3].max()) > 0.5


def _dense_case():
    case = harness.small_case(seed=9, n=6000, size=96)
    scene = dataclasses.replace(case.scene, scales=case.scene.scales * np.float32(5.0))
    return harness.make_case(scene, case.camera, case.pose)


def test_hierarchy_reorders_a_dense_scene():
    case = _dense_case()
    flat = harness.oracle_forward(case, 4, 0)
    sof = harness.oracle_forward(case, oracle.SOF_HIERARCHY, 0)
    full = harness.oracle_forward(case, 32, 0)
    assert not np.array_equal(sof["rgba"], flat["rgba"])
    # closer to the deep k-buffer than the flat 4-buffer is (the hierarchy sorts deeper windows)
    err_sof = np.abs(sof["rgba"] - full["rgba"]).mean()
    err_flat = np.abs(flat["rgba"] - full["rgba"]).mean()
    assert err_sof < err_flat
    np.testing.assert_allclose(sof["rgba"][..., 3], flat["rgba"][..., 3], atol=0.02)
