"""Accuracy of the shared elementary functions (gf_elementary.h) against
float64 references, through the oracle's exports."""

import math

import numpy as np
import pytest

import oracle


def _ulp_error(got: float, exact: float) -> float:
    if math.isinf(exact) or math.isinf(got):
        return 0.0 if got == exact else math.inf
    e32 = np.float32(exact)
    if e32 == 0.0:
        return abs(got) / float(np.finfo(np.float32).smallest_subnormal)
    spacing = float(np.spacing(np.abs(e32)))
    return abs(float(got) - exact) / spacing


@pytest.fixture(scope="module")
def lib():
    return oracle.load()


def test_expf_accuracy(lib):
    rng = np.random.default_rng(0)
    xs = np.concatenate([rng.uniform(-20, 5, 20000), rng.uniform(-103, -80, 2000), np.linspace(-9, 0, 4001),
                         [0.0, -0.0, 1.0, -1.0, 88.0, -4.5, -87.3]]).astype(np.float32)
    worst = 0.0
    for x in xs:
        got = lib.oracle_expf(float(x))
        worst = max(worst, _ulp_error(got, math.exp(float(x))))
    assert worst <= 2.0, worst
    assert lib.oracle_expf(-200.0) == 0.0
    assert math.isinf(lib.oracle_expf(100.0))
    assert math.isnan(lib.oracle_expf(float("nan")))


def test_logf_accuracy(lib):
    rng = np.random.default_rng(1)
    xs = np.concatenate([np.exp(rng.uniform(-80, 80, 20000)), rng.uniform(0.5, 2.0, 5000),
                         [1.0, 2.0, 0.5, 1e-40, 255.0, 3.4e38]]).astype(np.float32)
    worst = 0.0
    for x in xs:
        got = lib.oracle_logf(float(x))
        worst = max(worst, _ulp_error(got, math.log(float(x))))
    assert worst <= 2.0, worst
    assert lib.oracle_logf(1.0) == 0.0
    assert math.isinf(lib.oracle_logf(0.0)) and lib.oracle_logf(0.0) < 0
    assert math.isnan(lib.oracle_logf(-1.0))


def test_atan2f_accuracy(lib):
    rng = np.random.default_rng(2)
    ys = rng.uniform(0, 10, 20000).astype(np.float32)
    xs = rng.uniform(-10, 10, 20000).astype(np.float32)
    worst = 0.0
    for y, x in zip(ys, xs):
        got = lib.oracle_atan2f(float(y), float(x))
        worst = max(worst, _ulp_error(got, math.atan2(float(y), float(x))))
    assert worst <= 2.5, worst
    for y, x in [(0.0, 1.0), (1.0, 0.0), (0.0, -1.0), (1.0, -1e-30), (1e-30, 1.0), (float("inf"), 1.0)]:
        assert abs(lib.oracle_atan2f(y, x) - math.atan2(y, x)) <= 4e-7 * max(1.0, abs(math.atan2(y, x)))
