"""The client's float32 wire codec against test/f32-test.el's boundaries."""
import numpy as np

from nelisp_cuda.f32codec import bits_f32, f32_bits

MIN_NORMAL = 1.1754943508222875e-38
STEP = 1.401298464324817e-45


def rt(x):
    return bits_f32(f32_bits(x))


def test_normals_round_trip(f32_fixture):
    x = f32_fixture["normals"]
    assert np.max(np.abs(rt(x) - x) / np.abs(x)) < 1e-7


def test_subnormals_within_half_step(f32_fixture):
    x = f32_fixture["subnormals"]
    assert np.max(np.abs(rt(x) - x) / STEP) <= 0.5


def test_small_stays_small(f32_fixture):
    assert np.max(np.abs(rt(f32_fixture["small"]))) < MIN_NORMAL


def test_underflow_flushes(f32_fixture):
    assert np.all(rt(f32_fixture["flush"]) == 0.0)


def test_overflow_is_signed_infinity(f32_fixture):
    r = rt(f32_fixture["overflow"])
    assert r[0] == np.inf and r[1] == -np.inf


def test_flt_max_stays_finite(f32_fixture):
    m = rt(f32_fixture["flt_max"])[0]
    assert np.isfinite(m) and m > 3.4e38


def test_zero_and_nan():
    assert f32_bits(0.0)[0] == 0 and f32_bits(-0.0)[0] == 0
    assert f32_bits(float("nan"))[0] == 0x7FC00000
    assert np.isnan(rt(float("nan"))[0])


def test_softmax_tail_no_blowup(f32_fixture):
    x = f32_fixture["softmax_tail"]
    r = rt(x)
    normal = x >= MIN_NORMAL
    assert np.all(r[normal] / x[normal] <= 1.001)
    assert np.all(np.abs(r[~normal] - x[~normal]) <= 0.5 * STEP)
