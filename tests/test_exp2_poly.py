"""The attention softmax's FMA-pipe exponential (exp2_poly2 in julia1-rs_b200/csrc/attention.cu),
restated in float32 with fused multiply-adds and checked against exact powers of two.

The kernel evaluates part of each block's 2^x this way instead of on the MUFU
(ex2.approx.ftz.f32, whose relative error is of the order of 2^-22). The bound asserted here
is 2^-21.5 relative over the kernel's argument range [-125, 10]. Arguments below -125 give
2^-125 instead of 0 (or a denormal): in a softmax row whose sum is at least 1 that changes the
sum and the output far below their rounding. Masked keys (-inf) never reach it: blocks with a
masked key keep every exponential on the MUFU."""
import numpy as np

COEF = np.array([1.0000001, 6.9314694e-1, 2.4022120e-1, 5.5507131e-2, 9.6755410e-3, 1.3276472e-3],
                dtype=np.float32)  # degree 0 .. 5, as in the kernel


def _fma(a, b, c):
    # float32 fused multiply-add: the float64 product of two float32 values is exact
    return (a.astype(np.float64) * b.astype(np.float64) + c.astype(np.float64)).astype(np.float32)


def exp2_poly(x):
    x = np.maximum(x.astype(np.float32), np.float32(-125.0))
    t = (x + np.float32(12582912.0)).astype(np.float32)
    j = (t + np.float32(-12582912.0)).astype(np.float32)
    f = _fma(j, np.full_like(j, -1.0), x)
    p = np.full_like(f, COEF[5])
    for k in (4, 3, 2, 1, 0):
        p = _fma(p, f, np.full_like(f, COEF[k]))
    bits = (p.view(np.uint32).astype(np.uint64) + (t.view(np.uint32).astype(np.uint64) << 23)) & 0xFFFFFFFF
    return bits.astype(np.uint32).view(np.float32), f, j


def test_range_reduction_is_exact():
    x = np.random.default_rng(0).uniform(-125.0, 10.0, 200000).astype(np.float32)
    _, f, j = exp2_poly(x)
    assert np.all(np.abs(f) <= 0.5)
    assert np.array_equal(f.astype(np.float64) + j.astype(np.float64), x.astype(np.float64))
    assert np.array_equal(j, np.rint(x))


def test_relative_error_bound():
    rng = np.random.default_rng(1)
    x = np.concatenate([np.linspace(-125.0, 10.0, 2_000_001), rng.uniform(-8.0, 8.0, 1_000_000),
                        np.arange(-125, 11)]).astype(np.float32)
    y, _, _ = exp2_poly(x)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(y.astype(np.float64) - ref) / ref
    assert rel.max() < 2.0 ** -21.5, rel.max()
    assert np.all(np.isfinite(y)) and np.all(y > 0)


def test_masked_and_tiny_arguments():
    y, _, _ = exp2_poly(np.array([-np.inf, -1e30, -200.0, -125.0], np.float32))
    assert np.all(y == y[-1]) and abs(y[-1] / 2.0 ** -125 - 1.0) < 1e-6
