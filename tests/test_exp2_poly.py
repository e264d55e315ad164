"""The FMA-pipe exponential of the kernel (exp2_poly_x2 in
not-cute-zig_b200/csrc/sm100_ptx.cuh, used only when NCZ_EXP2_EMU_COUNT > 0)
checked against its stated error bound on the CPU.  The coefficients are read
from the header as shipped; the float32 steps are restated in numpy: round e
to n with the 1.5 * 2^23 trick, f = e - n, the degree-4 polynomial in f by
Horner's rule with fused multiply-adds (computed in float64, then rounded
once to float32), then scaled by 2^n."""
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "not-cute-zig_b200", "csrc", "sm100_ptx.cuh")


def coefficients():
    text = open(HEADER).read()
    body = text[text.index("void exp2_poly_x2"):]
    found = dict(re.findall(r"k(C[1-4]) = ([0-9.eE+-]+)f", body[:600]))
    return [np.float32(found[f"C{i}"]) for i in range(1, 5)]


def fma32(a, b, c):
    return (a.astype(np.float64) * b + c).astype(np.float32)


def exp2_poly(e):
    c1, c2, c3, c4 = coefficients()
    e = np.maximum(e.astype(np.float32), np.float32(-125.0))
    r = np.float32(12582912.0)  # 1.5 * 2^23
    t = (e + r).astype(np.float32)
    n = (t - r).astype(np.float32)
    f = fma32(n, np.float32(-1.0), e)
    q = fma32(f, c4, c3)
    q = fma32(q, f, c2)
    q = fma32(q, f, c1)
    q = fma32(q, f, np.float32(1.0))
    return (q.astype(np.float64) * np.exp2(n.astype(np.float64))).astype(np.float32), f


def test_reduction_is_exact_and_in_range():
    e = np.linspace(-125.0, 8.0, 200_001, dtype=np.float32)
    _, f = exp2_poly(e)
    assert np.all(np.abs(f) <= 0.5)
    n = e.astype(np.float64) - f.astype(np.float64)
    assert np.array_equal(n, np.rint(n))  # n is an integer and e - n lost nothing


def test_relative_error_within_the_stated_bound():
    e = np.concatenate([np.linspace(-125.0, 8.0, 2_000_001, dtype=np.float32),
                        np.arange(-125, 9, dtype=np.float32) + np.float32(0.5),
                        np.float32([-1e-7, 1e-7, -0.25, 0.25, -0.4999999, 0.4999999])])
    got, _ = exp2_poly(e)
    want = np.exp2(e.astype(np.float64))
    rel = np.abs(got.astype(np.float64) - want) / want
    assert rel.max() <= 3.8e-6, rel.max()  # stated: 3.7e-6 in f32


def test_exact_at_integers_and_clamped_below():
    e = np.arange(-125, 9, dtype=np.float32)
    got, _ = exp2_poly(e)
    assert np.array_equal(got.astype(np.float64), np.exp2(e.astype(np.float64)))  # 2^0 == 1 held exactly
    low, _ = exp2_poly(np.float32([-np.inf, -300.0, -126.0]))
    assert np.all(low == np.float32(2.0 ** -125))


def coefficients3():
    text = open(HEADER).read()
    body = text[text.index("void exp2_poly3_x2"):]
    found = dict(re.findall(r"k(C[1-3]) = ([0-9.eE+-]+)f", body[:400]))
    return [np.float32(found[f"C{i}"]) for i in range(1, 4)]


def exp2_poly3(e):
    c1, c2, c3 = coefficients3()
    e = np.maximum(e.astype(np.float32), np.float32(-125.0))
    r = np.float32(12582912.0)
    t = (e + r).astype(np.float32)
    n = (t - r).astype(np.float32)
    f = fma32(n, np.float32(-1.0), e)
    q = fma32(f, c3, c2)
    q = fma32(q, f, c1)
    q = fma32(q, f, np.float32(1.0))
    return (q.astype(np.float64) * np.exp2(n.astype(np.float64))).astype(np.float32)


def test_degree3_relative_error_within_a_fifth_of_the_f16_unit_roundoff():
    """exp2_poly3_x2 (NCZ_EXP2_EMU_DEGREE=3): stated 1.02e-4, under 2^-11 / 4."""
    e = np.concatenate([np.linspace(-125.0, 8.0, 2_000_001, dtype=np.float32),
                        np.arange(-125, 9, dtype=np.float32) + np.float32(0.5)])
    got = exp2_poly3(e)
    want = np.exp2(e.astype(np.float64))
    rel = np.abs(got.astype(np.float64) - want) / want
    assert rel.max() <= 1.03e-4, rel.max()
    assert rel.max() < 2.0 ** -11 / 4
    ints = np.arange(-125, 9, dtype=np.float32)
    assert np.array_equal(exp2_poly3(ints).astype(np.float64), np.exp2(ints.astype(np.float64)))
