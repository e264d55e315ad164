"""Shared case generation and parity checks for the flash-attention tests.

Inputs are generated on the host by the oracle's generators (bit-identical
f16), uploaded for the kernel, and compared with the oracle (a restatement of
computeFlashReferenceOne, src/main.zig:1271-1307) on the active region.

Tolerance (north star: max-abs 2e-3 and max-rel 1e-2), on every active element:

- |gpu - oracle| <= 2e-3;
- the per-element relative error rel = |gpu - oracle| / max(|oracle|, 1e-3)
  <= 1e-2, except for the part of the difference that the reference's own
  algorithm makes: its GPU kernels round every weight P to f16 before the PV
  product (src/flash_h64_bn32.zig:185), the oracle (src/main.zig:1271-1307)
  does not, and that rounding changes an output by at most u * sum_k w_k |v_k|
  (u = 2^-11, the f16 unit roundoff; the oracle reports the sum per element
  as `mag`).  So each element must satisfy
      |gpu - oracle| <= 1e-2 * max(|oracle|, 1e-3) + u * mag.
  Where an output is near zero (|O| < 1e-2, about 1 % of the elements of an
  N(0, s^2) workload) the rounding term is the larger one: the plain
  per-element rel then exceeds 1e-2 by design, and the check logs how often;
- the norm-relative error max|gpu - oracle| / max|oracle| <= 1e-2.

The reference's own checks (0.008 smoke, src/main.zig:279; 0.02 compare,
src/main.zig:1042) are looser and implied.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass, field

import numpy as np

ATOL = 2e-3
RTOL = 1e-2
NORM_RTOL = 1e-2
REL_FLOOR = 1e-3
# Unit roundoff of the weights P before the PV product: f16 as the reference
# kernels round them (src/flash_h64_bn32.zig:185), bf16 for bf16 inputs.
P_UNIT_F16 = 2.0 ** -11
P_UNIT_BF16 = 2.0 ** -8
# bf16 inputs (an extension: the reference is f16 only).  The kernel rounds P
# to bf16 before PV (a tensor-core MMA takes A and B of one type), 3 mantissa
# bits fewer than f16, so the bound is 4x the f16 one; the oracle reads the same
# bf16 Q/K/V bits and does not round P.
ATOL_BF16 = 8e-3

# The reference smoke cases, src/main.zig:190-193:
# (batch_heads, seq_len, head_dim, q/k/v/o slice strides, causal)
SMOKE_CASES = [
    (2, 32, 32, (32 * 32 + 17, 32 * 32 + 19, 32 * 32 + 23, 32 * 32 + 29), True),
    (1, 17, 16, (17 * 16 + 3, 17 * 16 + 5, 17 * 16 + 7, 17 * 16 + 11), False),
    (3, 49, 16, (49 * 16, 49 * 16 + 13, 49 * 16 + 17, 49 * 16 + 19), True),
    (1, 33, 64, (33 * 64 + 3, 33 * 64 + 5, 33 * 64 + 7, 33 * 64 + 11), False),
]

# The reference compare shapes, src/main.zig:141-170 (= tools/cuda_baselines.cu:780-794):
# (batch_heads, seq_len, head_dim, causal)
COMPARE_CASES = [
    (2, 32, 16, False), (2, 32, 32, True), (2, 64, 16, False), (2, 64, 32, True), (2, 128, 32, True),
    (8, 128, 16, False), (8, 128, 32, True), (8, 256, 16, False), (8, 256, 32, True), (16, 256, 32, False),
    (16, 512, 32, True), (8, 256, 64, False), (8, 512, 64, True), (16, 512, 64, False), (8, 1024, 64, True),
]


@dataclass
class Problem:
    bh: int
    seq: int
    d: int
    strides: tuple  # q, k, v, o slice strides (elements)
    causal: bool
    scale: float
    row_strides: tuple = None  # q, k, v, o row strides (None = head_dim)
    q: np.ndarray = field(default=None, repr=False)
    k: np.ndarray = field(default=None, repr=False)
    v: np.ndarray = field(default=None, repr=False)

    @property
    def rows(self):
        return self.row_strides if self.row_strides is not None else (self.d,) * 4


def pattern_problem(bh, seq, d, strides, causal, oracle):
    """fillFlashInput inputs (src/main.zig:219-221): Q (3,1,1/8), K (5,2,1/16), V (7,3,1/32)."""
    qs, ks, vs, os_ = strides
    p = Problem(bh, seq, d, strides, causal, 1.0 / math.sqrt(d))
    p.q = oracle.fill_pattern(bh * qs, 3, 1, 0.125)
    p.k = oracle.fill_pattern(bh * ks, 5, 2, 0.0625)
    p.v = oracle.fill_pattern(bh * vs, 7, 3, 0.03125)
    return p


def normal_problem(bh, seq, d, causal, seed, oracle, std=0.5, k_mul=1.0, strides=None, scale=None):
    """Contiguous N(0, std^2) inputs from splitmix64(seed), (seed, seed+1, seed+2) for Q, K, V."""
    n = bh * seq * d
    st = strides or (seq * d,) * 4
    p = Problem(bh, seq, d, st, causal, scale if scale is not None else 1.0 / math.sqrt(d))
    p.q = oracle.fill_normal(bh * st[0], seed * 3 + 0, 0.0, std)
    p.k = oracle.fill_normal(bh * st[1], seed * 3 + 1, 0.0, std * k_mul)
    p.v = oracle.fill_normal(bh * st[2], seed * 3 + 2, 0.0, std)
    del n
    return p


def normal_problem_bf16(bh, seq, d, causal, seed, oracle, std=0.5, k_mul=1.0, strides=None, scale=None):
    """normal_problem with bf16 Q/K/V (uint16 bit patterns, same random stream)."""
    st = strides or (seq * d,) * 4
    p = Problem(bh, seq, d, st, causal, scale if scale is not None else 1.0 / math.sqrt(d))
    p.q = oracle.fill_normal_bf16(bh * st[0], seed * 3 + 0, 0.0, std)
    p.k = oracle.fill_normal_bf16(bh * st[1], seed * 3 + 1, 0.0, std * k_mul)
    p.v = oracle.fill_normal_bf16(bh * st[2], seed * 3 + 2, 0.0, std)
    return p


class Reference(np.ndarray):
    """The oracle's output, with `.mag` (per element sum_k w_k |v_k|, same layout)."""

    mag = None


def reference(p: Problem, oracle, slices=None, rows=None):
    """Oracle output (float32, bh * o_stride elements, zeros outside the active
    region) as a Reference carrying the per-element magnitude `.mag`.

    slices: optional list of slice indices to compute (others stay 0)."""
    qs, ks, vs, os_ = p.strides
    out = np.zeros(p.bh * os_, dtype=np.float32)
    mag = np.zeros(p.bh * os_, dtype=np.float32)
    if slices is None:
        oracle.flash_reference(p.q, p.k, p.v, batch_heads=p.bh, seq_len=p.seq, head_dim=p.d, q_stride=qs,
                               k_stride=ks, v_stride=vs, o_stride=os_, scale=p.scale, causal=p.causal,
                               row_strides=p.rows, out=out, rows=rows, mag=mag)
    else:
        for s in slices:
            oracle.flash_reference(p.q[s * qs:], p.k[s * ks:], p.v[s * vs:], batch_heads=1, seq_len=p.seq,
                                   head_dim=p.d, q_stride=qs, k_stride=ks, v_stride=vs, o_stride=os_,
                                   scale=p.scale, causal=p.causal, row_strides=p.rows, out=out[s * os_:],
                                   rows=rows, mag=mag[s * os_:])
    ref = out.view(Reference)
    ref.mag = mag
    return ref


def active_index(p: Problem, slices=None, rows=None):
    """Flat indices of the active O elements (slice, row, col < d)."""
    os_ = p.strides[3]
    orow = p.rows[3]
    sl = np.arange(p.bh) if slices is None else np.asarray(slices)
    r0, r1 = rows if rows is not None else (0, p.seq)
    r = np.arange(r0, r1)
    c = np.arange(p.d)
    return (sl[:, None, None] * os_ + r[None, :, None] * orow + c[None, None, :]).reshape(-1)


def compare(got: np.ndarray, want: np.ndarray, idx: np.ndarray):
    g = got[idx].astype(np.float64)
    w = np.asarray(want)[idx].astype(np.float64)
    assert np.all(np.isfinite(g)), "non-finite output"
    err = np.abs(g - w)
    max_abs = float(err.max()) if err.size else 0.0
    norm_rel = max_abs / max(float(np.abs(w).max()), 1e-30) if err.size else 0.0
    return max_abs, norm_rel


def elementwise(got, want, idx, p_unit=P_UNIT_F16, rtol=RTOL):
    """Per-element figures over idx: max rel = |a-b| / max(|b|, REL_FLOOR), the
    count of elements with rel > rtol, and the worst ratio of |a-b| to the
    allowance rtol * max(|b|, REL_FLOOR) + p_unit * mag (None without mag)."""
    g = got[idx].astype(np.float64)
    w = np.asarray(want)[idx].astype(np.float64)
    err = np.abs(g - w)
    if err.size == 0:
        return 0.0, 0, 0.0
    rel = err / np.maximum(np.abs(w), REL_FLOOR)
    mag = getattr(want, "mag", None)
    ratio = None
    if mag is not None:
        allow = rtol * np.maximum(np.abs(w), REL_FLOOR) + p_unit * mag[idx].astype(np.float64)
        ratio = float((err / allow).max())
    return float(rel.max()), int((rel > rtol).sum()), ratio


def check(got, want, idx, what="", atol=ATOL, rtol=NORM_RTOL, p_unit=P_UNIT_F16, o_unit=0.0):
    """The parity gate (module docstring).  o_unit: unit roundoff of a 16-bit
    O (2^-11 f16, 2^-8 bf16), allowed as o_unit * |oracle| on top of atol."""
    max_abs, norm_rel = compare(got, want, idx)
    w = np.abs(np.asarray(want)[idx].astype(np.float64))
    err = np.abs(got[idx].astype(np.float64) - np.asarray(want)[idx].astype(np.float64))
    abs_ok = bool(np.all(err <= atol + o_unit * w)) if err.size else True
    max_rel, n_rel, ratio = elementwise(got, want, idx, p_unit, RTOL)
    log = os.environ.get("NCZ_PARITY_LOG")
    if log:
        with open(log, "a") as f:
            f.write(f"{what}\tmax_abs={max_abs:.3e}\tnorm_rel={norm_rel:.3e}\tmax_rel={max_rel:.3e}"
                    f"\trel_over={n_rel}\tallowance_ratio={ratio if ratio is None else f'{ratio:.3f}'}"
                    f"\telements={idx.size}\n")
    assert abs_ok and norm_rel <= rtol, f"{what}: max_abs={max_abs:.3e} norm_rel={norm_rel:.3e}"
    # o_unit * |b| of a 16-bit O is below rtol * |b|, so the allowance covers it too.
    assert ratio is None or ratio <= 1.0, (f"{what}: per-element error above 1e-2 * max(|b|, 1e-3) + "
                                           f"u * mag (worst ratio {ratio:.3f}, max rel {max_rel:.3e})")
    return max_abs, norm_rel
