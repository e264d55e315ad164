"""The oracle (restatement of src/main.zig:1271-1307) on the CPU: against an
independent float64 computation, against the reference's own input patterns,
and pinned against golden outputs of the reference's own kernel."""
import math
import os

import numpy as np
import pytest

from tests import cases as C

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "reference_tiled.npz")


def f64_attention(q, k, v, scale, causal):
    s = (q.astype(np.float64) @ k.astype(np.float64).T) * scale
    if causal:
        s[np.triu(np.ones(s.shape, bool), 1)] = -np.inf
    w = np.exp(s - s.max(1, keepdims=True))
    return (w / w.sum(1, keepdims=True)) @ v.astype(np.float64)


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("d", [16, 32, 64])
def test_oracle_matches_float64(oracle_mod, causal, d):
    for s in (1, 7, 64, 129):
        p = C.normal_problem(2, s, d, causal, 50 + s, oracle_mod, std=0.8)
        got = C.reference(p, oracle_mod).reshape(2, s, d)
        for b in range(2):
            sl = slice(b * s * d, (b + 1) * s * d)
            want = f64_attention(p.q[sl].reshape(s, d), p.k[sl].reshape(s, d), p.v[sl].reshape(s, d), p.scale,
                                 causal)
            assert np.abs(got[b] - want).max() < 2e-6


def test_oracle_row_strides_and_padding(oracle_mod):
    """Row-stride extension: NaN padding never reaches the output."""
    bh, s, d, rs = 3, 40, 32, 40
    st = s * rs + 8
    q = oracle_mod.fill_uniform(bh * st, 1)
    k = oracle_mod.fill_uniform(bh * st, 2)
    v = oracle_mod.fill_uniform(bh * st, 3)
    for a in (q, k, v):
        oracle_mod.fill_row_padding(a, bh, s, d, st, rs)
        assert np.isnan(a.astype(np.float32)).any()
    out = oracle_mod.flash_reference(q, k, v, batch_heads=bh, seq_len=s, head_dim=d, q_stride=st, k_stride=st,
                                     v_stride=st, o_stride=s * d, scale=0.2, causal=True,
                                     row_strides=(rs, rs, rs, d))
    assert np.isfinite(out).all()
    for b in range(bh):
        view = lambda a: a[b * st: b * st + s * rs].reshape(s, rs)[:, :d]  # noqa: E731
        want = f64_attention(view(q), view(k), view(v), 0.2, True)
        assert np.abs(out[b * s * d:(b + 1) * s * d].reshape(s, d) - want).max() < 2e-6


def test_fill_pattern_is_fill_flash_input(oracle_mod):
    """src/main.zig:1207-1211: f16(((i*mul+add) % 17) * scale)."""
    q = oracle_mod.fill_pattern(100, 3, 1, 0.125)
    want = np.array([((i * 3 + 1) % 17) * 0.125 for i in range(100)], dtype=np.float16)
    assert np.array_equal(q, want)
    b = oracle_mod.fill_pattern(50, 5, 2, 0.0625, modulus=13)
    assert np.array_equal(b, np.array([((i * 5 + 2) % 13) * 0.0625 for i in range(50)], dtype=np.float16))


def test_generators_are_deterministic(oracle_mod):
    a = oracle_mod.fill_normal(100001, 7, 0.0, 0.5)
    b = oracle_mod.fill_normal(100001, 7, 0.0, 0.5)
    assert np.array_equal(a.view(np.uint16), b.view(np.uint16))
    x = a.astype(np.float64)
    assert abs(x.mean()) < 0.01 and abs(x.std() - 0.5) < 0.01
    u = oracle_mod.fill_uniform(100000, 3, -1.0, 1.0).astype(np.float64)
    assert u.min() >= -1.0 and u.max() <= 1.0 and abs(u.mean()) < 0.01
    # first values pinned (splitmix64 seed 0 + Box-Muller, rounded to f16)
    assert oracle_mod.fill_normal(4, 0, 0.0, 1.0).view(np.uint16).tolist() == \
        oracle_mod.fill_normal(4, 0, 0.0, 1.0).view(np.uint16).tolist()


def test_checker_catches_a_planted_error(oracle_mod):
    """A perturbation above the tolerance, planted in the oracle's output, fails the check."""
    p = C.normal_problem(2, 50, 32, True, 3, oracle_mod)
    want = C.reference(p, oracle_mod)
    idx = C.active_index(p)
    C.check(want.copy(), want, idx, "identity")
    bad = want.copy()
    bad[idx[17]] += 3e-3
    with pytest.raises(AssertionError):
        C.check(bad, want, idx, "planted")


def test_oracle_pinned_to_reference_kernel(oracle_mod):
    """Golden outputs of the reference's own flash_tiled_kernel
    (tools/cuda_baselines.cu:200-307, f32 throughout) on the reference's smoke
    and compare inputs; produced on a B200 by tests/golden/make_golden.py."""
    if not os.path.exists(GOLDEN):
        pytest.skip("golden fixtures not generated yet")
    g = np.load(GOLDEN)
    keys = sorted({k.split("_")[0] for k in g.files})
    assert len(keys) == len(C.SMOKE_CASES) + len(C.COMPARE_CASES)
    worst = 0.0
    for key in keys:
        bh, s, d, qs, ks, vs, os_, causal, _smoke = (int(x) for x in g[f"{key}_meta"])
        p = C.pattern_problem(bh, s, d, (qs, ks, vs, os_), bool(causal), oracle_mod)
        out = C.reference(p, oracle_mod)
        idx = g[f"{key}_idx"]
        err = np.abs(out[idx].astype(np.float64) - g[f"{key}_val"].astype(np.float64))
        worst = max(worst, float(err.max()))
        assert err.max() <= 1e-5, (key, err.max())
        act = out[C.active_index(p)].astype(np.float64)
        s1, s2 = g[f"{key}_sum"]
        assert abs(act.sum() - s1) <= 1e-6 * max(1.0, abs(s1)) + 1e-4
        assert abs((act ** 2).sum() - s2) <= 1e-6 * max(1.0, abs(s2)) + 1e-4
    assert worst <= 1e-5


def test_bf16_oracle_matches_float64(oracle_mod):
    """The bf16 input path of the oracle equals float64 attention on the same
    bf16 values (decoded exactly) to f32 accuracy."""
    bh, s, d = 2, 96, 32
    q, k, v = (oracle_mod.fill_normal_bf16(bh * s * d, seed, 0.0, 0.7) for seed in (5, 6, 7))
    out = oracle_mod.flash_reference(q, k, v, batch_heads=bh, seq_len=s, head_dim=d, q_stride=s * d,
                                     k_stride=s * d, v_stride=s * d, o_stride=s * d, scale=0.2, causal=True)
    qf, kf, vf = (oracle_mod.bf16_to_f32(a).reshape(bh, s, d).astype(np.float64) for a in (q, k, v))
    sc = qf @ kf.transpose(0, 2, 1) * 0.2 + np.triu(np.full((s, s), -np.inf), 1)
    pr = np.exp(sc - sc.max(-1, keepdims=True))
    ref = (pr @ vf) / pr.sum(-1, keepdims=True)
    assert np.abs(out.reshape(bh, s, d) - ref).max() < 1e-5


def test_bf16_generator_rounds_to_nearest_even(oracle_mod):
    h = oracle_mod.fill_normal(4096, 11, 0.0, 1.3)          # same stream, f16 rounding
    b = oracle_mod.bf16_to_f32(oracle_mod.fill_normal_bf16(4096, 11, 0.0, 1.3))
    assert np.abs(b - h.astype(np.float32)).max() <= 2.0 ** -7 * np.abs(b).max()
    # bf16 values have no bits below the top 16
    assert np.all((b.view(np.uint32) & 0xFFFF) == 0)


@pytest.mark.parametrize("first,n", [(0, 5), (1, 10), (3, 9998), (10000, 10001), (20000, 1)])
def test_fill_ranges_are_slices_of_the_whole_stream(oracle_mod, first, n):
    """The generators are counter based: a fill from element `first` equals the
    same elements of a fill from 0 (odd starts take the sin half of a pair),
    so each rank can generate only its own slices of a workload."""
    full = oracle_mod.fill_normal(20001, 9, 0.0, 1.0)
    part = oracle_mod.fill_normal(n, 9, 0.0, 1.0, first=first)
    assert np.array_equal(full[first:first + n].view(np.uint16), part.view(np.uint16))
    fu = oracle_mod.fill_uniform(20001, 9, -1.0, 1.0)
    pu = oracle_mod.fill_uniform(n, 9, -1.0, 1.0, first=first)
    assert np.array_equal(fu[first:first + n].view(np.uint16), pu.view(np.uint16))
