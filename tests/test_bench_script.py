"""bench.py's host-side pieces on the CPU: workload table, FLOP formula, the
padded config-3 inputs, and the reference arm's JSON line (the oracle port on
a bounded sample; no GPU involved)."""
import importlib.util
import json
import os
import subprocess
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module")
def bench():
    spec = importlib.util.spec_from_file_location("bench_script", os.path.join(ROOT, "bench.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def test_flops_follow_the_reference_formula(bench):
    """bh * 4 * eff * d, eff = S(S+1)/2 causal, S^2 otherwise (src/main.zig:843-844)."""
    assert bench.flops_of(64, 8192, 64, True) == 64 * 4 * (8192 * 8193 // 2) * 64
    assert bench.flops_of(512, 128, 32, False) == 512 * 4 * 128 * 128 * 32


def test_workload_table(bench):
    assert bench.WORKLOADS["c4"][:4] == (64, 8192, 64, True)
    assert bench.WORKLOADS["c3"][:4] == (512, 128, 32, False)
    assert set(bench.PADDED) <= set(bench.WORKLOADS)
    assert bench.PADDED["c3"]["row"] == 40


def test_padded_inputs_match_the_config3_parity_case(bench, oracle_mod):
    """Seeds 6, 7, 8 and U(-1, 1), as tests/test_flash_gpu.py's config 3 case;
    NaN exactly in the padding columns."""
    bh, s, d, row = 3, 16, 32, 40
    q, k, v = bench.make_padded_inputs(oracle_mod, bh, s, d, row, -1.0, 1.0, 2)
    for a, seed in ((q, 6), (k, 7), (v, 8)):
        want = oracle_mod.fill_uniform(bh * s * row, seed, -1.0, 1.0).reshape(bh, s, row)
        got = a.reshape(bh, s, row)
        assert np.array_equal(got[:, :, :d], want[:, :, :d])
        assert np.isnan(got[:, :, d:]).all() and np.isfinite(got[:, :, :d]).all()


def test_reference_arm_json_line():
    """The reference arm on config 3 (128 rows per slice bound its sample, so
    it ends in seconds; the c4 arm spends its full 90 s CPU budget)."""
    out = subprocess.run([sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
                          "c3", "--steps", "1", "--warmup", "3"], capture_output=True, text=True, timeout=600,
                         cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference" and line["unit"] == "TFLOP/s" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"] == {"value": line["value"], "unit": "TFLOP/s", "h2d_bytes_per_step": 0,
                           "d2h_bytes_per_step": 0}
    assert line["config"]["head_dim"] == 32 and "row stride 40" in line["config"]["workload"]


def test_parity_check_gate(bench, oracle_mod):
    """bench.py's per-rank parity record: the oracle's own output passes; an
    error just inside both bounds (ATOL, and 1e-2 * max(|O|, 1e-3) + u * mag)
    passes, twice that fails; the slice checked is the middle one of the
    rank's range."""
    name = "c2"
    bh, s, d = 3, 300, 64
    _, _, _, causal, std, k_mul, seed, _, _ = bench.WORKLOADS[name]
    hq, hk, hv = bench.make_inputs(oracle_mod, bh, s, d, std, k_mul, seed)
    want = np.zeros(bh * s * d, dtype=np.float32)
    mag = np.zeros_like(want)
    oracle_mod.flash_reference(hq, hk, hv, batch_heads=bh, seq_len=s, head_dim=d, q_stride=s * d, k_stride=s * d,
                               v_stride=s * d, o_stride=s * d, scale=d ** -0.5, causal=causal, out=want, mag=mag)
    old = bench.WORKLOADS[name]
    bench.WORKLOADS[name] = (bh, s, d) + old[3:]
    try:
        rec = bench.parity_check(oracle_mod, name, hq, hk, hv, want.copy(), 5, 5 + bh)
        assert rec["ok"] and rec["max_abs"] == 0.0 and rec["slice"] == 6 and rec["rows"] == [[0, 128], [172, 300]]
        edge = 0.99 * np.minimum(bench.RTOL * np.maximum(np.abs(want), bench.REL_FLOOR) + bench.P_UNIT * mag,
                                 bench.ATOL)
        assert bench.parity_check(oracle_mod, name, hq, hk, hv, want + edge, 5, 5 + bh)["ok"]
        bad = bench.parity_check(oracle_mod, name, hq, hk, hv, want + 2 * edge, 5, 5 + bh)
        assert not bad["ok"] and bad["violations"] > 0 and bad["max_abs"] > bench.ATOL
    finally:
        bench.WORKLOADS[name] = old
