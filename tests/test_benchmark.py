"""benchmark.py / compare.py host logic on the CPU: the reference's rate
formulas (src/benchmark.zig:79-86), the compare record schema
(src/main.zig:873-881) and fillFlashInput (src/main.zig:1207-1211)."""
import importlib
import json

import numpy as np
import pytest


@pytest.fixture(scope="module")
def bench():
    return importlib.import_module("not-cute-zig_b200.benchmark")


@pytest.fixture(scope="module")
def compare():
    return importlib.import_module("not-cute-zig_b200.compare")


def test_summarize_rates_follow_the_reference_formulas(bench):
    r = bench.summarize([2.0, 1.0, 3.0], bytes_processed=4_000_000_000, flops_processed=6_000_000_000_000)
    assert (r.mean_ms, r.min_ms, r.max_ms) == (2.0, 1.0, 3.0)
    assert r.throughput_gbps == pytest.approx(4e9 / (2.0 * 1e6))  # 2000 GB/s
    assert r.tflops == pytest.approx(6e12 / (2.0 * 1e9))          # 3000 TFLOP/s
    assert bench.summarize([1.0]).tflops is None
    with pytest.raises(ValueError):
        bench.summarize([])


def test_record_keeps_the_reference_field_order(bench):
    r = bench.summarize([1.5], bytes_processed=10, flops_processed=20)
    rec = r.record("flash_attention", "not_cute_zig_b200", "batch_heads=2,seq=32,head=16,causal=false", True, 10, 20,
                   1e-4, gpus=1, max_rel_error=2e-3)
    keys = list(rec)
    assert keys[:12] == ["kernel", "implementation", "shape", "correct", "mean_ms", "min_ms", "max_ms", "gbps",
                         "tflops", "bytes", "flops", "max_abs_error"]
    assert rec["gpus"] == 1 and rec["max_rel_error"] == 2e-3
    json.dumps(rec)


def test_emit_writes_jsonl(bench, tmp_path):
    p = tmp_path / "out.jsonl"
    bench.emit([{"a": 1}, {"b": 2}], str(p))
    assert [json.loads(x) for x in p.read_text().splitlines()] == [{"a": 1}, {"b": 2}]


def test_fill_flash_input_matches_the_oracle(compare, oracle_mod):
    for mul, add, scale in ((3, 1, 0.125), (5, 2, 0.0625), (7, 3, 0.03125)):
        assert np.array_equal(compare.fill_flash_input(1000, mul, add, scale),
                              oracle_mod.fill_pattern(1000, mul, add, scale))


def test_reference_shape_list(compare):
    from tests import cases as C

    assert compare.REFERENCE_SHAPES == C.COMPARE_CASES


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("row", [0, 40])
def test_compare_cross_check_agrees_with_the_oracle(compare, oracle_mod, causal, row):
    """compare.py judges correctness against its own fp32 torch attention; on the
    CPU that reference must agree with the oracle (float32 rounding only), also
    with padded rows (--row-stride)."""
    torch = pytest.importorskip("torch")
    bh, s, d = 3, 77, 32
    r = row or d
    rng = np.random.default_rng(5)
    q, k, v = (rng.standard_normal(bh * s * r).astype(np.float16) for _ in range(3))
    scale = d ** -0.5
    got = compare.torch_attention(*(torch.from_numpy(a) for a in (q, k, v)), bh, s, d, scale, causal, row).numpy()
    want = oracle_mod.flash_reference(q, k, v, batch_heads=bh, seq_len=s, head_dim=d, q_stride=s * r, k_stride=s * r,
                                      v_stride=s * r, o_stride=s * d, scale=scale, causal=causal,
                                      row_strides=(r, r, r, d))
    assert np.allclose(got, want, atol=2e-5, rtol=1e-4), float(np.abs(got - want).max())


def test_host_reference_time(compare):
    """cpu_ms: the cross-check attention timed on the host CPU."""
    torch = pytest.importorskip("torch")
    q, k, v = (torch.randn(2 * 64 * 32).half() for _ in range(3))
    ms = compare.host_reference_ms(q, k, v, 2, 64, 32, 32 ** -0.5, True)
    assert 0.0 < ms < 60_000.0


def test_join_table_pairs_our_records_with_each_baseline(compare, tmp_path):
    """--join: one row per (kernel, shape, other implementation), ratio other / ours;
    multi-GPU records and shapes without a record of ours are left out."""
    shape = "batch_heads=8,seq=1024,head=64,causal=true"
    recs = [
        {"kernel": "flash_attention", "implementation": compare.OURS, "shape": shape, "mean_ms": 0.02, "correct": True},
        {"kernel": "flash_attention", "implementation": compare.OURS, "shape": shape, "mean_ms": 0.5, "correct": True,
         "gpus": 2},
        {"kernel": "flash_attention", "implementation": "torch_sdpa_flash", "shape": shape, "mean_ms": 0.05,
         "correct": True},
        {"kernel": "flash_attention", "implementation": "cuda_wmma", "shape": shape, "mean_ms": 0.4, "correct": False},
        {"kernel": "flash_attention", "implementation": "torch_sdpa_math", "shape": "other", "mean_ms": 1.0,
         "correct": True},
    ]
    a, b = tmp_path / "a.jsonl", tmp_path / "b.jsonl"
    a.write_text("\n".join(json.dumps(r) for r in recs[:2]) + "\nnot json\n")
    b.write_text("\n".join(json.dumps(r) for r in recs[2:]) + "\n")
    rows = compare.join_table(compare.read_records([str(a), str(b)]))
    assert len(rows) == 4
    assert "| cuda_wmma | 0.0200 | 0.4000 | 20.00x | no |" in rows[2]
    assert "| torch_sdpa_flash | 0.0200 | 0.0500 | 2.50x | yes |" in rows[3]
