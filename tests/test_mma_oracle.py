"""GEMM + epilogue oracle (oracle/mma_oracle.c) pinned to the reference's
fixtures, and the C ABI's argument validation, on the CPU."""
import numpy as np
import pytest

from tests import mma_cases as M


def ref(oracle_mod, a, b, c, **kw):
    return oracle_mod.mma_reference(a, b, c, **kw)


@pytest.mark.parametrize("k_iters", [1, 4])
@pytest.mark.parametrize("relu", [False, True])
def test_oracle_matches_pipeline_demo_exactly(oracle_mod, k_iters, relu):
    """runEpilogueDemo (k_iters 1, relu) and runPipelinedMma (k_iters 4, none),
    src/main.zig:289-395: alpha 1, beta 0; also beta 1 so C takes part."""
    a, b, c = M.fill_pipeline_inputs(k_iters)
    for alpha, beta in ((1.0, 0.0), (1.0, 1.0), (-0.5, 2.0)):
        got = ref(oracle_mod, a, b, c, alpha=alpha, beta=beta, batch_stride_a=0, batch_stride_b=0, batch_stride_c=0,
                  k_iters=k_iters, epilogue=1 if relu else 0, batches=1)
        want = M.exact_gemm(a, b, c, alpha=alpha, beta=beta, k_iters=k_iters, relu=relu)
        assert np.array_equal(got.astype(np.float64), want)


def test_oracle_matches_batched_and_single_mma_demos_exactly(oracle_mod):
    """runBatchedMma (4 batches, seeds 0..3, B column-major) and runMmaMatmul
    (alpha 1.25, beta 0.5), src/main.zig:396-460 and :1049-1110."""
    parts = [M.fill_mma_inputs(s) for s in range(4)]
    a = np.concatenate([p[0] for p in parts])
    b = np.concatenate([p[1] for p in parts])
    c = np.concatenate([p[2] for p in parts])
    got = ref(oracle_mod, a, b, c, alpha=1.0, beta=0.0, batch_stride_a=256, batch_stride_b=128, batch_stride_c=128,
              k_iters=1, epilogue=0, batches=4, b_col=True)
    want = M.exact_gemm(a, b, c, alpha=1.0, beta=0.0, k_iters=1, batches=4, b_col=True)
    assert np.array_equal(got.astype(np.float64), want)
    a, b, c = M.fill_mma_inputs(0)
    got = ref(oracle_mod, a, b, c, alpha=1.25, beta=0.5, batch_stride_a=0, batch_stride_b=0, batch_stride_c=0,
              k_iters=1, epilogue=0, batches=1, b_col=True)
    assert np.array_equal(got.astype(np.float64), M.exact_gemm(a, b, c, alpha=1.25, beta=0.5, k_iters=1, b_col=True))


def test_oracle_matches_reference_gemm_baseline(oracle_mod):
    """tools/cuda_baselines.cu:580-617 (16x8x16, B row-major, alpha 1, beta 0)."""
    a, b, c = M.gemm_baseline_inputs()
    got = ref(oracle_mod, a, b, c, alpha=1.0, beta=0.0, batch_stride_a=0, batch_stride_b=0, batch_stride_c=0,
              k_iters=1, epilogue=0, batches=1)
    want = M.exact_gemm(a, b, c, alpha=1.0, beta=0.0, k_iters=1)
    assert np.array_equal(got.astype(np.float64), want)
    assert want.max() > 0 and float(want[0]) == sum((i % 5) * 0.25 * ((i * 8) % 7) * 0.125 for i in range(16))


@pytest.mark.parametrize("kind,fn", [(2, M.silu64), (3, M.gelu64)])
def test_oracle_activations_follow_device_formulas(oracle_mod, kind, fn):
    """silu / gelu of src/device.zig:62-80 on a spread of pre-activations (f32
    rounding of each step: within a few ulp of the float64 formula)."""
    rng = np.random.default_rng(5)
    a = rng.uniform(-1, 1, 256).astype(np.float16)
    b = rng.uniform(-1, 1, 128).astype(np.float16)
    c = rng.uniform(-4, 4, 128).astype(np.float32)
    got = ref(oracle_mod, a, b, c, alpha=1.5, beta=1.0, batch_stride_a=0, batch_stride_b=0, batch_stride_c=0,
              k_iters=1, epilogue=kind, batches=1)
    lin = ref(oracle_mod, a, b, c, alpha=1.5, beta=1.0, batch_stride_a=0, batch_stride_b=0, batch_stride_c=0,
              k_iters=1, epilogue=0, batches=1)
    want = fn(lin)
    assert np.allclose(got, want, rtol=2e-6, atol=1e-6)


def test_oracle_unknown_epilogue_is_identity(oracle_mod):
    a, b, c = M.fill_pipeline_inputs(2)
    kw = dict(alpha=1.0, beta=1.0, batch_stride_a=0, batch_stride_b=0, batch_stride_c=0, k_iters=2, batches=1)
    assert np.array_equal(ref(oracle_mod, a, b, c, epilogue=7, **kw), ref(oracle_mod, a, b, c, epilogue=0, **kw))


def test_abi_validation_without_gpu(ncz):
    """Rejected before any CUDA call: null pointers with work to do, k_iters 0;
    zero batches is a no-op."""
    lib = ncz.mma.lib()
    assert lib.ncz_mma_matmul_pipelined(None, None, None, None, 1.0, 0.0, 0, 0, 0, 1, 0, 0, None) == 0
    assert lib.ncz_mma_matmul_batched(None, None, None, None, 1.0, 0.0, 0, 0, 0, 0, None) == 0
    st = lib.ncz_mma_matmul_pipelined(None, None, None, None, 1.0, 0.0, 0, 0, 0, 1, 0, 3, None)
    assert ncz.flash.STATUS_NAMES[st] == "InvalidValue"
    st = lib.ncz_mma_matmul_pipelined(16, 16, 16, 16, 1.0, 0.0, 0, 0, 0, 0, 0, 3, None)
    assert ncz.flash.STATUS_NAMES[st] == "InvalidValue"
    st = lib.ncz_mma_matmul(None, 16, 16, 16, 1.0, 0.0, None)
    assert ncz.flash.STATUS_NAMES[st] == "InvalidValue"


def test_python_wrapper_checks_sizes(ncz):
    torch = pytest.importorskip("torch")
    a = torch.zeros(255, dtype=torch.float16)
    with pytest.raises(ncz.FlashError):
        ncz.mma.mma_matmul(a, a, a, a, 1.0, 0.0)  # CPU tensors are rejected before any launch
    assert ncz.mma.flops(4, 10) == 2 * 16 * 8 * 16 * 4 * 10
    assert ncz.mma.bytes_moved(1, 1) == (256 + 128) * 2 + 2 * 128 * 4
