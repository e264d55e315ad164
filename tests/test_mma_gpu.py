"""GEMM + epilogue on the GPU against the oracle (oracle/mma_oracle.c).
The warp MMA sums each 16-term block in its own order, so results agree with
the oracle's sequential f32 sum within 1e-5 (relative and absolute); on the
reference's dyadic fixtures every partial sum is exact, so there they agree
bit for bit.  silu / gelu: ex2.approx on the GPU, exp2f in the oracle."""
import numpy as np
import pytest

from tests import mma_cases as M

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x)).cuda()


def run_pipelined(ncz, a, b, c, *, alpha, beta, sa, sb, sc, k_iters, epilogue, batches, offsets=(0, 0, 0, 0)):
    """Runs ncz_mma_matmul_pipelined; `offsets` shifts each operand's start by
    that many elements inside a larger buffer (misaligned layouts)."""
    oa, ob, oc, od = offsets
    ta = dev(np.concatenate([np.zeros(oa, np.float16), a]))
    tb = dev(np.concatenate([np.zeros(ob, np.float16), b]))
    tc = dev(np.concatenate([np.zeros(oc, np.float32), c]))
    # D starts as a copy of C: elements between the batches' tiles (padded
    # strides) must come back untouched, as the oracle leaves them.
    td = dev(np.concatenate([np.zeros(od, np.float32), c]))
    ptr = lambda t, o: t.data_ptr() + o * t.element_size()  # noqa: E731
    ncz.mma.pipelined_mma_matmul(ptr(ta, oa), ptr(tb, ob), ptr(tc, oc), ptr(td, od), alpha, beta, sa, sb, sc,
                                 k_iters, epilogue, batches)
    assert ncz.mma.sync_status() == 0
    return td[od:].cpu().numpy()


def check(got, want, epilogue, what):
    assert np.array_equal(np.isnan(got), np.isnan(want)), what
    ok = ~np.isnan(want)
    assert np.allclose(got[ok], want[ok], rtol=1e-5, atol=1e-5), (what, float(np.abs(got[ok] - want[ok]).max()))


def problem(batches, k_iters, seed, sa=None, sb=None, sc=None):
    sa = k_iters * 256 if sa is None else sa
    sb = k_iters * 128 if sb is None else sb
    sc = 128 if sc is None else sc
    rng = np.random.default_rng(seed)
    a = rng.uniform(-1, 1, (batches - 1) * sa + k_iters * 256).astype(np.float16)
    b = rng.uniform(-1, 1, (batches - 1) * sb + k_iters * 128).astype(np.float16)
    c = rng.uniform(-2, 2, (batches - 1) * sc + 128).astype(np.float32)
    return a, b, c, sa, sb, sc


def test_reference_demos_bit_exact(ncz):
    """runEpilogueDemo (relu, k_iters 1), runPipelinedMma (k_iters 4),
    runBatchedMma (4 column-major batches), runMmaMatmul (alpha 1.25, beta 0.5)
    and the reference's GEMM baseline: exact answers (src/main.zig:289-460,
    :1049-1110; tools/cuda_baselines.cu:580-617)."""
    for k_iters, epi in ((1, 1), (4, 0)):
        a, b, c = M.fill_pipeline_inputs(k_iters)
        got = run_pipelined(ncz, a, b, c, alpha=1.0, beta=0.0, sa=0, sb=0, sc=0, k_iters=k_iters, epilogue=epi,
                            batches=1)
        assert np.array_equal(got.astype(np.float64), M.exact_gemm(a, b, c, alpha=1.0, beta=0.0, k_iters=k_iters,
                                                                   relu=epi == 1))
    parts = [M.fill_mma_inputs(s) for s in range(4)]
    a, b, c = (np.concatenate([p[i] for p in parts]) for i in range(3))
    td = torch.zeros(c.size, dtype=torch.float32, device="cuda")
    ncz.mma.batched_mma_matmul(dev(a), dev(b), dev(c), td, 1.0, 0.0, 256, 128, 128, batches=4)
    assert ncz.mma.sync_status() == 0
    assert np.array_equal(td.cpu().numpy().astype(np.float64),
                          M.exact_gemm(a, b, c, alpha=1.0, beta=0.0, k_iters=1, batches=4, b_col=True))
    a, b, c = M.fill_mma_inputs(0)
    td = torch.zeros(128, dtype=torch.float32, device="cuda")
    ncz.mma.mma_matmul(dev(a), dev(b), dev(c), td, 1.25, 0.5)
    assert ncz.mma.sync_status() == 0
    assert np.array_equal(td.cpu().numpy().astype(np.float64),
                          M.exact_gemm(a, b, c, alpha=1.25, beta=0.5, k_iters=1, b_col=True))
    a, b, c = M.gemm_baseline_inputs()
    got = run_pipelined(ncz, a, b, c, alpha=1.0, beta=0.0, sa=0, sb=0, sc=0, k_iters=1, epilogue=0, batches=1)
    assert np.array_equal(got.astype(np.float64), M.exact_gemm(a, b, c, alpha=1.0, beta=0.0, k_iters=1))


@pytest.mark.parametrize("epilogue", [0, 1, 2, 3, 7])
@pytest.mark.parametrize("k_iters,batches", [(1, 1), (3, 5), (4, 600), (5, 37), (9, 300), (17, 9)])
def test_random_problems(ncz, oracle_mod, epilogue, k_iters, batches):
    a, b, c, sa, sb, sc = problem(batches, k_iters, 100 * k_iters + batches)
    alpha, beta = 1.75, -0.625
    got = run_pipelined(ncz, a, b, c, alpha=alpha, beta=beta, sa=sa, sb=sb, sc=sc, k_iters=k_iters,
                        epilogue=epilogue, batches=batches)
    want = oracle_mod.mma_reference(a, b, c, alpha=alpha, beta=beta, batch_stride_a=sa, batch_stride_b=sb,
                                    batch_stride_c=sc, k_iters=k_iters, epilogue=epilogue, batches=batches)
    check(got, want, epilogue, f"k_iters={k_iters} batches={batches} epilogue={epilogue}")


@pytest.mark.parametrize("case", ["padded_aligned", "odd_strides", "misaligned_bases", "odd_c_stride", "broadcast"])
def test_layouts(ncz, oracle_mod, case):
    """Bulk-copy path (16-byte multiples), plain-load path (odd strides or
    bases), scalar C/D path (odd C stride), and stride 0 (one A and B for all)."""
    k_iters, batches = 6, 211
    offsets = (0, 0, 0, 0)
    if case == "padded_aligned":
        sa, sb, sc = k_iters * 256 + 8, k_iters * 128 + 24, 128 + 4
    elif case == "odd_strides":
        sa, sb, sc = k_iters * 256 + 3, k_iters * 128 + 5, 128
    elif case == "misaligned_bases":
        sa, sb, sc = k_iters * 256, k_iters * 128, 128
        offsets = (1, 3, 1, 1)
    elif case == "odd_c_stride":
        sa, sb, sc = k_iters * 256, k_iters * 128, 131
    else:
        sa, sb, sc = 0, 0, 128
    a, b, c, sa, sb, sc = problem(batches, k_iters, 7, sa, sb, sc)
    for epilogue in (0, 2):
        got = run_pipelined(ncz, a, b, c, alpha=0.5, beta=1.0, sa=sa, sb=sb, sc=sc, k_iters=k_iters,
                            epilogue=epilogue, batches=batches, offsets=offsets)
        want = oracle_mod.mma_reference(a, b, c, alpha=0.5, beta=1.0, batch_stride_a=sa, batch_stride_b=sb,
                                        batch_stride_c=sc, k_iters=k_iters, epilogue=epilogue, batches=batches)
        check(got, want, epilogue, case)


def test_nan_c_with_zero_beta_propagates(ncz, oracle_mod):
    """beta * c is computed even when beta is 0, as in the reference
    (src/kernels.zig:128-131): NaN in C gives NaN in D."""
    a, b, c, sa, sb, sc = problem(3, 2, 11)
    c[5] = np.nan
    got = run_pipelined(ncz, a, b, c, alpha=1.0, beta=0.0, sa=sa, sb=sb, sc=sc, k_iters=2, epilogue=0, batches=3)
    want = oracle_mod.mma_reference(a, b, c, alpha=1.0, beta=0.0, batch_stride_a=sa, batch_stride_b=sb,
                                    batch_stride_c=sc, k_iters=2, epilogue=0, batches=3)
    assert np.isnan(got[5])
    check(got, want, 0, "nan in C")


def test_many_batches_grid_stride(ncz, oracle_mod):
    """More batches than warps of the grid (296 CTAs x 8 warps): each warp
    walks several batches through one ring of stages."""
    k_iters, batches = 2, 40000
    a, b, c, sa, sb, sc = problem(batches, k_iters, 13)
    got = run_pipelined(ncz, a, b, c, alpha=1.0, beta=0.5, sa=sa, sb=sb, sc=sc, k_iters=k_iters, epilogue=1,
                        batches=batches)
    want = oracle_mod.mma_reference(a, b, c, alpha=1.0, beta=0.5, batch_stride_a=sa, batch_stride_b=sb,
                                    batch_stride_c=sc, k_iters=k_iters, epilogue=1, batches=batches)
    check(got, want, 1, "40000 batches")


def test_stage_wait_times_out_cleanly(ncz):
    """Failure detection without a GPU fault: with a short wait limit and one
    bulk copy withheld, the stage wait runs out, the kernel stops cleanly and
    the status reads DeviceTimeout; the next launch is correct."""
    lib = ncz.mma.lib()
    a, b, c, sa, sb, sc = problem(64, 4, 21)
    try:
        assert lib.ncz_mma_test_set_wait_limit(-1, 2_000_000) == 0  # about 1 ms
        assert lib.ncz_mma_test_drop_copy(-1, 1) == 0
        ta, tb, tc = dev(a), dev(b), dev(c)
        td = torch.zeros_like(tc)
        ncz.mma.pipelined_mma_matmul(ta, tb, tc, td, 1.0, 0.0, sa, sb, sc, 4, 0, 64)
        with pytest.raises(ncz.FlashError) as err:
            ncz.mma.sync_status()
        assert "DeviceTimeout" in str(err.value)
    finally:
        lib.ncz_mma_test_drop_copy(-1, 0)
        lib.ncz_mma_test_set_wait_limit(-1, 0)
    got = run_pipelined(ncz, a, b, c, alpha=1.0, beta=0.0, sa=sa, sb=sb, sc=sc, k_iters=4, epilogue=0, batches=64)
    want = ncz_oracle_mma(a, b, c, sa, sb, sc)
    check(got, want, 0, "after timeout")


def ncz_oracle_mma(a, b, c, sa, sb, sc):
    from oracle import oracle as o

    return o.mma_reference(a, b, c, alpha=1.0, beta=0.0, batch_stride_a=sa, batch_stride_b=sb, batch_stride_c=sc,
                           k_iters=4, epilogue=0, batches=64)
