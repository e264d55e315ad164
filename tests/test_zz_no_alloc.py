"""ncz_flash_fwd_static, the forward entry point that allocates nothing, through
the C ABI.

Some callers cannot let this library allocate device memory. A host whose own
allocator owns every device buffer (the reference's Zig host allocates each one
with cuda.malloc) wants no memory it did not hand out, and a request loop must
not block on an allocation or fail on one mid-request when memory is tight. For
them the split-KV partials go to a fixed 16 MiB array of the library's device
image instead of the memory pool of ncz_flash_fwd_splits.

The test runs the new entry point on three calls in a row, with different
shapes and inputs. The shared array then holds the previous call's partials,
so stale contents would show. Each output is checked against the oracle on the
same f16 inputs (the parity gate of the other GPU tests) and against the
allocating entry point. An explicit split count too large for the array must
be refused with OutOfMemory before any launch.

This file is collected last, so a run that stops at its first failure has
already run every other test.
"""
import ctypes

import pytest

from tests import cases as C

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

ATOL = 2e-3  # the parity tolerance of the GPU tests (max-abs, f32 O)


def _inputs(bh, s, d, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    return tuple((torch.randn(bh * s * d, generator=g, device="cuda") * 0.7).half() for _ in range(3))


def _desc(ncz, q, k, v, o, bh, s, d, causal):
    x = ncz.flash._Desc()
    x.q, x.k, x.v, x.o = q.data_ptr(), k.data_ptr(), v.data_ptr(), o.data_ptr()
    x.batch_heads, x.seq_len, x.head_dim = bh, s, d
    x.q_stride = x.k_stride = x.v_stride = x.o_stride = s * d
    x.scale, x.causal = d ** -0.5, int(causal)
    x.o_dtype, x.in_dtype, x.producer, x.device = 0, 1, 0, torch.cuda.current_device()
    x.stream = torch.cuda.current_stream().cuda_stream
    return x


def test_no_alloc_entry_matches_oracle_on_calls_in_a_row(ncz, oracle_mod):
    lib = ncz.flash.lib()
    # (bh, S, d, causal, seed): each splits its K range, so the scratch is used;
    # the third call repeats the first shape with new inputs.
    calls = [(1, 4096, 64, True, 1), (2, 3000, 32, False, 2), (1, 4096, 64, True, 3)]
    for bh, s, d, causal, seed in calls:
        p = C.normal_problem(bh, s, d, causal, 40 + seed, oracle_mod, std=0.7)
        q, k, v = (torch.from_numpy(a).cuda() for a in (p.q, p.k, p.v))
        got = torch.full((bh * s * d,), float("nan"), device="cuda")
        want = torch.zeros(bh * s * d, device="cuda")
        before = lib.ncz_launch_count()
        assert lib.ncz_flash_fwd_static(ctypes.byref(_desc(ncz, q, k, v, got, bh, s, d, causal)), 0) == 0
        assert lib.ncz_launch_count() - before == 2  # split forward + merge: partials went through the scratch
        assert lib.ncz_flash_fwd_splits(ctypes.byref(_desc(ncz, q, k, v, want, bh, s, d, causal)), 0) == 0
        assert ncz.sync_status() == 0
        assert bool(torch.isfinite(got).all())
        C.check(got.cpu().numpy(), C.reference(p, oracle_mod), C.active_index(p), f"static {bh}x{s}x{d}")
        err = float((got - want).abs().max())
        assert err <= ATOL, (bh, s, d, causal, err)


def test_no_alloc_entry_refuses_a_split_count_beyond_its_scratch(ncz):
    lib = ncz.flash.lib()
    bh, s, d = 2, 8192, 64  # 4 splits need 4 * 2 * 8192 * 66 floats > 16 MiB
    q, k, v = _inputs(bh, s, d, 4)
    o = torch.zeros(bh * s * d, device="cuda")
    torch.cuda.synchronize()
    before = lib.ncz_launch_count()
    st = lib.ncz_flash_fwd_static(ctypes.byref(_desc(ncz, q, k, v, o, bh, s, d, True)), 4)
    assert ncz.flash.STATUS_NAMES[st] == "OutOfMemory" and lib.ncz_launch_count() == before
    assert ncz.sync_status() == 0 and bool((o == 0).all())
