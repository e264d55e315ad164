"""Property tests (hypothesis) of the host-side rules of the C ABI, on the CPU:
validation against the reference rule and against a restatement of the
row-stride extension, and the kernel's work-item order over random shapes."""
import ctypes

import pytest

hypothesis = pytest.importorskip("hypothesis")
from hypothesis import given, settings, strategies as st  # noqa: E402

from tests.test_item_order import check_item_order  # noqa: E402

U64 = (1 << 64) - 1
sizes = st.one_of(st.integers(0, 300), st.integers(0, 1 << 20), st.integers(0, U64),
                  st.sampled_from([0, 1, 15, 16, 17, 32, 48, 64, 1 << 31, 1 << 32, U64]))
dims = st.one_of(st.sampled_from([0, 8, 16, 24, 32, 64, 128]), st.integers(0, U64))
near = st.sampled_from([-1, 0, 0, 1, 7])  # offsets from an exact bound
small = st.one_of(st.integers(0, 5000), st.integers(0, U64))


def clamp(x):
    return min(max(x, 0), U64)


@st.composite
def reference_args(draw):
    """Mostly shapes near the rule's edges (valid head_dim, strides at the bound
    +-1), sometimes anything at all."""
    if draw(st.integers(0, 3)) == 0:
        return draw(sizes), draw(sizes), draw(dims), draw(st.lists(sizes, min_size=4, max_size=4))
    bh = draw(st.one_of(st.integers(1, 5000), st.sampled_from([0, 1 << 40, U64])))
    s = draw(st.one_of(st.integers(1, 100000), st.sampled_from([0, 1 << 58, 1 << 62, U64])))
    d = draw(st.one_of(st.sampled_from([16, 32, 64]), dims))
    return bh, s, d, [clamp(s * d + draw(near)) for _ in range(4)]


@st.composite
def extended_args(draw):
    """The descriptor's fields, mostly near the extended rule's edges."""
    wild = draw(st.integers(0, 4)) == 0
    bh = draw(st.one_of(st.integers(1, 4096), st.sampled_from([0, 1 << 28, 0x7FFFFFFF + 1, U64])))
    s = draw(st.one_of(st.integers(1, 9000), st.sampled_from([0, 1 << 30, (1 << 30) + 1, 1 << 62, U64])))
    d = draw(st.sampled_from([16, 32, 64]) if not wild else st.sampled_from([0, 16, 32, 48, 64]))
    rows, slices = [], []
    for _ in range(4):
        row = draw(st.sampled_from([0, d, d + 8, d - 1, 3 * d]))
        r = row or d
        rows.append(row)
        slices.append(draw(small) if wild else clamp((s - 1) * r + d + draw(near)))
    pick = st.sampled_from([0, 1, 2]) if not wild else st.integers(-1, 3)
    return bh, s, d, slices, rows, draw(pick), draw(pick), draw(pick)


def ref_validate(bh, s, d, strides):
    """src/flash.zig:16-28, with seq_len * head_dim overflow reported as Overflow
    (a safety panic in the reference's checked build)."""
    if bh == 0 or s == 0 or d not in (16, 32, 64):
        return "InvalidValue"
    if s * d > U64:
        return "Overflow"
    return "InvalidValue" if min(strides) < s * d else "Success"


@settings(max_examples=400, deadline=None)
@given(args=reference_args())
def test_validate_matches_the_reference_rule(ncz, args):
    bh, s, d, strides = args
    got = ncz.flash.lib().ncz_flash_validate(bh, s, d, *strides)
    assert ncz.flash.STATUS_NAMES[got] == ref_validate(bh, s, d, strides)


def ref_validate_ex(bh, s, d, slices, rows, o_dtype, in_dtype, producer):
    """The extended rule: each row stride >= d, each slice stride >= the last
    element a slice touches ((s-1)*row + d), checked operand by operand
    (q, k, v, o) with 64-bit overflow reported; then dtypes, producer and the
    32-bit launch limits."""
    if bh == 0 or s == 0 or d not in (16, 32, 64):
        return "InvalidValue"
    for sl, row in zip(slices, rows):
        row = row or d
        if row < d:
            return "InvalidValue"
        span = (s - 1) * row
        if span > U64 or span + d > U64:
            return "Overflow"
        if sl < span + d:
            return "InvalidValue"
        if sl * bh > U64:
            return "Overflow"
    if o_dtype not in (0, 1, 2) or (in_dtype or 1) not in (1, 2) or producer not in (0, 1, 2):
        return "InvalidValue"
    if s > 1 << 30:
        return "InvalidValue"
    groups = -(-s // 256)
    if groups * bh > U64 or groups * bh > 0x7FFFFFFF // 8 or bh > 0x7FFFFFFF:
        return "InvalidValue"
    return "Success"


@settings(max_examples=400, deadline=None)
@given(args=extended_args())
def test_validate_ex_matches_the_row_stride_rule(ncz, args):
    bh, s, d, slices, rows, o_dtype, in_dtype, producer = args
    x = ncz.flash._Desc()
    x.batch_heads, x.seq_len, x.head_dim = bh, s, d
    x.q_stride, x.k_stride, x.v_stride, x.o_stride = slices
    x.q_row_stride, x.k_row_stride, x.v_row_stride, x.o_row_stride = rows
    x.o_dtype, x.in_dtype, x.producer, x.device = o_dtype, in_dtype, producer, -1
    got = ncz.flash.lib().ncz_flash_validate_ex(ctypes.byref(x))
    assert ncz.flash.STATUS_NAMES[got] == ref_validate_ex(bh, s, d, slices, rows, o_dtype, in_dtype, producer)


@settings(max_examples=40, deadline=None)
@given(bh=st.integers(1, 24), s=st.integers(1, 2600), causal=st.booleans(), splits=st.integers(1, 9),
       chunk=st.integers(1, 30))
def test_item_order_is_a_permutation_for_random_shapes(ncz, bh, s, causal, splits, chunk):
    check_item_order(ncz.flash.lib(), bh, s, causal, splits, chunk)


def ref_gemm(ptrs_ok, k_iters, batches, strides):
    """ncz_mma_matmul_pipelined's argument rule: zero batches launch nothing;
    otherwise every pointer and k_iters >= 1 are required, and k_iters <= 2^24,
    batches and strides <= 2^40 (64-bit element offsets stay exact)."""
    if batches == 0:
        return "Success", 0
    if not ptrs_ok or k_iters == 0:
        return "InvalidValue", 0
    if k_iters > 1 << 24 or batches > 1 << 40 or max(strides) > 1 << 40:
        return "Overflow", 0
    return "Success", 1


@settings(max_examples=300, deadline=None,
          suppress_health_check=[hypothesis.HealthCheck.function_scoped_fixture])
@given(ptrs_ok=st.booleans(), k_iters=st.one_of(st.integers(0, 40), st.sampled_from([1 << 24, (1 << 24) + 1, U64])),
       batches=st.one_of(st.integers(0, 100000), st.sampled_from([1 << 40, (1 << 40) + 1, U64])),
       strides=st.lists(st.one_of(st.integers(0, 4096), st.sampled_from([1 << 40, (1 << 40) + 1])), min_size=3,
                        max_size=3),
       epilogue=st.integers(0, 7))
def test_gemm_arguments_and_launch_shape(ncz, fake, ptrs_ok, k_iters, batches, strides, epilogue):
    """Under the fake devices: the status follows the rule, and a valid call
    launches one mma_gemm<row_b> of min(ceil(batches / 10), 2 x SMs) CTAs of
    10 warps."""
    lib = ncz.mma.lib()
    before = len(fake.launches)
    ptr = 0x1000_0000 if ptrs_ok else None
    st_ = lib.ncz_mma_matmul_pipelined(0x1000_0000, ptr, 0x3000_0000, 0x4000_0000, 1.0, 0.5, *strides, k_iters,
                                       epilogue, batches, None)
    want, launches = ref_gemm(ptrs_ok, k_iters, batches, strides)
    assert ncz.flash.STATUS_NAMES[st_] == want
    new = fake.launches[before:]
    assert len(new) == launches
    if launches:
        assert new[0].grid == min(-(-batches // 10), 2 * fake.sms) and new[0].block == 320
        assert ncz.driver.kernel_label(new[0].kernel) == "mma_gemm<row_b>"
