"""Race check of the launch-control item walk on the GPU.

Every CTA of the forward takes further work items at run time (cluster launch
control), so which CTA runs which item changes from launch to launch.  The
debug build libncz_flash_debug.so (NCZ_DEBUG_ITEM_VISITS) counts, per item,
the CTAs whose producer started it.  A correct walk starts every item exactly
once: a count of 0 is a lost item, 2 an item run twice.  The shapes below give
many items per CTA, empty split-KV ranges and both producers, each launched
twice.  O must equal the product library's output bit for bit, since the
counter is the only difference between the two builds.
"""
import ctypes
import os

import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DEBUG_LIB = os.path.join(ROOT, "not-cute-zig_b200", "libncz_flash_debug.so")

CASES = [  # (bh, S, d, causal, producer, in_dtype, splits)
    (64, 2048, 64, True, "tma", torch.float16, 0),    # 512 items, several per CTA
    (900, 256, 32, False, "tma", torch.float16, 0),   # 900 one-group items
    (1, 8192, 64, True, "tma", torch.float16, 0),     # split-KV with empty ranges
    (37, 1000, 16, True, "lsu", torch.float16, 0),    # plain-load producer
    (20, 4096, 64, True, "tma", torch.bfloat16, 3),   # bf16 inputs, explicit split
    (513, 128, 32, False, "tma", torch.float16, 0),   # twin items, odd slice count
    (9, 100, 64, True, "lsu", torch.bfloat16, 0),     # twin items, plain-load producer
]


@pytest.fixture(scope="module")
def debug_lib():
    if not os.path.exists(DEBUG_LIB):
        pytest.fail(f"{DEBUG_LIB} is not built (run __graft_entry__.build())")
    lib = ctypes.CDLL(DEBUG_LIB)
    lib.ncz_debug_item_visits.restype = ctypes.c_int
    lib.ncz_debug_item_visits.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_size_t,
                                          ctypes.POINTER(ctypes.c_size_t)]
    lib.ncz_flash_sync_status.restype = ctypes.c_int
    lib.ncz_flash_sync_status.argtypes = [ctypes.c_int, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]
    return lib


@pytest.mark.parametrize("case", CASES, ids=lambda c: f"bh{c[0]}_s{c[1]}_d{c[2]}_{c[4]}_split{c[6]}")
def test_every_item_started_exactly_once(ncz, debug_lib, case):
    check_items(ncz, debug_lib, case)


QSPLIT_CASES = [  # split-Q items forced in both libraries
    (64, 2048, 64, True, "tma", torch.float16, 0),    # 1024 items of one Q tile
    (300, 600, 32, False, "lsu", torch.float16, 0),   # 1500 items, plain-load producer
]
MIXED_CASES = [  # (case, split-Q groups forced in both libraries)
    ((10, 4096, 64, True, "tma", torch.float16, 1), 3),     # top 3 of 16 groups split: 190 items
    ((8, 8192, 64, True, "tma", torch.float16, 1), 4),      # two-tile items before and after the split-Q ones
    ((6, 2000, 32, False, "lsu", torch.float16, 1), 2),     # ragged S, plain-load producer
]


@pytest.mark.parametrize("case", QSPLIT_CASES, ids=lambda c: f"qsplit_bh{c[0]}_s{c[1]}_d{c[2]}_{c[4]}")
def test_split_q_items_started_exactly_once(ncz, debug_lib, case):
    """The same check with split-Q items: each CTA's two pipelines share one Q
    tile per item and merge their states through barriers whose phases run
    over all the items a CTA walks."""
    lib = ncz.flash.lib()
    debug_lib.ncz_test_set_qsplit.argtypes = [ctypes.c_int]
    assert lib.ncz_test_set_qsplit(1) == 0 and debug_lib.ncz_test_set_qsplit(1) == 0
    try:
        check_items(ncz, debug_lib, case)
    finally:
        assert lib.ncz_test_set_qsplit(0) == 0 and debug_lib.ncz_test_set_qsplit(0) == 0


def check_items(ncz, debug_lib, case):
    bh, s, d, causal, producer, in_dtype, splits = case
    g = torch.Generator(device="cuda")
    g.manual_seed(bh * 7 + s)
    q, k, v = ((torch.randn(bh * s * d, generator=g, device="cuda") * 0.7).to(in_dtype) for _ in range(3))
    opts = ncz.Options(seq_len=s, head_dim=d, q_stride=s * d, k_stride=s * d, v_stride=s * d, o_stride=s * d,
                       scale=d ** -0.5, batch_heads=bh, causal=causal)
    want = torch.zeros(bh * s * d, device="cuda")
    ncz.launch_splits(q, k, v, want, opts, splits, producer=producer)
    cap = 1 << 16
    for _ in range(2):
        o = torch.full_like(want, float("nan"))
        visits = torch.zeros(cap, dtype=torch.int32, device="cuda")
        desc = ncz.flash.make_desc(q, k, v, o, opts, producer=producer)
        items = ctypes.c_size_t(0)
        st = debug_lib.ncz_debug_item_visits(ctypes.addressof(desc), splits, visits.data_ptr(), cap,
                                             ctypes.byref(items))
        assert st == 0, ncz.flash.STATUS_NAMES.get(st, st)
        word = ctypes.c_uint32(0)
        assert debug_lib.ncz_flash_sync_status(-1, desc.stream, ctypes.byref(word)) == 0, hex(word.value)
        n = items.value
        assert 0 < n <= cap
        counts = visits[:n]
        lost = int((counts == 0).sum())
        repeated = int((counts > 1).sum())
        assert lost == 0 and repeated == 0, (n, lost, repeated)
        assert int(visits[n:].abs().sum()) == 0
        assert ncz.sync_status() == 0
        assert torch.equal(o, want)


@pytest.mark.parametrize("case,groups", MIXED_CASES, ids=["bh10_s4096_g3", "bh8_s8192_g4", "bh6_s2000_g2_lsu"])
def test_mixed_items_started_exactly_once(ncz, debug_lib, case, groups):
    """A launch whose top groups run as split-Q items and the others as items
    of two Q tiles, in one item order: every item started once, O identical to
    the product library's."""
    lib = ncz.flash.lib()
    debug_lib.ncz_test_set_qsplit_groups.argtypes = [ctypes.c_int]
    assert lib.ncz_test_set_qsplit_groups(groups) == 0 and debug_lib.ncz_test_set_qsplit_groups(groups) == 0
    try:
        check_items(ncz, debug_lib, case)
    finally:
        assert lib.ncz_test_set_qsplit_groups(-1) == 0 and debug_lib.ncz_test_set_qsplit_groups(-1) == 0
