"""Work-item order of the flash kernel on the CPU (ncz_test_item_work runs the
kernel's own make_work on the host): every (Q-tile group, slice, K range) is
one item exactly once; items come in chunks of slices, the heaviest group
first inside a chunk; each Q tile visits the K tiles up to its causal
diagonal (reference tile_end, src/flash_h64_bn32.zig:80-84) inside its range."""
import ctypes
import math

import pytest


def work(lib, bh, s, causal, splits, chunk, i):
    out = (ctypes.c_int32 * 8)()
    assert lib.ncz_test_item_work(bh, s, int(causal), splits, chunk, i, out) == 0
    return list(out)


@pytest.mark.parametrize("bh,s,causal,splits,chunk", [
    (64, 8192, True, 1, 16),   # config 4 with its 32 MB chunks
    (20, 8192, True, 1, 16),   # short last chunk
    (1024, 2048, False, 1, 64),
    (7, 600, True, 1, 3),      # ragged S, empty second Q tile in the last group
    (2, 4096, True, 8, 1),     # split-KV
    (3, 1000, False, 3, 2),
    (5, 100, True, 1, 5),      # one group
])
def test_item_order(ncz, bh, s, causal, splits, chunk):
    check_item_order(ncz.flash.lib(), bh, s, causal, splits, chunk)


def check_item_order(lib, bh, s, causal, splits, chunk):
    """Every (slice, Q group, K range) once, chunks in order, heaviest group
    first inside a chunk, each Q tile's K tiles inside its range and causal
    bound; one item past the end is refused."""
    groups = math.ceil(s / 256)
    n_kv = math.ceil(s / 128)
    ns = work(lib, bh, s, causal, splits, chunk, 0)[7]
    per = math.ceil(n_kv / min(splits, n_kv))
    assert ns == math.ceil(n_kv / per)
    items = groups * bh * ns
    chunk = min(chunk, bh)
    seen = set()
    prev_chunk, prev_group = -1, None
    for i in range(items):
        sl, q_base, sp, kv0, n0, n1, nmax, _ = work(lib, bh, s, causal, splits, chunk, i)
        key = (sl, q_base, sp)
        assert key not in seen and 0 <= sl < bh and q_base % 256 == 0 and q_base < s and 0 <= sp < ns
        seen.add(key)
        c = sl // chunk
        assert c >= prev_chunk  # chunks in order
        g = q_base // 256
        if c == prev_chunk:
            assert g <= prev_group  # heaviest (last) group first inside a chunk
        prev_chunk, prev_group = c, g
        assert kv0 == sp * per
        for w, n in ((0, n0), (1, n1)):
            q0 = q_base + 128 * w
            total = 0 if q0 >= s else ((min(q0 + 128, s) - 1) // 128 + 1 if causal else n_kv)
            assert n == max(0, min(total, kv0 + per) - kv0)
        assert nmax == max(n0, n1)
    assert len(seen) == items
    out = (ctypes.c_int32 * 8)()
    assert lib.ncz_test_item_work(bh, s, int(causal), splits, chunk, items, out) != 0  # past the end


def qsplit_work(lib, bh, s, causal, chunk, i):
    out = (ctypes.c_int32 * 6)()
    assert lib.ncz_test_qsplit_work(bh, s, int(causal), chunk, i, out) == 0
    return list(out)


@pytest.mark.parametrize("bh,s,causal,chunk", [
    (8, 1024, True, 8),        # config 2
    (8, 8192, True, 16),       # config 4 on 8 GPUs
    (20, 8192, True, 16),      # short last chunk
    (3, 1000, False, 2),       # ragged S
    (5, 100, True, 5),         # one Q tile: one K tile, the second slot empty
    (2, 129, True, 1),
])
def test_split_q_item_order(ncz, bh, s, causal, chunk):
    """Split-Q launches (one Q tile per item): every (slice, Q tile) once,
    chunks of slices in order, heaviest Q tile first inside a chunk; the item
    streams all K tiles of its Q tile (up to the causal diagonal) and its two
    slots take the even (ceil half) and the odd (floor half) of them."""
    lib = ncz.flash.lib()
    n_qt = math.ceil(s / 128)
    n_kv = math.ceil(s / 128)
    items = n_qt * bh
    chunk = min(chunk, bh)
    seen = set()
    prev_chunk, prev_qt = -1, None
    for i in range(items):
        sl, q_base, n0, n1, nmax, kstride = qsplit_work(lib, bh, s, causal, chunk, i)
        assert kstride == 2 and q_base % 128 == 0 and 0 <= q_base < s and 0 <= sl < bh
        key = (sl, q_base)
        assert key not in seen
        seen.add(key)
        c, qt = sl // chunk, q_base // 128
        assert c >= prev_chunk
        if c == prev_chunk:
            assert qt <= prev_qt
        prev_chunk, prev_qt = c, qt
        total = (min(q_base + 128, s) - 1) // 128 + 1 if causal else n_kv
        assert nmax == total and n0 == (total + 1) // 2 and n1 == total // 2
    assert len(seen) == items
    out = (ctypes.c_int32 * 6)()
    assert lib.ncz_test_qsplit_work(bh, s, int(causal), chunk, items, out) != 0


def test_split_q_mode_hook(ncz):
    lib = ncz.flash.lib()
    assert lib.ncz_test_set_qsplit(3) != 0 and lib.ncz_test_set_qsplit(-1) != 0
    for mode in (1, 2, 0):
        assert lib.ncz_test_set_qsplit(mode) == 0
