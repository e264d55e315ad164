"""Work-item order of the flash kernel on the CPU (ncz_test_item_work runs the
kernel's own make_work on the host): every (Q-tile group, slice, K range) is
one item exactly once; items come in chunks of slices, the heaviest group
first inside a chunk; each Q tile visits the K tiles up to its causal
diagonal (reference tile_end, src/flash_h64_bn32.zig:80-84) inside its range."""
import ctypes
import math

import pytest


def key_tile(lib):
    """Keys per K/V tile of the kernel (the unit of the hooks' tile counts)."""
    out = (ctypes.c_int32 * 2)()
    assert lib.ncz_test_tile_shape(out) == 0 and out[0] == 128
    return out[1]


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
    kt = key_tile(lib)
    n_kv = math.ceil(s / kt)
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
            total = 0 if q0 >= s else ((min(q0 + 128, s) - 1) // kt + 1 if causal else n_kv)
            assert n == max(0, min(total, kv0 + per) - kv0)
        assert nmax == max(n0, n1)
    assert len(seen) == items
    out = (ctypes.c_int32 * 8)()
    assert lib.ncz_test_item_work(bh, s, int(causal), splits, chunk, items, out) != 0  # past the end


def qsplit_work(lib, bh, s, causal, chunk, groups, i):
    out = (ctypes.c_int32 * 6)()
    assert lib.ncz_test_qsplit_work(bh, s, int(causal), chunk, groups, i, out) == 0
    return list(out)


def k_tiles(q_base, s, causal, kt):
    """K tiles (of kt keys) a Q tile starting at q_base visits (reference tile_end)."""
    if q_base >= s:
        return 0
    return (min(q_base + 128, s) - 1) // kt + 1 if causal else math.ceil(s / kt)


@pytest.mark.parametrize("bh,s,causal,chunk,groups", [
    (8, 1024, True, 8, 4),       # config 2: every group split
    (8, 8192, True, 16, 4),      # config 4 on 8 GPUs: the top 4 of 32 groups split
    (8, 8192, True, 16, 32),
    (20, 8192, True, 16, 3),     # short last chunk
    (3, 1000, False, 2, 4),      # ragged S, all split
    (3, 1000, False, 2, 1),      # ragged S: the top group has one Q tile
    (5, 100, True, 5, 1),        # one Q tile: one K tile, the second slot empty
    (2, 129, True, 1, 1),
])
def test_split_q_item_order(ncz, bh, s, causal, chunk, groups):
    """Launches with split-Q items for the top `groups` groups: every Q tile of
    those groups is one split-Q item (its K tiles split: slot 0 the even ceil
    half, slot 1 the odd floor half), every other group one item of two Q tiles,
    each exactly once; chunks of slices in order; inside a chunk by K tiles
    per pipeline: the two-tile items heavier than the heaviest split-Q item
    (half of its K tiles, rounded up), then the split-Q items, heaviest Q tile
    first, then the other two-tile items, heaviest group first."""
    lib = ncz.flash.lib()
    n_groups = math.ceil(s / 256)
    n_qt = math.ceil(s / 128)
    low = n_groups - groups
    split_qt = n_qt - 2 * low
    items = bh * (split_qt + low)
    chunk = min(chunk, bh)
    kt = key_tile(lib)
    top_half = (k_tiles((n_qt - 1) * 128, s, causal, kt) + 1) // 2  # heaviest split-Q item, per pipeline
    seen = set()
    prev_chunk, prev_key = -1, None
    for i in range(items):
        sl, q_base, n0, n1, nmax, kstride = qsplit_work(lib, bh, s, causal, chunk, groups, i)
        assert 0 <= sl < bh and 0 <= q_base < s
        c = sl // chunk
        assert c >= prev_chunk
        if kstride == 2:
            assert q_base % 128 == 0 and q_base // 128 >= 2 * low
            key = (sl, q_base, "q")
            total = k_tiles(q_base, s, causal, kt)
            assert nmax == total and n0 == (total + 1) // 2 and n1 == total // 2
            order = (1, -q_base)  # heaviest Q tile first
        else:
            assert kstride == 1 and q_base % 256 == 0 and q_base // 256 < low
            key = (sl, q_base, "g")
            assert (n0, n1) == (k_tiles(q_base, s, causal, kt), k_tiles(q_base + 128, s, causal, kt))
            assert nmax == max(n0, n1)
            order = (0 if nmax > top_half else 2, -q_base)
        assert key not in seen
        seen.add(key)
        if c == prev_chunk:
            assert order >= prev_key
        prev_chunk, prev_key = c, order
    assert len(seen) == items
    out = (ctypes.c_int32 * 6)()
    assert lib.ncz_test_qsplit_work(bh, s, int(causal), chunk, groups, items, out) != 0
    assert lib.ncz_test_qsplit_work(bh, s, int(causal), chunk, n_groups + 1, 0, out) != 0


@pytest.mark.parametrize("bh,s,sms,groups", [
    (8, 1024, 148, 4),       # config 2: 32 items, all split
    (5, 8192, 148, 32),      # 160 items < 1.25 per SM: all split
    (8, 8192, 148, 0),       # config 4's 8-GPU shard: 256 items
    (6, 8192, 148, 0),       # 192 items
    (16, 8192, 148, 0),      # 4-GPU shard
    (64, 8192, 148, 0),      # config 4 on one GPU
    (128, 2048, 148, 0),
    (184, 256, 148, 1),      # 184 one-group items < 185
    (185, 256, 148, 0),      # 185 = 1.25 * 148
    (4, 1024, 148, 4),
])
def test_split_q_plan(ncz, bh, s, sms, groups):
    """Every group split-Q when the items of two Q tiles number fewer than
    1.25 per SM, else none (causal masking or not)."""
    out = (ctypes.c_int32 * 2)()
    assert ncz.flash.lib().ncz_test_qsplit_plan(bh, s, sms, out) == 0
    assert out[0] == groups
    n_groups, n_qt = math.ceil(s / 256), math.ceil(s / 128)
    low = n_groups - groups
    assert out[1] == (bh * (n_qt - 2 * low + low) if groups else bh * n_groups)


def test_split_q_mode_hook(ncz):
    lib = ncz.flash.lib()
    assert lib.ncz_test_set_qsplit(3) != 0 and lib.ncz_test_set_qsplit(-1) != 0
    for mode in (1, 2, 0):
        assert lib.ncz_test_set_qsplit(mode) == 0
    assert lib.ncz_test_set_qsplit_groups(-2) != 0
    for groups in (0, 7, 1 << 20, -1):
        assert lib.ncz_test_set_qsplit_groups(groups) == 0


@pytest.mark.parametrize("bh", [1, 2, 5, 512, 513])
@pytest.mark.parametrize("s,causal", [(1, True), (77, False), (128, True), (128, False)])
def test_twin_item_order(ncz, bh, s, causal):
    """Twin items (seq_len <= 128): item i holds slices 2i and 2i + 1, one per
    slot, each against all of its K tiles; the ring alternates between the two
    slices; the last item of an odd count is an item of one slice."""
    lib = ncz.flash.lib()
    kt = key_tile(lib)
    total = math.ceil(s / kt)
    out = (ctypes.c_int32 * 8)()
    items = (bh + 1) // 2
    seen = []
    for i in range(items):
        assert lib.ncz_test_twin_work(bh, s, int(causal), i, out) == 0
        s0, s1, n0, n1, n_max, r0, r1, kind = list(out)
        assert s0 == 2 * i and n0 == total and r0 == s0
        if 2 * i + 1 < bh:
            assert (kind, s1, n1, n_max) == (2, 2 * i + 1, total, 2 * total)
            assert r1 == 2 * i + 1
            seen += [s0, s1]
        else:
            assert (kind, s1, n1, n_max) == (0, -1, 0, total)
            assert r1 == (s0 if total > 1 else -1)
            seen.append(s0)
    assert seen == list(range(bh))
    assert lib.ncz_test_twin_work(bh, s, int(causal), items, out) != 0
    assert lib.ncz_test_twin_work(bh, 129, int(causal), 0, out) != 0


def test_twin_hook(ncz):
    lib = ncz.flash.lib()
    assert lib.ncz_test_set_twin(2) != 0 and lib.ncz_test_set_twin(-1) != 0
    for v in (0, 1):
        assert lib.ncz_test_set_twin(v) == 0
