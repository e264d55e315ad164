"""Host-side launch planning on the CPU: the split-KV plan (split_plan) and the
host-buffer pipeline's slice chunks (chunk_plan), through their test hooks."""
import ctypes
import math

import pytest


def key_tile(lib):
    out = (ctypes.c_int32 * 2)()
    assert lib.ncz_test_tile_shape(out) == 0
    return out[1]


def split_plan(lib, bh, seq, requested, sms=148):
    out = (ctypes.c_int32 * 2)()
    assert lib.ncz_test_split_plan(bh, seq, requested, sms, out) == 0
    return out[0], out[1]


@pytest.mark.parametrize("bh,seq", [(1, 128), (1, 2047), (1, 2048), (1, 4096), (8, 1024), (8, 4096), (2, 8192),
                                    (64, 8192), (37, 5000), (100, 16384)])
def test_automatic_split_policy(ncz, bh, seq):
    """Split only when the grid fills at most half the SMs and the K range has
    at least 2048 keys; at most 8 ranges of at least 512 keys; ranges cover all
    K tiles."""
    lib = ncz.flash.lib()
    kt = key_tile(lib)
    n_kv = math.ceil(seq / kt)
    items = math.ceil(seq / 256) * bh
    splits, per = split_plan(lib, bh, seq, 0)
    if items * 2 <= 148 and n_kv >= 2048 // kt:
        assert splits > 1 and per >= 512 // kt and splits <= 8
        assert splits <= math.ceil(148 / items)
    else:
        assert splits == 1 and per == n_kv
    assert per * splits >= n_kv and (splits - 1) * per < n_kv


@pytest.mark.parametrize("requested", [1, 2, 3, 5, 8, 9, 64])
@pytest.mark.parametrize("seq", [128, 1000, 4096])
def test_requested_splits(ncz, requested, seq):
    lib = ncz.flash.lib()
    n_kv = math.ceil(seq / key_tile(lib))
    splits, per = split_plan(lib, 3, seq, requested)
    assert splits <= min(requested, n_kv, 8)
    assert per == math.ceil(n_kv / min(requested, n_kv, 8))
    assert per * splits >= n_kv and (splits - 1) * per < n_kv


def chunk_plan(lib, bh, chunk, taper):
    out = (ctypes.c_size_t * 1024)()
    count = ctypes.c_size_t(0)
    assert lib.ncz_test_chunk_plan(bh, chunk, int(taper), out, 1024, ctypes.byref(count)) == 0
    return list(out[:count.value])


@pytest.mark.parametrize("bh,chunk", [(64, 8), (64, 1), (7, 3), (1, 4), (100, 16), (20, 8), (12, 4)])
@pytest.mark.parametrize("taper", [False, True])
def test_chunk_plan(ncz, bh, chunk, taper):
    """Chunks cover the slices in order, none above the chunk size; with taper
    (and room for it) the first two and last two chunks are a quarter and a
    half of the chunk size."""
    plan = chunk_plan(ncz.flash.lib(), bh, chunk, taper)
    assert sum(plan) == bh and all(0 < c <= chunk for c in plan)
    a, b = max(1, chunk // 4), max(1, chunk // 2)
    if taper and chunk >= 4 and bh >= 2 * (a + b) + chunk:
        assert plan[:2] == [a, b] and plan[-2:] == [b, a]
    else:
        assert plan == [min(chunk, bh - s0) for s0 in range(0, bh, chunk)]


def test_plan_hooks_reject_bad_input(ncz):
    lib = ncz.flash.lib()
    out = (ctypes.c_int32 * 2)()
    assert lib.ncz_test_split_plan(0, 128, 0, 148, out) != 0
    count = ctypes.c_size_t(0)
    small = (ctypes.c_size_t * 2)()
    assert ncz.flash.STATUS_NAMES[lib.ncz_test_chunk_plan(64, 1, 0, small, 2, ctypes.byref(count))] == "Overflow"
    assert count.value == 64
