"""Parity of the sm_100a kernel with the oracle, through the C ABI.

Every launch goes through the reference-shaped Python mirror
(not-cute-zig_b200.flash.launch / launch_ex -> libncz_flash.so).  Inputs are
generated on the host, so the kernel and the oracle read identical f16 bits.
"""
import ctypes
import math

import numpy as np
import pytest

from tests import cases as C

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

SENTINEL = 12345.0


def run(ncz, p: C.Problem, *, o_dtype="float32", producer="auto", via="auto", splits=None):
    dev = torch.device("cuda:0")
    q = torch.from_numpy(p.q).to(dev)
    k = torch.from_numpy(p.k).to(dev)
    v = torch.from_numpy(p.v).to(dev)
    o = torch.full((p.bh * p.strides[3],), SENTINEL, dtype=getattr(torch, o_dtype), device=dev)
    opts = ncz.Options(seq_len=p.seq, head_dim=p.d, q_stride=p.strides[0], k_stride=p.strides[1],
                       v_stride=p.strides[2], o_stride=p.strides[3], scale=p.scale, batch_heads=p.bh,
                       causal=p.causal)
    plain = p.row_strides is None and o_dtype == "float32" and producer == "auto"
    if splits is not None:
        ncz.launch_splits(q, k, v, o, opts, splits, row_strides=p.row_strides, producer=producer)
    elif via == "launch" or (via == "auto" and plain):
        ncz.launch(q, k, v, o, opts)
    else:
        ncz.launch_ex(q, k, v, o, opts, row_strides=p.row_strides, producer=producer)
    assert ncz.sync_status() == 0
    return o.float().cpu().numpy()


def untouched(got, p, idx):
    mask = np.ones(got.size, dtype=bool)
    mask[idx] = False
    return bool(np.all(got[mask] == SENTINEL))


@pytest.mark.parametrize("case", C.SMOKE_CASES, ids=lambda c: f"bh{c[0]}_s{c[1]}_d{c[2]}_c{int(c[4])}")
def test_reference_smoke_cases(ncz, oracle_mod, case):
    """src/main.zig:189-287: odd slice strides (LSU producer), 0.008 there, 2e-3 here."""
    bh, s, d, strides, causal = case
    p = C.pattern_problem(bh, s, d, strides, causal, oracle_mod)
    got = run(ncz, p)
    want = C.reference(p, oracle_mod)
    idx = C.active_index(p)
    C.check(got, want, idx, f"smoke {case}")
    assert untouched(got, p, idx), "kernel wrote outside the active rows"


@pytest.mark.parametrize("case", C.COMPARE_CASES, ids=lambda c: f"bh{c[0]}_s{c[1]}_d{c[2]}_c{int(c[3])}")
def test_reference_compare_cases(ncz, oracle_mod, case):
    """src/main.zig:141-170 shapes with fillFlashInput data (0.02 there, 2e-3 here)."""
    bh, s, d, causal = case
    p = C.pattern_problem(bh, s, d, (s * d,) * 4, causal, oracle_mod)
    got = run(ncz, p)
    C.check(got, C.reference(p, oracle_mod), C.active_index(p), f"compare {case}")


def test_config1_smoke(ncz, oracle_mod):
    """bh=2, S=64, d=32, causal, N(0, 0.5^2) seed 0, O f32."""
    p = C.normal_problem(2, 64, 32, True, 0, oracle_mod, std=0.5)
    got = run(ncz, p)
    C.check(got, C.reference(p, oracle_mod), C.active_index(p), "config1")


def test_config2_profile_f16_out(ncz, oracle_mod):
    """bh=8, S=1024, d=64, causal, N(0, 0.5^2) seed 1, f16 O."""
    p = C.normal_problem(8, 1024, 64, True, 1, oracle_mod, std=0.5)
    got = run(ncz, p, o_dtype="float16")
    # f16 output adds at most half an f16 ulp of |O| on top of the f32 tolerance.
    C.check(got, C.reference(p, oracle_mod), C.active_index(p), "config2 f16 O", o_unit=2.0 ** -11)


def test_config3_padded_rows_nan_pad(ncz, oracle_mod):
    """bh=512, S=128, d=32, row stride 40 with NaN padding,
    slice stride 128*40, U(-1,1) seed 2, non-causal.  NaN over-reads would poison O."""
    bh, s, d, rs = 512, 128, 32, 40
    st = s * rs
    p = C.Problem(bh, s, d, (st, st, st, s * d), False, 1.0 / math.sqrt(d), row_strides=(rs, rs, rs, d))
    p.q = oracle_mod.fill_uniform(bh * st, 6, -1.0, 1.0)
    p.k = oracle_mod.fill_uniform(bh * st, 7, -1.0, 1.0)
    p.v = oracle_mod.fill_uniform(bh * st, 8, -1.0, 1.0)
    for a in (p.q, p.k, p.v):
        oracle_mod.fill_row_padding(a, bh, s, d, st, rs)
    got = run(ncz, p)
    C.check(got, C.reference(p, oracle_mod), C.active_index(p), "config3")


def test_config4_long_causal_sampled(ncz, oracle_mod):
    """bh=64, S=8192, d=64, causal, N(0,1), K x2 (peaked rows).
    The oracle runs on slices {0, 63} (all rows) and a row band of slice 31;
    all slices are checked for finiteness and the convex-hull property."""
    p = C.normal_problem(64, 8192, 64, True, 3, oracle_mod, std=1.0, k_mul=2.0)
    got = run(ncz, p)
    want = C.reference(p, oracle_mod, slices=[0, 63])
    C.check(got, want, C.active_index(p, slices=[0, 63]), "config4 slices 0,63")
    band = C.reference(p, oracle_mod, slices=[31], rows=(4000, 4200))
    C.check(got, band, C.active_index(p, slices=[31], rows=(4000, 4200)), "config4 slice 31 band")
    o = got.reshape(64, 8192, 64)
    v = p.v.astype(np.float32).reshape(64, 8192, 64)
    assert np.all(np.isfinite(o))
    # O is a convex combination of V rows up to P's f16 rounding (relative 2^-11 per weight).
    slack = 2.0 ** -11 * float(np.abs(v).max()) + 1e-4
    assert np.all(o <= v.max(axis=1, keepdims=True) + slack) and np.all(o >= v.min(axis=1, keepdims=True) - slack)


@pytest.mark.parametrize("d,seed", [(64, 4), (16, 5)])
def test_config5_sweep_sampled(ncz, oracle_mod, d, seed):
    """bh=1024, S=2048, non-causal, N(0, 0.5^2); oracle on 3 slices."""
    p = C.normal_problem(1024, 2048, d, False, seed, oracle_mod, std=0.5)
    got = run(ncz, p)
    sl = [0, 517, 1023]
    C.check(got, C.reference(p, oracle_mod, slices=sl), C.active_index(p, slices=sl), f"config5 d{d}")
    assert np.all(np.isfinite(got))


SEQS = [1, 2, 15, 16, 17, 127, 128, 129, 255, 256, 257, 383, 385, 512, 640, 1000]


@pytest.mark.parametrize("d", [16, 32, 64])
@pytest.mark.parametrize("causal", [False, True])
def test_sequence_residues(ncz, oracle_mod, d, causal):
    """Residue tiles, single-row sequences, odd Q-tile pairs, diagonal tiles."""
    for s in SEQS:
        p = C.normal_problem(3, s, d, causal, 100 + s, oracle_mod, std=0.7)
        got = run(ncz, p)
        C.check(got, C.reference(p, oracle_mod), C.active_index(p), f"S={s} d={d} causal={causal}")


@pytest.mark.parametrize("d", [16, 32, 64])
def test_tma_and_lsu_producers_agree(ncz, oracle_mod, d):
    """Both producers fill identical swizzled tiles, so outputs are bit-identical."""
    p = C.normal_problem(5, 300, d, True, 7, oracle_mod, std=0.6)
    a = run(ncz, p, producer="tma")
    b = run(ncz, p, producer="lsu")
    C.check(a, C.reference(p, oracle_mod), C.active_index(p), "tma")
    assert np.array_equal(a, b)


@pytest.mark.parametrize("scale", [-0.125, 0.0, 2.0])
def test_scale_edge_cases(ncz, oracle_mod, scale):
    """Non-positive scales take the scale-then-mask path; a large scale peaks rows."""
    p = C.normal_problem(2, 200, 32, True, 9, oracle_mod, std=0.5, scale=scale)
    C.check(run(ncz, p), C.reference(p, oracle_mod), C.active_index(p), f"scale={scale}")


def test_multi_descriptor_launch(ncz, oracle_mod):
    """ncz_flash_fwd_multi: two slice shards (on device 0) in one call."""
    p = C.normal_problem(6, 333, 64, False, 11, oracle_mod)
    dev = torch.device("cuda:0")
    n = 333 * 64
    q, k, v = (torch.from_numpy(a).to(dev) for a in (p.q, p.k, p.v))
    o = torch.full((6 * n,), SENTINEL, dtype=torch.float32, device=dev)
    descs = []
    for lo, hi in ((0, 4), (4, 6)):
        opts = ncz.Options(seq_len=333, head_dim=64, q_stride=n, k_stride=n, v_stride=n, o_stride=n,
                           scale=p.scale, batch_heads=hi - lo)
        descs.append(ncz.flash.make_desc(q[lo * n:hi * n], k[lo * n:hi * n], v[lo * n:hi * n], o[lo * n:hi * n],
                                         opts, device=0))
    ncz.launch_multi(descs)
    assert ncz.sync_status() == 0
    C.check(o.cpu().numpy(), C.reference(p, oracle_mod), C.active_index(p), "multi")


def test_invalid_arguments_raise_before_launch(ncz):
    dev = torch.device("cuda:0")
    t = torch.zeros(64 * 16, dtype=torch.float16, device=dev)
    o = torch.zeros(64 * 16, dtype=torch.float32, device=dev)
    before = ncz.flash.launch_count()
    bad = [
        dict(seq_len=64, head_dim=48, q_stride=64 * 48, k_stride=64 * 48, v_stride=64 * 48, o_stride=64 * 48),
        dict(seq_len=0, head_dim=16, q_stride=0, k_stride=0, v_stride=0, o_stride=0),
        dict(seq_len=64, head_dim=16, q_stride=64 * 16 - 1, k_stride=1024, v_stride=1024, o_stride=1024),
        dict(seq_len=64, head_dim=16, q_stride=1024, k_stride=1024, v_stride=1024, o_stride=1024, batch_heads=2),
    ]
    for kw in bad:
        with pytest.raises(ncz.FlashError) as e:
            ncz.launch(t, t, t, o, ncz.Options(scale=0.25, **kw))
        assert e.value.name == "InvalidValue"
    assert ncz.flash.launch_count() == before


def test_status_word_clean(ncz):
    assert ncz.sync_status() == 0


@pytest.mark.parametrize("d", [16, 32, 64])
@pytest.mark.parametrize("producer", ["tma", "lsu"])
def test_causal_first_row_is_exact(ncz, oracle_mod, d, producer):
    """Under causal masking row 0 sees only key 0: p = 2^0 = 1 exactly, so O[0] == V[0]
    bit for bit in every slice.  Size-independent; catches any stray value in the row max."""
    bh, s = 48, 700
    p = C.normal_problem(bh, s, d, True, 31, oracle_mod, std=0.8)
    got = run(ncz, p, producer=producer).reshape(bh, s, d)
    v = p.v.astype(np.float32).reshape(bh, s, d)
    assert np.array_equal(got[:, 0, :], v[:, 0, :])


@pytest.mark.parametrize("d", [16, 32, 64])
def test_repeated_launches_are_bit_identical(ncz, oracle_mod, d):
    """No data races: the same launch repeated gives identical bits (both producers)."""
    p = C.normal_problem(24, 1100, d, False, 41, oracle_mod, std=0.6)
    for producer in ("tma", "lsu"):
        first = run(ncz, p, producer=producer)
        assert np.isfinite(first).all()
        for _ in range(3):
            assert np.array_equal(run(ncz, p, producer=producer), first)
    assert np.array_equal(run(ncz, p, producer="tma"), run(ncz, p, producer="lsu"))


@pytest.mark.parametrize("chunk", [0, 1, 3, 7, 64])
@pytest.mark.parametrize("o_dtype", ["float32", "float16"])
def test_host_pipeline_matches_device_launch(ncz, oracle_mod, qsplit_mode, chunk, o_dtype):
    """ncz_flash_fwd_host (chunked upload / forward / download on three streams)
    gives exactly the device-path result (with items of two Q tiles in every
    launch: a small chunk would otherwise take split-Q items, which sum in
    another order), for chunk sizes that do and do not
    divide batch_heads, with padded slice strides (the last chunk copies only up
    to its last row)."""
    qsplit_mode(2)
    bh, s, d = 7, 333, 64
    strides = (s * d + 24, s * d + 40, s * d + 8, s * d + 16)
    p = C.normal_problem(bh, s, d, True, 61, oracle_mod, std=0.7, strides=strides)
    dev = torch.device("cuda:0")
    q, k, v = (torch.from_numpy(a).to(dev) for a in (p.q, p.k, p.v))
    o_ref = torch.full((bh * strides[3],), SENTINEL, dtype=getattr(torch, o_dtype), device=dev)
    opts = ncz.Options(seq_len=s, head_dim=d, q_stride=strides[0], k_stride=strides[1], v_stride=strides[2],
                       o_stride=strides[3], scale=p.scale, batch_heads=bh, causal=True)
    ncz.launch_ex(q, k, v, o_ref, opts)
    assert ncz.sync_status() == 0
    want = o_ref.cpu()

    qh, kh, vh = (torch.from_numpy(a).pin_memory() for a in (p.q, p.k, p.v))
    oh = torch.full((bh * strides[3],), SENTINEL, dtype=getattr(torch, o_dtype)).pin_memory()
    qd, kd, vd = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)
    od = torch.full_like(o_ref, SENTINEL)
    stream = torch.cuda.Stream(dev)
    ncz.launch_host(qh, kh, vh, oh, qd, kd, vd, od, opts, chunk_slices=chunk, stream=stream)
    stream.synchronize()
    assert ncz.sync_status() == 0
    got = oh.clone()
    idx = C.active_index(p)
    ti = torch.from_numpy(idx)
    assert torch.equal(got[ti], want[ti])
    C.check(got.float().numpy(), C.reference(p, oracle_mod), idx, f"host pipeline chunk={chunk} {o_dtype}",
            o_unit=2.0 ** -11 if o_dtype == "float16" else 0.0)


@pytest.mark.parametrize("chunk", [0, 1, 3, 8])
def test_host_pipeline_twin_items_match_device_launch(ncz, oracle_mod, chunk):
    """seq_len <= 128 through ncz_flash_fwd_host: every chunk runs twin items
    (two slices per item), chunks of an odd slice count end with an item of
    one slice; the result equals the device-path launch bit for bit and meets
    the parity bound."""
    bh, s, d = 37, 100, 32
    p = C.normal_problem(bh, s, d, True, 63, oracle_mod, std=0.7)
    dev = torch.device("cuda:0")
    q, k, v = (torch.from_numpy(a).to(dev) for a in (p.q, p.k, p.v))
    opts = C_opts(p)
    o_ref = torch.full((bh * s * d,), SENTINEL, dtype=torch.float32, device=dev)
    ncz.launch_ex(q, k, v, o_ref, opts)
    assert ncz.sync_status() == 0
    qh, kh, vh = (torch.from_numpy(a).pin_memory() for a in (p.q, p.k, p.v))
    oh = torch.full((bh * s * d,), SENTINEL, dtype=torch.float32).pin_memory()
    qd, kd, vd, od = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty_like(o_ref)
    ncz.launch_host(qh, kh, vh, oh, qd, kd, vd, od, opts, chunk_slices=chunk)
    torch.cuda.synchronize()
    assert ncz.sync_status() == 0
    assert torch.equal(oh, o_ref.cpu())
    C.check(oh.numpy(), C.reference(p, oracle_mod), C.active_index(p), f"host pipeline twin chunk={chunk}")


SPLIT_CASES = [(4, 1024, 64, True), (3, 1000, 64, False), (2, 777, 32, True), (5, 1300, 16, True),
               (1, 4096, 64, True)]


@pytest.mark.parametrize("case", SPLIT_CASES, ids=lambda c: f"bh{c[0]}_s{c[1]}_d{c[2]}_c{int(c[3])}")
@pytest.mark.parametrize("splits", [2, 3, 8])
def test_split_kv_matches_oracle(ncz, oracle_mod, case, splits):
    """Split-KV (K ranges on separate CTAs, merged by combine_splits) against the
    oracle, next to the unsplit launch; nothing outside the active rows is written."""
    bh, s, d, causal = case
    p = C.normal_problem(bh, s, d, causal, 71, oracle_mod, std=0.8)
    want = C.reference(p, oracle_mod)
    idx = C.active_index(p)
    for sp in (1, splits):
        got = run(ncz, p, splits=sp)
        C.check(got, want, idx, f"split-KV splits={sp} {case}")
        assert untouched(got, p, idx)


def test_config2_split_and_unsplit_match(ncz, oracle_mod):
    """BASELINE config 2 (bh=8, S=1024, d=64, causal, f16 O): the automatic
    choice does not split (8 K tiles are too few to pay for a second launch);
    a forced 4-way split gives the same result within tolerance."""
    p = C.normal_problem(8, 1024, 64, True, 1, oracle_mod, std=0.5)
    want = C.reference(p, oracle_mod)
    idx = C.active_index(p)
    before = ncz.flash.launch_count()
    auto = run(ncz, p, o_dtype="float16", splits=0)
    assert ncz.flash.launch_count() - before == 1
    C.check(auto, want, idx, "config 2 auto (f16 O)", o_unit=2.0 ** -11)
    before = ncz.flash.launch_count()
    split = run(ncz, p, o_dtype="float16", splits=4)
    assert ncz.flash.launch_count() - before == 2  # forward + combine
    C.check(split, want, idx, "config 2 split 4 (f16 O)", o_unit=2.0 ** -11)


def test_long_sequence_few_slices_splits_automatically(ncz, oracle_mod):
    """bh=1, S=4096 causal: 16 CTAs for 32 K tiles, so the automatic choice splits
    (forward + combine) and matches the oracle."""
    p = C.normal_problem(1, 4096, 64, True, 5, oracle_mod, std=0.7)
    before = ncz.flash.launch_count()
    got = run(ncz, p, splits=0)
    assert ncz.flash.launch_count() - before == 2
    C.check(got, C.reference(p, oracle_mod), C.active_index(p), "bh=1 S=4096 auto split")


@pytest.mark.parametrize("d", [16, 32, 64])
def test_split_kv_tma_equals_lsu(ncz, oracle_mod, d):
    """Both producers give bit-identical split results (same partials, same merge)."""
    p = C.normal_problem(3, 900, d, True, 81, oracle_mod, std=0.6)
    a = run(ncz, p, splits=4, producer="tma")
    b = run(ncz, p, splits=4, producer="lsu")
    assert np.array_equal(a, b)
    assert np.array_equal(run(ncz, p, splits=4, producer="tma"), a)


def test_split_kv_repeated_launches_and_streams(ncz, oracle_mod):
    """Repeated split launches (partials in the stream-ordered pool) on one stream
    and on a second stream stay bit-identical."""
    p = C.normal_problem(4, 2048, 64, True, 91, oracle_mod, std=0.7)
    first = run(ncz, p, splits=4)
    for _ in range(3):
        assert np.array_equal(run(ncz, p, splits=4), first)
    dev = torch.device("cuda:0")
    q, k, v = (torch.from_numpy(a).to(dev) for a in (p.q, p.k, p.v))
    opts = ncz.Options(seq_len=p.seq, head_dim=p.d, q_stride=p.strides[0], k_stride=p.strides[1],
                       v_stride=p.strides[2], o_stride=p.strides[3], scale=p.scale, batch_heads=p.bh, causal=True)
    side = torch.cuda.Stream(dev)
    for _ in range(2):
        o = torch.full((p.bh * p.strides[3],), SENTINEL, dtype=torch.float32, device=dev)
        ncz.launch_splits(q, k, v, o, opts, 4, stream=side)
        side.synchronize()
        assert np.array_equal(o.cpu().numpy(), first)
    assert ncz.sync_status() == 0


def _dev_inputs(p):
    dev = torch.device("cuda:0")
    q, k, v = (torch.from_numpy(a).to(dev) for a in (p.q, p.k, p.v))
    opts = C_opts(p)
    return q, k, v, opts


def C_opts(p):
    import importlib

    ncz = importlib.import_module("not-cute-zig_b200")
    return ncz.Options(seq_len=p.seq, head_dim=p.d, q_stride=p.strides[0], k_stride=p.strides[1],
                       v_stride=p.strides[2], o_stride=p.strides[3], scale=p.scale, batch_heads=p.bh,
                       causal=p.causal)


def _out(p, dtype=torch.float32):
    return torch.full((p.bh * p.strides[3],), SENTINEL, dtype=dtype, device=torch.device("cuda:0"))


def test_static_scratch_entry_matches_pool_path(ncz, oracle_mod):
    """ncz_flash_fwd_static (partials in the static device scratch, no allocation)
    gives the pool path's bits when the same split count fits, and the oracle's values."""
    p = C.normal_problem(1, 4096, 64, True, 5, oracle_mod, std=0.7)
    q, k, v, opts = _dev_inputs(p)
    a, b = _out(p), _out(p)
    before = ncz.flash.launch_count()
    ncz.launch_static(q, k, v, a, opts, 0)
    assert ncz.flash.launch_count() - before == 2  # split forward + combine
    ncz.launch_splits(q, k, v, b, opts, 0)
    assert ncz.sync_status() == 0
    assert torch.equal(a, b)
    C.check(a.cpu().numpy(), C.reference(p, oracle_mod), C.active_index(p), "static scratch bh=1 S=4096")


@pytest.mark.parametrize("bh,splits,fits", [(2, 0, 3), (2, 3, 3), (2, 4, 0), (4, 8, 0), (4, 0, 1), (8, 1, 1)])
def test_static_scratch_split_count_must_fit(ncz, oracle_mod, bh, splits, fits):
    """16 MiB of scratch holds 4 Mi floats: at S=8192, d=64 one split of bh slices
    needs bh*8192*66 floats.  The automatic count (0) runs what fits (bh=2: 3
    splits; bh=4: unsplit); an explicit count that fits runs as asked; one that
    does not raises OutOfMemory and launches nothing.  Results equal the pool
    path run with the same split count, bit for bit."""
    p = C.normal_problem(bh, 8192, 64, True, 13, oracle_mod, std=0.7)
    q, k, v, opts = _dev_inputs(p)
    a, b = _out(p), _out(p)
    before = ncz.flash.launch_count()
    if fits == 0:
        with pytest.raises(ncz.FlashError) as err:
            ncz.launch_static(q, k, v, a, opts, splits)
        assert err.value.name == "OutOfMemory" and ncz.flash.launch_count() == before
        assert bool((a == SENTINEL).all())
        return
    ncz.launch_static(q, k, v, a, opts, splits)
    assert ncz.flash.launch_count() - before == (2 if fits > 1 else 1)
    ncz.launch_splits(q, k, v, b, opts, fits)
    assert ncz.sync_status() == 0
    assert torch.equal(a, b)


@pytest.mark.parametrize("kind", ["split_q", "two_tile", "twin"])
def test_expired_wait_reports_device_timeout_and_context_survives(ncz, oracle_mod, qsplit_mode, kind):
    """Failure detection without a GPU fault: with a short wait limit and the
    first scores never signalled (a barrier that nothing completes), the CTA
    aborts cleanly, ncz_flash_sync_status returns DeviceTimeout with the wait
    site (s_full = 5) in the status word, and the same context then runs a
    correct launch.  For each item kind: split-Q (one item of bh=1, S=200:
    the merge hand-offs wait too), two Q tiles (split-Q off), twin (S=100,
    three slices: two items)."""
    import ctypes

    lib = ncz.flash.lib()
    if kind == "twin":
        p = C.normal_problem(3, 100, 64, True, 3, oracle_mod, std=0.6)
    else:
        p = C.normal_problem(1, 200, 64, True, 3, oracle_mod, std=0.6)
    if kind == "two_tile":
        qsplit_mode(2)
    assert lib.ncz_test_set_wait_limit(-1, 20_000_000) == 0  # about 10 ms
    assert lib.ncz_test_drop_arrive(-1, 1) == 0
    try:
        dev = torch.device("cuda:0")
        q, k, v = (torch.from_numpy(a).to(dev) for a in (p.q, p.k, p.v))
        o = torch.full((p.bh * p.strides[3],), SENTINEL, dtype=torch.float32, device=dev)
        ncz.launch(q, k, v, o, C_opts(p))
        detail = ctypes.c_uint32(0)
        rc = lib.ncz_flash_sync_status(-1, None, ctypes.byref(detail))
        assert ncz.flash.STATUS_NAMES[rc] == "DeviceTimeout"
        assert detail.value >> 31 == 1 and (detail.value >> 24) & 0x7F == 5
    finally:
        assert lib.ncz_test_drop_arrive(-1, 0) == 0
        assert lib.ncz_test_set_wait_limit(-1, 0) == 0
    assert ncz.sync_status() == 0  # the word was cleared
    got = run(ncz, p)
    C.check(got, C.reference(p, oracle_mod), C.active_index(p), "launch after an expired wait")


def test_reference_kernel_names(ncz, oracle_mod):
    """launch_named with the reference's kernel names: the same bits as
    flash.launch (itself checked against the oracle) for every name that takes
    the head_dim; h64_causal is causal with the flag off; a head_dim the name
    does not take leaves O untouched."""
    dev = torch.device("cuda:0")

    def problem(bh, s, d, seed):
        p = C.normal_problem(bh, s, d, True, seed, oracle_mod, std=1.0)
        q, k, v = (torch.from_numpy(a).to(dev) for a in (p.q, p.k, p.v))
        return p, q, k, v, ncz.Options(seq_len=s, head_dim=d, q_stride=s * d, k_stride=s * d, v_stride=s * d,
                                       o_stride=s * d, scale=1.0 / math.sqrt(d), batch_heads=bh, causal=True)

    for d in (16, 32, 64):
        p, q, k, v, opts = problem(3, 700, d, 11 + d)
        want = torch.zeros(q.numel(), dtype=torch.float32, device=dev)
        ncz.launch(q, k, v, want, opts)
        C.check(want.cpu().numpy(), C.reference(p, oracle_mod), C.active_index(p), f"flash.launch d={d}")
        for name in ncz.flash.REFERENCE_KERNELS:
            dims, always_causal = ncz.flash.kernel_info(name)
            o = torch.full_like(want, 7.0)
            ncz.launch_named(name, q, k, v, o, opts)
            torch.cuda.synchronize()
            if d in dims:
                assert torch.equal(o, want), (name, d)
            else:
                assert bool((o == 7.0).all()), (name, d)
    _, q, k, v, opts = problem(2, 513, 64, 91)
    want = torch.zeros(q.numel(), dtype=torch.float32, device=dev)
    ncz.launch(q, k, v, want, opts)
    opts.causal = False
    o = torch.zeros_like(want)
    ncz.launch_named("flash_attention_fwd_h64_causal", q, k, v, o, opts)
    other = torch.zeros_like(want)
    ncz.launch_named("flash_attention_fwd_h64_bn32", q, k, v, other, opts)
    torch.cuda.synchronize()
    assert torch.equal(o, want) and not torch.equal(other, want)
    assert ncz.sync_status() == 0


def test_compare_harness_records(ncz):
    """compare.py (the reference's compareFlash + JSONL record) on three of the
    reference shapes: correct against fp32 torch attention, rates consistent."""
    import importlib

    compare = importlib.import_module("not-cute-zig_b200.compare")
    for bh, s, d, causal in ((2, 32, 16, False), (8, 256, 32, True), (8, 1024, 64, True)):
        rec = compare.compare_shape(ncz, bh, s, d, causal)
        assert rec["correct"] and rec["max_abs_error"] <= 2e-3
        assert rec["tflops"] == pytest.approx(rec["flops"] / (rec["mean_ms"] * 1e9))
        assert rec["min_ms"] <= rec["mean_ms"] <= rec["max_ms"] and rec["gpus"] == 1
        assert rec["label"] == f"flash_fwd_sm100a_d{d}"


def test_compare_cli_layout_and_type_flags(ncz, tmp_path):
    """compare.py's --seed / --in-dtype / --o-dtype / --row-stride: N(0,1)
    inputs, padded rows (O padding untouched), bf16 inputs, f16 and bf16 O,
    each within the compare bound against fp32 torch attention."""
    import importlib
    import json

    compare = importlib.import_module("not-cute-zig_b200.compare")
    out = tmp_path / "records.jsonl"
    argv = ["--shape", "4,1000,32,1", "--shape", "2,300,64,0", "--row-stride", "72", "--seed", "7",
            "--jsonl", str(out)]
    for in_dtype, o_dtype in (("f16", "f32"), ("bf16", "f16"), ("f16", "bf16")):
        assert compare.main(argv + ["--in-dtype", in_dtype, "--o-dtype", o_dtype]) == 0
    recs = [json.loads(line) for line in out.read_text().splitlines()]
    assert len(recs) == 6 and all(r["correct"] for r in recs)
    assert all("row_stride=72" in r["shape"] and "seed=7" in r["shape"] for r in recs)
    assert max(r["max_abs_error"] for r in recs[:2]) <= 2e-3  # f32 O: the parity bound


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_compare_harness_multi_device(ncz):
    import importlib

    compare = importlib.import_module("not-cute-zig_b200.compare")
    rec = compare.compare_shape(ncz, 8, 1024, 64, True, gpus=2)
    assert rec["correct"] and rec["gpus"] == 2 and len(rec["device_ms"]) == 2
    assert rec["mean_ms"] >= max(rec["device_ms"]) - 1e-6  # the slowest device per iteration


def test_host_pipeline_tapered_default_matches_device_launch(ncz, oracle_mod, qsplit_mode):
    """bh=96, S=1024: the default plan tapers (3, 6, 12 x 6, 6, 6, 3 slices); the
    result equals the device path bit for bit (items of two Q tiles in every
    launch), and with the automatic item kinds (split-Q in the small chunks)
    it meets the parity bound."""
    qsplit_mode(2)
    bh, s, d = 96, 1024, 64
    p = C.normal_problem(bh, s, d, True, 67, oracle_mod, std=0.7)
    dev = torch.device("cuda:0")
    q, k, v = (torch.from_numpy(a).to(dev) for a in (p.q, p.k, p.v))
    opts = C_opts(p)
    o_ref = torch.empty(bh * s * d, dtype=torch.float32, device=dev)
    ncz.launch(q, k, v, o_ref, opts)
    qh, kh, vh = (torch.from_numpy(a).pin_memory() for a in (p.q, p.k, p.v))
    oh = torch.full((bh * s * d,), SENTINEL, dtype=torch.float32).pin_memory()
    qd, kd, vd, od = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v), torch.empty_like(o_ref)
    before = ncz.flash.launch_count()
    ncz.launch_host(qh, kh, vh, oh, qd, kd, vd, od, opts)
    torch.cuda.synchronize()
    assert ncz.flash.launch_count() - before == 11
    assert ncz.sync_status() == 0
    assert torch.equal(oh, o_ref.cpu())
    qsplit_mode(0)
    ncz.launch_host(qh, kh, vh, oh, qd, kd, vd, od, opts)
    torch.cuda.synchronize()
    assert ncz.sync_status() == 0
    C.check(oh.numpy(), C.reference(p, oracle_mod), C.active_index(p), "host pipeline, automatic item kinds")


def _run_bf16(ncz, p, o_dtype=torch.float32, producer="auto", splits=None):
    dev = torch.device("cuda:0")
    q, k, v = (torch.from_numpy(a.view(np.int16)).to(dev).view(torch.bfloat16) for a in (p.q, p.k, p.v))
    o = torch.full((p.bh * p.strides[3],), SENTINEL, dtype=o_dtype, device=dev)
    if splits is None:
        ncz.launch_ex(q, k, v, o, C_opts(p), row_strides=p.row_strides, producer=producer)
    else:
        ncz.launch_splits(q, k, v, o, C_opts(p), splits, producer=producer)
    assert ncz.sync_status() == 0
    return o.float().cpu().numpy()


BF16_CASES = [(2, 200, 64, True), (3, 333, 32, False), (2, 129, 16, True), (1, 1024, 64, False),
              (4, 1000, 64, True)]


@pytest.mark.parametrize("case", BF16_CASES, ids=lambda c: f"bh{c[0]}_s{c[1]}_d{c[2]}_c{int(c[3])}")
@pytest.mark.parametrize("producer", ["tma", "lsu"])
def test_bf16_inputs_match_oracle(ncz, oracle_mod, case, producer):
    """bf16 Q/K/V (the kernel's bf16 variant: bf16 MMAs, P rounded to bf16)
    against the oracle's bf16 path, within the bf16 bound; TMA = LSU bit-exact."""
    bh, s, d, causal = case
    p = C.normal_problem_bf16(bh, s, d, causal, 23, oracle_mod, std=0.8)
    got = _run_bf16(ncz, p, producer=producer)
    idx = C.active_index(p)
    C.check(got, C.reference(p, oracle_mod), idx, f"bf16 {case} {producer}", atol=C.ATOL_BF16,
            p_unit=C.P_UNIT_BF16)
    assert untouched(got, p, idx)
    if producer == "lsu":
        assert np.array_equal(got, _run_bf16(ncz, p, producer="tma"))


@pytest.mark.parametrize("o_dtype", [torch.float16, torch.bfloat16])
def test_bf16_inputs_16bit_outputs(ncz, oracle_mod, o_dtype):
    p = C.normal_problem_bf16(3, 700, 64, True, 29, oracle_mod, std=0.7)
    got = _run_bf16(ncz, p, o_dtype=o_dtype)
    C.check(got, C.reference(p, oracle_mod), C.active_index(p), f"bf16 in, {o_dtype} out", atol=C.ATOL_BF16,
            p_unit=C.P_UNIT_BF16)


def test_bf16_split_kv(ncz, oracle_mod):
    p = C.normal_problem_bf16(1, 4096, 64, True, 31, oracle_mod, std=0.7)
    got = _run_bf16(ncz, p, splits=4)
    C.check(got, C.reference(p, oracle_mod), C.active_index(p), "bf16 split-KV", atol=C.ATOL_BF16,
            p_unit=C.P_UNIT_BF16)


def test_bf16_output_from_f16_inputs(ncz, oracle_mod):
    """bf16 O from f16 inputs (O type is independent of the input type)."""
    p = C.normal_problem(2, 300, 32, False, 37, oracle_mod, std=0.7)
    got = run(ncz, p, o_dtype="bfloat16")
    C.check(got, C.reference(p, oracle_mod), C.active_index(p), "f16 in, bf16 out", atol=C.ATOL_BF16,
            o_unit=2.0 ** -8)


def test_many_items_per_cta_with_empty_q_tiles(ncz, oracle_mod):
    """bh=300, S=600, causal: 900 work items, one resident CTA per SM taking
    further items through launch control (Q double-buffered across them,
    pipelines swapping Q tiles per item), and every slice's last item has an
    empty second Q tile (rows 640.. >= S); all rows against the oracle."""
    p = C.normal_problem(300, 600, 32, True, 71, oracle_mod, std=0.8)
    got = run(ncz, p)
    idx = C.active_index(p)
    C.check(got, C.reference(p, oracle_mod), idx, "bh=300 S=600 causal (item walk)")
    assert untouched(got, p, idx)


def test_item_walk_split_kv_with_empty_ranges(ncz, oracle_mod):
    """bh=2, S=8192, causal, 8 forced splits: 512 items, most early groups' later
    K ranges empty (items without work taken and passed on); two slices' head
    and tail rows against the oracle."""
    p = C.normal_problem(2, 8192, 64, True, 73, oracle_mod, std=0.7)
    got = run(ncz, p, splits=8)
    for rows in ((0, 300), (7900, 8192)):
        idx = C.active_index(p, rows=rows)
        C.check(got, C.reference(p, oracle_mod, rows=rows), idx, f"split 8 rows {rows}")


def test_item_order_chunks_with_short_last_chunk(ncz, oracle_mod):
    """bh=20, S=8192, d=64, causal: 2 MB of K/V per slice, so the item order runs
    a chunk of 16 slices, then a short chunk of 4; head, middle and tail rows of
    slices on both sides of the chunk edge against the oracle."""
    p = C.normal_problem(20, 8192, 64, True, 79, oracle_mod, std=0.7)
    got = run(ncz, p)
    sl = [0, 15, 16, 19]
    for rows in ((0, 130), (4000, 4100), (8100, 8192)):
        idx = C.active_index(p, slices=sl, rows=rows)
        want = C.reference(p, oracle_mod, slices=sl, rows=rows)
        C.check(got, want, idx, f"chunked order rows {rows}")


def test_item_walk_lsu_equals_tma(ncz, oracle_mod):
    """bh=300, S=600, d=32, causal: 900 items walked through launch control with
    each producer (TMA, and plain loads that request the next item the same
    way); bit-identical outputs, against the oracle."""
    p = C.normal_problem(300, 600, 32, True, 83, oracle_mod, std=0.8)
    a = run(ncz, p, producer="tma")
    b = run(ncz, p, producer="lsu")
    C.check(a, C.reference(p, oracle_mod), C.active_index(p), "item walk, TMA producer")
    assert np.array_equal(a, b)


QSPLIT_CASES = [(8, 1024, 64, True), (3, 1000, 64, False), (2, 129, 32, True), (5, 100, 16, True),
                (4, 777, 64, True), (1, 4096, 32, True), (300, 600, 64, True)]


@pytest.fixture
def qsplit_mode(ncz):
    """Sets the split-Q choice for one test and restores the automatic one."""
    lib = ncz.flash.lib()

    def set_mode(mode):
        assert lib.ncz_test_set_qsplit(mode) == 0

    yield set_mode
    assert lib.ncz_test_set_qsplit(0) == 0


@pytest.mark.parametrize("case", QSPLIT_CASES, ids=lambda c: f"bh{c[0]}_s{c[1]}_d{c[2]}_c{int(c[3])}")
def test_split_q_items_match_oracle(ncz, oracle_mod, qsplit_mode, case):
    """Split-Q items (one Q tile per item, its K tiles alternating between the
    two pipelines, states merged in the CTA) against the oracle, next to items
    of two Q tiles; nothing outside the active rows written.  bh=300, S=600
    gives 1500 items walked by 148 CTAs (merge barriers over many items)."""
    bh, s, d, causal = case
    p = C.normal_problem(bh, s, d, causal, 83, oracle_mod, std=0.8)
    want = C.reference(p, oracle_mod)
    idx = C.active_index(p)
    for mode in (1, 2):
        qsplit_mode(mode)
        got = run(ncz, p)
        C.check(got, want, idx, f"split-Q mode {mode} {case}")
        assert untouched(got, p, idx)


def test_split_q_producers_and_output_types(ncz, oracle_mod, qsplit_mode):
    """Split-Q with the plain-load producer (bit-identical to TMA), f16 O and
    bf16 inputs."""
    qsplit_mode(1)
    p = C.normal_problem(3, 555, 64, True, 89, oracle_mod, std=0.7)
    want = C.reference(p, oracle_mod)
    idx = C.active_index(p)
    a = run(ncz, p, producer="tma")
    b = run(ncz, p, producer="lsu")
    assert np.array_equal(a, b)
    C.check(a, want, idx, "split-Q tma")
    C.check(run(ncz, p, o_dtype="float16"), want, idx, "split-Q f16 O", o_unit=2.0 ** -11)
    pb = C.normal_problem_bf16(2, 700, 32, True, 97, oracle_mod, std=0.7)
    C.check(_run_bf16(ncz, pb), C.reference(pb, oracle_mod), C.active_index(pb), "split-Q bf16",
            atol=C.ATOL_BF16, p_unit=C.P_UNIT_BF16)


def test_mixed_split_q_and_two_tile_items(ncz, oracle_mod, qsplit_mode):
    """bh=5, S=8192, causal, the top 15 of 32 groups forced to split-Q items
    and the rest run as items of two Q tiles in one launch (two-tile items
    heavier than the heaviest split-Q item first, then the split-Q items, then
    the lighter two-tile items).  Slices 0 and 4 against the oracle, next to
    the automatic plan (every group split: 160 two-tile items are fewer than
    1.25 per SM) and to two-tile items only."""
    lib = ncz.flash.lib()
    out = (ctypes.c_int32 * 2)()
    assert lib.ncz_test_qsplit_plan(5, 8192, 148, out) == 0 and out[0] == 32
    p = C.normal_problem(5, 8192, 64, True, 101, oracle_mod, std=1.0, k_mul=2.0)
    want = C.reference(p, oracle_mod, slices=[0, 4])
    idx = C.active_index(p, slices=[0, 4])
    assert lib.ncz_test_set_qsplit_groups(15) == 0
    try:
        C.check(run(ncz, p), want, idx, "mixed split-Q items")
    finally:
        assert lib.ncz_test_set_qsplit_groups(-1) == 0
    qsplit_mode(0)
    C.check(run(ncz, p), want, idx, "automatic plan")
    qsplit_mode(2)
    C.check(run(ncz, p), want, idx, "two-tile items only")


TWIN_CASES = [(513, 128, 32, False), (7, 77, 64, True), (2, 1, 16, True), (64, 128, 64, True), (5, 100, 16, False),
              (1, 128, 64, True)]


@pytest.fixture
def twin_mode(ncz):
    """Sets the twin-item choice for one test and restores the default."""
    lib = ncz.flash.lib()

    def set_mode(enable):
        assert lib.ncz_test_set_twin(enable) == 0

    yield set_mode
    assert lib.ncz_test_set_twin(1) == 0


@pytest.mark.parametrize("case", TWIN_CASES, ids=lambda c: f"bh{c[0]}_s{c[1]}_d{c[2]}_c{int(c[3])}")
def test_twin_items_match_oracle(ncz, oracle_mod, twin_mode, qsplit_mode, case):
    """seq_len <= 128: items of two slices, one per pipeline (an odd count
    ends with an item of one slice), against the oracle; both producers give
    the same bits, and so do items of one slice (with split-Q items off too:
    those merge two states, which rounds differently)."""
    bh, s, d, causal = case
    p = C.normal_problem(bh, s, d, causal, 61 + bh, oracle_mod, std=0.7)
    want = C.reference(p, oracle_mod)
    idx = C.active_index(p)
    a = run(ncz, p, producer="tma")
    assert np.array_equal(a, run(ncz, p, producer="lsu"))
    C.check(a, want, idx, "twin items")
    C.check(run(ncz, p, o_dtype="float16"), want, idx, "twin items f16 O", o_unit=2.0 ** -11)
    twin_mode(0)
    C.check(run(ncz, p, producer="tma"), want, idx, "twin off (automatic plan)")
    qsplit_mode(2)
    assert np.array_equal(a, run(ncz, p, producer="tma"))


def test_twin_items_bf16(ncz, oracle_mod, twin_mode, qsplit_mode):
    """bf16 inputs through twin items, against the oracle; items of one slice
    (split-Q items off) give the same bits."""
    pb = C.normal_problem_bf16(9, 100, 32, True, 71, oracle_mod, std=0.7)
    got = _run_bf16(ncz, pb)
    C.check(got, C.reference(pb, oracle_mod), C.active_index(pb), "twin bf16", atol=C.ATOL_BF16,
            p_unit=C.P_UNIT_BF16)
    twin_mode(0)
    qsplit_mode(2)
    assert np.array_equal(got, _run_bf16(ncz, pb))
