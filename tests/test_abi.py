"""C ABI of libncz_flash.so on the CPU: symbols, validation, dispatch labels,
descriptor encodings.  No compute call needs a GPU here."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "ncz_flash.h")
HEADERS = sorted(os.path.join(ROOT, "include", f) for f in os.listdir(os.path.join(ROOT, "include")) if f.endswith(".h"))


def declared_functions():
    text = "".join(open(h).read() for h in HEADERS)
    return sorted(set(re.findall(r"\b(ncz_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(ncz):
    lib = ncz.flash.lib()
    names = declared_functions()
    assert len(names) >= 19
    assert {"ncz_mma_matmul_pipelined", "ncz_mma_matmul_batched", "ncz_mma_matmul"} <= set(names)
    for name in names:
        assert hasattr(lib, name), name
    out = subprocess.run(["nm", "-D", "--defined-only", ncz.flash.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\b(ncz_[a-z0-9_]+)\b", out))
    assert set(names) <= exported


def test_no_link_time_libcuda_dependency(ncz):
    out = subprocess.run(["ldd", ncz.flash.LIB_PATH], capture_output=True, text=True).stdout
    assert "libcuda.so" not in out


def ref_validate(bh, s, d, qs, ks, vs, os_):
    """src/flash.zig:16-28 restated."""
    if bh == 0 or s == 0:
        return False
    if d not in (16, 32, 64):
        return False
    m = s * d
    return not (qs < m or ks < m or vs < m or os_ < m)


@pytest.mark.parametrize("bh", [0, 1, 3])
@pytest.mark.parametrize("s", [0, 1, 17, 128])
@pytest.mark.parametrize("d", [0, 8, 16, 24, 32, 48, 64, 128])
def test_validate_matches_reference(ncz, bh, s, d):
    lib = ncz.flash.lib()
    for delta in (-1, 0, 5):
        st = max(0, s * d + delta)
        for strides in ((st, st, st, st), (st + 3, st, st, st), (s * d + 7, s * d + 1, st, s * d + 2)):
            want = ref_validate(bh, s, d, *strides)
            got = lib.ncz_flash_validate(bh, s, d, *strides)
            assert (got == 0) == want, (bh, s, d, strides, got)
            if not want:
                assert ncz.flash.STATUS_NAMES[got] == "InvalidValue"


def test_options_validate_raises(ncz):
    with pytest.raises(ncz.FlashError) as e:
        ncz.Options(seq_len=64, head_dim=40, q_stride=4096, k_stride=4096, v_stride=4096, o_stride=4096,
                    scale=0.1).validate()
    assert e.value.name == "InvalidValue"
    ncz.Options(seq_len=64, head_dim=64, q_stride=4096, k_stride=4096, v_stride=4096, o_stride=4096,
                scale=0.1).validate()


@pytest.mark.parametrize("d", [16, 32, 64])
def test_select_kernel(ncz, d):
    sel = ncz.select_kernel(ncz.Options(seq_len=512, head_dim=d, q_stride=512 * d, k_stride=512 * d,
                                        v_stride=512 * d, o_stride=512 * d, scale=0.1, batch_heads=8, causal=True))
    assert sel.label == f"flash_fwd_sm100a_d{d}" and sel.threads == 384


def test_select_rejects_bad_head_dim(ncz):
    with pytest.raises(ncz.FlashError):
        ncz.select_kernel(ncz.Options(seq_len=8, head_dim=128, q_stride=1024, k_stride=1024, v_stride=1024,
                                      o_stride=1024, scale=0.1))


def test_require_len(ncz):
    """src/flash.zig:40-43: each buffer must hold batch_heads * stride elements."""
    lib = ncz.flash.lib()
    bh, s, d = 2, 16, 16
    st = s * d
    args = dict(bh=bh, s=s, d=d)
    base = [bh * st] * 4
    for i in range(4):
        lens = list(base)
        lens[i] -= 1
        rc = lib.ncz_flash_launch(None, lens[0], None, lens[1], None, lens[2], None, lens[3], bh, s, d, st, st, st,
                                  st, ctypes.c_float(0.25), 0, None)
        assert ncz.flash.STATUS_NAMES[rc] == "InvalidValue", (i, rc, args)


def test_overflow_is_reported(ncz):
    lib = ncz.flash.lib()
    huge = 2 ** 63
    rc = lib.ncz_flash_validate(1, huge, 64, 1, 1, 1, 1)
    assert ncz.flash.STATUS_NAMES[rc] == "Overflow"


def test_launch_without_gpu_fails_loudly(ncz):
    """No CPU fallback: with no device the call returns an error, never success."""
    import torch

    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    lib = ncz.flash.lib()
    st = 64 * 16
    rc = lib.ncz_flash_fwd(1, 1, 1, 1, 1, 64, 16, st, st, st, st, ctypes.c_float(0.25), 0, None)
    assert rc != 0
    assert ncz.flash.STATUS_NAMES[rc] in ("NoDevice", "NotInitialized", "NotFound", "UnknownError")


def test_validate_ex_row_strides(ncz):
    lib = ncz.flash.lib()
    D = ncz.flash._Desc

    def desc(**kw):
        d = D()
        d.batch_heads, d.seq_len, d.head_dim = 4, 128, 32
        d.q_stride = d.k_stride = d.v_stride = 128 * 40
        d.o_stride = 128 * 32
        d.q_row_stride = d.k_row_stride = d.v_row_stride = 40
        d.scale, d.device = 0.1, -1
        for key, val in kw.items():
            setattr(d, key, val)
        return d

    assert lib.ncz_flash_validate_ex(ctypes.byref(desc())) == 0
    # last row needs (S-1)*row + d <= slice stride
    assert lib.ncz_flash_validate_ex(ctypes.byref(desc(q_stride=127 * 40 + 32))) == 0
    assert lib.ncz_flash_validate_ex(ctypes.byref(desc(q_stride=127 * 40 + 31))) == 5
    assert lib.ncz_flash_validate_ex(ctypes.byref(desc(k_row_stride=31))) == 5
    assert lib.ncz_flash_validate_ex(ctypes.byref(desc(o_dtype=7))) == 5
    assert lib.ncz_flash_validate_ex(ctypes.byref(desc(producer=9))) == 5
    assert lib.ncz_flash_validate_ex(None) == 5


def test_status_strings(ncz):
    lib = ncz.flash.lib()
    for code, name in ncz.flash.STATUS_NAMES.items():
        assert lib.ncz_status_string(code).decode() == name


def test_umma_smem_descriptor_bits(ncz):
    """tcgen05 shared-memory descriptor fields (PTX ISA): start>>4 @0, LBO>>4 @16,
    SBO>>4 @32, version 1 @46, layout @61."""
    lib = ncz.flash.lib()
    desc = lib.ncz_umma_smem_desc(0x1400, 16, 1024, 2)
    assert desc & 0x3FFF == 0x140
    assert (desc >> 16) & 0x3FFF == 1
    assert (desc >> 32) & 0x3FFF == 64
    assert (desc >> 46) & 3 == 1
    assert (desc >> 49) & 7 == 0
    assert (desc >> 61) & 7 == 2
    # advancing K by 16 f16 (32 bytes) inside a swizzled row adds 2 to the start field
    assert lib.ncz_umma_smem_desc(0x1400 + 32, 16, 1024, 2) == desc + 2
    for layout, span in ((2, 128), (4, 64), (6, 32)):
        d = lib.ncz_umma_smem_desc(0x8000, 16, 8 * span, layout)
        assert (d >> 32) & 0x3FFF == 8 * span // 16 and (d >> 61) == layout


def test_umma_instr_descriptor_bits(ncz):
    """kind::f16 instruction descriptor: D f32 @4, A/B f16 @7/@10, majors @15/@16, N>>3 @17, M>>4 @24."""
    lib = ncz.flash.lib()
    assert lib.ncz_umma_instr_desc_f16(128, 128, 0, 0) == (1 << 4) | (16 << 17) | (8 << 24)
    assert lib.ncz_umma_instr_desc_f16(128, 64, 0, 1) == (1 << 4) | (1 << 16) | (8 << 17) | (8 << 24)
    assert lib.ncz_umma_instr_desc_f16(128, 16, 0, 1) == (1 << 4) | (1 << 16) | (2 << 17) | (8 << 24)


def xor_swizzle(source_bit, target_bit, width, value):
    """layout.XorSwizzle.apply (src/layout.zig:349-357) restated."""
    out = value
    for b in range(width):
        out ^= ((value >> (source_bit + b)) & 1) << (target_bit + b)
    return out


@pytest.mark.parametrize("span", [32, 64, 128])
def test_tma_swizzle_offsets(ncz, span):
    """TMA SWIZZLE_{32,64,128}B: 16-byte chunk index ^= row phase, within 8-row atoms."""
    lib = ncz.flash.lib()
    chunks = span // 16
    seen = set()
    for row in range(16):
        for c in range(chunks):
            for b in (0, 5, 15):
                off = row * span + c * 16 + b
                phase = (off >> 7) & (chunks - 1)
                want = row * span + ((c ^ phase) * 16) + b
                got = lib.ncz_tma_swizzle_offset(span, off)
                assert got == want
                # the reference's XOR hook, generalised to byte addresses: bits [7, 7+w) into [4, 4+w)
                assert got == xor_swizzle(7, 4, chunks.bit_length() - 1, off)
                seen.add(got)
    assert len(seen) == 16 * chunks * 3  # bijective on the tile


def test_shard_ranges(ncz):
    from importlib import import_module

    shard = import_module("not-cute-zig_b200.shard")
    for bh in (1, 7, 64, 1024):
        for world in (1, 2, 4, 8):
            ranges = [shard.slice_range(bh, world, r) for r in range(world)]
            assert ranges[0][0] == 0 and ranges[-1][1] == bh
            assert all(a[1] == b[0] for a, b in zip(ranges, ranges[1:]))
            sizes = [hi - lo for lo, hi in ranges]
            assert max(sizes) - min(sizes) <= 1


def test_host_pipeline_validates_before_any_device_work(ncz):
    """ncz_flash_fwd_host: null host buffers and invalid shapes are rejected
    before the library touches a device; with no device it fails loudly."""
    import torch

    lib = ncz.flash.lib()
    D = ncz.flash._Desc
    st = 64 * 16
    good = D(q=1, k=1, v=1, o=1, batch_heads=2, seq_len=64, head_dim=16, q_stride=st, k_stride=st, v_stride=st,
             o_stride=st, scale=0.25, causal=1, o_dtype=0, producer=0, device=-1, stream=None)
    assert ncz.flash.STATUS_NAMES[lib.ncz_flash_fwd_host(ctypes.byref(good), None, 1, 1, 1, 0)] == "InvalidValue"
    assert ncz.flash.STATUS_NAMES[lib.ncz_flash_fwd_host(None, 1, 1, 1, 1, 0)] == "InvalidValue"
    bad = D.from_buffer_copy(good)
    bad.head_dim = 48
    assert ncz.flash.STATUS_NAMES[lib.ncz_flash_fwd_host(ctypes.byref(bad), 1, 1, 1, 1, 0)] == "InvalidValue"
    if not torch.cuda.is_available():
        rc = lib.ncz_flash_fwd_host(ctypes.byref(good), 1, 1, 1, 1, 0)
        assert ncz.flash.STATUS_NAMES[rc] in ("NoDevice", "NotInitialized", "NotFound", "UnknownError")


def test_split_entry_points_validate(ncz):
    lib = ncz.flash.lib()
    D = ncz.flash._Desc
    st = 64 * 16
    good = D(q=1, k=1, v=1, o=1, batch_heads=2, seq_len=64, head_dim=16, q_stride=st, k_stride=st, v_stride=st,
             o_stride=st, scale=0.25, causal=1, o_dtype=0, producer=0, device=-1, stream=None)
    for fn in (lib.ncz_flash_fwd_splits, lib.ncz_flash_fwd_static):
        assert ncz.flash.STATUS_NAMES[fn(None, 0)] == "InvalidValue"
        assert ncz.flash.STATUS_NAMES[fn(ctypes.byref(good), -1)] == "InvalidValue"
        bad = D.from_buffer_copy(good)
        bad.seq_len = 0
        assert ncz.flash.STATUS_NAMES[fn(ctypes.byref(bad), 2)] == "InvalidValue"


def test_umma_instr_descriptor_bf16(ncz):
    lib = ncz.flash.lib()
    assert lib.ncz_umma_instr_desc_bf16(128, 128, 0, 0) == lib.ncz_umma_instr_desc_f16(128, 128, 0, 0) | (1 << 7) | (1 << 10)
    assert lib.ncz_umma_instr_desc_bf16(128, 64, 0, 1) == lib.ncz_umma_instr_desc_f16(128, 64, 0, 1) | (1 << 7) | (1 << 10)


def test_validate_ex_dtypes(ncz):
    lib = ncz.flash.lib()
    D = ncz.flash._Desc
    st = 64 * 16
    for in_dt, o_dt, ok in ((0, 0, True), (1, 1, True), (2, 2, True), (2, 0, True), (1, 2, True),
                            (3, 0, False), (2, 3, False), (-1, 0, False)):
        d = D(q=1, k=1, v=1, o=1, batch_heads=2, seq_len=64, head_dim=16, q_stride=st, k_stride=st, v_stride=st,
              o_stride=st, scale=0.25, causal=1, o_dtype=o_dt, producer=0, device=-1, stream=None, in_dtype=in_dt)
        assert (lib.ncz_flash_validate_ex(ctypes.byref(d)) == 0) == ok, (in_dt, o_dt)
