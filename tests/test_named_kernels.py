"""The reference's kernel names as aliases (module.getFunction(name) +
Function.launch, src/main.zig:93-94, :820-852) on the CPU, through the fake
devices of the driver-call table: which names launch, for which head_dim,
and which return without launching as the named kernel's entry guard does."""
import ctypes

import pytest

BASE = 0x1000_0000


def named(ncz, kernel, *, bh=4, seq=1024, d=64, causal=1, stride=None):
    stride = seq * d if stride is None else stride
    n = bh * stride
    return ncz.flash.lib().ncz_flash_fwd_named(kernel.encode(), BASE, BASE + 2 * n, BASE + 4 * n, BASE + 6 * n, bh,
                                               seq, d, stride, stride, stride, stride, 0.125, causal, None)


def status(ncz, st):
    return ncz.flash.STATUS_NAMES[st]


def test_every_reference_kernel_name_is_known(ncz):
    info = {name: ncz.flash.kernel_info(name) for name in ncz.flash.REFERENCE_KERNELS}
    assert info == {
        "flash_attention_fwd": ((16, 32, 64), False),
        "flash_attention_fwd_opt": ((16, 32, 64), False),
        "flash_attention_fwd_v2": ((16, 32, 64), False),
        "flash_attention_fwd_h64": ((64,), False),
        "flash_attention_fwd_h64_bn32": ((64,), False),
        "flash_attention_fwd_h64_causal": ((64,), True),
    }
    for d in (16, 32, 64):
        assert ncz.flash.kernel_info(f"flash_fwd_sm100a_d{d}") == ((d,), False)
    with pytest.raises(ncz.FlashError) as err:
        ncz.flash.kernel_info("flash_attention_fwd_h128")
    assert err.value.name == "NotFound"


@pytest.mark.parametrize("kernel", ["flash_attention_fwd", "flash_attention_fwd_opt", "flash_attention_fwd_v2",
                                    "flash_attention_fwd_h64", "flash_attention_fwd_h64_bn32",
                                    "flash_attention_fwd_h64_causal", "flash_fwd_sm100a_d16",
                                    "flash_fwd_sm100a_d32", "flash_fwd_sm100a_d64"])
@pytest.mark.parametrize("d", [16, 32, 64])
def test_name_launches_only_the_head_dims_it_takes(ncz, fake, kernel, d):
    dims, _ = ncz.flash.kernel_info(kernel)
    assert named(ncz, kernel, d=d) == 0
    if d in dims:
        assert [ncz.driver.kernel_label(x.kernel) for x in fake.launches] == [f"flash_fwd<{d},tma,f16>"]
    else:
        assert fake.launches == []  # the named kernel's guard returns without writing O


def test_guards_and_errors(ncz, fake):
    assert named(ncz, "flash_attention_fwd_h64", seq=0) == 0  # seq_len 0: the kernel returns
    assert named(ncz, "flash_attention_fwd_opt", d=48) == 0  # head_dim outside 16/32/64: returns
    assert fake.launches == []
    assert status(ncz, named(ncz, "flash_attention_fwd_h65")) == "NotFound"
    assert status(ncz, named(ncz, "flash_attention_fwd_h64", bh=0)) == "InvalidValue"  # grid.y = 0
    assert status(ncz, named(ncz, "flash_attention_fwd_h64", stride=100)) == "InvalidValue"  # stride < S*d
    lib = ncz.flash.lib()
    st = lib.ncz_flash_fwd_named(None, BASE, BASE, BASE, BASE, 1, 16, 16, 256, 256, 256, 256, 1.0, 0, None)
    assert status(ncz, st) == "InvalidValue"
    assert fake.launches == []
    assert named(ncz, "flash_attention_fwd_h64_causal", causal=0) == 0
    assert len(fake.launches) == 1 and fake.launches[0].grid == 8 * 4  # split-Q items: 8 Q tiles x 4 slices


def test_python_mirror_checks_tensors(ncz):
    torch = pytest.importorskip("torch")
    t = torch.zeros(16, dtype=torch.float16)
    opts = ncz.Options(seq_len=1, head_dim=16, q_stride=16, k_stride=16, v_stride=16, o_stride=16, scale=1.0)
    with pytest.raises(ncz.FlashError):
        ncz.launch_named("flash_attention_fwd_opt", t, t, t, t, opts)  # CPU tensors: rejected before any call
