"""Failure detection on the host: the library's CUDA calls go through an
injectable driver-call table (include/ncz_driver.h).  These CPU tests install
a fake of eight devices (tests/fake_driver.py), make chosen calls fail on
chosen devices, and check that the error reaches the caller as the
reference's CudaError name, that the caller's device is restored, that the
calls after the failing one never run, and that workspace, streams, events
and pools are released.  Nothing here needs a GPU."""
import ctypes
import threading

import pytest

from tests import fake_driver as F

BASE = 0x1000_0000          # fake device addresses (never dereferenced)
SPAN = 0x0100_0000
HOST = 0x2000_0000          # fake host addresses
AUTO, TMA, LSU = 0, 1, 2
F16, BF16 = 1, 2


def status(ncz, st):
    return ncz.flash.STATUS_NAMES[st]


def desc(ncz, device, *, bh=4, seq=1024, d=64, base=BASE, producer=AUTO, in_dtype=F16):
    n = seq * d
    x = ncz.flash._Desc()
    x.q, x.k, x.v, x.o = base, base + bh * n * 2, base + 2 * bh * n * 2, base + 3 * bh * n * 2
    x.batch_heads, x.seq_len, x.head_dim = bh, seq, d
    x.q_stride = x.k_stride = x.v_stride = x.o_stride = n
    x.scale, x.causal, x.o_dtype, x.producer, x.device = 0.125, 1, 0, producer, device
    x.stream, x.in_dtype = None, in_dtype
    return x


def fwd(ncz, x):
    return ncz.flash.lib().ncz_flash_fwd_ex(ctypes.byref(x))


def fwd_host(ncz, x, chunk):
    return ncz.flash.lib().ncz_flash_fwd_host(ctypes.byref(x), HOST, HOST + SPAN, HOST + 2 * SPAN, HOST + 3 * SPAN,
                                              chunk)


def labels(ncz, launches):
    return [ncz.driver.kernel_label(x.kernel) for x in launches]


def split_plan(ncz, bh, seq):
    out = (ctypes.c_int32 * 2)()
    assert ncz.flash.lib().ncz_test_split_plan(bh, seq, 0, 148, out) == 0
    return out[0]


def test_table_layout_and_rejected_tables(ncz):
    lib = ncz.driver.lib()
    assert ctypes.sizeof(ncz.driver.DriverTable) == ctypes.sizeof(ctypes.c_size_t) + 24 * ctypes.sizeof(
        ctypes.c_void_p)
    before = ctypes.cast(ncz.driver.current().launch_kernel, ctypes.c_void_p).value
    empty = ncz.driver.DriverTable()
    empty.size = ctypes.sizeof(empty)
    assert status(ncz, lib.ncz_set_driver(ctypes.byref(empty), None)) == "InvalidValue"
    short = ncz.driver.make_table(F.FakeDevices().table())
    short.size -= 8
    assert status(ncz, lib.ncz_set_driver(ctypes.byref(short), None)) == "InvalidValue"
    assert ctypes.cast(ncz.driver.current().launch_kernel, ctypes.c_void_p).value == before
    bad = ncz.driver.DriverTable()
    bad.size = 3
    assert status(ncz, lib.ncz_get_driver(ctypes.byref(bad))) == "InvalidValue"
    with pytest.raises(ValueError):
        ncz.driver.make_table({})
    assert ncz.driver.kernel_label(0x1234) is None


def test_one_shard_per_device(ncz, fake):
    before = ncz.flash.launch_count()
    ncz.flash.launch_multi([desc(ncz, dev, base=BASE + dev * SPAN) for dev in range(8)])
    assert [x.device for x in fake.launches] == list(range(8))
    assert set(labels(ncz, fake.launches)) == {"flash_fwd<64,tma,f16>"}
    # 4 row groups x 4 slices would leave SMs idle: split-Q items, 8 Q tiles x 4 slices
    assert all(x.grid == 8 * 4 and x.block == 384 for x in fake.launches)
    assert ncz.flash.launch_count() - before == 8
    assert len(fake.encodes) == 24 and {e[2] for e in fake.encodes} == {128}
    assert fake.current() == 0


def test_launch_failure_on_device_3_of_8(ncz, fake):
    fake.fail("launch_kernel", device=3, error=F.LAUNCH_FAILURE)
    with pytest.raises(ncz.FlashError) as err:
        ncz.flash.launch_multi([desc(ncz, dev, base=BASE + dev * SPAN) for dev in range(8)])
    assert err.value.name == "LaunchFailed"
    assert [x.device for x in fake.launches] == [0, 1, 2]
    assert fake.calls[("launch_kernel", 3)] == 1
    assert all(fake.calls[("launch_kernel", dev)] == 0 for dev in range(4, 8))
    assert fake.current() == 0


def test_split_workspace_out_of_memory_on_device_5(ncz, fake):
    x = desc(ncz, 5, bh=1, seq=8192)
    splits = split_plan(ncz, 1, 8192)
    assert splits > 1
    fake.fail("pool_alloc_async", device=5, error=F.MEMORY_ALLOCATION)
    assert status(ncz, fwd(ncz, x)) == "OutOfMemory"
    assert fake.launches == [] and fake.live()["allocs"] == 0 and fake.current() == 0
    assert fwd(ncz, x) == 0  # the same call again: forward, then the merge of the ranges
    assert labels(ncz, fake.launches) == ["flash_fwd<64,tma,f16>", "combine_splits<64>"]
    assert fake.launches[0].grid == 32 * splits and {x.device for x in fake.launches} == {5}
    assert fake.created["alloc"] == 1 and fake.live()["allocs"] == 0
    assert fake.created["pool"] == 1


def test_merge_launch_failure_still_frees_workspace(ncz, fake):
    fake.fail("launch_kernel", device=2, nth=2)
    assert status(ncz, fwd(ncz, desc(ncz, 2, bh=1, seq=8192))) == "LaunchFailed"
    assert labels(ncz, fake.launches) == ["flash_fwd<64,tma,f16>"]
    assert fake.calls[("free_async", 2)] == 1 and fake.live()["allocs"] == 0


def test_pool_creation_failure_then_recovery(ncz, fake):
    fake.fail("pool_create", device=4, error=F.MEMORY_ALLOCATION)
    x = desc(ncz, 4, bh=1, seq=8192)
    assert status(ncz, fwd(ncz, x)) == "OutOfMemory"
    assert fake.live()["pools"] == 0 and fake.launches == []
    assert fwd(ncz, x) == 0 and fwd(ncz, x) == 0
    assert fake.created["pool"] == 1 and len(fake.launches) == 4


def test_static_scratch_allocates_nothing(ncz, fake):
    lib = ncz.flash.lib()
    x = desc(ncz, 0, bh=1, seq=8192)
    assert lib.ncz_flash_fwd_static(ctypes.byref(x), 0) == 0
    assert lib.ncz_flash_fwd_static(ctypes.byref(x), 0) == 0
    assert labels(ncz, fake.launches) == ["flash_fwd<64,tma,f16>", "combine_splits<64>"] * 2
    assert fake.created["alloc"] == 0 and fake.created["pool"] == 0
    assert fake.calls[("symbol_address", 0)] == 1  # resolved once per device
    # an explicit split count whose partials exceed the 16 MiB scratch: refused before any launch
    assert status(ncz, lib.ncz_flash_fwd_static(ctypes.byref(x), 8)) == "OutOfMemory"
    assert len(fake.launches) == 4 and fake.created["alloc"] == 0


def test_static_scratch_unsplit_request_runs_when_one_split_does_not_fit(ncz, fake):
    """bh=8, S=8192, d=64: one split's partials (8*8192*66 floats) exceed the
    scratch.  A request that makes no split (1, or the automatic count, which
    the plan leaves at 1 for a grid this full) writes no partials and runs;
    an explicit 2 still has to fit and is refused."""
    lib = ncz.flash.lib()
    x = desc(ncz, 0, bh=8, seq=8192)
    assert lib.ncz_flash_fwd_static(ctypes.byref(x), 1) == 0
    assert lib.ncz_flash_fwd_static(ctypes.byref(x), 0) == 0
    assert labels(ncz, fake.launches) == ["flash_fwd<64,tma,f16>"] * 2
    assert status(ncz, lib.ncz_flash_fwd_static(ctypes.byref(x), 2)) == "OutOfMemory"
    assert len(fake.launches) == 2 and fake.created["alloc"] == 0 and fake.created["pool"] == 0


def test_device_selection_failures(ncz, fake):
    fake.fail("set_device", device=6, error=F.INVALID_DEVICE)
    assert status(ncz, fwd(ncz, desc(ncz, 6))) == "InvalidDevice"
    assert status(ncz, fwd(ncz, desc(ncz, 9))) == "InvalidDevice"   # past the fake's 8 devices
    assert status(ncz, fwd(ncz, desc(ncz, 64))) == "InvalidDevice"  # past the library's device table
    assert fake.launches == [] and fake.current() == 0
    assert fake.calls[("set_device", 0)] == 0


def test_caller_device_restored_after_success_and_failure(ncz, fake):
    fake.set_current(4)
    assert fwd(ncz, desc(ncz, 1)) == 0
    assert fake.current() == 4
    fake.fail("launch_kernel", device=7)
    assert status(ncz, fwd(ncz, desc(ncz, 7))) == "LaunchFailed"
    assert fake.current() == 4
    assert fwd(ncz, desc(ncz, -1)) == 0  # -1: the caller's device
    assert [x.device for x in fake.launches] == [1, 4]


def test_tensor_map_failure_falls_back_to_plain_loads(ncz, fake):
    fake.fail("encode_tensor_map", times=None)
    assert fwd(ncz, desc(ncz, 0, producer=AUTO)) == 0
    assert labels(ncz, fake.launches) == ["flash_fwd<64,lsu,f16>"]
    assert status(ncz, fwd(ncz, desc(ncz, 0, producer=TMA, base=BASE + SPAN))) == "Misaligned"
    assert len(fake.launches) == 1


def test_unaligned_operands_take_plain_loads_without_encoding(ncz, fake):
    assert fwd(ncz, desc(ncz, 0, base=BASE + 2)) == 0
    assert labels(ncz, fake.launches) == ["flash_fwd<64,lsu,f16>"] and fake.encodes == []
    assert status(ncz, fwd(ncz, desc(ncz, 0, base=BASE + 2, producer=TMA))) == "Misaligned"
    assert fwd(ncz, desc(ncz, 0, producer=LSU)) == 0
    assert labels(ncz, fake.launches)[-1] == "flash_fwd<64,lsu,f16>" and fake.encodes == []


@pytest.mark.parametrize("d", [16, 32, 64])
@pytest.mark.parametrize("in_dtype,name", [(F16, "f16"), (BF16, "bf16")])
def test_variant_by_head_dim_and_input_type(ncz, fake, d, in_dtype, name):
    assert fwd(ncz, desc(ncz, 0, d=d, in_dtype=in_dtype)) == 0
    assert labels(ncz, fake.launches) == [f"flash_fwd<{d},tma,{name}>"]
    assert {e[2] for e in fake.encodes} == {2 * d}  # swizzle span = one row


def test_host_pipeline_copies_and_copy_failure(ncz, fake):
    n = 1024 * 64
    x = desc(ncz, 1, bh=16, seq=1024)
    assert fwd_host(ncz, x, 4) == 0
    # each 4-slice chunk: 16 items of two Q tiles would leave SMs idle, so 8 Q tiles x 4 slices
    assert [l.device for l in fake.launches] == [1] * 4 and all(l.grid == 32 for l in fake.launches)
    up = [c for c in fake.copies if c[1] == ncz.driver.COPY_HOST_TO_DEVICE]
    down = [c for c in fake.copies if c[1] == ncz.driver.COPY_DEVICE_TO_HOST]
    assert len(up) == 12 and sum(c[2] for c in up) == 3 * 16 * n * 2
    assert len(down) == 4 and sum(c[2] for c in down) == 16 * n * 4
    assert {c[0] for c in fake.copies} == {1} and fake.current() == 0
    assert fake.created["stream"] == 2 and fake.created["event"] == 4
    fake.fail("memcpy_async", device=1, nth=5, error=F.ILLEGAL_ADDRESS)  # chunk 2, second upload
    launched = len(fake.launches)
    assert status(ncz, fwd_host(ncz, x, 4)) == "IllegalAddress"
    assert len(fake.launches) - launched == 1 and fake.current() == 0
    assert fwd_host(ncz, x, 4) == 0  # the pipe stays usable: no new streams or events
    assert len(fake.launches) - launched == 5
    assert fake.created["stream"] == 2 and fake.created["event"] == 4


def test_host_pipeline_setup_failure_releases_what_it_made(ncz, fake):
    fake.fail("event_create", device=2, nth=3, error=F.MEMORY_ALLOCATION)
    x = desc(ncz, 2, bh=8, seq=1024)
    assert status(ncz, fwd_host(ncz, x, 0)) == "OutOfMemory"
    assert fake.live()["streams"] == 0 and fake.live()["events"] == 0 and fake.launches == []
    assert fwd_host(ncz, x, 0) == 0
    assert fake.live()["streams"] == 2 and fake.live()["events"] == 4


@pytest.mark.parametrize("error,name", [(F.NO_DEVICE, "NoDevice"), (F.INITIALIZATION_ERROR, "NotInitialized"),
                                        (35, "NotInitialized")])
def test_initialisation_failures_are_retried(ncz, fake, error, name):
    fake.device_count_error = error
    assert status(ncz, fwd(ncz, desc(ncz, 0))) == name
    fake.device_count_error = 0
    fake.count = 0
    assert status(ncz, fwd(ncz, desc(ncz, 0))) == "NoDevice"
    fake.count = 8
    fake.encoder_error = 500
    assert status(ncz, fwd(ncz, desc(ncz, 0))) == "NotFound"
    fake.encoder_error = 0
    assert fwd(ncz, desc(ncz, 0)) == 0 and len(fake.launches) == 1


def test_sync_status_reads_and_clears_the_device_word(ncz, fake):
    lib = ncz.flash.lib()
    detail = ctypes.c_uint32(0)
    fake.symbol_words[3] = 5
    assert status(ncz, lib.ncz_flash_sync_status(3, None, ctypes.byref(detail))) == "DeviceTimeout"
    assert detail.value == 5 and fake.symbol_writes == [(3, b"\0\0\0\0")]
    assert lib.ncz_flash_sync_status(3, None, ctypes.byref(detail)) == 0 and detail.value == 0
    fake.fail("stream_synchronize", device=1, error=F.ILLEGAL_ADDRESS)
    assert status(ncz, lib.ncz_flash_sync_status(1, None, ctypes.byref(detail))) == "IllegalAddress"
    assert fake.current() == 0
    assert lib.ncz_test_set_wait_limit(6, 1000) == 0 and fake.symbol_writes[-1][0] == 6
    assert fake.current() == 0


def test_gemm_launch_and_status_per_device(ncz, fake):
    lib = ncz.mma.lib()
    fake.set_current(2)
    a, b, c, d = BASE, BASE + SPAN, BASE + 2 * SPAN, BASE + 3 * SPAN
    assert lib.ncz_mma_matmul_pipelined(a, b, c, d, 1.0, 0.0, 1024, 512, 128, 4, 0, 100000, None) == 0
    assert lib.ncz_mma_matmul_batched(a, b, c, d, 1.0, 0.0, 256, 128, 128, 4, None) == 0
    assert labels(ncz, fake.launches) == ["mma_gemm<row_b>", "mma_gemm<col_b>"]
    assert [x.grid for x in fake.launches] == [2 * 148, 1] and {x.device for x in fake.launches} == {2}
    fake.fail("launch_kernel", device=2)
    assert status(ncz, lib.ncz_mma_matmul(a, b, c, d, 1.0, 0.0, None)) == "LaunchFailed"
    fake.symbol_words[5] = 1
    assert status(ncz, lib.ncz_mma_sync_status(5)) == "DeviceTimeout" and fake.current() == 2
    assert lib.ncz_mma_sync_status(5) == 0
    fake.fail("device_synchronize", device=2, error=F.LAUNCH_FAILURE)
    assert status(ncz, lib.ncz_mma_sync_status(-1)) == "LaunchFailed"


def test_threads_as_ranks_one_failing(ncz, fake):
    """Four host threads stand in for four ranks, each on its own device; the
    launch on device 2 fails and only that rank sees the error."""
    fake.fail("launch_kernel", device=2)
    results = {}

    def rank(r):
        fake.set_current(r)
        st = fwd(ncz, desc(ncz, -1, base=BASE + r * SPAN))
        results[r] = (status(ncz, st), fake.current())

    threads = [threading.Thread(target=rank, args=(r,)) for r in range(4)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=60)
    assert results == {0: ("Success", 0), 1: ("Success", 1), 2: ("LaunchFailed", 2), 3: ("Success", 3)}
    assert sorted(x.device for x in fake.launches) == [0, 1, 3]


def test_switching_tables_releases_through_the_old_one(ncz, fake):
    assert fwd_host(ncz, desc(ncz, 1, bh=8), 0) == 0
    assert fwd_host(ncz, desc(ncz, 3, bh=8, base=BASE + SPAN), 0) == 0
    assert fwd(ncz, desc(ncz, 5, bh=1, seq=8192, base=BASE + 2 * SPAN)) == 0
    assert fake.live() == {"streams": 4, "events": 8, "pools": 1, "allocs": 0}
    other = F.FakeDevices(2)
    assert ncz.driver.install(other.table()) == 0
    assert fake.live() == {"streams": 0, "events": 0, "pools": 0, "allocs": 0}
    assert fwd(ncz, desc(ncz, 1)) == 0  # initialised again through the new table
    assert other.calls[("get_device_count", 0)] == 1 and len(other.launches) == 1
    assert ncz.driver.install(None) == 0 and other.errors == []


def test_shutdown_releases_everything_and_the_next_call_starts_over(ncz, fake):
    lib = ncz.flash.lib()
    assert fwd_host(ncz, desc(ncz, 2, bh=8), 0) == 0
    assert fwd(ncz, desc(ncz, 6, bh=1, seq=8192, base=BASE + SPAN)) == 0
    assert fake.live() == {"streams": 2, "events": 4, "pools": 1, "allocs": 0}
    assert lib.ncz_shutdown() == 0
    assert fake.live() == {"streams": 0, "events": 0, "pools": 0, "allocs": 0}
    counted = fake.calls[("get_device_count", 0)]
    assert fwd(ncz, desc(ncz, 0)) == 0  # initialised again
    assert fake.calls[("get_device_count", 0)] == counted + 1
    fake.fail("pool_destroy", error=F.ILLEGAL_ADDRESS)
    assert fwd(ncz, desc(ncz, 6, bh=1, seq=8192, base=BASE + SPAN)) == 0
    assert status(ncz, lib.ncz_shutdown()) == "IllegalAddress" and fake.live()["pools"] == 0


def test_release_error_is_reported_and_the_rest_released(ncz, fake):
    before = F.FakeDevices()  # a table to go back to after the failing release
    assert fwd_host(ncz, desc(ncz, 1, bh=8), 0) == 0
    fake.fail("stream_destroy", error=F.ILLEGAL_ADDRESS)
    released = ncz.driver.install(before.table())
    assert status(ncz, released) == "IllegalAddress"
    assert fake.live() == {"streams": 0, "events": 0, "pools": 0, "allocs": 0}
    assert ncz.driver.install(None) == 0 and before.errors == []
