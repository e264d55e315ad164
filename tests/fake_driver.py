"""A fake of N CUDA devices behind the library's driver-call table, for CPU
tests of per-device error propagation and resource release.

Nothing runs: launches, copies and allocations are recorded, handles and
device addresses are distinct integers that are never dereferenced, and the
current device is per host thread, as in the CUDA runtime.  `fail(...)` makes
chosen calls on chosen devices return a CUDA runtime error number.
"""
from __future__ import annotations

import ctypes
import itertools
import threading
from collections import Counter
from dataclasses import dataclass
from typing import Dict, List, Optional

# CUDA runtime error numbers the tests inject.
MEMORY_ALLOCATION = 2
INITIALIZATION_ERROR = 3
INVALID_VALUE = 1
NO_DEVICE = 100
INVALID_DEVICE = 101
ILLEGAL_ADDRESS = 700
LAUNCH_FAILURE = 719
UNKNOWN = 999


@dataclass
class Rule:
    call: str
    device: Optional[int]   # None = any device
    nth: int                # the first matching call that fails (1-based)
    error: int
    times: Optional[int]    # failures left; None = every call from the nth on
    seen: int = 0


@dataclass
class Launch:
    device: int
    kernel: int
    grid: int
    block: int
    smem: int
    stream: int


class FakeDevices:
    def __init__(self, count: int = 8, sms: int = 148):
        self.count = count
        self.sms = sms
        self.device_count_error = 0
        self.encoder_error = 0
        self.lock = threading.RLock()
        self.tls = threading.local()
        self.ids = itertools.count(0x10000, 0x100)
        self.rules: List[Rule] = []
        self.calls: Counter = Counter()          # (entry, device) -> calls
        self.launches: List[Launch] = []
        self.copies: List[tuple] = []            # (device, kind, bytes, stream)
        self.encodes: List[tuple] = []           # (device, base, swizzle)
        self.streams: Dict[int, int] = {}        # live handle -> device
        self.events: Dict[int, int] = {}
        self.pools: Dict[int, int] = {}
        self.allocs: Dict[int, tuple] = {}       # live address -> (device, bytes)
        self.created: Counter = Counter()        # "stream" / "event" / "pool" / "alloc" -> count
        self.symbol_words: Dict[int, int] = {}   # device -> word that symbol_read returns
        self.symbol_writes: List[tuple] = []     # (device, bytes written)
        self.errors: List[str] = []              # misuse seen by the fake (must stay empty)

    # ---- test controls -------------------------------------------------
    def fail(self, call: str, device: Optional[int] = None, nth: int = 1, error: int = LAUNCH_FAILURE,
             times: Optional[int] = 1) -> None:
        self.rules.append(Rule(call, device, nth, error, times))

    def clear_failures(self) -> None:
        self.rules.clear()

    def current(self) -> int:
        return getattr(self.tls, "device", 0)

    def set_current(self, device: int) -> None:
        self.tls.device = device

    def launches_on(self, device: int) -> List[Launch]:
        return [x for x in self.launches if x.device == device]

    def live(self) -> Dict[str, int]:
        return {"streams": len(self.streams), "events": len(self.events), "pools": len(self.pools),
                "allocs": len(self.allocs)}

    # ---- plumbing ---------------------------------------------------------
    def _new(self) -> int:
        return next(self.ids)

    def _check(self, call: str, device: int) -> int:
        """Counts the call and returns the injected error for it, or 0."""
        self.calls[(call, device)] += 1
        for r in self.rules:
            if r.call != call or (r.device is not None and r.device != device):
                continue
            r.seen += 1
            if r.seen >= r.nth and (r.times is None or r.times > 0):
                if r.times is not None:
                    r.times -= 1
                return r.error
        return 0

    def _entry(self, name, fn):
        def call(*args):
            try:
                with self.lock:
                    return fn(*args)
            except Exception as exc:  # a fake bug must fail the test, not read as success
                self.errors.append(f"{name}: {exc!r}")
                return UNKNOWN
        return call

    # ---- the table ------------------------------------------------------------
    def table(self) -> dict:
        entries = {
            "get_device_count": self._get_device_count,
            "get_device": self._get_device,
            "set_device": self._set_device,
            "sm_count": self._sm_count,
            "load_tensor_map_encoder": self._load_encoder,
            "encode_tensor_map": self._encode,
            "set_max_dynamic_smem": lambda kernel, nbytes: self._check("set_max_dynamic_smem", self.current()),
            "launch_kernel": self._launch,
            "stream_create": lambda out: self._create("stream_create", "stream", self.streams, out),
            "stream_destroy": lambda h: self._destroy("stream_destroy", self.streams, h),
            "event_create": lambda out: self._create("event_create", "event", self.events, out),
            "event_destroy": lambda h: self._destroy("event_destroy", self.events, h),
            "event_record": lambda ev, st: self._use("event_record", self.events, ev),
            "stream_wait_event": lambda st, ev: self._use("stream_wait_event", self.events, ev),
            "stream_synchronize": lambda st: self._check("stream_synchronize", self.current()),
            "device_synchronize": lambda: self._check("device_synchronize", self.current()),
            "memcpy_async": self._memcpy,
            "symbol_read": self._symbol_read,
            "symbol_write": self._symbol_write,
            "symbol_address": self._symbol_address,
            "pool_create": self._pool_create,
            "pool_destroy": lambda h: self._destroy("pool_destroy", self.pools, h),
            "pool_alloc_async": self._alloc,
            "free_async": self._free,
        }
        return {name: self._entry(name, fn) for name, fn in entries.items()}

    def _get_device_count(self, out):
        e = self.device_count_error or self._check("get_device_count", self.current())
        if e == 0:
            out[0] = self.count
        return e

    def _get_device(self, out):
        e = self._check("get_device", self.current())
        if e == 0:
            out[0] = self.current()
        return e

    def _set_device(self, device):
        if not 0 <= device < self.count:
            return INVALID_DEVICE
        e = self._check("set_device", device)
        if e == 0:
            self.set_current(device)
        return e

    def _sm_count(self, device, out):
        e = self._check("sm_count", device)
        if e == 0:
            out[0] = self.sms
        return e

    def _load_encoder(self):
        return self.encoder_error or self._check("load_tensor_map_encoder", self.current())

    def _encode(self, tmap, bf16, base, dims, strides, box, swizzle):
        e = self._check("encode_tensor_map", self.current())
        if e == 0:
            ctypes.memset(tmap, 0, 128)
            self.encodes.append((self.current(), base, swizzle))
        return e

    def _launch(self, kernel, grid, block, smem, stream, args):
        e = self._check("launch_kernel", self.current())
        if e == 0:
            self.launches.append(Launch(self.current(), kernel, grid, block, smem, stream or 0))
        return e

    def _create(self, call, kind, live, out):
        e = self._check(call, self.current())
        if e == 0:
            h = self._new()
            live[h] = self.current()
            self.created[kind] += 1
            out[0] = h
        return e

    def _destroy(self, call, live, handle):
        if handle not in live:
            self.errors.append(f"{call} of unknown handle {handle}")
            return INVALID_VALUE
        e = self._check(call, live[handle])
        del live[handle]  # released even when the call reports an error
        return e

    def _use(self, call, live, handle):
        if handle not in live:
            self.errors.append(f"{call} of unknown event {handle}")
            return INVALID_VALUE
        return self._check(call, self.current())

    def _memcpy(self, dst, src, nbytes, kind, stream):
        e = self._check("memcpy_async", self.current())
        if e == 0:
            self.copies.append((self.current(), kind, nbytes, stream or 0))
        return e

    def _symbol_read(self, dst, symbol, nbytes):
        e = self._check("symbol_read", self.current())
        if e == 0:
            word = self.symbol_words.get(self.current(), 0)
            ctypes.memmove(dst, (ctypes.c_uint32 * 1)(word), min(nbytes, 4))
        return e

    def _symbol_write(self, symbol, src, nbytes):
        e = self._check("symbol_write", self.current())
        if e == 0:
            self.symbol_writes.append((self.current(), ctypes.string_at(src, nbytes)))
            if nbytes == 4 and ctypes.string_at(src, 4) == b"\0\0\0\0":
                self.symbol_words.pop(self.current(), None)
        return e

    def _symbol_address(self, out, symbol):
        e = self._check("symbol_address", self.current())
        if e == 0:
            out[0] = 0x7000_0000 + 0x100_0000 * self.current()
        return e

    def _pool_create(self, out, device, threshold):
        e = self._check("pool_create", device)
        if e == 0:
            h = self._new()
            self.pools[h] = device
            self.created["pool"] += 1
            out[0] = h
        return e

    def _alloc(self, out, nbytes, pool, stream):
        if pool not in self.pools:
            self.errors.append(f"alloc from unknown pool {pool}")
            return INVALID_VALUE
        e = self._check("pool_alloc_async", self.current())
        if e == 0:
            addr = 0x4000_0000 + self._new() * 0x1000
            self.allocs[addr] = (self.current(), nbytes)
            self.created["alloc"] += 1
            out[0] = addr
        return e

    def _free(self, ptr, stream):
        if ptr not in self.allocs:
            self.errors.append(f"free of unknown address {ptr}")
            return INVALID_VALUE
        e = self._check("free_async", self.current())
        if e == 0:
            del self.allocs[ptr]
        return e
