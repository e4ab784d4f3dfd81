"""Offload staging: copies from pinned host memory into device slots on a copy
queue beside compute, ordered with events.

The Transfer trait of the engine (projects/oom-inference/crates/oominf-core/src/
backend.rs:945-1018, CUDA body crates/oominf-cuda/src/memory.rs:300-398) under
the same method names, on the C ABI of liboomb.so.  TieredExperts uses it to
bring cold expert records into device slots while resident experts compute
(crates/oominf-tiers/src/tiered.rs:1105-1116, 1494-1510): copies wait for the
compute that last read a slot (record_compute + copies_wait), and the compute
that reads a staged record waits for its copy (record_copies + compute_wait).

HostArena is the PinnedArena counterpart (crates/oominf-tiers/src/host.rs:30-120):
one page-locked host allocation holding expert records at fixed strides.
"""
from __future__ import annotations

import ctypes as C

import torch

from . import _lib
from ._lib import check


class Event:
    def __init__(self, handle):
        self.handle = handle

    def __del__(self):
        if self.handle:
            _lib.lib().oomb_event_destroy(self.handle)
            self.handle = None


class Transfer:
    """A copy queue on `device` and the event operations around it."""

    def __init__(self, device=0):
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        self.L = _lib.lib()
        q = C.c_void_p()
        check(self.L.oomb_copy_queue_create(C.byref(q)), "copy_queue")
        self.queue = q.value

    def close(self):
        if self.queue:
            self.L.oomb_copy_queue_destroy(self.queue)
            self.queue = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def _compute(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def pin_host(self, ptr: int, n_bytes: int):
        check(self.L.oomb_pin_host(ptr, n_bytes), "pin_host")

    def unpin_host(self, ptr: int):
        check(self.L.oomb_unpin_host(ptr), "unpin_host")

    def copy_to_device(self, dst: int, src: int, n_bytes: int):
        check(self.L.oomb_copy_to_device(self.queue, dst, src, n_bytes), "copy_to_device")

    def copy_on_device(self, dst: int, src: int, n_bytes: int):
        check(self.L.oomb_copy_on_device(self.queue, dst, src, n_bytes), "copy_on_device")

    def record_compute(self) -> Event:
        ev = C.c_void_p()
        check(self.L.oomb_record_compute(self._compute(), C.byref(ev)), "record_compute")
        return Event(ev.value)

    def record_copies(self) -> Event:
        ev = C.c_void_p()
        check(self.L.oomb_record_copies(self.queue, C.byref(ev)), "record_copies")
        return Event(ev.value)

    def copies_wait(self, ev: Event):
        check(self.L.oomb_copies_wait(self.queue, ev.handle), "copies_wait")

    def compute_wait(self, ev: Event):
        check(self.L.oomb_compute_wait(self._compute(), ev.handle), "compute_wait")

    def event_done(self, ev: Event) -> bool:
        r = self.L.oomb_event_done(ev.handle)
        if r < 0:
            check(r, "event_done")
        return r == 1

    def event_wait(self, ev: Event):
        check(self.L.oomb_event_wait(ev.handle), "event_wait")

    def copies_sync(self):
        check(self.L.oomb_copies_sync(self.queue), "copies_sync")


class HostArena:
    """`count` expert records of `stride` bytes in one pinned host allocation."""

    def __init__(self, count: int, stride: int):
        self.count, self.stride = count, stride
        self.buf = torch.empty(count * stride, dtype=torch.uint8).pin_memory()

    def record(self, i: int) -> torch.Tensor:
        return self.buf[i * self.stride:(i + 1) * self.stride]

    def address(self, i: int) -> int:
        return self.buf.data_ptr() + i * self.stride


def stage_records(transfer: Transfer, arena: HostArena, which, slots_addr, after: Event | None = None) -> Event:
    """Copies arena records `which` into the device slots at `slots_addr` (one
    per record, in order) on the copy queue, after `after` (the compute that
    last read those slots) if given; returns the event compute waits on."""
    if after is not None:
        transfer.copies_wait(after)
    for i, dst in zip(which, slots_addr):
        transfer.copy_to_device(int(dst), arena.address(int(i)), arena.stride)
    return transfer.record_copies()


class Policy:
    """A replacement policy of the expert cache (oomb_policy: the Policy trait of
    crates/oominf-tiers/src/policy.rs:9-129): "lru", "lfu" or "lrfu:<half_life>".
    Host-only (no GPU needed)."""

    def __init__(self, spec: str = "lru"):
        self.L = _lib.lib()
        h = C.c_void_p()
        check(self.L.oomb_policy_create(spec.encode(), C.byref(h)), f"policy {spec!r}")
        self.h = h.value

    def touch(self, key: int, now: int):
        check(self.L.oomb_policy_touch(self.h, key, now), "policy_touch")

    def remove(self, key: int):
        check(self.L.oomb_policy_remove(self.h, key), "policy_remove")

    def victim(self, pinned=()) -> int | None:
        arr = (C.c_uint32 * max(len(pinned), 1))(*pinned)
        v = self.L.oomb_policy_victim(self.h, arr, len(pinned))
        return None if v < 0 else int(v)

    def __del__(self):
        if getattr(self, "h", None):
            self.L.oomb_policy_destroy(self.h)
            self.h = None


class ExpertTier:
    """Expert records of `layers` x `experts` in a pinned host arena, served from
    `slots` device slots (oomb_tier): the ExpertSource two-phase fetch
    (crates/oominf-core/src/experts.rs:12-41) with the cache policy `policy`.

        addrs, ready = tier.begin_fetch(layer, experts)   # ready[i]: usable by work issued now
        ... issue the work of the ready experts ...
        tier.finish_fetch()                                # the rest are usable after this
        ... issue the work of the others ...
    """

    def __init__(self, arena: HostArena, layers: int, experts: int, slots: int, device=0, policy: str = "lru"):
        if arena.count < layers * experts:
            raise ValueError("the arena holds fewer records than layers x experts")
        self.L = _lib.lib()
        self.device = torch.device("cuda", device) if isinstance(device, int) else torch.device(device)
        self.arena, self.stride = arena, arena.stride
        self.slots = torch.empty(slots * arena.stride, dtype=torch.uint8, device=self.device)
        h = C.c_void_p()
        check(self.L.oomb_tier_create(arena.buf.data_ptr(), arena.stride, layers, experts, self.slots.data_ptr(),
                                      slots, policy.encode(), C.byref(h)), "tier_create")
        self.h = h.value

    def _compute(self):
        return torch.cuda.current_stream(self.device).cuda_stream

    def begin_fetch(self, layer: int, experts):
        n = len(experts)
        ids = (C.c_int32 * max(n, 1))(*[int(e) for e in experts])
        addrs = (C.c_uint64 * max(n, 1))()
        ready = (C.c_uint8 * max(n, 1))()
        check(self.L.oomb_tier_begin_fetch(self.h, self._compute(), layer, ids, n, addrs, ready), "tier_begin_fetch")
        return [int(addrs[i]) for i in range(n)], [bool(ready[i]) for i in range(n)]

    def finish_fetch(self):
        check(self.L.oomb_tier_finish_fetch(self.h, self._compute()), "tier_finish_fetch")

    def stats(self) -> dict:
        v = (C.c_uint64 * 5)()
        check(self.L.oomb_tier_stats(self.h, v), "tier_stats")
        return dict(zip(("requests", "hits", "misses", "evictions", "bytes_copied"), (int(x) for x in v)))

    def close(self):
        if getattr(self, "h", None):
            self.L.oomb_tier_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
