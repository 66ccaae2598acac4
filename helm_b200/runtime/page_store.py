"""Physical page storage behind KVAllocator: one slab per device.

A slab is a tensor [capacity, 2 (K/V), Hkv, P, D].  A page's slot is its
int32 index in the slab; that index is what the device page tables hold and
what the attention kernel dereferences, so every page of one device lives in
one allocation and one kernel launch can reach all of them.  On the host
(device type 'cpu') the slab is pinned when CUDA is available, so page
transfers are true asynchronous DMA.

Slots are recycled through a free list.  The slab grows by reallocation when a
request exceeds its capacity (slot indices stay valid; tensors handed out as
page views before a growth keep pointing at the old storage, which is why
KVPage materialises its views lazily).  Large pools should be sized up front
with reserve().

Evictions (device -> pinned host) are batched: KVAllocator.move_page queues
the page copy on the host store (defer_move) instead of copying it, and
flush_moves() issues every queued copy as one helm_move_pages launch on the
device's transfer stream, ordered after the work already queued on the
current stream.  Until their copy has completed, the source slots stay out of
the free list (quarantine) and the host slab's readers wait for its events
(pending_events): a CPU-side view, a host slab growth and a staging copy all
flush and wait first.
"""
from __future__ import annotations

from typing import List, Optional

import torch

_TRANSFER_STREAMS = {}

# Queued migrations flushed as soon as this many are pending (one kernel launch carries 2048).
MAX_PENDING_MOVES = 2048


def transfer_stream(device) -> "torch.cuda.Stream":
    """The side stream of `device` that carries page migrations and host-page staging copies
    (the reference's per-device copy stream, kv_cache.py:315)."""
    dev = device_key(device)
    st = _TRANSFER_STREAMS.get(dev)
    if st is None:
        st = torch.cuda.Stream(device=dev)
        _TRANSFER_STREAMS[dev] = st
    return st


def device_key(device) -> torch.device:
    """Canonical device of a storage request: cuda -> cuda:<current>, anything else -> cpu."""
    if isinstance(device, str):
        device = torch.device(device)
    if getattr(device, "type", None) == "cuda":
        idx = device.index if device.index is not None else torch.cuda.current_device()
        return torch.device("cuda", idx)
    return torch.device("cpu")


class PageStore:
    def __init__(self, device: torch.device, num_kv_heads: int, page_size: int, head_dim: int,
                 dtype: torch.dtype, initial: int = 0):
        self.device = device_key(device)
        self.Hkv, self.P, self.D, self.dtype = num_kv_heads, page_size, head_dim, dtype
        self.slab: Optional[torch.Tensor] = None
        self.capacity = 0
        self.next_slot = 0           # slots [0, next_slot) have been handed out at least once
        self.free_slots: List[int] = []
        self.growths = 0
        self.pending_events = []     # events after which host pages written by D2H copies are valid
        self.pending_moves = []      # queued migrations into this store: (source store, source slot, slot)
        self.quarantine = []         # (event, slots): sources of migrations still in flight
        self.last_reader = None      # event after the last staging copy that read this (host) slab
        self.outbound = {}           # host stores holding queued migrations out of this store
        if initial:
            self.reserve(initial)

    # ---- geometry ------------------------------------------------------------
    @property
    def page_elems(self) -> int:
        """Elements per slot (K and V)."""
        return 2 * self.Hkv * self.P * self.D

    @property
    def page_bytes(self) -> int:
        return self.page_elems * torch.tensor([], dtype=self.dtype).element_size()

    @property
    def head_stride(self) -> int:
        return self.P * self.D

    @property
    def pinned(self) -> bool:
        return self.slab is not None and self.slab.is_pinned()

    # ---- capacity --------------------------------------------------------------
    def _alloc(self, n: int) -> torch.Tensor:
        shape = (n, 2, self.Hkv, self.P, self.D)
        if self.device.type == "cpu":
            # pinned from the start (no pageable copy first: host slabs can be tens of GB)
            return torch.empty(shape, dtype=self.dtype, pin_memory=torch.cuda.is_available())
        return torch.empty(shape, dtype=self.dtype, device=self.device)

    def reserve(self, capacity: int) -> None:
        """Makes room for `capacity` slots in total (no-op if already there)."""
        if capacity <= self.capacity:
            return
        # The old slab is copied below and then dropped: a host slab must first receive every
        # queued and in-flight migration (the copy runs on the CPU), and no staging copy may still
        # be reading it when its pinned block goes back to the allocator.
        self.sync_host()
        if self.last_reader is not None:
            self.last_reader.synchronize()
            self.last_reader = None
        new = self._alloc(capacity)
        if self.slab is not None and self.next_slot > 0:
            new[:self.next_slot].copy_(self.slab[:self.next_slot])
            self.growths += 1
        self.slab = new
        self.capacity = capacity

    def take(self, n: int) -> List[int]:
        """n slots, contiguous and ascending when the free list cannot serve them all."""
        out: List[int] = []
        while self.free_slots and len(out) < n:
            out.append(self.free_slots.pop())
        if len(out) < n and (self.quarantine or self.outbound):
            for dst in list(self.outbound.values()):
                dst.flush_moves()            # queued migrations hold slots of this store
            self._release_quarantine()
            while self.free_slots and len(out) < n:
                out.append(self.free_slots.pop())
        need = n - len(out)
        if need:
            if self.next_slot + need > self.capacity:
                self.reserve(max(2 * self.capacity, self.next_slot + need, 16))
            out.extend(range(self.next_slot, self.next_slot + need))
            self.next_slot += need
        return out

    def release(self, slot: int) -> None:
        self.free_slots.append(slot)

    # ---- views -------------------------------------------------------------------
    def k_view(self, slot: int) -> torch.Tensor:
        self.sync_host()
        return self.slab[slot, 0].unsqueeze(0)

    def v_view(self, slot: int) -> torch.Tensor:
        self.sync_host()
        return self.slab[slot, 1].unsqueeze(0)

    def sync_host(self) -> None:
        """Host slabs written by asynchronous D2H copies: issue the queued ones and wait for all of
        them before a CPU-side read."""
        self.flush_moves()
        evs, self.pending_events = self.pending_events, []
        for ev in evs:
            ev.synchronize()

    # ---- batched migrations ---------------------------------------------------------
    def defer_move(self, src: "PageStore", src_slot: int, dst_slot: int) -> None:
        """Queues the copy of slot src_slot of `src` (a device store) into slot dst_slot of this
        (host) store.  The source slot is held until the copy has run, then quarantined."""
        self.pending_moves.append((src, src_slot, dst_slot))
        src.outbound[id(self)] = self
        if len(self.pending_moves) >= MAX_PENDING_MOVES:
            self.flush_moves()

    def flush_moves(self) -> None:
        """Issues every queued migration: per source store, one helm_move_pages on that device's
        transfer stream after the work queued so far on its current stream; the event that ends
        it guards this slab's readers and the source slots."""
        moves, self.pending_moves = self.pending_moves, []
        if not moves:
            return
        from .. import ops
        self.pending_events = [e for e in self.pending_events if not e.query()]
        groups = {}
        for src, s_slot, d_slot in moves:
            groups.setdefault(id(src), (src, [], []))
            groups[id(src)][1].append(s_slot)
            groups[id(src)][2].append(d_slot)
        for src, s_slots, d_slots in groups.values():
            dev = src.device
            side = transfer_stream(dev)
            side.wait_stream(torch.cuda.current_stream(dev))
            ops.move_pages(self.slab, d_slots, src.slab, s_slots, self.page_bytes, stream=side.cuda_stream)
            ev = torch.cuda.Event()
            ev.record(side)
            src.slab.record_stream(side)     # a reallocation of the source slab waits for these reads
            self.pending_events.append(ev)
            src.quarantine.append((ev, s_slots))
            src.outbound.pop(id(self), None)

    def _release_quarantine(self) -> None:
        """Returns migrated-out slots to the free list; the current stream waits (on the device, not
        the host) for the copies that read them, so any later write to them comes after."""
        q, self.quarantine = self.quarantine, []
        cur = torch.cuda.current_stream(self.device)
        for ev, slots in q:
            cur.wait_event(ev)
            self.free_slots.extend(slots)

    def base_ptrs(self):
        """(k_base, v_base) views whose data_ptr()s are the kernel's pool bases."""
        return self.slab[:, 0], self.slab[:, 1]
