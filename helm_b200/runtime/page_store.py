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
"""
from __future__ import annotations

from typing import List, Optional

import torch


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
        self.pending_event = None    # event after which host pages written by D2H copies are valid
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
        """Host slabs written by asynchronous D2H copies: wait for them before a CPU-side read."""
        ev = self.pending_event
        if ev is not None:
            ev.synchronize()
            self.pending_event = None

    def base_ptrs(self):
        """(k_base, v_base) views whose data_ptr()s are the kernel's pool bases."""
        return self.slab[:, 0], self.slab[:, 1]
