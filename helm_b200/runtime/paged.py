"""Device-side decode state and page-list attention on top of the C ABI.

* attend_page_list(): attention of a query over an arbitrary list of KVPages
  (what perform_streaming_attention receives).  Pages held by a device
  PageStore are read in place; pages in a host store are first copied into
  a double-buffered range of staging slots of the device store on a side
  stream (helm_copy_pages; Staging below); pages given as loose tensors are
  gathered into a temporary pool.
* DecodeBatch: the int32 page tables [layers, B, width] of a batch of
  KVCacheManagers (one row per sequence), kept on the device and updated
  incrementally: a decode append writes its token and its table entry in the
  same kernel (helm_kv_append, host-directed rows), so an all-GPU decode step
  moves no table data from the host; rows are re-uploaded only after a
  structural change (prefill, eviction, clear).
"""
from __future__ import annotations

from typing import List, Optional

import numpy as np
import torch

from .. import ops
from .page_store import PageStore, transfer_stream


def _is_cuda(device) -> bool:
    return getattr(device, "type", None) == "cuda"


class Staging:
    """Host pages in flight to the device: two ranges of slots of a device PageStore (a double
    buffer, alternating per call), filled on a dedicated side stream with helm_copy_pages.

    Ordering is by events only -- no host synchronisation:
    * a copy into a range waits for the last consumer of that range (the event recorded by
      consumed()) and for the host store's pending D2H copies (pages just evicted), not for the
      rest of the consumer stream, so it can run ahead of kernels still queued there;
    * the consumer stream waits for the copy's completion event before stage() returns.
    The reference keeps one copy stream per device for the same purpose (kv_cache.py:315,413-414)."""

    def __init__(self, store: PageStore):
        self.store = store
        self.ranges = [[-1, 0], [-1, 0]]     # (first slot, slots) of each half
        self.turn = 0
        self.stream = None
        self.ready = [None, None]
        self.done = [None, None]             # consumer-side events: the half's last reader finished
        self.slab_seen = None                # the device slab the side stream last wrote into

    def _reserve(self, r: int, n: int) -> bool:
        """Makes half r hold >= n slots; True when the slab had to grow (a reallocation copy on
        the consumer stream that the side stream must then wait for)."""
        start, have = self.ranges[r]
        if n <= have:
            return False
        st = self.store
        if have:
            for s in range(start, start + have):
                st.release(s)
        grew = False
        if st.next_slot + n > st.capacity:
            st.reserve(max(st.capacity * 2, st.next_slot + n))
            grew = True
        self.ranges[r] = [st.next_slot, n]
        st.next_slot += n
        return grew

    def reserve(self, n: int) -> int:
        """First slot of the next half, sized for n pages (no copy)."""
        r = self.turn
        self._reserve(r, n)
        return self.ranges[r][0]

    def stage(self, host_store: PageStore, host_slots: List[int]) -> int:
        """Copies host pages into the next half's first len(host_slots) slots on the side stream and
        makes the current stream wait for them; returns the first slot.  Call consumed() after
        enqueueing the kernel that reads them."""
        r = self.turn
        self.turn ^= 1
        self._reserve(r, len(host_slots))
        start = self.ranges[r][0]
        if not host_slots:
            return start
        if host_store.slab.shape[1:] != self.store.slab.shape[1:] or host_store.dtype != self.store.dtype:
            raise ValueError("staging: host and device page geometry differ")
        dev = self.store.device
        cur = torch.cuda.current_stream(dev)
        if self.stream is None:
            self.stream = transfer_stream(dev)
            self.ready = [torch.cuda.Event(), torch.cuda.Event()]
        side = self.stream
        # Evictions queued into the host store must be issued before their pages are read.
        host_store.flush_moves()
        slab = self.store.slab
        if slab is not self.slab_seen or self.done[r] is None:
            # The device slab is new to the side stream (first use, or reallocated by a growth
            # anywhere: its old -> new copy sits on the consumer stream), or this half has no
            # reader event yet: wait for everything queued so far.
            side.wait_stream(cur)
            slab.record_stream(side)
            self.slab_seen = slab
        else:
            side.wait_event(self.done[r])     # the half's previous reader has finished
        for ev in host_store.pending_events:
            side.wait_event(ev)               # pages evicted just now: their D2H copies
        ops.copy_pages(slab, start, host_store.slab, host_slots, self.store.page_bytes, stream=side.cuda_stream)
        self.ready[r].record(side)
        host_store.last_reader = self.ready[r]
        cur.wait_event(self.ready[r])
        self._last = r
        return start

    def consumed(self) -> None:
        """Records, on the current stream, that the half filled by the last stage() may be reused."""
        r = getattr(self, "_last", None)
        if r is None:
            return
        ev = self.done[r] if self.done[r] is not None else torch.cuda.Event()
        ev.record(torch.cuda.current_stream(self.store.device))
        self.done[r] = ev


_STAGING = {}


def staging_for(store: PageStore) -> Staging:
    st = _STAGING.get(id(store))
    if st is None or st.store is not store:
        st = Staging(store)
        _STAGING[id(store)] = st
    return st


def _launch(q3: torch.Tensor, store: PageStore, table: torch.Tensor, used: torch.Tensor, npages: torch.Tensor,
            scale: float, out: torch.Tensor, max_pages: int, error_flag: Optional[torch.Tensor] = None):
    k_base, v_base = store.base_ptrs()
    return ops.paged_decode_attention(
        q3, k_base, v_base, table, used, npages, num_kv_heads=store.Hkv, page_size=store.P,
        page_stride=store.page_elems, head_stride=store.head_stride, num_pool_pages=store.capacity,
        scale=scale, max_pages=max_pages, out=out, error_flag=error_flag)


def attend_page_list(query: torch.Tensor, pages: list, scale: float) -> torch.Tensor:
    """query [B, Hq, 1, D] on a CUDA device; pages = the active pages (GPU ones, then CPU ones)."""
    dev = query.device
    B, Hq, Sq, D = query.shape
    if Sq != 1:
        raise ValueError("perform_streaming_attention: decode attention takes one query token (q_len == 1)")
    q3 = query.reshape(B, Hq, D).contiguous()
    out = torch.empty((B, Hq, D), dtype=query.dtype, device=dev)

    dev_store = None
    host_store = None
    direct = True
    for p in pages:
        if not p.has_store():
            direct = False
            break
        st = p.store
        if _is_cuda(p.device):
            if st.device != dev or (dev_store is not None and st is not dev_store):
                direct = False
                break
            dev_store = st
        else:
            if host_store is not None and st is not host_store:
                direct = False
                break
            host_store = st
    if direct and host_store is not None:
        if dev_store is None:
            # host pages only: stage them through a device store of the same geometry
            from .kv_allocator import KVAllocator  # noqa: F401  (documentation of the owner)
            dev_store = _scratch_store(host_store, dev)
        if host_store.slab.shape[1:] != dev_store.slab.shape[1:] or host_store.dtype != dev_store.dtype:
            direct = False

    if direct:
        slots = []
        host_slots = []
        for p in pages:
            if _is_cuda(p.device):
                slots.append(p.slot)
            else:
                host_slots.append(p.slot)
        if host_slots:
            start = staging_for(dev_store).stage(host_store, host_slots)
            slots += list(range(start, start + len(host_slots)))
        used = [p.used_tokens for p in pages if _is_cuda(p.device)] + \
               [p.used_tokens for p in pages if not _is_cuda(p.device)]
        n = len(slots)
        table = torch.tensor([slots] * B, dtype=torch.int32).to(dev, non_blocking=False)
        usedt = torch.tensor([used] * B, dtype=torch.int32).to(dev, non_blocking=False)
        npg = torch.full((B,), n, dtype=torch.int32, device=dev)
        _launch(q3, dev_store, table, usedt, npg, scale, out, n)
        if host_slots:
            staging_for(dev_store).consumed()
        return out.reshape(B, Hq, 1, D)

    # Loose tensors (or mixed stores): gather the used tokens into a temporary pool.
    Hkv = pages[0].k_tensor.shape[1]
    Pm = max(p.used_tokens for p in pages)
    kv_dtype = pages[0].k_tensor.dtype
    n = len(pages)
    pool = torch.empty((n, 2, Hkv, Pm, D), dtype=kv_dtype, device=dev)
    for i, p in enumerate(pages):
        u = p.used_tokens
        pool[i, 0, :, :u].copy_(p.k_tensor[0, :, :u], non_blocking=True)
        pool[i, 1, :, :u].copy_(p.v_tensor[0, :, :u], non_blocking=True)
    table = torch.arange(n, dtype=torch.int32, device=dev).repeat(B, 1)
    usedt = torch.tensor([[p.used_tokens for p in pages]] * B, dtype=torch.int32).to(dev)
    npg = torch.full((B,), n, dtype=torch.int32, device=dev)
    ops.paged_decode_attention(q3, pool[:, 0], pool[:, 1], table, usedt, npg, num_kv_heads=Hkv, page_size=Pm,
                               page_stride=2 * Hkv * Pm * D, head_stride=Pm * D, num_pool_pages=n, scale=scale,
                               max_pages=n, out=out)
    return out.reshape(B, Hq, 1, D)


_SCRATCH = {}


def _scratch_store(like: PageStore, dev) -> PageStore:
    key = (id(like), dev)
    st = _SCRATCH.get(key)
    if st is None:
        st = PageStore(dev, like.Hkv, like.P, like.D, like.dtype)
        _SCRATCH[key] = st
    return st


class DecodeBatch:
    """Device page tables of one batch of KVCacheManagers (row b = kvcms[b])."""

    def __init__(self, kvcms, num_layers: int, device, width: int = 64):
        self.kvcms = list(kvcms)
        self.L = num_layers
        self.B = len(self.kvcms)
        self.device = torch.device(device)
        self.width = max(1, width)
        self.table = torch.zeros((self.L, self.B, self.width), dtype=torch.int32, device=self.device)
        self.used = torch.zeros_like(self.table)
        self.npages = torch.zeros((self.L, self.B), dtype=torch.int32, device=self.device)
        self.synced = [[None] * self.B for _ in range(self.L)]   # layer._version mirrored per row
        self.error_flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self.dest = np.zeros((self.B, 3), dtype=np.int32)
        self.cont = None          # ContiguousBatch when the contiguous fast path is active
        self.graph = None         # DecodeGraph while a decode step is being captured or warmed up
        self._rec = None
        for i, m in enumerate(self.kvcms):
            m._batch = (self, i)

    # ---- table maintenance ------------------------------------------------------------
    def _grow(self, need: int) -> None:
        w = self.width
        while w < need:
            w *= 2
        if w == self.width:
            return
        t = torch.zeros((self.L, self.B, w), dtype=torch.int32, device=self.device)
        u = torch.zeros_like(t)
        t[:, :, :self.width] = self.table
        u[:, :, :self.width] = self.used
        self.table, self.used, self.width = t, u, w

    def _upload_row(self, l: int, b: int, slots, used) -> None:
        n = len(slots)
        self._grow(max(n, 1))
        if n:
            self.table[l, b, :n].copy_(torch.from_numpy(np.asarray(slots, dtype=np.int32)))
            self.used[l, b, :n].copy_(torch.from_numpy(np.asarray(used, dtype=np.int32)))
        self.npages[l, b].fill_(n)

    def sync_row(self, l: int, b: int) -> None:
        """Re-uploads row (l, b) from the manager's page list; entry i is layer.pages[i], the index
        helm_kv_append writes.  Only valid while every page of the layer is GPU-resident."""
        m = self.kvcms[b]
        layer = m.layers.get(l)
        if layer is None:
            self._upload_row(l, b, [], [])
            self.synced[l][b] = None
            return
        self._upload_row(l, b, [p.slot for p in layer.pages], [p.used_tokens for p in layer.pages])
        self.synced[l][b] = (id(layer), layer._version)

    def record_buffer(self, rows: int, D: int) -> torch.Tensor:
        """Scratch [rows, D+2] fp32 for the per-rank attention record of sharded decode."""
        if self._rec is None or tuple(self._rec.shape) != (rows, D + 2):
            self._rec = torch.empty((rows, D + 2), dtype=torch.float32, device=self.device)
        return self._rec

    def in_sync(self, l: int, b: int) -> bool:
        layer = self.kvcms[b].layers.get(l)
        return layer is not None and self.synced[l][b] == (id(layer), layer._version)
