"""KVAllocator: the page pool, with HELM's API and bookkeeping, over device-indexed storage.

Mirrors helm/runtime/kv_allocator.py:6-163 exactly in its observable
bookkeeping -- page ids handed out in creation order, LIFO free pools,
batches of 8 GPU / 16 CPU pages reserved on demand, move_page semantics
(GPU -> CPU leaves a DEAD source page and decrements gpu_total_pages) and the
report_usage() figures -- so that eviction traces are bit-identical.

What differs is storage: a page does not own two tensors.  It owns a slot in
the per-device slab of a PageStore ([slots, 2, Hkv, P, D]), and its k_tensor
/ v_tensor are views of that slot, so the GPU pages of every layer and
sequence are addressable by one int32 page table in one kernel launch.  A
DEAD page's slot returns to the store for reuse by later pages.
"""
from __future__ import annotations

from typing import Dict

import torch

from .page_store import PageStore, device_key


def _is_cuda(device) -> bool:
    return getattr(device, "type", None) == "cuda"


class KVAllocator:
    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, page_size: int = 64,
                 dtype=torch.bfloat16):
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.page_size = page_size
        self.dtype = dtype

        self.gpu_free_pool = []
        self.cpu_free_pool = []

        self.gpu_total_pages = 0
        self.cpu_total_pages = 0

        self._next_page_id = 0
        self._stores: Dict[torch.device, PageStore] = {}

    # ---- storage ---------------------------------------------------------------
    def store(self, device) -> PageStore:
        """The PageStore that holds pages of `device` (created on first use).

        `device` is a torch.device (or string).  Any other object is treated as a device of
        its own whose `type` attribute says what it stands for; its pages are stored on the
        torch device named by its `_helm_storage` attribute (default: the CPU).  The CPU test
        suite uses such a stand-in 'cuda' device to run eviction without a GPU."""
        if isinstance(device, (torch.device, str)):
            key = device_key(device)
            storage = key
        else:
            key = device
            storage = getattr(device, "_helm_storage", torch.device("cpu"))
        st = self._stores.get(key)
        if st is None:
            st = PageStore(storage, self.num_kv_heads, self.page_size, self.head_dim, self.dtype)
            self._stores[key] = st
        return st

    def flush_migrations(self) -> None:
        """Issues every queued eviction copy (batched helm_move_pages launches on the transfer
        streams); nothing waits for them here."""
        for st in self._stores.values():
            if st.pending_moves:
                st.flush_moves()

    def reserve_capacity(self, device, pages: int) -> None:
        """Pre-sizes the slab of `device` for `pages` slots (avoids growth copies later).
        No bookkeeping changes: page ids and pool counters are untouched."""
        self.store(device).reserve(pages)

    # ---- reference API ------------------------------------------------------------
    def _create_page(self, device, slot: int = None):
        from .kv_cache import KVPage
        st = self.store(device)
        if slot is None:
            slot = st.take(1)[0]
        page = KVPage(page_id=self._next_page_id, layer_id=-1, start_token=0, used_tokens=0,
                      capacity_tokens=self.page_size, device=device, state="FREE", store=st, slot=slot)
        self._next_page_id += 1
        if _is_cuda(device):
            self.gpu_total_pages += 1
        else:
            self.cpu_total_pages += 1
        return page

    def reserve_batch(self, batch_size: int, device):
        """Allocate a batch of free pages on the specified device."""
        if batch_size <= 0:
            return
        # Pages are popped LIFO, so the last one created is handed out first: give it the lowest
        # slot, so that consecutive allocations read consecutive slots.
        slots = self.store(device).take(batch_size)
        slots.sort(reverse=True)
        pool = self.gpu_free_pool if _is_cuda(device) else self.cpu_free_pool
        for s in slots:
            pool.append(self._create_page(device, slot=s))

    def allocate(self, device):
        """Get a free page from the pool, allocating if necessary."""
        if _is_cuda(device):
            if not self.gpu_free_pool:
                self.reserve_batch(8, device)
            page = self.gpu_free_pool.pop()
            page.state = "GPU"
        else:
            if not self.cpu_free_pool:
                self.reserve_batch(16, device)
            page = self.cpu_free_pool.pop()
            page.state = "CPU"
        page.layer_id = -1
        page.start_token = 0
        page.used_tokens = 0
        page.device = device
        return page

    def free(self, page):
        """Recycle a page back to the free pool (its slot keeps stale data, never read)."""
        page.state = "FREE"
        page.layer_id = -1
        page.start_token = 0
        page.used_tokens = 0
        if _is_cuda(page.device):
            self.gpu_free_pool.append(page)
        else:
            self.cpu_free_pool.append(page)

    def move_page(self, page, target_device):
        """Move a page between CPU and GPU: allocate on the target, copy the used tokens, recycle
        the source (GPU -> CPU: the source becomes DEAD and its slot is released)."""
        if page.device == target_device:
            return page
        new_page = self.allocate(target_device)
        used = page.used_tokens
        queued = False
        if used > 0:
            queued = copy_page_tokens(page, new_page, used)
        new_page.layer_id = page.layer_id
        new_page.start_token = page.start_token
        new_page.used_tokens = used
        new_page.device = target_device

        if _is_cuda(page.device) and not _is_cuda(target_device):
            # a queued copy still has to read the source slot: its store quarantines the slot when
            # the copy is issued, instead of freeing it now
            page.detach_storage(release=not queued)
            page.k_tensor = torch.empty(0, dtype=self.dtype)
            page.v_tensor = torch.empty(0, dtype=self.dtype)
            page.state = "DEAD"
            self.gpu_total_pages -= 1
        else:
            self.free(page)
        return new_page

    def report_usage(self) -> dict:
        bytes_per_page = 2 * (1 * self.num_kv_heads * self.page_size * self.head_dim
                              * torch.finfo(self.dtype).bits // 8)
        gpu_used_pages = self.gpu_total_pages - len(self.gpu_free_pool)
        cpu_used_pages = self.cpu_total_pages - len(self.cpu_free_pool)
        return {
            "gpu_pool_size": self.gpu_total_pages,
            "cpu_pool_size": self.cpu_total_pages,
            "active_gpu_pages": gpu_used_pages,
            "active_cpu_pages": cpu_used_pages,
            "gpu_free_pages": len(self.gpu_free_pool),
            "cpu_free_pages": len(self.cpu_free_pool),
            "gpu_reserved_bytes": self.gpu_total_pages * bytes_per_page,
            "cpu_reserved_bytes": self.cpu_total_pages * bytes_per_page,
            "gpu_used_bytes": gpu_used_pages * bytes_per_page,
            "cpu_used_bytes": cpu_used_pages * bytes_per_page,
        }


def copy_page_tokens(src, dst, used: int) -> bool:
    """Copies the first `used` tokens of every head of src into dst; True when the copy was queued.

    A device -> pinned-host copy between store-backed pages is queued on the host store
    (PageStore.defer_move) and issued with the other queued evictions as one batched launch on the
    device's transfer stream; every CPU-side view, host slab growth and staging copy of the host
    store flushes and waits first, so a later read never sees the copy in flight (the hazard the
    reference avoids with synchronous copies, kv_allocator.py:108-110).  The whole slot is moved:
    tokens past `used` are never read.  Other store-backed pairs copy the [2, Hkv, used, D] block
    slot to slot."""
    if src.has_store() and dst.has_store():
        s_st, d_st = src.store, dst.store
        if d_st.pinned and s_st.device.type == "cuda" and s_st.page_bytes == d_st.page_bytes:
            d_st.defer_move(s_st, src.slot, dst.slot)
            return True
        s_st.sync_host()   # a host source may still be receiving its own queued copy
        s_blk = s_st.slab[src.slot, :, :, :used]
        d_blk = d_st.slab[dst.slot, :, :, :used]
        d_blk.copy_(s_blk)
        return False
    dst.k_tensor[:, :, :used, :].copy_(src.k_tensor[:, :, :used, :])
    dst.v_tensor[:, :, :used, :].copy_(src.v_tensor[:, :, :used, :])
    return False
