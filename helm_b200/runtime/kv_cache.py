"""KVPage, LayerKVCache, KVCacheManager and perform_streaming_attention.

Drop-in mirror of helm/runtime/kv_cache.py.  Observable behaviour -- page
lists, start_token / used_tokens, states, eviction order (global oldest
start_token first, stable, tail and partial pages protected, the byte budget
checked before each page, bytes counted at full page capacity), report dicts
-- follows the reference line by line (cited per method).  Two things are
different by design:

* storage: pages are views of slots in a device-indexed slab (see
  kv_allocator.py), and the attention runs in one CUDA kernel over an int32
  page table (helm_paged_attn_decode) instead of torch.cat + SDPA / a Python
  loop over pages;
* cost: the reference rescans every page of every layer on each append
  (kv_cache.py:161-172, 195-202).  Here each layer keeps its eviction
  candidates (non-tail, full, GPU pages, in page order) and a count of its
  non-GPU pages as pages are appended and moved, so the residency check is
  O(1) and an eviction sorts only the candidates.  The candidate set is the
  reference's scan result by construction, for every sequence of
  append_prefill / append_decode / evict_pages / clear calls.
"""
from __future__ import annotations

import heapq
import itertools
import math
from typing import List, Optional

import torch

_SLOTS = ("page_id", "layer_id", "start_token", "used_tokens", "capacity_tokens", "_k", "_v", "device",
          "state", "store", "slot")


def _is_cuda(device) -> bool:
    return getattr(device, "type", None) == "cuda"


class KVPage:
    """A KV page (kv_cache.py:7-17).  Constructed like the reference dataclass; pages made by
    KVAllocator additionally carry (store, slot) and expose k_tensor / v_tensor as [1, Hkv, P, D]
    views of that slot."""
    __slots__ = _SLOTS

    def __init__(self, page_id: int, layer_id: int, start_token: int, used_tokens: int, capacity_tokens: int,
                 k_tensor: Optional[torch.Tensor] = None, v_tensor: Optional[torch.Tensor] = None,
                 device=None, state: str = "FREE", *, store=None, slot: int = -1):
        self.page_id = page_id
        self.layer_id = layer_id
        self.start_token = start_token
        self.used_tokens = used_tokens
        self.capacity_tokens = capacity_tokens
        self._k = k_tensor
        self._v = v_tensor
        if device is None and k_tensor is not None:
            device = k_tensor.device
        self.device = device
        self.state = state
        self.store = store
        self.slot = slot

    @property
    def k_tensor(self) -> torch.Tensor:
        if self._k is None and self.store is not None:
            return self.store.k_view(self.slot)
        return self._k

    @k_tensor.setter
    def k_tensor(self, value):
        self._k = value

    @property
    def v_tensor(self) -> torch.Tensor:
        if self._v is None and self.store is not None:
            return self.store.v_view(self.slot)
        return self._v

    @v_tensor.setter
    def v_tensor(self, value):
        self._v = value

    def has_store(self) -> bool:
        """True when the page's data lives in a PageStore slot (no explicit tensors set)."""
        return self.store is not None and self._k is None and self._v is None

    def detach_storage(self, release: bool = False) -> None:
        if self.store is not None and release and self.slot >= 0:
            self.store.release(self.slot)
        self.store = None
        self.slot = -1

    def __repr__(self):
        return (f"KVPage(page_id={self.page_id}, layer_id={self.layer_id}, start_token={self.start_token}, "
                f"used_tokens={self.used_tokens}, capacity_tokens={self.capacity_tokens}, "
                f"device={self.device}, state={self.state!r}, slot={self.slot})")


def _candidate(page) -> bool:
    """The reference's eviction filter for a non-tail page (kv_cache.py:129-133)."""
    return page.state == "GPU" and _is_cuda(page.device) and page.used_tokens == page.capacity_tokens


class LayerKVCache:
    """Per-layer page list (kv_cache.py:19-28), plus a count of non-GPU pages maintained as pages
    are appended and moved."""

    def __init__(self, layer_id: int):
        self.layer_id = layer_id
        self.pages: List[KVPage] = []
        self.tail_page: Optional[KVPage] = None
        self.total_tokens: int = 0
        self._n_off: int = 0      # pages with state != 'GPU' and used_tokens > 0
        self._version: int = 0    # bumped on changes the device page table must resync

    def append_page(self, page: KVPage) -> Optional[KVPage]:
        """Appends `page` as the new tail; returns the old tail if it just became an eviction
        candidate (full, GPU-resident, no longer the tail)."""
        old = self.tail_page
        if page.state != "GPU" and page.used_tokens > 0:
            self._n_off += 1
        self.pages.append(page)
        self.tail_page = page
        return old if old is not None and _candidate(old) else None


class KVCacheManager:
    """Owns all layer KV state of one sequence (kv_cache.py:30-310)."""

    def __init__(self, allocator, gpu_high_watermark_bytes: int = 0.25 * 1024 * 1024):
        self.allocator = allocator
        self.layers = {}
        self.gpu_high_watermark_bytes = gpu_high_watermark_bytes
        self.cont_K: dict = {}
        self.cont_V: dict = {}
        self.cont_capacity: int = 0
        self.cont_num_layers: int = 0
        self.cont_seq_len: int = 0
        self.cont_prefill_len: int = 0
        self.use_contiguous: bool = False
        # Set by KVOffloadManager: (DecodeBatch, row) when this sequence is one row of a batch
        # whose page tables live on the device.
        self._batch = None
        # Eviction candidates in the reference's eviction order: a heap keyed by (start_token,
        # layer order in self.layers, page position) -- exactly the order of its stable sort by
        # start_token over the layer-by-layer, page-by-page scan (kv_cache.py:121-159) -- so an
        # eviction costs O(log n) instead of a rescan and sort of every page per call.
        self._heap: list = []
        self._rank: dict = {}            # layer id -> position among self.layers' keys
        self._tie = itertools.count()
        self._n_evictable = 0            # live entries of the heap
        self._prefill_writes = None      # the append_prefill chunks not yet written (during the call)

    def _page_bytes(self) -> int:
        a = self.allocator
        elem = torch.tensor([], dtype=a.dtype).element_size()
        return a.num_kv_heads * a.page_size * a.head_dim * elem * 2

    def _layer(self, layer_id: int) -> LayerKVCache:
        layer = self.layers.get(layer_id)
        if layer is None:
            layer = self.layers[layer_id] = LayerKVCache(layer_id)
            self._rank.setdefault(layer_id, len(self._rank))
        return layer

    def initialize_layer_caches(self, num_layers: int):
        replaced = False
        for i in range(num_layers):
            replaced |= i in self.layers
            self.layers[i] = LayerKVCache(layer_id=i)   # a replaced key keeps its dict position
            self._rank.setdefault(i, len(self._rank))
        if replaced:
            # pages of a replaced layer belong to no layer any more: the reference's scan never
            # sees them again, so they leave the candidates (and the evictable byte count)
            self._heap = [e for e in self._heap if self._live(e)]
            heapq.heapify(self._heap)
            self._n_evictable = len(self._heap)

    # ---- appends (kv_cache.py:55-113) ------------------------------------------------
    def append_prefill(self, layer_id: int, K_prefill: torch.Tensor, V_prefill: torch.Tensor):
        """Append prefill KV in page-sized chunks; residency enforced after every page."""
        layer = self._layer(layer_id)
        seq_len = K_prefill.size(2)
        page_size = self.allocator.page_size
        device = K_prefill.device
        pending = _PrefillWrites(K_prefill, V_prefill)
        self._prefill_writes = pending    # an eviction of a page still in it writes it first
        try:
            for start_idx in range(0, seq_len, page_size):
                chunk_len = min(page_size, seq_len - start_idx)
                page = self.allocator.allocate(device)
                page.layer_id = layer_id
                page.start_token = layer.total_tokens
                page.used_tokens = chunk_len
                pending.add(page, start_idx, chunk_len)
                self._append_page(layer, page)
                layer._version += 1
                layer.total_tokens += chunk_len
                self._enforce_residency_policy()
            pending.flush()
        finally:
            self._prefill_writes = None
        # the evictions of this call leave as batched copies on the transfer stream
        flush = getattr(self.allocator, "flush_migrations", None)
        if flush is not None:
            flush()

    def append_decode(self, layer_id: int, K_new: torch.Tensor, V_new: torch.Tensor,
                      skip_residency: bool = False):
        """Append a single token KV pair for the given layer."""
        page, idx, new_page = self._reserve_decode_slot(layer_id, K_new.device)
        _write_tokens(page, idx, K_new, V_new)
        self._commit_decode_slot(layer_id, page, skip_residency)

    # The two halves of append_decode, so that a batched caller can write the token of every
    # sequence with one kernel launch between them.
    def _reserve_decode_slot(self, layer_id: int, device):
        layer = self._layer(layer_id)
        new_page = False
        if layer.tail_page is None or layer.tail_page.used_tokens == layer.tail_page.capacity_tokens:
            page = self.allocator.allocate(device)
            page.layer_id = layer_id
            page.start_token = layer.total_tokens
            page.used_tokens = 0
            self._append_page(layer, page)
            new_page = True
        page = layer.tail_page
        return page, page.used_tokens, new_page

    def _commit_decode_slot(self, layer_id: int, page, skip_residency: bool):
        layer = self.layers[layer_id]
        if page.used_tokens == 0 and page.state != "GPU":
            layer._n_off += 1
        page.used_tokens += 1
        layer.total_tokens += 1
        if not skip_residency:
            self._enforce_residency_policy()

    def _append_page(self, layer: LayerKVCache, page: KVPage) -> None:
        cand = layer.append_page(page)
        if cand is not None:
            rank = self._rank.get(layer.layer_id, len(self._rank))
            heapq.heappush(self._heap, (cand.start_token, rank, len(layer.pages) - 2, next(self._tie), layer, cand))
            self._n_evictable += 1

    def iterate_layer_pages(self, layer_id: int):
        if layer_id not in self.layers:
            return []
        return list(self.layers[layer_id].pages)

    # ---- eviction (kv_cache.py:121-172) ------------------------------------------------
    def _candidates(self):
        """(layer, page) pairs the reference scan would collect, in its eviction order."""
        return [(e[4], e[5]) for e in sorted(self._heap) if self._live(e)]

    def _live(self, entry) -> bool:
        """The entry is still a candidate: its layer is current, the page still sits at its
        position and is full, GPU-resident and not the tail."""
        _, _, pos, _, layer, page = entry
        return (self.layers.get(layer.layer_id) is layer and pos < len(layer.pages) and layer.pages[pos] is page
                and page is not layer.tail_page and _candidate(page))

    def evict_pages(self, bytes_to_evict: int):
        """Global oldest-page-first eviction to the CPU; the byte budget is checked before each page."""
        if bytes_to_evict <= 0:
            return
        evicted_bytes = 0
        heap = self._heap
        while heap and evicted_bytes < bytes_to_evict:
            entry = heapq.heappop(heap)
            self._n_evictable -= 1
            if not self._live(entry):
                continue
            _, _, idx, _, layer, page = entry
            pw = self._prefill_writes
            if pw is not None and pw.holds(page):
                pw.flush()                # the page's data must be written before it is copied out
            original_start_token = page.start_token
            new_page = self.allocator.move_page(page, torch.device("cpu"))
            assert new_page.start_token == original_start_token, "Page invariant broken during migration"
            layer.pages[idx] = new_page
            if new_page.state != "GPU" and new_page.used_tokens > 0:
                layer._n_off += 1
            layer._version += 1
            # full page capacity, as the reference counts it from the new page's tensors
            evicted_bytes += self._page_bytes()

    def _gpu_evictable_bytes(self) -> int:
        return self._n_evictable * self._page_bytes()

    def _enforce_residency_policy(self):
        # The watermark applies to evictable pages only (kv_cache.py:162-163).
        gpu_bytes = self._gpu_evictable_bytes()
        if gpu_bytes > self.gpu_high_watermark_bytes:
            self.evict_pages(gpu_bytes - self.gpu_high_watermark_bytes)

    # ---- queries (kv_cache.py:174-202) ------------------------------------------------
    def seq_len(self):
        if 0 in self.layers:
            return self.layers[0].total_tokens
        return 0

    def num_layers(self):
        return len(self.layers)

    def clear(self):
        for layer in self.layers.values():
            for page in layer.pages:
                if page.state != "DEAD":
                    self.allocator.free(page)
            layer.pages.clear()
            layer.tail_page = None
            layer.total_tokens = 0
            layer._n_off = 0
            layer._version += 1
        self.layers.clear()
        self._heap = []
        self._rank = {}
        self._n_evictable = 0

    def all_gpu_resident(self, layer_id: int) -> bool:
        """True if every used page of this layer is GPU-resident."""
        if layer_id not in self.layers:
            return True
        return self.layers[layer_id]._n_off == 0

    # ---- contiguous fast path (kv_cache.py:206-289) -------------------------------------
    def build_contiguous(self, num_layers: int, num_kv_heads: int, head_dim: int, capacity: int,
                         device: torch.device, dtype: torch.dtype) -> bool:
        """Pre-allocate [1, Hkv, capacity, D] K/V buffers per layer; on OOM halve the capacity
        down to 1024 (kv_cache.py:206-234)."""
        cap = capacity
        while cap >= 1024:
            try:
                self.cont_K.clear()
                self.cont_V.clear()
                for lid in range(num_layers):
                    self.cont_K[lid] = torch.zeros(1, num_kv_heads, cap, head_dim, device=device, dtype=dtype)
                    self.cont_V[lid] = torch.zeros(1, num_kv_heads, cap, head_dim, device=device, dtype=dtype)
                self.cont_capacity = cap
                self.cont_num_layers = num_layers
                self.use_contiguous = True
                return True
            except (torch.cuda.OutOfMemoryError, RuntimeError):
                self.cont_K.clear()
                self.cont_V.clear()
                if getattr(device, "type", None) == "cuda":
                    torch.cuda.empty_cache()
                cap //= 2
        self.use_contiguous = False
        return False

    def prefill_contiguous(self, layer_id: int, K: torch.Tensor, V: torch.Tensor):
        n = K.shape[2]
        self.cont_K[layer_id][:, :, :n, :].copy_(K)
        self.cont_V[layer_id][:, :, :n, :].copy_(V)
        if layer_id == 0:
            self.cont_prefill_len = n
            self.cont_seq_len = n

    def write_decode_contiguous(self, layer_id: int, K_new: torch.Tensor, V_new: torch.Tensor):
        idx = self.cont_seq_len
        self.cont_K[layer_id][:, :, idx:idx + 1, :].copy_(K_new)
        self.cont_V[layer_id][:, :, idx:idx + 1, :].copy_(V_new)

    def get_kv_contiguous(self, layer_id: int):
        n = self.cont_seq_len + 1
        return self.cont_K[layer_id][:, :, :n, :], self.cont_V[layer_id][:, :, :n, :]

    def advance_contiguous(self):
        self.cont_seq_len += 1

    def migrate_contiguous_to_pages(self):
        """Bulk-copy decode tokens from the contiguous buffers into pages, then drop the buffers
        (kv_cache.py:260-276)."""
        if not self.cont_K:
            return
        decode_start = self.cont_prefill_len
        decode_end = self.cont_seq_len
        if decode_end > decode_start:
            for layer_id in range(self.cont_num_layers):
                decode_K = self.cont_K[layer_id][:, :, decode_start:decode_end, :]
                decode_V = self.cont_V[layer_id][:, :, decode_start:decode_end, :]
                self.append_prefill(layer_id, decode_K, decode_V)
        self.drop_contiguous()

    def drop_contiguous(self):
        self.cont_K.clear()
        self.cont_V.clear()
        self.use_contiguous = False

    def reset_contiguous(self):
        if self.cont_K:
            self.use_contiguous = True
            self.cont_seq_len = 0
            self.cont_prefill_len = 0

    def layers_keys(self):
        return sorted(self.layers.keys())

    def report_bytes_per_tier(self) -> dict:
        gpu_bytes = 0
        cpu_bytes = 0
        for layer in self.layers.values():
            for page in layer.pages:
                if page.state == "DEAD":
                    continue
                page_bytes = page.k_tensor.numel() * page.k_tensor.element_size() * 2
                if page.state == "GPU":
                    gpu_bytes += page_bytes
                elif page.state == "CPU":
                    cpu_bytes += page_bytes
        return {"gpu_active_bytes": gpu_bytes, "cpu_active_bytes": cpu_bytes}


class _PrefillWrites:
    """Prefill chunks waiting to be written.  Store-backed pages on the prompt's CUDA device are
    written by one helm_kv_write_pages launch per flush (every chunk's slot in the launch's page
    list); other pages (host stores, loose tensors) with slab copies, runs of consecutive slots
    with one copy per K and V."""

    def __init__(self, K: torch.Tensor, V: torch.Tensor):
        self.K, self.V = K, V
        self.items = []   # (page, start token in K, tokens)
        self.ids = set()

    def add(self, page, start: int, n: int) -> None:
        self.items.append((page, start, n))
        self.ids.add(id(page))

    def holds(self, page) -> bool:
        return id(page) in self.ids

    def flush(self) -> None:
        items, self.items = self.items, []
        self.ids = set()
        K = self.K
        if K.device.type == "cuda" and items:
            dev_items = [it for it in items if it[0].has_store() and it[0].store.device == K.device
                         and it[0].store.dtype == K.dtype]
            if dev_items:
                st = dev_items[0][0].store
                if all(it[0].store is st for it in dev_items):
                    from .. import ops
                    kb, vb = st.base_ptrs()
                    ops.kv_write_pages(K, self.V, kb, vb, [(pg.slot, start, n) for pg, start, n in dev_items],
                                       page_stride=st.page_elems, head_stride=st.head_stride,
                                       num_pool_pages=st.capacity, page_size=st.P)
                    done = set(id(it[0]) for it in dev_items)
                    items = [it for it in items if id(it[0]) not in done]
        i = 0
        while i < len(items):
            page, start, n = items[i]
            j = i + 1
            if page.has_store() and n == page.capacity_tokens:
                P = n
                while (j < len(items) and items[j][0].has_store() and items[j][0].store is page.store
                       and items[j][0].slot == page.slot + (j - i) and items[j][2] == P
                       and items[j][1] == start + (j - i) * P):
                    j += 1
            if j - i > 1:
                run = j - i
                st = page.store
                Hkv, D = self.K.shape[1], self.K.shape[3]
                src_k = self.K[0, :, start:start + run * P].reshape(Hkv, run, P, D).transpose(0, 1)
                src_v = self.V[0, :, start:start + run * P].reshape(Hkv, run, P, D).transpose(0, 1)
                st.slab[page.slot:page.slot + run, 0].copy_(src_k)
                st.slab[page.slot:page.slot + run, 1].copy_(src_v)
            else:
                _write_tokens(page, 0, self.K[:, :, start:start + n, :], self.V[:, :, start:start + n, :])
            i = j


def _write_tokens(page: KVPage, idx: int, K: torch.Tensor, V: torch.Tensor) -> None:
    """page.k_tensor[:, :, idx:idx+n, :] = K (same for V), in one slab copy for store-backed pages."""
    n = K.size(2)
    if page.has_store():
        st = page.store
        blk = st.slab[page.slot, :, :, idx:idx + n]  # [2, Hkv, n, D]
        src = torch.stack((K[0], V[0]))
        blk.copy_(src)
        return
    page.k_tensor[:, :, idx:idx + n, :].copy_(K)
    page.v_tensor[:, :, idx:idx + n, :].copy_(V)


# ---------------------------------------------------------------------------------------------
# perform_streaming_attention
# ---------------------------------------------------------------------------------------------

def perform_streaming_attention(query: torch.Tensor, pages: List[KVPage], scale: float = None):
    """Single-query attention over a list of KV pages (kv_cache.py:318-442), on the GPU.

    query [B, Hq, 1, D] (the reference uses B = 1) on a CUDA device; pages with used_tokens > 0
    and state 'GPU' on a CUDA device or 'CPU' off it are attended, the rest skipped
    (kv_cache.py:350-351); no such page -> zeros_like(query) (kv_cache.py:353-354).  Every batch
    row of query attends to the same pages.  GPU pages are read in place from their slab; CPU
    pages are copied to device staging slots first (kv_cache.py:412-423).  The result has
    query's dtype.  A CPU query raises: this path has no CPU implementation."""
    if query.device.type != "cuda":
        raise RuntimeError("helm_b200.perform_streaming_attention: the query must be on a CUDA device "
                           "(the B200 path has no CPU implementation)")
    if scale is None:
        scale = 1.0 / math.sqrt(query.size(-1))
    gpu_pages = [p for p in pages if p.used_tokens > 0 and p.state == "GPU" and _is_cuda(p.device)]
    cpu_pages = [p for p in pages if p.used_tokens > 0 and p.state == "CPU" and not _is_cuda(p.device)]
    if not gpu_pages and not cpu_pages:
        return torch.zeros_like(query)
    from .paged import attend_page_list
    return attend_page_list(query, gpu_pages + cpu_pages, scale)
