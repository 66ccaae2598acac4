"""CUDA-graph decode for a model patched by KVOffloadManager (extension; HELM's runtime is eager).

An eager decode step of an HF decoder issues a few hundred small launches from Python, so at
batch 1 the host, not HBM, sets the step time.  DecodeGraph captures the whole step -- every
layer's projections, norms, RoPE, the KV append and the paged attention, the MLP and the
logits -- in one CUDA graph and replays it per token:

    mgr = KVOffloadManager(model, KVOffloadConfig.from_model(model, cont_capacity=0), batch_size=B)
    model(prompt ...)                        # prefill as usual (eager)
    g = DecodeGraph(mgr, model)
    logits = g.step(next_ids)                # next_ids [B, 1] int64 on the device -> [B, 1, vocab]
    ...
    g.close()                                # back to eager decode (the caches stay consistent)

How the step stays replayable: inside the graph the new token of every (layer, sequence) is
appended in device-directed mode (helm_kv_append with spare pages): the kernel writes the token
into the tail page, or into the next spare page when the tail is full, and updates the device page
table itself.  The spare pages are allocated ahead by the host (two per (layer, sequence)), and
after every replay the host mirrors the same append in the KVCacheManager objects -- the tail
page's used count, or the spare page attached as the new tail -- so page lists, token counts and
report_usage() stay exact.  Positions live in a device buffer that the graph itself advances.

Scope: paged mode (cont_capacity=0), one GPU, every page GPU-resident (the reference's all-GPU
decode path also appends without enforcing the watermark, kv_offload.py:133-138).  Spare pages
are allocated when they are reserved, so page ids are handed out in a different order than an
eager decode would, and report_usage() counts the reserved spares as active GPU pages.
"""
from __future__ import annotations

from typing import Optional

import numpy as np
import torch

from .. import ops


class DecodeGraph:
    SPARES = 2   # spare pages per (layer, sequence); one is consumed at most per step

    def __init__(self, mgr, model, headroom_tokens: int = 1024):
        batch = mgr.batch
        if batch is None or batch.cont is not None or mgr.kvcms[0].use_contiguous:
            raise RuntimeError("DecodeGraph needs KVOffloadManager in paged mode (cont_capacity=0) on a CUDA device")
        if mgr.shard_group is not None and getattr(mgr.shard_group, "world", 1) > 1:
            raise RuntimeError("DecodeGraph does not support sharded decode")
        self.mgr, self.model, self.batch = mgr, model, batch
        self.dev = batch.device
        self.L, self.B = batch.L, batch.B
        kvcms = batch.kvcms
        for l in range(self.L):
            for b, m in enumerate(kvcms):
                layer = m.layers.get(l)
                if layer is None or not layer.pages:
                    raise RuntimeError("DecodeGraph: prefill every sequence first")
                if layer._n_off:
                    raise RuntimeError("DecodeGraph: every page must be GPU-resident")
        self.alloc = mgr.allocator
        self.store = self.alloc.store(self.dev)
        P = self.alloc.page_size
        self.headroom = max(P, headroom_tokens)
        self._make_room()
        for l in range(self.L):
            for b in range(self.B):
                if not batch.in_sync(l, b):
                    batch.sync_row(l, b)
        # spare pages: device ids [L, B, SPARES] + next index [L, B]; the host keeps the page objects
        self.spare_ids = torch.zeros((self.L, self.B, self.SPARES), dtype=torch.int32, device=self.dev)
        self.spare_next = torch.zeros((self.L, self.B), dtype=torch.int32, device=self.dev)
        self.spare_pages = [[[] for _ in range(self.B)] for _ in range(self.L)]
        self._ids_host = np.zeros((self.L, self.B, self.SPARES), dtype=np.int32)
        self._refill(list(range(self.B)))
        # per-sequence positions (= tokens cached so far), advanced by the graph
        self.pos = torch.tensor([[kvcms[b].layers[0].total_tokens] for b in range(self.B)], dtype=torch.long,
                                device=self.dev)
        self.ids = torch.zeros((self.B, 1), dtype=torch.long, device=self.dev)
        self.graph: Optional[torch.cuda.CUDAGraph] = None
        self.logits = None

    def _make_room(self) -> None:
        """Grows the page tables and the device slab for the tokens decodable before the next
        capture.  A captured graph holds the tables' and the slab's addresses, so neither may be
        reallocated while it lives: step() recaptures when either has moved or is about to run out."""
        P = self.alloc.page_size
        need = max(len(m.layers[l].pages) for m in self.batch.kvcms for l in range(self.L))
        self.batch._grow(need + self.headroom // P + self.SPARES + 1)
        self.width = self.batch.width
        st = self.store
        st.reserve(st.next_slot + self.L * self.B * (self.headroom // P + self.SPARES + 1))
        self._slab_ptr = st.slab.data_ptr()
        self._slot_limit = st.capacity

    # ---- spare pages ----------------------------------------------------------------------
    def _refill(self, seqs) -> None:
        """Tops the spare lists of sequences `seqs` (all layers) back up to SPARES pages, unconsumed
        pages first, and rewinds the device index.  The host holds the device's spare state
        exactly (the kernel takes spares in order), so nothing is read back."""
        for l in range(self.L):
            for b in seqs:
                lst = self.spare_pages[l][b]
                while len(lst) < self.SPARES:
                    lst.append(self.alloc.allocate(self.dev))
                for j, page in enumerate(lst):
                    self._ids_host[l, b, j] = page.slot
        self.spare_ids.copy_(torch.from_numpy(self._ids_host.copy()).pin_memory(), non_blocking=True)
        self.spare_next.zero_()

    # ---- host mirror of one device-directed append per (layer, sequence) -----------------
    def _mirror(self) -> None:
        batch = self.batch
        refill = []
        for b, m in enumerate(batch.kvcms):
            crossed = False
            for l in range(self.L):
                layer = m.layers[l]
                tail = layer.tail_page
                if tail is None or tail.used_tokens == tail.capacity_tokens:
                    page = self.spare_pages[l][b].pop(0)
                    page.layer_id = l
                    page.start_token = layer.total_tokens
                    page.used_tokens = 0
                    m._append_page(layer, page)
                    crossed = True
                layer.tail_page.used_tokens += 1
                layer.total_tokens += 1
                batch.synced[l][b] = (id(layer), layer._version)
            if crossed:
                refill.append(b)
        if refill:
            self._refill(refill)

    # ---- capture / replay -------------------------------------------------------------------
    def _forward(self):
        return self.model(input_ids=self.ids, position_ids=self.pos, attention_mask=None, use_cache=False,
                          logits_to_keep=1).logits

    def _capture(self) -> None:
        self.batch.graph = self
        try:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                logits = self._forward()
                self.pos.add_(1)
        finally:
            self.batch.graph = None
        self.graph, self.logits = g, logits

    @torch.no_grad()
    def step(self, input_ids: torch.Tensor) -> torch.Tensor:
        """One decode step for every sequence: input_ids [B, 1] (device) -> logits [B, 1, vocab].
        The returned tensor is reused by the next step."""
        if tuple(input_ids.shape) != (self.B, 1):
            raise ValueError(f"DecodeGraph.step: input_ids must be [{self.B}, 1]")
        if self.graph is not None and (
                max(len(m.layers[0].pages) for m in self.batch.kvcms) + 2 > self.width
                or self.store.slab.data_ptr() != self._slab_ptr
                or self.store.next_slot + self.L * self.B * self.SPARES > self._slot_limit):
            self._recapture()   # tables or slab grew (or are about to): the graph holds their addresses
        self.ids.copy_(input_ids, non_blocking=True)
        if self.graph is None:
            # first step: run it eagerly in device-directed mode (warms up every library the graph
            # will hold), then capture the next ones
            self.batch.graph = self
            try:
                logits = self._forward()
                self.pos.add_(1)
            finally:
                self.batch.graph = None
            self._mirror()
            self._capture()
            return logits
        self.graph.replay()
        self._mirror()
        return self.logits

    def _recapture(self) -> None:
        torch.cuda.synchronize(self.dev)
        self.graph = None
        self.logits = None
        self._make_room()

    def close(self) -> None:
        """Returns the unused spare pages to the allocator; decode continues eagerly."""
        torch.cuda.synchronize(self.dev)
        self.graph = None
        self.logits = None
        for l in range(self.L):
            for b in range(self.B):
                for page in self.spare_pages[l][b]:
                    self.alloc.free(page)
                self.spare_pages[l][b] = []


def device_append(batch, l: int, k, v, store, prologue=None, q_out=None) -> None:
    """The graph-mode append of layer l: one token per sequence, destination chosen on the device
    (tail page, or the next spare page when the tail is full), page table updated by the kernel.
    With a prologue, the same launch also normalises / rotates q (into q_out) and k."""
    g = batch.graph
    B = batch.B
    k_base, v_base = store.base_ptrs()
    dest_kw = dict(page_stride=store.page_elems, head_stride=store.head_stride, num_pool_pages=store.capacity,
                   page_size=store.P, page_table=batch.table[l], page_used=batch.used[l],
                   num_pages=batch.npages[l], spare_pages=g.spare_ids[l], spare_next=g.spare_next[l],
                   error_flag=batch.error_flag)
    if prologue is not None:
        prologue.run(q_out, k_base, v_base, True, **dest_kw)
        return
    k3 = k.reshape(B, k.shape[1], k.shape[-1])
    v3 = v.reshape(B, v.shape[1], v.shape[-1])
    if not k3.is_contiguous():
        k3 = k3.contiguous()
    if not v3.is_contiguous():
        v3 = v3.contiguous()
    ops.kv_append(k3, v3, k_base, v_base, **dest_kw)
