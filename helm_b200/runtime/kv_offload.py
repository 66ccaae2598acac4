"""KV offload integration: KVOffloadConfig, KVOffloadManager and the patched attention forwards.

Drop-in mirror of helm/runtime/kv_offload.py: the same config fields and
defaults, the same class-level patch of Qwen3/Qwen2/Llama attention forwards,
the same three decode paths selected in the same order (contiguous buffers,
all-GPU pages, mixed residency).  The decode attention of every path is the
paged kernel (helm_paged_attn_decode) over device page tables, launched once
per layer for the whole batch, and the new token's K/V is written by one
helm_kv_append launch that also updates those tables.  Prefill keeps torch
SDPA (kv_offload.py:201-214 etc.), as in the reference.
"""
from __future__ import annotations

import ctypes

import math
from dataclasses import dataclass
from typing import Optional

import numpy as np
import torch
import torch.nn.functional as F

from .. import _native as N
from .. import ops
from .kv_allocator import KVAllocator
from .kv_cache import KVCacheManager, perform_streaming_attention
from .paged import DecodeBatch, staging_for


# ---------------------------------------------------------------------------------------------
# Config (kv_offload.py:31-75)
# ---------------------------------------------------------------------------------------------

@dataclass
class KVOffloadConfig:
    num_layers: int
    num_kv_heads: int
    head_dim: int
    page_size: int = 64
    dtype: torch.dtype = torch.float16
    gpu_watermark_bytes: Optional[int] = None
    cont_capacity: int = 32768

    def __post_init__(self):
        if self.gpu_watermark_bytes is None:
            elem = torch.tensor([], dtype=self.dtype).element_size()
            per_token_bytes = 2 * self.num_kv_heads * self.head_dim * elem
            self.gpu_watermark_bytes = 512 * per_token_bytes * self.num_layers

    @staticmethod
    def from_model(model, page_size: int = 64, gpu_watermark_bytes: Optional[int] = None,
                   cont_capacity: Optional[int] = None) -> "KVOffloadConfig":
        cfg = model.config
        num_layers = cfg.num_hidden_layers
        num_kv_heads = getattr(cfg, "num_key_value_heads", cfg.num_attention_heads)
        head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        dtype = next(model.parameters()).dtype
        if cont_capacity is None:
            cont_capacity = getattr(cfg, "max_position_embeddings", 32768)
        return KVOffloadConfig(num_layers=num_layers, num_kv_heads=num_kv_heads, head_dim=head_dim,
                               page_size=page_size, dtype=dtype, gpu_watermark_bytes=gpu_watermark_bytes,
                               cont_capacity=cont_capacity)


# ---------------------------------------------------------------------------------------------
# Batched decode (kv_offload.py:82-167)
# ---------------------------------------------------------------------------------------------

class _Prologue:
    """The decode step's raw q/k/v projections ([B, 1, H, D]) and what turns them into the
    attention inputs: the per-head RMSNorm modules (Qwen3's q_norm / k_norm, or None) and the
    rotary tables (cos, sin [B, 1, D]).  On the paged batch path one helm_decode_prologue launch
    applies them and appends K/V; elsewhere materialize() applies the model's own functions."""

    def __init__(self, q, k, v, cos, sin, rope_fn, q_norm=None, k_norm=None):
        self.q, self.k, self.v = q, k, v
        self.cos, self.sin, self.rope_fn = cos, sin, rope_fn
        self.q_norm, self.k_norm = q_norm, k_norm

    def materialize(self):
        """(q [B, Hq, 1, D], k, v [B, Hkv, 1, D]) as the unfused forward computes them."""
        q = (self.q_norm(self.q) if self.q_norm is not None else self.q).transpose(1, 2)
        k = (self.k_norm(self.k) if self.k_norm is not None else self.k).transpose(1, 2)
        v = self.v.transpose(1, 2)
        q, k = self.rope_fn(q, k, self.cos, self.sin)
        return q, k, v

    def fusable(self) -> bool:
        q, k, v, cos = self.q, self.k, self.v, self.cos
        ok = (q.dim() == 4 and q.shape[1] == 1 and q.dtype in (torch.float16, torch.bfloat16)
              and k.dtype == q.dtype and v.dtype == q.dtype and cos.dim() == 3 and cos.shape[1] == 1
              and cos.shape[0] in (1, q.shape[0]) and tuple(self.sin.shape) == tuple(cos.shape))
        if self.q_norm is not None:
            ok = ok and hasattr(self.q_norm, "variance_epsilon") and hasattr(self.k_norm, "variance_epsilon")
        return ok

    def run(self, q_out, k_base, v_base, do_append: bool, **append_kw) -> None:
        B, _, Hq, D = self.q.shape
        Hkv = self.k.shape[2]
        cos = self.cos.reshape(self.cos.shape[0], D)
        sin = self.sin.reshape(self.sin.shape[0], D)
        if cos.stride(-1) != 1 or sin.stride(-1) != 1:
            cos, sin = cos.contiguous(), sin.contiguous()
        if cos.shape[0] != B:      # one position shared by the batch: broadcast rows (stride 0)
            cos, sin = cos.expand(B, D), sin.expand(B, D)
        elif cos.stride(0) != sin.stride(0):
            cos, sin = cos.contiguous(), sin.contiguous()
        qn = self.q_norm
        ops.decode_prologue(self.q.view(B, Hq, D), self.k.view(B, Hkv, D), self.v.view(B, Hkv, D), q_out,
                            k_base, v_base, q_norm_w=None if qn is None else qn.weight,
                            k_norm_w=None if qn is None else self.k_norm.weight,
                            eps=1e-6 if qn is None else qn.variance_epsilon, cos=cos, sin=sin,
                            do_append=do_append, **append_kw)


def _batch_of(kvcms):
    b0 = getattr(kvcms[0], "_batch", None)
    if b0 is None:
        return None
    batch = b0[0]
    if batch.B != len(kvcms):
        return None
    for i, m in enumerate(kvcms):
        if getattr(m, "_batch", None) != (batch, i):
            return None
    return batch


def _decode_batched(kvcms, q, k, v, layer_idx: int, scale: float, *, shard=None, prologue=None):
    """Decode step shared by all architecture forward patches; returns [bsz, Hq, 1, D].

    Path selection follows the reference: (1) contiguous buffers while the sequence fits,
    else migrate them to pages; (2)/(3) paged, appending with skip_residency when every
    page of the layer is GPU-resident (kv_offload.py:133-138).

    shard (a KVShardGroup, multi-GPU only): the managers hold this rank's share of every
    sequence's pages; only the last rank appends the new token, and the per-rank records are
    exchanged and merged so that every rank returns the full attention output.

    prologue (a _Prologue, instead of q/k/v): the raw projections plus their norms and rotary
    tables; the paged batch path fuses them into the append launch (helm_decode_prologue)."""
    x = q if q is not None else prologue.q
    bsz = x.shape[0]
    if x.device.type != "cuda":
        raise RuntimeError("helm_b200 decode attention runs on CUDA devices only")
    batch = _batch_of(kvcms)
    fuse = prologue is not None and prologue.fusable()
    if prologue is not None and not fuse:
        q, k, v = prologue.materialize()
        prologue = None
    if shard is not None and shard.world > 1:
        if batch is None or kvcms[0].use_contiguous:
            raise RuntimeError("sharded decode needs a registered batch in paged mode (cont_capacity=0)")
        all_gpu = all(kvcms[i].all_gpu_resident(layer_idx) for i in range(bsz))
        return _decode_paged_batch(batch, layer_idx, q, k, v, scale, all_gpu, shard=shard, prologue=prologue)

    if prologue is not None and (kvcms[0].use_contiguous or batch is None):
        q, k, v = prologue.materialize()
        prologue = None
    if kvcms[0].use_contiguous:
        if kvcms[0].cont_seq_len < kvcms[0].cont_capacity:
            return _decode_contiguous(kvcms, q, k, v, layer_idx, scale, batch)
        for kvcm in kvcms:
            kvcm.migrate_contiguous_to_pages()
        if batch is not None:
            batch.cont = None

    all_gpu = all(kvcms[i].all_gpu_resident(layer_idx) for i in range(bsz))
    if batch is not None:
        return _decode_paged_batch(batch, layer_idx, q, k, v, scale, all_gpu, prologue=prologue)

    outs = []
    for i in range(bsz):
        kvcms[i].append_decode(layer_idx, k[i:i + 1], v[i:i + 1], skip_residency=all_gpu)
        pages = kvcms[i].iterate_layer_pages(layer_idx)
        outs.append(perform_streaming_attention(q[i:i + 1], pages, scale=scale))
    return torch.cat(outs, dim=0)


def _decode_paged_batch(batch: DecodeBatch, l: int, q, k, v, scale: float, all_gpu: bool, shard=None,
                        prologue=None):
    kvcms = batch.kvcms
    B = batch.B
    x = q if q is not None else prologue.q
    dev = x.device
    alloc = kvcms[0].allocator
    store = alloc.store(dev)
    if prologue is not None:
        Hq, D = prologue.q.shape[2], prologue.q.shape[-1]
        q3 = torch.empty((B, Hq, D), dtype=x.dtype, device=dev)
    else:
        Hq, D = q.shape[1], q.shape[-1]
        q3 = q.reshape(B, Hq, D)
        if not q3.is_contiguous():
            q3 = q3.contiguous()
    if batch.graph is not None:
        # CUDA-graph decode (runtime/graph.py): the append picks its page on the device and the
        # host mirrors it after the step, so nothing here reads or changes host state
        from .graph import device_append
        device_append(batch, l, k, v, store, prologue=prologue, q_out=q3)
        out = torch.empty((B, Hq, D), dtype=x.dtype, device=dev)
        _attend_batch(batch, l, q3, scale, store, False, out=out, out_record=None)
        return out.reshape(B, Hq, 1, D)
    append = shard is None or shard.rank == shard.world - 1
    if append:
        _append_batch(batch, l, k, v, all_gpu, store, dev, prologue=prologue, q_out=q3)
    else:
        if prologue is not None:   # q only: this rank holds no tail page
            prologue.run(q3, *store.base_ptrs(), do_append=False, page_stride=store.page_elems,
                         head_stride=store.head_stride, num_pool_pages=store.capacity, page_size=store.P)
        for b, m in enumerate(kvcms):
            layer = m.layers.get(l)
            if layer is not None and not batch.in_sync(l, b) and not layer._n_off:
                batch.sync_row(l, b)
    mixed = any(m.layers[l]._n_off for m in kvcms if l in m.layers)
    out = torch.empty((B, Hq, D), dtype=x.dtype, device=dev)
    if shard is not None and shard.fused and not getattr(shard, "_fused_unsupported", False):
        try:
            _attend_batch(batch, l, q3, scale, store, mixed, out=out, out_record=None,
                          exchange=shard.xparams_ptr)
            return out.reshape(B, Hq, 1, D)
        except N.HelmError as e:
            if e.code != N.ERR_UNSUPPORTED:
                raise
            shard._fused_unsupported = True   # e.g. fp32 pages: exchange as a separate kernel
    if shard is not None:
        rec = batch.record_buffer(B * Hq, D)
        _attend_batch(batch, l, q3, scale, store, mixed, out=None, out_record=rec)
        shard.gather_merge(rec, out=out.view(B * Hq, D))
    else:
        _attend_batch(batch, l, q3, scale, store, mixed, out=out, out_record=None)
    return out.reshape(B, Hq, 1, D)


def _append_batch(batch: DecodeBatch, l: int, k, v, all_gpu: bool, store, dev, prologue=None, q_out=None):
    """Host bookkeeping of append_decode for every sequence + one kernel writing the tokens and
    their device page-table entries; rows changed structurally are re-uploaded."""
    kvcms = batch.kvcms
    B = batch.B
    reserved = []
    dest = batch.dest
    max_li = 0
    for b, m in enumerate(kvcms):
        page, idx, _new = m._reserve_decode_slot(l, dev)
        li = len(m.layers[l].pages) - 1
        dest[b, 0], dest[b, 1], dest[b, 2] = page.slot, li, idx
        max_li = max(max_li, li)
        reserved.append(page)
    batch._grow(max_li + 1)
    k_base, v_base = store.base_ptrs()
    dest_kw = dict(page_stride=store.page_elems, head_stride=store.head_stride, num_pool_pages=store.capacity,
                   page_size=store.P, dest_host=dest, page_table=batch.table[l], page_used=batch.used[l],
                   num_pages=batch.npages[l], error_flag=batch.error_flag)
    if prologue is not None:
        prologue.run(q_out, k_base, v_base, True, **dest_kw)
    else:
        k3 = k.reshape(B, k.shape[1], k.shape[-1])
        v3 = v.reshape(B, v.shape[1], v.shape[-1])
        if not k3.is_contiguous():
            k3 = k3.contiguous()
        if not v3.is_contiguous():
            v3 = v3.contiguous()
        ops.kv_append(k3, v3, k_base, v_base, **dest_kw)
    in_sync = [batch.in_sync(l, b) for b in range(B)]
    for b, m in enumerate(kvcms):
        m._commit_decode_slot(l, reserved[b], all_gpu)
    # The append mirrored the new token on the device; after a structural change (prefill,
    # eviction, clear) the row is rebuilt from the page list.
    for b, m in enumerate(kvcms):
        layer = m.layers[l]
        if in_sync[b] and batch.synced[l][b] == (id(layer), layer._version):
            continue
        if layer._n_off:
            continue
        batch.sync_row(l, b)


def _attend_batch(batch: DecodeBatch, l: int, q3, scale, store, mixed: bool, out, out_record, exchange=None):
    if not mixed:
        _attend_cached(batch, l, q3, scale, store, out, out_record, exchange)
        return
    _decode_mixed(batch, l, q3, scale, out, store, out_record=out_record, exchange=exchange)


def _attend_cached(batch: DecodeBatch, l: int, q3, scale, store, out, out_record, exchange):
    """One helm_paged_attn_decode call over the batch's device tables.  The parameter block of each
    layer is built once and kept on the batch (with one workspace shared by the layers) while the
    pool, the tables and the shapes stay the same; a call then only sets q, the outputs and the
    scale."""
    cache = batch.__dict__.setdefault("_attn_params", {})
    key = (store.slab.data_ptr(), store.capacity, batch.table.data_ptr(), batch.width, tuple(q3.shape), q3.dtype,
           None if out is None else out.dtype, out_record is None,
           None if exchange is None else ctypes.addressof(exchange.contents))
    ent = cache.get(l)
    ws = batch.__dict__.get("_attn_ws")
    if ent is None or ent[0] != key or (ent[2] is not None and ent[2] != ws.data_ptr()):
        k_base, v_base = store.base_ptrs()
        p = ops.make_attn_params(q3, k_base, v_base, batch.table[l], batch.used[l], batch.npages[l],
                                 num_kv_heads=store.Hkv, page_size=store.P, page_stride=store.page_elems,
                                 head_stride=store.head_stride, num_pool_pages=store.capacity, scale=scale,
                                 max_pages=batch.width, out=out, out_record=out_record,
                                 error_flag=batch.error_flag)
        if exchange is not None:
            p.exchange = exchange
        lib = N.lib()
        S = ctypes.c_int32(0)
        need = lib.helm_paged_attn_workspace_bytes(ctypes.byref(p), ctypes.byref(S))
        if need < 0:
            N.check("helm_paged_attn_workspace_bytes", N.ERR_INVALID_ARGUMENT)
        p.num_splits = S.value
        ws_ptr = None
        if need > 0:
            # one workspace per batch, shared by the layers' calls (they run in stream order)
            if ws is None or ws.numel() * 4 < need:
                ws = torch.empty((need + 3) // 4, dtype=torch.float32, device=q3.device)
                batch._attn_ws = ws
            p.workspace, p.workspace_bytes = ws.data_ptr(), ws.numel() * 4
            ws_ptr = ws.data_ptr()
        ent = (key, p, ws_ptr, ctypes.byref(p), lib.helm_paged_attn_decode)
        cache[l] = ent
    p = ent[1]
    p.q = q3.data_ptr()
    p.out = None if out is None else out.data_ptr()
    p.out_record = None if out_record is None else out_record.data_ptr()
    p.scale = scale
    N.check("helm_paged_attn_decode", ent[4](ent[3], torch.cuda.current_stream(q3.device).cuda_stream))


def _decode_mixed(batch: DecodeBatch, l: int, q3, scale, out, store, out_record=None, exchange=None):
    """Some pages of layer l live on the host: stage them into device slots and attend over a
    per-call table (the reference's Path 3, kv_cache.py:382-442)."""
    kvcms = batch.kvcms
    rows = []
    host_store = None
    host_slots = []
    for b, m in enumerate(kvcms):
        row = []
        for p in m.layers[l].pages:
            if p.used_tokens <= 0:
                continue
            if p.state == "GPU" and p.device.type == "cuda":
                row.append((p.slot, p.used_tokens))
            elif p.state == "CPU":
                host_store = p.store
                row.append((-1 - len(host_slots), p.used_tokens))
                host_slots.append(p.slot)
        rows.append(row)
    start = staging_for(store).stage(host_store, host_slots) if host_slots else 0
    width = max(1, max(len(r) for r in rows))
    table = np.zeros((batch.B, width), dtype=np.int32)
    used = np.zeros((batch.B, width), dtype=np.int32)
    npg = np.zeros((batch.B,), dtype=np.int32)
    for b, row in enumerate(rows):
        for i, (s, u) in enumerate(row):
            table[b, i] = s if s >= 0 else start + (-1 - s)
            used[b, i] = u
        npg[b] = len(row)
    dev = q3.device
    t = torch.from_numpy(table).to(dev)
    u = torch.from_numpy(used).to(dev)
    n = torch.from_numpy(npg).to(dev)
    k_base, v_base = store.base_ptrs()
    ops.paged_decode_attention(q3, k_base, v_base, t, u, n, num_kv_heads=store.Hkv, page_size=store.P,
                               page_stride=store.page_elems, head_stride=store.head_stride,
                               num_pool_pages=store.capacity, scale=scale, max_pages=width, out=out,
                               out_record=out_record, error_flag=batch.error_flag, exchange=exchange)
    if host_slots:
        staging_for(store).consumed()
    return out


class ContiguousBatch:
    """Contiguous per-layer K/V buffers of a whole batch, laid out [Hkv, B, cap, D], so that each
    sequence's [1, Hkv, cap, D] buffer (KVCacheManager.cont_K[layer]) is a view and one kernel
    launch covers the batch: pages of P tokens with page stride P*D and head stride B*cap*D."""

    def __init__(self, kvcms, num_layers, num_kv_heads, head_dim, capacity, page_size, device, dtype):
        self.B = len(kvcms)
        self.P = page_size
        self.cap = capacity
        self.L = num_layers
        self.Hkv, self.D = num_kv_heads, head_dim
        self.ppr = capacity // page_size          # pages per row
        self.K = [torch.zeros((num_kv_heads, self.B, capacity, head_dim), dtype=dtype, device=device)
                  for _ in range(num_layers)]
        self.V = [torch.zeros_like(self.K[0]) for _ in range(num_layers)]
        for b, m in enumerate(kvcms):
            m.cont_K.clear()
            m.cont_V.clear()
            for lid in range(num_layers):
                m.cont_K[lid] = self.K[lid][:, b].unsqueeze(0)
                m.cont_V[lid] = self.V[lid][:, b].unsqueeze(0)
            m.cont_capacity = capacity
            m.cont_num_layers = num_layers
            m.use_contiguous = True
        ids = torch.arange(self.B * self.ppr, dtype=torch.int32, device=device).reshape(self.B, self.ppr)
        self.table = ids
        self.used = torch.zeros((num_layers, self.B, self.ppr), dtype=torch.int32, device=device)
        self.npages = torch.zeros((num_layers, self.B), dtype=torch.int32, device=device)
        self.synced_len = [-1] * num_layers
        self.dest = np.zeros((self.B, 3), dtype=np.int32)

    def sync(self, l: int, n: int) -> None:
        """Device rows of layer l describe n tokens per sequence."""
        full, rem = divmod(n, self.P)
        used = np.zeros((self.ppr,), dtype=np.int32)
        used[:full] = self.P
        if rem:
            used[full] = rem
        self.used[l].copy_(torch.from_numpy(np.broadcast_to(used, (self.B, self.ppr)).copy()))
        self.npages[l].fill_(full + (1 if rem else 0))
        self.synced_len[l] = n


def _decode_contiguous(kvcms, q, k, v, layer_idx, scale, batch):
    """Path 1 (kv_offload.py:106-126): write the token in place at cont_seq_len, attend over
    cont_seq_len + 1 tokens, advance after the last layer."""
    bsz = q.shape[0]
    cb = batch.cont if batch is not None else None
    Hq, D = q.shape[1], q.shape[-1]
    if cb is None:
        for i in range(bsz):
            kvcms[i].write_decode_contiguous(layer_idx, k[i:i + 1], v[i:i + 1])
        outs = []
        for i in range(bsz):
            K = kvcms[i].cont_K[layer_idx]
            V = kvcms[i].cont_V[layer_idx]
            outs.append(_attend_contiguous_single(q[i:i + 1], K, V, kvcms[i].cont_seq_len + 1, scale))
        out = torch.cat(outs, dim=0)
    else:
        n = kvcms[0].cont_seq_len
        if cb.synced_len[layer_idx] != n:
            cb.sync(layer_idx, n)
        dest = cb.dest
        pi, slot = divmod(n, cb.P)
        for b in range(bsz):
            dest[b, 0], dest[b, 1], dest[b, 2] = b * cb.ppr + pi, pi, slot
        k3 = k.reshape(bsz, k.shape[1], D).contiguous()
        v3 = v.reshape(bsz, v.shape[1], D).contiguous()
        Kl, Vl = cb.K[layer_idx], cb.V[layer_idx]
        ops.kv_append(k3, v3, Kl, Vl, page_stride=cb.P * D, head_stride=cb.B * cb.cap * D,
                      num_pool_pages=cb.B * cb.ppr, page_size=cb.P, dest_host=dest, page_table=cb.table,
                      page_used=cb.used[layer_idx], num_pages=cb.npages[layer_idx], error_flag=batch.error_flag)
        cb.synced_len[layer_idx] = n + 1
        q3 = q.reshape(bsz, Hq, D).contiguous()
        out = torch.empty((bsz, Hq, D), dtype=q.dtype, device=q.device)
        ops.paged_decode_attention(q3, Kl, Vl, cb.table, cb.used[layer_idx], cb.npages[layer_idx],
                                   num_kv_heads=cb.Hkv, page_size=cb.P, page_stride=cb.P * D,
                                   head_stride=cb.B * cb.cap * D, num_pool_pages=cb.B * cb.ppr, scale=scale,
                                   max_pages=cb.ppr, out=out, error_flag=batch.error_flag)
        out = out.reshape(bsz, Hq, 1, D)
    if layer_idx == kvcms[0].cont_num_layers - 1:
        for kvcm in kvcms:
            kvcm.advance_contiguous()
    return out


def _attend_contiguous_single(q, K, V, n, scale):
    """One sequence over its own [1, Hkv, cap, D] buffer (no batch layout): pages of P=64 rows."""
    Hkv, cap, D = K.shape[1], K.shape[2], K.shape[3]
    P = 64 if cap % 64 == 0 else cap
    npg = (n + P - 1) // P
    dev = q.device
    table = torch.arange(npg, dtype=torch.int32, device=dev).reshape(1, npg)
    used = torch.full((1, npg), P, dtype=torch.int32)
    used[0, -1] = n - P * (npg - 1)
    out = torch.empty((1, q.shape[1], D), dtype=q.dtype, device=dev)
    ops.paged_decode_attention(q.reshape(1, q.shape[1], D).contiguous(), K[0], V[0], table, used.to(dev),
                               torch.tensor([npg], dtype=torch.int32, device=dev), num_kv_heads=Hkv,
                               page_size=P, page_stride=P * D, head_stride=K.stride(1),
                               num_pool_pages=max(npg, cap // P), scale=scale, max_pages=npg, out=out)
    return out.reshape(1, q.shape[1], 1, D)


# ---------------------------------------------------------------------------------------------
# Patched forwards (kv_offload.py:174-322)
# ---------------------------------------------------------------------------------------------

def _shard_tokens(n_tokens: int, page_size: int, shard):
    """Token range [lo, hi) of the prompt that this rank stores: its share of whole pages."""
    if shard is None or shard.world == 1:
        return 0, n_tokens
    from .sharded import shard_bounds
    npg = (n_tokens + page_size - 1) // page_size
    plo, phi = shard_bounds(npg, shard.rank, shard.world)
    return plo * page_size, min(phi * page_size, n_tokens)


def _prefill(attn_self, kvcms, q, k, v, attention_mask, scale, k_exp, v_exp, shard=None):
    bsz = q.shape[0]
    lo, hi = _shard_tokens(k.shape[2], kvcms[0].allocator.page_size, shard)
    for i in range(bsz):
        if hi > lo:
            kvcms[i].append_prefill(attn_self.layer_idx, k[i:i + 1, :, lo:hi], v[i:i + 1, :, lo:hi])
        if kvcms[i].use_contiguous:
            kvcms[i].prefill_contiguous(attn_self.layer_idx, k[i:i + 1], v[i:i + 1])
    return F.scaled_dot_product_attention(
        q, k_exp, v_exp, attn_mask=attention_mask,
        dropout_p=attn_self.attention_dropout if attn_self.training else 0.0, scale=scale)


def _project_qkv(attn_self, hidden_states, hidden_shape):
    """The decode step's q, k and v projections, [B, 1, H, D] each: one launch when
    patch_int8_linears fused the module's projections (Int8QKV; q, k and v are then strided views
    of one output), else the three projection modules."""
    fused = getattr(attn_self, "_helm_qkv", None)
    if fused is not None:
        return tuple(t.view(hidden_shape) for t in fused(hidden_states))
    return (attn_self.q_proj(hidden_states).view(hidden_shape), attn_self.k_proj(hidden_states).view(hidden_shape),
            attn_self.v_proj(hidden_states).view(hidden_shape))


def _make_qwen2_forward(kvcms, shard=None):
    def forward(attn_self, hidden_states, position_embeddings, attention_mask=None, past_key_values=None,
                cache_position=None, **kwargs):
        from transformers.models.qwen2.modeling_qwen2 import apply_rotary_pos_emb
        bsz, q_len, _ = hidden_states.shape
        hidden_shape = (bsz, q_len, -1, attn_self.head_dim)
        cos, sin = position_embeddings
        scale = 1.0 / math.sqrt(attn_self.head_dim)
        if q_len == 1:
            pro = _Prologue(*_project_qkv(attn_self, hidden_states, hidden_shape), cos, sin, apply_rotary_pos_emb)
            out = _decode_batched(kvcms, None, None, None, attn_self.layer_idx, scale, shard=shard, prologue=pro)
        else:
            q = attn_self.q_proj(hidden_states).view(hidden_shape).transpose(1, 2)
            k = attn_self.k_proj(hidden_states).view(hidden_shape).transpose(1, 2)
            v = attn_self.v_proj(hidden_states).view(hidden_shape).transpose(1, 2)
            q, k = apply_rotary_pos_emb(q, k, cos, sin)
            groups = q.shape[1] // k.shape[1]
            out = _prefill(attn_self, kvcms, q, k, v, attention_mask, scale,
                           k.repeat_interleave(groups, dim=1), v.repeat_interleave(groups, dim=1), shard)
        out = out.transpose(1, 2).contiguous().reshape(bsz, q_len, -1)
        return attn_self.o_proj(out), None
    return forward


def _make_qwen3_forward(kvcms, shard=None):
    def forward(attn_self, hidden_states, position_embeddings, attention_mask=None, past_key_values=None,
                cache_position=None, **kwargs):
        from transformers.models.qwen3.modeling_qwen3 import apply_rotary_pos_emb, repeat_kv
        bsz, q_len, _ = hidden_states.shape
        hidden_shape = (bsz, q_len, -1, attn_self.head_dim)
        cos, sin = position_embeddings
        scale = 1.0 / math.sqrt(attn_self.head_dim)
        if q_len == 1:
            pro = _Prologue(*_project_qkv(attn_self, hidden_states, hidden_shape), cos, sin, apply_rotary_pos_emb,
                            q_norm=attn_self.q_norm, k_norm=attn_self.k_norm)
            out = _decode_batched(kvcms, None, None, None, attn_self.layer_idx, scale, shard=shard, prologue=pro)
        else:
            q = attn_self.q_norm(attn_self.q_proj(hidden_states).view(hidden_shape)).transpose(1, 2)
            k = attn_self.k_norm(attn_self.k_proj(hidden_states).view(hidden_shape)).transpose(1, 2)
            v = attn_self.v_proj(hidden_states).view(hidden_shape).transpose(1, 2)
            q, k = apply_rotary_pos_emb(q, k, cos, sin)
            out = _prefill(attn_self, kvcms, q, k, v, attention_mask, scale,
                           repeat_kv(k, attn_self.num_key_value_groups), repeat_kv(v, attn_self.num_key_value_groups),
                           shard)
        out = out.transpose(1, 2).contiguous().reshape(bsz, q_len, -1)
        return attn_self.o_proj(out), None
    return forward


def _make_llama_forward(kvcms, shard=None):
    def forward(attn_self, hidden_states, position_embeddings, attention_mask=None, past_key_values=None,
                cache_position=None, **kwargs):
        from transformers.models.llama.modeling_llama import apply_rotary_pos_emb
        bsz, q_len, _ = hidden_states.shape
        hidden_shape = (bsz, q_len, -1, attn_self.head_dim)
        cos, sin = position_embeddings
        scale = 1.0 / math.sqrt(attn_self.head_dim)
        if q_len == 1:
            pro = _Prologue(*_project_qkv(attn_self, hidden_states, hidden_shape), cos, sin, apply_rotary_pos_emb)
            out = _decode_batched(kvcms, None, None, None, attn_self.layer_idx, scale, shard=shard, prologue=pro)
        else:
            q = attn_self.q_proj(hidden_states).view(hidden_shape).transpose(1, 2)
            k = attn_self.k_proj(hidden_states).view(hidden_shape).transpose(1, 2)
            v = attn_self.v_proj(hidden_states).view(hidden_shape).transpose(1, 2)
            q, k = apply_rotary_pos_emb(q, k, cos, sin)
            groups = q.shape[1] // k.shape[1]
            out = _prefill(attn_self, kvcms, q, k, v, attention_mask, scale,
                           k.repeat_interleave(groups, dim=1), v.repeat_interleave(groups, dim=1), shard)
        out = out.transpose(1, 2).contiguous().reshape(bsz, q_len, -1)
        return attn_self.o_proj(out), None
    return forward


def _make_rmsnorm_forward(orig):
    """RMSNorm forward as one helm_rmsnorm launch (16-bit CUDA inputs; anything else runs the
    module's own forward).  Same arithmetic as the HF modules: fp32 statistics, the normalised
    value cast to the input dtype, then scaled by the weight."""
    def forward(norm_self, hidden_states):
        if (hidden_states.device.type == "cuda" and hidden_states.dtype in (torch.float16, torch.bfloat16)
                and norm_self.weight.dtype == hidden_states.dtype and hasattr(norm_self, "variance_epsilon")):
            return ops.rmsnorm(hidden_states, norm_self.weight, norm_self.variance_epsilon)
        return orig(norm_self, hidden_states)
    return forward


# ---------------------------------------------------------------------------------------------
# Manager (kv_offload.py:329-433)
# ---------------------------------------------------------------------------------------------

class KVOffloadManager:
    """Installs the paged-KV attention patches on the model and manages the cache lifecycle.
    One KVCacheManager per batch item, all sharing one KVAllocator; the batch's page tables
    live on the device (DecodeBatch)."""

    def __init__(self, model, config: KVOffloadConfig, batch_size: int = 1, shard_group=None,
                 fused_norms: bool = False):
        """shard_group (a KVShardGroup; extension, multi-GPU only): store this rank's share of every
        sequence's KV pages and merge the ranks' attention records on each decode step.  Requires
        config.cont_capacity == 0 (paged mode).

        fused_norms (extension): also patch the architecture's RMSNorm module (Qwen3RMSNorm /
        Qwen2RMSNorm / LlamaRMSNorm) to run as one helm_rmsnorm launch for 16-bit CUDA inputs
        instead of five elementwise kernels; restore() undoes it too."""
        self.fused_norms = fused_norms
        self.config = config
        self.batch_size = batch_size
        self.shard_group = shard_group
        if shard_group is not None and shard_group.world > 1 and config.cont_capacity > 0:
            raise ValueError("KVOffloadManager: sharded decode needs cont_capacity=0")
        self.allocator = KVAllocator(num_layers=config.num_layers, num_kv_heads=config.num_kv_heads,
                                     head_dim=config.head_dim, page_size=config.page_size, dtype=config.dtype)
        watermark_per_item = max(config.gpu_watermark_bytes // batch_size, 1)
        self.kvcms = [KVCacheManager(self.allocator, gpu_high_watermark_bytes=watermark_per_item)
                      for _ in range(batch_size)]
        self._patched: dict = {}
        self._apply_patches(model)
        device = next(model.parameters()).device
        self.batch = DecodeBatch(self.kvcms, config.num_layers, device) if device.type == "cuda" else None

        if config.cont_capacity > 0 and device.type == "cuda":
            cap = config.cont_capacity - config.cont_capacity % config.page_size
            built = False
            while cap >= 1024 and not built:
                try:
                    self.batch.cont = ContiguousBatch(self.kvcms, config.num_layers, config.num_kv_heads,
                                                      config.head_dim, cap, config.page_size, device,
                                                      config.dtype)
                    built = True
                except (torch.cuda.OutOfMemoryError, RuntimeError):
                    self.batch.cont = None
                    torch.cuda.empty_cache()
                    cap //= 2
                    cap -= cap % config.page_size
            if not built:
                for kvcm in self.kvcms:
                    kvcm.drop_contiguous()

    def reset(self):
        """Clear all paged caches and re-arm the contiguous path for the next generate()."""
        for kvcm in self.kvcms:
            kvcm.clear()
            kvcm.reset_contiguous()
        if self.batch is not None and self.batch.cont is not None:
            self.batch.cont.synced_len = [-1] * self.batch.cont.L

    def restore(self):
        """Restore the original attention forwards."""
        for arch, (cls, orig) in self._patched.items():
            cls.forward = orig
        self._patched.clear()

    def report(self) -> dict:
        return self.allocator.report_usage()

    def _apply_patches(self, model):
        name = model.__class__.__name__.lower()
        if "qwen3" in name:
            self._patch("qwen3")
        elif "qwen2" in name:
            self._patch("qwen2")
        elif "llama" in name or "mistral" in name:
            self._patch("llama")
        else:
            raise NotImplementedError(f"KVOffloadManager: no attention patch for {model.__class__.__name__}")

    def _patch(self, arch: str):
        if arch == "qwen2":
            import transformers.models.qwen2.modeling_qwen2 as m
            cls, new_fwd = m.Qwen2Attention, _make_qwen2_forward(self.kvcms, self.shard_group)
        elif arch == "qwen3":
            import transformers.models.qwen3.modeling_qwen3 as m
            cls, new_fwd = m.Qwen3Attention, _make_qwen3_forward(self.kvcms, self.shard_group)
        elif arch == "llama":
            import transformers.models.llama.modeling_llama as m
            cls, new_fwd = m.LlamaAttention, _make_llama_forward(self.kvcms, self.shard_group)
        else:
            raise ValueError(arch)
        self._patched[arch] = (cls, cls.forward)
        cls.forward = new_fwd
        if self.fused_norms:
            norm_cls = {"qwen2": "Qwen2RMSNorm", "qwen3": "Qwen3RMSNorm", "llama": "LlamaRMSNorm"}[arch]
            ncls = getattr(m, norm_cls)
            self._patched[arch + "_norm"] = (ncls, ncls.forward)
            ncls.forward = _make_rmsnorm_forward(ncls.forward)
