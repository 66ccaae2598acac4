"""Torch-facing wrappers of the C-ABI kernels (one call = one C-ABI call).

Every function takes CUDA tensors, launches on the current torch stream of
the tensors' device and raises when the native library is missing or returns
an error.  Nothing here computes on the CPU.
"""
from __future__ import annotations

import ctypes
import math
from typing import Optional

import torch

from . import _native as N

_DT = {torch.float32: N.F32, torch.float16: N.F16, torch.bfloat16: N.BF16, torch.int8: N.I8}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise TypeError(f"helm_b200: unsupported dtype {dt}") from None


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _need_cuda(name: str, *ts: Optional[torch.Tensor]) -> torch.device:
    dev = None
    for t in ts:
        if t is None:
            continue
        if t.device.type != "cuda":
            raise ValueError(f"helm_b200.{name}: tensors must be on a CUDA device (got {t.device}); "
                             "this path has no CPU implementation")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise ValueError(f"helm_b200.{name}: tensors on different devices {dev} and {t.device}")
    if dev is None:
        raise ValueError(f"helm_b200.{name}: no tensor given")
    return dev


class _Workspace:
    """Per-device scratch buffer for split-KV records, grown on demand."""

    def __init__(self):
        self.bufs: dict = {}

    def get(self, dev: torch.device, nbytes: int) -> torch.Tensor:
        key = (dev.type, dev.index)
        buf = self.bufs.get(key)
        if buf is None or buf.numel() * 4 < nbytes:
            buf = torch.empty((max(nbytes, 1 << 20) + 3) // 4, dtype=torch.float32, device=dev)
            self.bufs[key] = buf
        return buf


WORKSPACE = _Workspace()


def make_attn_params(q: torch.Tensor, k_base: torch.Tensor, v_base: torch.Tensor, page_table: torch.Tensor,
                     page_used: torch.Tensor, num_pages: torch.Tensor, *, num_kv_heads: int, page_size: int,
                     page_stride: int, head_stride: int, num_pool_pages: int, scale: Optional[float] = None,
                     max_pages: Optional[int] = None, num_splits: int = 0, out: Optional[torch.Tensor] = None,
                     out_record: Optional[torch.Tensor] = None,
                     error_flag: Optional[torch.Tensor] = None) -> N.PagedAttnParams:
    B, Hq, D = q.shape
    p = N.PagedAttnParams()
    p.q = q.data_ptr()
    p.k_base = k_base.data_ptr()
    p.v_base = v_base.data_ptr()
    p.page_stride = int(page_stride)
    p.head_stride = int(head_stride)
    p.num_pool_pages = int(num_pool_pages)
    p.page_table = page_table.data_ptr()
    p.page_used = page_used.data_ptr()
    p.num_pages = num_pages.data_ptr()
    p.page_table_stride = page_table.stride(0) if page_table.dim() == 2 else page_table.shape[-1]
    p.max_pages = int(page_table.shape[-1] if max_pages is None else max_pages)
    p.B, p.Hq, p.Hkv, p.D, p.P = B, Hq, int(num_kv_heads), D, int(page_size)
    p.q_dtype = dtype_code(q.dtype)
    p.kv_dtype = dtype_code(k_base.dtype)
    p.out_dtype = dtype_code(out.dtype) if out is not None else N.F32
    p.scale = float(1.0 / math.sqrt(D) if scale is None else scale)
    p.num_splits = int(num_splits)
    p.out = _ptr(out)
    p.out_record = _ptr(out_record)
    p.error_flag = _ptr(error_flag)
    return p


def paged_decode_attention(q: torch.Tensor, k_base: torch.Tensor, v_base: torch.Tensor, page_table: torch.Tensor,
                           page_used: torch.Tensor, num_pages: torch.Tensor, *, num_kv_heads: int,
                           page_size: int, page_stride: int, head_stride: int, num_pool_pages: int,
                           scale: Optional[float] = None, max_pages: Optional[int] = None, num_splits: int = 0,
                           out: Optional[torch.Tensor] = None, out_dtype: Optional[torch.dtype] = None,
                           out_record: Optional[torch.Tensor] = None,
                           error_flag: Optional[torch.Tensor] = None,
                           workspace: Optional[torch.Tensor] = None, exchange=None,
                           records_only: bool = False) -> Optional[torch.Tensor]:
    """Single-query attention of q [B, Hq, D] over paged K/V (see helm_paged_attn_decode).

    ``page_table``/``page_used`` are int32 [B, max_pages] and ``num_pages``
    int32 [B], all on q's device.  Returns ``out`` [B, Hq, D] (allocated in
    ``out_dtype``, default q.dtype, unless given), or None when only
    ``out_record`` is requested.  ``exchange``: a ctypes pointer to a ShardExchange (KV sequence
    sharding with the cross-GPU exchange fused into the kernel).
    ``records_only``: write no output; return the split records [S, B*Hq, D+2]
    (fp32, a view of the workspace) for a later merge (KVShardGroup.gather_merge merges and
    exchanges them in one launch).  Consume them before the workspace is reused.
    """
    dev = _need_cuda("paged_decode_attention", q, k_base, v_base, page_table, page_used, num_pages)
    if not q.is_contiguous() or q.dim() != 3:
        raise ValueError("paged_decode_attention: q must be a contiguous [B, Hq, D] tensor")
    for name, t in (("page_table", page_table), ("page_used", page_used), ("num_pages", num_pages)):
        if t.dtype != torch.int32:
            raise TypeError(f"paged_decode_attention: {name} must be int32")
        if t.stride(-1) != 1:
            raise ValueError(f"paged_decode_attention: {name} must have unit inner stride")
    if page_table.dim() == 2 and page_used.stride(0) != page_table.stride(0):
        raise ValueError("paged_decode_attention: page_used must share page_table's row stride")
    if records_only:
        out = out_record = None
    elif out is None and out_record is None:
        out = torch.empty(q.shape, dtype=out_dtype or q.dtype, device=dev)
    p = make_attn_params(q, k_base, v_base, page_table, page_used, num_pages, num_kv_heads=num_kv_heads,
                         page_size=page_size, page_stride=page_stride, head_stride=head_stride,
                         num_pool_pages=num_pool_pages, scale=scale, max_pages=max_pages, num_splits=num_splits,
                         out=out, out_record=out_record, error_flag=error_flag)
    if exchange is not None:
        p.exchange = exchange
    lib = N.lib()
    S = ctypes.c_int32(0)
    need = lib.helm_paged_attn_workspace_bytes(ctypes.byref(p), ctypes.byref(S))
    if need < 0:
        N.check("helm_paged_attn_workspace_bytes", N.ERR_INVALID_ARGUMENT)
    p.num_splits = S.value
    ws = None
    if need > 0:
        ws = workspace if workspace is not None and workspace.numel() * 4 >= need else WORKSPACE.get(dev, need)
        p.workspace = ws.data_ptr()
        p.workspace_bytes = ws.numel() * ws.element_size()
    N.check("helm_paged_attn_decode", lib.helm_paged_attn_decode(ctypes.byref(p), _stream(dev)))
    if records_only:
        B, Hq, D = q.shape
        return ws.view(-1)[:S.value * B * Hq * (D + 2)].view(S.value, B * Hq, D + 2)
    return out


def lse_merge(partials: torch.Tensor, out: Optional[torch.Tensor] = None, out_dtype=torch.float32,
              out_record: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
    """Merges records [S, rows, D+2] (o..., m, l) into out [rows, D] and/or a merged record."""
    dev = _need_cuda("lse_merge", partials)
    if partials.dtype != torch.float32 or partials.dim() != 3 or not partials.is_contiguous():
        raise ValueError("lse_merge: partials must be contiguous float32 [S, rows, D+2]")
    S, rows, rl = partials.shape
    D = rl - 2
    if out is None and out_record is None:
        out = torch.empty((rows, D), dtype=out_dtype, device=dev)
    code = N.lib().helm_lse_merge(partials.data_ptr(), S, rows * rl, rows, D, _ptr(out),
                                  dtype_code(out.dtype) if out is not None else N.F32, _ptr(out_record),
                                  _stream(dev))
    N.check("helm_lse_merge", code)
    return out


class PackedInt8:
    """INT8 weights [N, K] in the packed block layout of helm_int8_pack_weight (``data``, a flat int8
    device tensor); ``rows(lo, hi)`` is the packed weight of rows [lo, hi) (multiples of 16), a view."""

    def __init__(self, data: torch.Tensor, N: int, K: int):
        self.data, self.N, self.K = data, N, K
        self.kb = (K + 127) // 128

    @property
    def device(self):
        return self.data.device

    @property
    def shape(self):
        return (self.N, self.K)

    def rows(self, lo: int, hi: int) -> "PackedInt8":
        if lo % 16 or (hi % 16 and hi != self.N):
            raise ValueError("PackedInt8.rows: bounds must be multiples of 16")
        blk = self.kb * 2048
        return PackedInt8(self.data[(lo // 16) * blk:((hi + 15) // 16) * blk], hi - lo, self.K)

    def unpack(self) -> torch.Tensor:
        """The row-major int8 [N, K] weight."""
        T = (self.N + 15) // 16
        b = self.data.view(T, self.kb, 16, 8, 16)
        r = torch.arange(16, device=self.data.device)[:, None]
        c = torch.arange(8, device=self.data.device)[None, :]
        src = (c ^ (r & 7))                       # stored chunk of logical chunk c in row r
        b = b[:, :, r, src]                       # [T, kb, 16, 8, 16]: logical chunk order
        return b.permute(0, 2, 1, 3, 4).reshape(T * 16, self.kb * 128)[:self.N, :self.K].contiguous()


def int8_pack_weight(weight: torch.Tensor) -> PackedInt8:
    """helm_int8_pack_weight of a contiguous int8 [N, K] tensor.  A weight still on the host (a
    module quantised before it is moved) is rearranged with the same index arithmetic in torch; the
    layout is the data's, not a compute path."""
    if weight.dtype != torch.int8 or weight.dim() != 2 or not weight.is_contiguous():
        raise ValueError("int8_pack_weight: weight must be a contiguous int8 [N, K] tensor")
    Nn, K = weight.shape
    nbytes = N.lib().helm_int8_packed_bytes(Nn, K)
    if nbytes < 0:
        raise ValueError(f"int8_pack_weight: K={K} must be a positive multiple of 16")
    if weight.device.type != "cuda":
        T, KB = (Nn + 15) // 16, (K + 127) // 128
        w = torch.zeros((T * 16, KB * 128), dtype=torch.int8)
        w[:Nn, :K] = weight
        b = w.view(T, 16, KB, 8, 16).permute(0, 2, 1, 3, 4)          # [T, KB, 16 rows, 8 chunks, 16]
        r = torch.arange(16)[:, None]
        c = torch.arange(8)[None, :]
        b = b[:, :, r, c ^ (r & 7)]                                      # stored chunk c <- logical c ^ (r & 7)
        return PackedInt8(b.contiguous().view(-1), Nn, K)
    dev = weight.device
    out = torch.empty(max(nbytes, 16), dtype=torch.int8, device=dev)
    N.check("helm_int8_pack_weight", N.lib().helm_int8_pack_weight(weight.data_ptr(), Nn, K, out.data_ptr(),
                                                                     _stream(dev)))
    return PackedInt8(out[:nbytes], Nn, K)


def int8_linear(x: torch.Tensor, weight, scale: torch.Tensor,
                bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None,
                gemm: bool = False) -> torch.Tensor:
    """y = (x @ weight.T) * scale + bias with int8 ``weight`` [N, K] (a row-major tensor or a
    PackedInt8) and per-row ``scale`` [N].  gemm=True (PackedInt8 only) runs the tcgen05 GEMM
    (helm_int8_gemm_packed) instead of the GEMV kernel."""
    packed = isinstance(weight, PackedInt8)
    if gemm and not packed:
        raise ValueError("int8_linear: the tensor-core GEMM takes packed weights")
    wt = weight.data if packed else weight
    dev = _need_cuda("int8_linear", x, wt, scale, bias)
    if not packed and (weight.dtype != torch.int8 or weight.dim() != 2 or not weight.is_contiguous()):
        raise ValueError("int8_linear: weight must be a contiguous int8 [N, K] tensor")
    Nn, K = weight.shape
    if x.shape[-1] != K:
        raise ValueError(f"int8_linear: input last dim ({x.shape[-1]}) != weight K ({K})")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    M = x2.shape[0]
    if scale.shape != (Nn,) or not scale.is_contiguous():
        raise ValueError("int8_linear: scale must be a contiguous [N] tensor")
    if bias is not None:
        if bias.dtype != x.dtype:
            bias = bias.to(x.dtype)
        bias = bias.contiguous()
    y = out if out is not None else torch.empty((M, Nn), dtype=x.dtype, device=dev)
    lib = N.lib()
    name = "helm_int8_gemm_packed" if gemm else "helm_int8_linear_packed" if packed else "helm_int8_linear"
    code = getattr(lib, name)(x2.data_ptr(), dtype_code(x.dtype), wt.data_ptr(), scale.data_ptr(),
                              dtype_code(scale.dtype), _ptr(bias), y.data_ptr(), M, Nn, K, _stream(dev))
    N.check(name, code)
    return y.reshape(*lead, Nn)


def int8_linear_glu(x: torch.Tensor, weight, scale: torch.Tensor,
                    bias: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """helm_int8_linear_glu: silu(x @ Wg.T * sg + bg) * (x @ Wu.T * su + bu) from the tile-interleaved
    int8 ``weight`` [2I, K] (see interleave_glu_rows; a row-major tensor or a PackedInt8) and
    ``scale`` / ``bias`` [2I]; returns [..., I]."""
    packed = isinstance(weight, PackedInt8)
    wt = weight.data if packed else weight
    dev = _need_cuda("int8_linear_glu", x, wt, scale, bias)
    if not packed and (weight.dtype != torch.int8 or weight.dim() != 2 or not weight.is_contiguous()):
        raise ValueError("int8_linear_glu: weight must be a contiguous int8 [2I, K] tensor")
    N2, K = weight.shape
    if x.shape[-1] != K or N2 % 32:
        raise ValueError(f"int8_linear_glu: weight [{N2}, {K}] does not fit input [..., {x.shape[-1]}] "
                         "(2I must be a multiple of 32)")
    lead = x.shape[:-1]
    x2 = x.reshape(-1, K)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    M = x2.shape[0]
    if scale.shape != (N2,) or not scale.is_contiguous():
        raise ValueError("int8_linear_glu: scale must be a contiguous [2I] tensor")
    if bias is not None:
        bias = bias.to(x.dtype).contiguous()
    y = out if out is not None else torch.empty((M, N2 // 2), dtype=x.dtype, device=dev)
    fn = N.lib().helm_int8_linear_glu_packed if packed else N.lib().helm_int8_linear_glu
    code = fn(x2.data_ptr(), dtype_code(x.dtype), wt.data_ptr(), scale.data_ptr(), dtype_code(scale.dtype),
              _ptr(bias), y.data_ptr(), M, N2 // 2, K, _stream(dev))
    N.check("helm_int8_linear_glu_packed" if packed else "helm_int8_linear_glu", code)
    return y.reshape(*lead, N2 // 2)


def interleave_glu_rows(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[2I, ...] rows in the order helm_int8_linear_glu reads them: 16 gate rows, then the same 16
    up rows, and so on (I a multiple of 16)."""
    I = gate.shape[0]
    if up.shape != gate.shape or I % 16:
        raise ValueError("interleave_glu_rows: gate and up must match, with a multiple of 16 rows")
    tail = gate.shape[1:]
    return torch.stack((gate.reshape(I // 16, 16, *tail), up.reshape(I // 16, 16, *tail)), 1).reshape(2 * I, *tail)


def int8_linear_error(reset: bool = True) -> int:
    """HELM_DEVERR_* bits raised by the INT8 kernels since the last reset (synchronises)."""
    v = ctypes.c_int32(0)
    N.check("helm_int8_linear_error", N.lib().helm_int8_linear_error(ctypes.byref(v), 1 if reset else 0))
    return v.value


def make_append_params(k_new, v_new, k_base, v_base, *, page_stride, head_stride, num_pool_pages, page_size,
                       dest=None, dest_host=None, page_table=None, page_used=None, num_pages=None,
                       spare_pages=None, spare_next=None, error_flag=None) -> N.KVAppendParams:
    """Parameter block of helm_kv_append.  ``dest_host`` is a C-contiguous int32 numpy array [B, 3]
    (kept alive by the caller until the call returns)."""
    B, Hkv, D = k_new.shape
    p = N.KVAppendParams()
    p.k_new, p.v_new = k_new.data_ptr(), v_new.data_ptr()
    p.src_dtype = dtype_code(k_new.dtype)
    p.k_base, p.v_base = k_base.data_ptr(), v_base.data_ptr()
    p.page_stride, p.head_stride = int(page_stride), int(head_stride)
    p.num_pool_pages = int(num_pool_pages)
    p.kv_dtype = dtype_code(k_base.dtype)
    p.B, p.Hkv, p.D, p.P = B, Hkv, D, int(page_size)
    p.dest = _ptr(dest)
    p.dest_host = None if dest_host is None else dest_host.ctypes.data
    p.page_table, p.page_used, p.num_pages = _ptr(page_table), _ptr(page_used), _ptr(num_pages)
    p.page_table_stride = page_table.stride(0) if page_table is not None and page_table.dim() == 2 else 0
    p.spare_pages, p.spare_next = _ptr(spare_pages), _ptr(spare_next)
    p.spare_stride = spare_pages.shape[-1] if spare_pages is not None else 0
    p.error_flag = _ptr(error_flag)
    return p


def kv_append(k_new: torch.Tensor, v_new: torch.Tensor, k_base: torch.Tensor, v_base: torch.Tensor, **kw) -> None:
    """Writes one token per sequence into the pool (see helm_kv_append)."""
    dev = _need_cuda("kv_append", k_new, v_new, k_base, v_base)
    if not (k_new.is_contiguous() and v_new.is_contiguous()) or k_new.dim() != 3 or k_new.shape != v_new.shape:
        raise ValueError("kv_append: k_new/v_new must be contiguous [B, Hkv, D] tensors of one shape")
    p = make_append_params(k_new, v_new, k_base, v_base, **kw)
    N.check("helm_kv_append", N.lib().helm_kv_append(ctypes.byref(p), _stream(dev)))


def decode_prologue(q_in: torch.Tensor, k_new: torch.Tensor, v_new: torch.Tensor, q_out: torch.Tensor, k_base,
                    v_base, *, q_norm_w=None, k_norm_w=None, eps: float = 1e-6, cos=None, sin=None,
                    do_append: bool = True, **append_kw) -> None:
    """helm_decode_prologue: q_in [B, Hq, D], k_new / v_new [B, Hkv, D] raw projections (rows may be
    strided, heads contiguous); q_out [B, Hq, D] contiguous; cos / sin [B, D] (rows may be strided);
    append_kw: the destination arguments of make_append_params."""
    dev = _need_cuda("decode_prologue", q_in, k_new, v_new, q_out)
    B, Hq, D = q_in.shape
    for name, t in (("q_in", q_in), ("k_new", k_new), ("v_new", v_new)):
        if t.dim() != 3 or t.stride(2) != 1 or t.stride(1) != D:
            raise ValueError(f"decode_prologue: {name} must be [B, H, D] with contiguous heads")
    if not q_out.is_contiguous() or tuple(q_out.shape) != (B, Hq, D) or q_out.dtype != q_in.dtype:
        raise ValueError("decode_prologue: q_out must be a contiguous [B, Hq, D] tensor of q's dtype")
    if k_new.dtype != q_in.dtype or v_new.dtype != q_in.dtype:
        raise ValueError("decode_prologue: q, k and v must share a dtype")
    p = N.DecodePrologueParams()
    p.append = make_append_params(k_new, v_new, k_base, v_base, **append_kw)
    p.q_in, p.q_out, p.Hq = q_in.data_ptr(), q_out.data_ptr(), Hq
    p.q_stride, p.k_stride, p.v_stride = q_in.stride(0), k_new.stride(0), v_new.stride(0)
    p.q_norm_w, p.k_norm_w = _ptr(q_norm_w), _ptr(k_norm_w)
    p.norm_dtype = dtype_code(q_norm_w.dtype) if q_norm_w is not None else N.F32
    p.eps = float(eps)
    if cos is not None:
        if cos.stride(-1) != 1 or sin.stride(-1) != 1 or cos.shape[-1] != D or cos.stride(0) != sin.stride(0):
            raise ValueError("decode_prologue: cos / sin must be [B, D] rows with unit inner stride")
        p.cos, p.sin, p.cs_dtype, p.cs_stride = cos.data_ptr(), sin.data_ptr(), dtype_code(cos.dtype), cos.stride(0)
    else:
        p.cs_dtype = N.F32
    p.do_append = 1 if do_append else 0
    N.check("helm_decode_prologue", N.lib().helm_decode_prologue(ctypes.byref(p), _stream(dev)))


def kv_write_pages(K: torch.Tensor, V: torch.Tensor, k_base: torch.Tensor, v_base: torch.Tensor, pages, *,
                   page_stride: int, head_stride: int, num_pool_pages: int, page_size: int,
                   table=None, error_flag: Optional[torch.Tensor] = None) -> None:
    """helm_kv_write_pages: K / V [1, Hkv, S, D] (one sequence; head and token strides free, dims
    contiguous) chunked into pool slots; pages = [(slot, first token, tokens), ...].  table:
    optional (page_table_row, page_used_row, num_pages_word, first_index) device tensors/int."""
    import numpy as np
    dev = _need_cuda("kv_write_pages", K, V, k_base, v_base)
    if K.dim() != 4 or K.shape[0] != 1 or K.shape != V.shape:
        raise ValueError("kv_write_pages: K and V must be [1, Hkv, S, D] of one shape")
    if K.stride(-1) != 1 or V.stride(-1) != 1 or K.stride(1) != V.stride(1) or K.stride(2) != V.stride(2):
        K, V = K.contiguous(), V.contiguous()
    arr = np.ascontiguousarray(np.asarray(pages, dtype=np.int32).reshape(-1, 3))
    p = N.KVPrefillParams()
    p.k_src, p.v_src, p.src_dtype = K.data_ptr(), V.data_ptr(), dtype_code(K.dtype)
    p.src_head_stride, p.src_tok_stride = K.stride(1), K.stride(2)
    p.k_base, p.v_base = k_base.data_ptr(), v_base.data_ptr()
    p.page_stride, p.head_stride = int(page_stride), int(head_stride)
    p.num_pool_pages, p.kv_dtype = int(num_pool_pages), dtype_code(k_base.dtype)
    p.Hkv, p.D, p.P = K.shape[1], K.shape[3], int(page_size)
    p.pages, p.count = arr.ctypes.data, len(arr)
    if table is not None:
        pt, pu, npg, first = table
        p.page_table, p.page_used, p.num_pages = pt.data_ptr(), pu.data_ptr(), npg.data_ptr()
        p.page_table_stride, p.first_index = pt.shape[-1], int(first)
    p.error_flag = _ptr(error_flag)
    N.check("helm_kv_write_pages", N.lib().helm_kv_write_pages(ctypes.byref(p), _stream(dev)))


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """helm_rmsnorm over the last dimension of x (rows may be strided; the last dim contiguous)."""
    dev = _need_cuda("rmsnorm", x, weight)
    dim = x.shape[-1]
    x2 = x.reshape(-1, dim) if x.dim() != 2 else x
    if x2.stride(-1) != 1:
        x2 = x2.contiguous()
    y = out if out is not None else torch.empty(x.shape, dtype=x.dtype, device=dev)
    y2 = y.view(-1, dim)
    N.check("helm_rmsnorm", N.lib().helm_rmsnorm(x2.data_ptr(), dtype_code(x.dtype), x2.stride(0), weight.data_ptr(),
                                                 dtype_code(weight.dtype), y2.data_ptr(), y2.stride(0), x2.shape[0],
                                                 dim, float(eps), _stream(dev)))
    return y


def copy_pages(dst: torch.Tensor, dst_first: int, src: torch.Tensor, src_ids, page_bytes: int,
               stream: Optional[int] = None) -> int:
    """Copies pages src[src_ids[i]] -> dst[dst_first + i] (runs merged); returns the copy count."""
    import numpy as np
    ids = np.ascontiguousarray(np.asarray(src_ids, dtype=np.int32))
    if len(ids):
        if int(ids.min()) < 0 or int(ids.max()) >= src.shape[0]:
            raise ValueError(f"copy_pages: source page ids must lie in [0, {src.shape[0]})")
        if dst_first < 0 or dst_first + len(ids) > dst.shape[0]:
            raise ValueError(f"copy_pages: destination pages [{dst_first}, {dst_first + len(ids)}) outside "
                             f"[0, {dst.shape[0]})")
    dev = dst.device if dst.device.type == "cuda" else src.device
    st = _stream(dev) if stream is None else stream
    n = ctypes.c_int32(0)
    code = N.lib().helm_copy_pages(dst.data_ptr(), int(dst_first), src.data_ptr(),
                                   ids.ctypes.data_as(ctypes.c_void_p), len(ids), int(page_bytes),
                                   ctypes.byref(n), st)
    N.check("helm_copy_pages", code)
    return n.value


def move_pages(dst: torch.Tensor, dst_ids, src: torch.Tensor, src_ids, page_bytes: int,
               stream: Optional[int] = None) -> int:
    """helm_move_pages: src[src_ids[i]] -> dst[dst_ids[i]] for slabs whose first dimension is the page
    (ids checked against both slabs' page counts); returns the launch / copy count."""
    import numpy as np
    s_ids = np.ascontiguousarray(np.asarray(src_ids, dtype=np.int32))
    d_ids = np.ascontiguousarray(np.asarray(dst_ids, dtype=np.int32))
    if s_ids.shape != d_ids.shape:
        raise ValueError("move_pages: src_ids and dst_ids differ in length")
    dev = src.device if src.device.type == "cuda" else dst.device
    if dev.type != "cuda":
        raise ValueError("helm_b200.move_pages: one slab must be on a CUDA device")
    st = _stream(dev) if stream is None else stream
    n = ctypes.c_int32(0)
    code = N.lib().helm_move_pages(dst.data_ptr(), d_ids.ctypes.data_as(ctypes.c_void_p), src.data_ptr(),
                                   s_ids.ctypes.data_as(ctypes.c_void_p), len(s_ids), int(page_bytes),
                                   int(dst.shape[0]), int(src.shape[0]), ctypes.byref(n), st)
    N.check("helm_move_pages", code)
    return n.value
