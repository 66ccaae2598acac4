"""helm_b200.kernels -- INT8 weight-only linear layers for the decode path.

The GPU counterpart of helm.kernels (helm/kernels/__init__.py): the same
module-swap pattern as patch_cpu_linears / _AVXLinear (__init__.py:107-157)
and the same availability probes (is_available / load_error, :91-100), with
int8 weights and one scale per output channel instead of fp16 weights.

    n = patch_int8_linears(model)        # nn.Linear -> Int8Linear, in place
    y = int8_linear(x, w_int8, scale)    # one call of helm_int8_linear

Quantisation is symmetric per output channel: scale[n] = max_k |W[n, k]| / 127,
W_q = round(W / scale) clipped to [-127, 127].  Decode-sized inputs
(rows <= 64 of x) run the INT8 GEMV kernel; larger (prefill) inputs run the
tcgen05 INT8 GEMM (helm_int8_gemm_packed) on the same packed weights.

Projections that read the same input are fused (fuse=True, the default):
an attention module's q_proj / k_proj / v_proj share one int8 weight, so a
decode step projects q, k and v with one launch (Int8QKV; the three modules
stay, as views of it, for prefill), and a SwiGLU MLP's gate_proj / up_proj and
silu(gate) * up become one launch with the activation in the epilogue
(Int8GLU, helm_int8_linear_glu).
"""
from __future__ import annotations

import types
from typing import Iterable, Optional, Tuple

import torch
import torch.nn as nn
import torch.nn.functional as F

from .. import _native
from .. import ops

# Rows of x up to which the INT8 GEMV kernel is used; above it the weight is dequantised once
# per call and a dense GEMM runs (prefill).
INT8_KERNEL_MAX_ROWS = 64


def is_available() -> bool:
    """True if libhelm_b200.so loads."""
    return _native.is_available()


def load_error() -> Optional[str]:
    """Why the library did not load, or None."""
    return _native.load_error()


@torch.no_grad()
def quantize_weight(weight: torch.Tensor, scale_dtype: Optional[torch.dtype] = None) -> Tuple[torch.Tensor, torch.Tensor]:
    """Symmetric per-output-channel int8 quantisation of weight [N, K]: (int8 [N, K], scale [N])."""
    w = weight.detach().float()
    amax = w.abs().amax(dim=1)
    scale = torch.where(amax > 0, amax / 127.0, torch.ones_like(amax))
    q = torch.clamp(torch.round(w / scale[:, None]), -127, 127).to(torch.int8)
    return q.contiguous(), scale.to(scale_dtype or weight.dtype).contiguous()


def int8_linear(input: torch.Tensor, weight, scale: torch.Tensor,
                bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = (input @ weight.T) * scale + bias, weight int8 [N, K] (a row-major tensor or an
    ops.PackedInt8), scale [N]; CUDA tensors only."""
    rows = input.numel() // input.shape[-1] if input.numel() else 0
    if rows <= INT8_KERNEL_MAX_ROWS:
        return ops.int8_linear(input, weight, scale, bias)
    if isinstance(weight, ops.PackedInt8):
        return ops.int8_linear(input, weight, scale, bias, gemm=True)   # tcgen05 GEMM
    w = weight.to(input.dtype) * scale.to(input.dtype)[:, None]
    return F.linear(input, w, None if bias is None else bias.to(input.dtype))


class _PackedWeight:
    """Mixin: the int8 weight lives packed (ops.PackedInt8, buffer `packed`); `weight` reads back
    the row-major int8 [N, K] and assigning it packs."""

    def _set_packed(self, pk: "ops.PackedInt8") -> None:
        self.packed = pk.data
        self._shape = (pk.N, pk.K)

    @property
    def pk(self) -> "ops.PackedInt8":
        return ops.PackedInt8(self.packed, *self._shape)

    @property
    def weight(self) -> torch.Tensor:
        return self.pk.unpack()

    @weight.setter
    def weight(self, w: torch.Tensor) -> None:
        self._set_packed(ops.int8_pack_weight(w.contiguous()))


class Int8Linear(_PackedWeight, nn.Module):
    """nn.Linear replacement holding an int8 weight [N, K] (stored packed for the kernel) and a
    per-channel scale [N]."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None,
                 dtype: torch.dtype = torch.bfloat16):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.register_buffer("packed", torch.zeros(0, dtype=torch.int8, device=device))
        self._shape = (out_features, in_features)
        self.register_buffer("scale", torch.ones((out_features,), dtype=dtype, device=device))
        if bias:
            self.register_buffer("bias", torch.zeros((out_features,), dtype=dtype, device=device))
        else:
            self.bias = None
        if device is not None and torch.device(device).type == "cuda":
            self.weight = torch.zeros((out_features, in_features), dtype=torch.int8, device=device)

    @classmethod
    def from_linear(cls, linear: nn.Linear, scale_dtype: Optional[torch.dtype] = None) -> "Int8Linear":
        m = cls(linear.in_features, linear.out_features, bias=linear.bias is not None,
                device=linear.weight.device, dtype=scale_dtype or linear.weight.dtype)
        q, s = quantize_weight(linear.weight, scale_dtype or linear.weight.dtype)
        m.weight = q
        m.scale = s
        if linear.bias is not None:
            m.bias = linear.bias.detach().clone()
        return m

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.device.type != "cuda":
            raise RuntimeError("Int8Linear runs on CUDA devices only (no CPU implementation)")
        return int8_linear(x, self.pk, self.scale, self.bias)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, int8=True")


class Int8QKV(_PackedWeight, nn.Module):
    """q_proj, k_proj and v_proj of one attention module as one int8 weight [Nq+Nk+Nv, K] (and one
    scale / bias vector): a decode step projects all three with one INT8 launch.  The module's own
    q_proj / k_proj / v_proj become Int8Linear views of the fused buffers (for prefill)."""

    def __init__(self, q: nn.Linear, k: nn.Linear, v: nn.Linear):
        super().__init__()
        parts = [quantize_weight(m.weight) for m in (q, k, v)]
        self.splits = tuple(m.out_features for m in (q, k, v))
        self.register_buffer("packed", torch.zeros(0, dtype=torch.int8, device=q.weight.device))
        self.weight = torch.cat([p[0] for p in parts]).contiguous()
        self.register_buffer("scale", torch.cat([p[1] for p in parts]).contiguous())
        if q.bias is not None:
            self.register_buffer("bias", torch.cat([m.bias.detach() for m in (q, k, v)]).contiguous())
        else:
            self.bias = None

    def views(self):
        """Int8Linear modules over the q, k and v rows of the fused buffers (row bounds are
        multiples of 16, so each view is a contiguous slice of the packed blocks)."""
        out, lo = [], 0
        K = self._shape[1]
        pk = self.pk
        for n in self.splits:
            m = Int8Linear(K, n, bias=self.bias is not None, device=None, dtype=self.scale.dtype)
            m._set_packed(pk.rows(lo, lo + n))
            m.scale = self.scale[lo:lo + n]
            if self.bias is not None:
                m.bias = self.bias[lo:lo + n]
            out.append(m)
            lo += n
        return out

    def forward(self, x: torch.Tensor):
        """(q, k, v) projections of x as views of one [..., Nq+Nk+Nv] output."""
        y = int8_linear(x, self.pk, self.scale, self.bias)
        nq, nk, _ = self.splits
        return y[..., :nq], y[..., nq:nq + nk], y[..., nq + nk:]


class Int8GLU(_PackedWeight, nn.Module):
    """gate_proj, up_proj and silu(gate) * up of a SwiGLU MLP as one tile-interleaved int8 weight
    [2I, K] (ops.interleave_glu_rows): decode-sized inputs run helm_int8_linear_glu (one launch, the
    activation in the epilogue); larger inputs run the tcgen05 GEMM over both halves and apply
    silu(gate) * up in the activation dtype, as the unfused MLP does."""

    def __init__(self, gate: nn.Linear, up: nn.Linear):
        super().__init__()
        qg, sg = quantize_weight(gate.weight)
        qu, su = quantize_weight(up.weight)
        self.I, self.K = gate.out_features, gate.in_features
        self.register_buffer("packed", torch.zeros(0, dtype=torch.int8, device=gate.weight.device))
        self.weight = ops.interleave_glu_rows(qg, qu).contiguous()
        self.register_buffer("scale", ops.interleave_glu_rows(sg, su).contiguous())
        if gate.bias is not None:
            self.register_buffer("bias", ops.interleave_glu_rows(gate.bias.detach(), up.bias.detach()).contiguous())
        else:
            self.bias = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if x.device.type != "cuda":
            raise RuntimeError("Int8GLU runs on CUDA devices only (no CPU implementation)")
        rows = x.numel() // x.shape[-1] if x.numel() else 0
        if rows <= INT8_KERNEL_MAX_ROWS:
            return ops.int8_linear_glu(x, self.pk, self.scale, self.bias)
        y = ops.int8_linear(x, self.pk, self.scale, self.bias, gemm=True)   # tcgen05 GEMM, [.., 2I]
        y = y.reshape(*x.shape[:-1], self.I // 16, 2, 16)
        return (F.silu(y[..., 0, :]) * y[..., 1, :]).reshape(*x.shape[:-1], self.I)


def _glu_mlp_forward(mlp_self, x):
    return mlp_self.down_proj(mlp_self._helm_glu(x))


def _is_silu(act) -> bool:
    return type(act).__name__ in ("SiLU", "SiLUActivation")


def _linear_ok(m, skip, name) -> bool:
    return (isinstance(m, nn.Linear) and name not in skip and m.weight.device.type == "cuda"
            and m.in_features % 16 == 0 and m.weight.dtype in (torch.float16, torch.bfloat16))


def patch_int8_linears(module: nn.Module, verbose: bool = False,
                       skip: Iterable[str] = (), fuse: bool = True) -> int:
    """Replaces, in place, every fp16/bf16 nn.Linear child on a CUDA device whose in_features is a
    multiple of 16 with Int8Linear -- the lm_head included, as patch_cpu_linears replaces every
    linear (helm/kernels/__init__.py:133-157); children named in `skip` are kept.  Returns how many
    were replaced.  With fuse=True, an
    attention module's q/k/v projections share one fused weight (Int8QKV, module attribute
    `_helm_qkv`) and a SwiGLU MLP's gate/up projections become one Int8GLU (`_helm_glu`, with the
    MLP's forward patched on the instance); each still counts as its replaced linears."""
    if not is_available():
        if verbose:
            print(f"[helm_b200 kernels] library unavailable ({load_error()}); skipping patch")
        return 0
    skip = set(skip)
    count = 0
    if fuse:
        kids = dict(module.named_children())
        qkv = [kids.get(n) for n in ("q_proj", "k_proj", "v_proj")]
        if (all(_linear_ok(m, skip, n) for m, n in zip(qkv, ("q_proj", "k_proj", "v_proj")))
                and len({(m.in_features, m.weight.dtype, m.bias is not None) for m in qkv}) == 1):
            fused = Int8QKV(*qkv)
            module._helm_qkv = fused
            for n, m in zip(("q_proj", "k_proj", "v_proj"), fused.views()):
                setattr(module, n, m)
            count += 3
        gate, up, down = kids.get("gate_proj"), kids.get("up_proj"), kids.get("down_proj")
        if (_linear_ok(gate, skip, "gate_proj") and _linear_ok(up, skip, "up_proj") and down is not None
                and _is_silu(getattr(module, "act_fn", None)) and gate.out_features % 16 == 0
                and gate.weight.shape == up.weight.shape and (gate.bias is None) == (up.bias is None)):
            module._helm_glu = Int8GLU(gate, up)
            del module.gate_proj, module.up_proj
            module.forward = types.MethodType(_glu_mlp_forward, module)
            count += 2
    for name, child in list(module.named_children()):
        if name == "_helm_qkv" or name == "_helm_glu":
            continue
        if isinstance(child, nn.Linear):
            if _linear_ok(child, skip, name):
                setattr(module, name, Int8Linear.from_linear(child))
                count += 1
        elif not isinstance(child, Int8Linear):
            count += patch_int8_linears(child, verbose=verbose, skip=skip, fuse=fuse)
    return count
