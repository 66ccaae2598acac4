"""helm_b200.kernels -- INT8 weight-only linear layers for the decode path.

The GPU counterpart of helm.kernels (helm/kernels/__init__.py): the same
module-swap pattern as patch_cpu_linears / _AVXLinear (__init__.py:107-157)
and the same availability probes (is_available / load_error, :91-100), with
int8 weights and one scale per output channel instead of fp16 weights.

    n = patch_int8_linears(model)        # nn.Linear -> Int8Linear, in place
    y = int8_linear(x, w_int8, scale)    # one call of helm_int8_linear

Quantisation is symmetric per output channel: scale[n] = max_k |W[n, k]| / 127,
W_q = round(W / scale) clipped to [-127, 127].  Decode-sized inputs
(rows <= 64 of x) run the INT8 kernel; larger (prefill) inputs dequantise the
weight to the activation dtype and use a dense GEMM.
"""
from __future__ import annotations

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


def int8_linear(input: torch.Tensor, weight: torch.Tensor, scale: torch.Tensor,
                bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = (input @ weight.T) * scale + bias, weight int8 [N, K], scale [N]; CUDA tensors only."""
    rows = input.numel() // input.shape[-1] if input.numel() else 0
    if rows <= INT8_KERNEL_MAX_ROWS:
        return ops.int8_linear(input, weight, scale, bias)
    w = weight.to(input.dtype) * scale.to(input.dtype)[:, None]
    return F.linear(input, w, None if bias is None else bias.to(input.dtype))


class Int8Linear(nn.Module):
    """nn.Linear replacement holding an int8 weight [N, K] and a per-channel scale [N]."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True, device=None,
                 dtype: torch.dtype = torch.bfloat16):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.register_buffer("weight", torch.zeros((out_features, in_features), dtype=torch.int8, device=device))
        self.register_buffer("scale", torch.ones((out_features,), dtype=dtype, device=device))
        if bias:
            self.register_buffer("bias", torch.zeros((out_features,), dtype=dtype, device=device))
        else:
            self.bias = None

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
        return int8_linear(x, self.weight, self.scale, self.bias)

    def extra_repr(self) -> str:
        return (f"in_features={self.in_features}, out_features={self.out_features}, "
                f"bias={self.bias is not None}, int8=True")


def patch_int8_linears(module: nn.Module, verbose: bool = False,
                       skip: Iterable[str] = ("lm_head",)) -> int:
    """Replaces, in place, every fp16/bf16 nn.Linear child on a CUDA device whose in_features is a
    multiple of 16 with Int8Linear; children named in `skip` are kept.  Returns how many were replaced
    (the contract of patch_cpu_linears, helm/kernels/__init__.py:133-157)."""
    if not is_available():
        if verbose:
            print(f"[helm_b200 kernels] library unavailable ({load_error()}); skipping patch")
        return 0
    skip = set(skip)
    count = 0
    for name, child in list(module.named_children()):
        if isinstance(child, nn.Linear):
            if (name not in skip and child.weight.device.type == "cuda" and child.in_features % 16 == 0
                    and child.weight.dtype in (torch.float16, torch.bfloat16)):
                setattr(module, name, Int8Linear.from_linear(child))
                count += 1
        else:
            count += patch_int8_linears(child, verbose=verbose, skip=skip)
    return count
