"""Helpers shared by the attention tests: pool construction and tolerances."""
from __future__ import annotations

import numpy as np
import torch

# bf16 / fp16 unit roundoff of the final cast of an attention output.
ROUNDOFF = {torch.float32: 0.0, torch.float16: 2.0 ** -11, torch.bfloat16: 2.0 ** -8}

# The north-star bar for fp16/bf16 attention: max abs error <= 2e-3 relative to
# an fp32 (here float64) reference, measured on an fp32 output; a 16-bit output
# additionally carries its own rounding of up to one unit roundoff.
ATTN_TOL_16BIT = 2e-3
ATTN_TOL_FP32 = 1e-4  # the reference test-suite's atol for fp32 attention


def attn_error(out: torch.Tensor, ref: torch.Tensor) -> float:
    """max |out - ref| / max(1, max |ref|)."""
    out = out.detach().double().cpu()
    ref = ref.detach().double().cpu()
    scale = max(1.0, float(ref.abs().max())) if ref.numel() else 1.0
    return float((out - ref).abs().max()) / scale if ref.numel() else 0.0


def assert_attn_close(out: torch.Tensor, ref: torch.Tensor, kv_dtype: torch.dtype, what: str = ""):
    """Asserts out (any dtype) matches the float64 reference within the bar for kv_dtype."""
    base = ATTN_TOL_FP32 if kv_dtype == torch.float32 else ATTN_TOL_16BIT
    tol = base + ROUNDOFF[out.dtype]
    err = attn_error(out, ref)
    assert err <= tol, f"{what}: attention error {err:.3e} > {tol:.3e}"
    return err


def pool_from_pages(k: np.ndarray, v: np.ndarray, dtype: torch.dtype, device, shuffle_seed=None):
    """Pool tensors [n, Hkv, P, D] from page arrays; optionally with the pages at shuffled ids.
    Returns (k_pool, v_pool, ids) where ids[i] is the pool id of page i."""
    n = k.shape[0]
    ids = np.arange(n)
    if shuffle_seed is not None:
        ids = np.random.default_rng(shuffle_seed).permutation(n)
    kp = torch.empty(k.shape, dtype=dtype)
    vp = torch.empty(v.shape, dtype=dtype)
    kp[torch.from_numpy(ids)] = torch.from_numpy(k).to(dtype)
    vp[torch.from_numpy(ids)] = torch.from_numpy(v).to(dtype)
    return kp.to(device), vp.to(device), ids
