"""CPU restatement of the INT8 weight-only linear.  TEST INFRASTRUCTURE ONLY.

The reference has no INT8 code (its only linear kernel is the fp16 CPU GEMV,
helm/kernels/fp16_gemv.cpp:45-100); this oracle states the new operator
y = (x @ W^T) * s + bias in float64 with W int8 [N, K] and per-output-channel
scales s [N].  Parity of the INT8 path is therefore pinned only by this
restatement and, on fp16-dequantised weights, by the reference's own GEMV
(tests/golden/fp16_gemv.npz).
"""
from __future__ import annotations

import numpy as np


def int8_linear_ref(x: np.ndarray, w: np.ndarray, s: np.ndarray, bias=None) -> np.ndarray:
    """float64 y [M, N] for x [M, K], int8 w [N, K], s [N], optional bias [N]."""
    y = x.astype(np.float64) @ w.astype(np.float64).T
    y *= s.astype(np.float64)[None, :]
    if bias is not None:
        y += np.asarray(bias, dtype=np.float64)[None, :]
    return y


def quantize_per_channel(w: np.ndarray):
    """Symmetric per-output-channel int8 quantisation: s = max|w_row| / 127, q = round(w / s)."""
    w = np.asarray(w, dtype=np.float64)
    amax = np.abs(w).max(axis=1)
    s = np.where(amax > 0, amax / 127.0, 1.0)
    q = np.clip(np.rint(w / s[:, None]), -127, 127).astype(np.int8)
    return q, s
