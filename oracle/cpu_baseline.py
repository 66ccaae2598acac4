"""Timed CPU baseline: the reference's own CPU decode-attention algorithm.  TEST/BENCH INFRASTRUCTURE ONLY.

bench.py's cpu_baseline leg and its `--impl reference` arm call this module;
nothing in helm_b200 does.  `path2_attention` restates, op for op, HELM's
all-CPU path of perform_streaming_attention (helm/runtime/kv_cache.py:376-380:
torch.cat of the used slices of every page, .float(), repeat_interleave of the
KV heads to the query heads, F.scaled_dot_product_attention, cast back) and
`path3_attention` its mixed-residency online-softmax loop
(kv_cache.py:387-442) without the CUDA copy stream.  The reference Python
package cannot travel to the GPU host, so this port is what is timed there.
"""
from __future__ import annotations

import math
import os
import time
from typing import List, Sequence, Tuple

import torch
import torch.nn.functional as F


def _expand(k: torch.Tensor, v: torch.Tensor, hq: int):
    hkv = k.size(1)
    if hkv != hq:
        g = hq // hkv
        k = k.repeat_interleave(g, dim=1)
        v = v.repeat_interleave(g, dim=1)
    return k, v


def path2_attention(query: torch.Tensor, pages: Sequence[Tuple[torch.Tensor, torch.Tensor, int]],
                    scale: float = None) -> torch.Tensor:
    """query [1, Hq, 1, D]; pages: (k [1, Hkv, P, D], v, used) on the CPU."""
    if scale is None:
        scale = 1.0 / math.sqrt(query.size(-1))
    act = [(k, v, u) for k, v, u in pages if u > 0]
    if not act:
        return torch.zeros_like(query)
    K = torch.cat([k[:, :, :u, :] for k, _, u in act], dim=2).float()
    V = torch.cat([v[:, :, :u, :] for _, v, u in act], dim=2).float()
    K, V = _expand(K, V, query.size(1))
    return F.scaled_dot_product_attention(query.float(), K, V, scale=scale).to(query.dtype)


def path3_attention(query: torch.Tensor, pages: Sequence[Tuple[torch.Tensor, torch.Tensor, int]],
                    scale: float = None) -> torch.Tensor:
    """The per-page online-softmax loop on the CPU."""
    if scale is None:
        scale = 1.0 / math.sqrt(query.size(-1))
    hq = query.size(1)
    q32 = query.float()
    out = torch.zeros(q32.shape, dtype=torch.float32)
    run_max = torch.full(q32.shape[:-1] + (1,), -float("inf"))
    run_sum = torch.zeros(q32.shape[:-1] + (1,))
    for k, v, u in pages:
        if u == 0:
            continue
        kk, vv = _expand(k[:, :, :u].float(), v[:, :, :u].float(), hq)
        s = torch.matmul(q32, kk.transpose(-2, -1)) * scale
        bmax = s.amax(dim=-1, keepdim=True)
        new_max = torch.maximum(run_max, bmax)
        old = torch.nan_to_num(torch.exp(run_max - new_max), nan=0.0)
        e = torch.exp(s - new_max)
        out = out * old + torch.matmul(e, vv)
        run_sum = run_sum * old + e.sum(dim=-1, keepdim=True)
        run_max = new_max
    return (out / torch.clamp(run_sum, min=1e-12)).to(query.dtype)


def host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


def time_decode_attention(Hq: int, Hkv: int, D: int, P: int, ctx: int, dtype=torch.bfloat16, path: int = 2,
                          min_seconds: float = 10.0, max_calls: int = 3, seed: int = 0):
    """Times one (layer, sequence) unit of decode attention over `ctx` cached tokens in pages of P
    on the host cores.  Returns (seconds per call, calls timed, threads)."""
    threads = host_threads()
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(seed)
    npg = (ctx + P - 1) // P
    pages: List[Tuple[torch.Tensor, torch.Tensor, int]] = []
    for i in range(npg):
        u = min(P, ctx - i * P)
        k = torch.randn(1, Hkv, P, D, generator=g).to(dtype)
        v = torch.randn(1, Hkv, P, D, generator=g).to(dtype)
        pages.append((k, v, u))
    q = torch.randn(1, Hq, 1, D, generator=g).to(dtype)
    fn = path2_attention if path == 2 else path3_attention
    fn(q, pages)  # warm-up
    times = []
    t_end = time.perf_counter() + min_seconds
    while len(times) < max_calls:
        t0 = time.perf_counter()
        fn(q, pages)
        times.append(time.perf_counter() - t0)
        if time.perf_counter() > t_end:
            break
    times.sort()
    return times[len(times) // 2], len(times), threads
