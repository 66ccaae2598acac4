"""Seeded case definitions shared by tests/golden/make_golden.py and the tests.

Inputs are drawn with numpy's PCG64 generator, so they are identical on every
host; the fixtures store only the reference outputs.
"""
from __future__ import annotations

import hashlib

import numpy as np

# (name, seed, Hq, Hkv, D, page capacity, used tokens per page, dtype, scale)
ATTN_CASES = [
    ("single_page", 1, 2, 2, 8, 4, [4], "float32", None),
    ("two_pages", 2, 2, 2, 8, 4, [4, 3], "float32", None),
    ("three_ragged", 3, 1, 1, 16, 5, [3, 5, 2], "float32", None),
    ("gqa_multi", 4, 4, 2, 8, 4, [4, 3], "float32", None),
    ("empty_then_real", 5, 2, 2, 8, 4, [0, 4], "float32", None),
    ("all_empty", 6, 2, 2, 8, 4, [0, 0], "float32", None),
    ("custom_scale", 7, 1, 1, 4, 3, [3], "float32", 0.25),
    ("fp16_gqa", 8, 8, 2, 64, 16, [16, 16, 9], "float16", None),
    ("bf16_d128_p64", 9, 32, 8, 128, 64, [64, 64, 64, 17], "bfloat16", None),
    ("bf16_gqa8_d128", 10, 64, 8, 128, 64, [64] * 6 + [33], "bfloat16", None),
    ("fp16_gqa5_d128", 13, 40, 8, 128, 64, [64, 64, 64, 40], "float16", None),
    ("fp32_d128_p64", 11, 32, 8, 128, 64, [64, 64, 5], "float32", None),
    ("large_logits", 12, 1, 1, 64, 8, [8], "float32", None),
]


def attn_case_inputs(case):
    """(q [1, Hq, 1, D], k, v [pages, Hkv, cap, D]) float32 arrays for one case (before the cast
    to the case dtype)."""
    name, seed, Hq, Hkv, D, cap, useds, _dt, _scale = case
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((1, Hq, 1, D)).astype(np.float32)
    k = rng.standard_normal((len(useds), Hkv, cap, D)).astype(np.float32)
    v = rng.standard_normal((len(useds), Hkv, cap, D)).astype(np.float32)
    if name == "large_logits":
        q[:] = 100.0
        k[:] = 100.0
    return q, k, v


def page_bytes(Hkv, P, D, elem):
    """Bytes of one page (K and V) as the reference counts them (kv_cache.py:159)."""
    return 2 * Hkv * P * D * elem


def trace_specs():
    """Op sequences replayed on KVAllocator / KVCacheManager (see make_golden.run_trace)."""
    specs = []
    # 1. one sequence, 3 layers, watermark of 2 full pages: steady prefill+decode eviction.
    ops = [["init_layers", 0, 3]]
    for lid in range(3):
        ops.append(["prefill", 0, lid, 10])
    for _step in range(14):
        for lid in range(3):
            ops.append(["decode", 0, lid, 1])
    ops += [["clear", 0]]
    for lid in range(3):
        ops.append(["prefill", 0, lid, 7])
    specs.append({"name": "steady_decode", "seed": 21,
                  "alloc": {"num_layers": 3, "Hkv": 2, "D": 8, "P": 4, "dtype": "float32"},
                  "watermarks": [2 * page_bytes(2, 4, 8, 4)], "ops": ops})
    # 2. batch of two sharing one allocator, different prefill lengths, skip_residency steps.
    ops = []
    for mi, n in ((0, 9), (1, 17)):
        for lid in range(2):
            ops.append(["prefill", mi, lid, n])
    for step in range(10):
        for mi in range(2):
            for lid in range(2):
                ops.append(["decode", mi, lid, 1, {"skip": step % 3 == 1}])
    ops += [["evict", 1, 10 ** 6], ["clear", 0], ["prefill", 0, 0, 5], ["decode", 0, 0, 1]]
    specs.append({"name": "batch_two", "seed": 22,
                  "alloc": {"num_layers": 2, "Hkv": 2, "D": 8, "P": 4, "dtype": "float16"},
                  "watermarks": [3 * page_bytes(2, 4, 8, 2), 1], "ops": ops})
    # 3. zero watermark: every full non-tail page leaves; explicit evictions of odd byte counts;
    #    a partial page left resident between evicted ones.
    ops = [["reserve", 3, "cuda"], ["reserve", 2, "cpu"], ["prefill", 0, 0, 13], ["prefill", 0, 1, 8],
           ["evict", 0, 1], ["evict", 0, 0], ["decode", 0, 0, 1], ["decode", 0, 1, 1], ["prefill", 0, 0, 6]]
    specs.append({"name": "zero_watermark", "seed": 23,
                  "alloc": {"num_layers": 2, "Hkv": 1, "D": 16, "P": 4, "dtype": "bfloat16"},
                  "watermarks": [0], "ops": ops})
    # 4. start_token ties across layers (stable sort keeps layer order), partial tails, and an
    #    eviction budget that stops mid-way.
    pb = page_bytes(2, 8, 4, 4)
    ops = [["prefill", 0, 0, 16], ["prefill", 0, 1, 16], ["prefill", 0, 0, 3], ["prefill", 0, 1, 3],
           ["evict", 0, 3 * pb], ["decode", 0, 1, 1], ["decode", 0, 0, 1], ["evict", 0, pb + 1],
           ["prefill", 0, 0, 6], ["evict", 0, 10 ** 6]]
    specs.append({"name": "ties_partial", "seed": 24,
                  "alloc": {"num_layers": 2, "Hkv": 2, "D": 4, "P": 8, "dtype": "float32"},
                  "watermarks": [10 ** 9], "ops": ops})
    return specs


def config1_inputs():
    """torch.manual_seed(0); q [1,32,1,128], k, v [1,8,4096,128] ~ N(0,1) fp32."""
    import torch
    torch.manual_seed(0)
    q = torch.randn(1, 32, 1, 128)
    k = torch.randn(1, 8, 4096, 128)
    v = torch.randn(1, 8, 4096, 128)
    return q, k, v


def sha256_tensors(*ts):
    h = hashlib.sha256()
    for t in ts:
        h.update(t.contiguous().numpy().tobytes())
    return h.hexdigest()
