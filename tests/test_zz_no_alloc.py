"""GPU test of helm_paged_attn_decode_noalloc, the attention entry point that allocates nothing.

Some callers cannot allocate device memory on their own: a plugin running
inside a host application that owns the device-memory budget, or a caller
from another language runtime with no CUDA allocator to draw a workspace from.
For them the split-KV records live in a static device array inside the
library.  This test calls that entry point through the C ABI, twice in a row
on the same inputs, and checks each result against the regular entry point
(which uses a caller-provided workspace).  It sits in its own file, collected
last, and must pass both alone in a fresh process and after the other tests.
"""
import ctypes

import pytest
import torch

from tests.attn_util import ATTN_TOL_16BIT

pytestmark = pytest.mark.gpu


def _noalloc_fn():
    from helm_b200 import _native as N
    fn = N.lib().helm_paged_attn_decode_noalloc
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.POINTER(N.PagedAttnParams), ctypes.c_void_p]
    return fn


def _inputs(cuda, B, Hq, Hkv, npages, seed):
    g = torch.Generator(device=cuda).manual_seed(seed)
    D, P = 128, 64
    total = B * npages + 3
    kp = torch.randn(total, Hkv, P, D, generator=g, device=cuda).to(torch.bfloat16)
    vp = torch.randn(total, Hkv, P, D, generator=g, device=cuda).to(torch.bfloat16)
    pt = torch.randperm(total, generator=g, device=cuda)[:B * npages].to(torch.int32).reshape(B, npages)
    pu = torch.full((B, npages), P, dtype=torch.int32, device=cuda)
    pu[:, -1] = 17
    npg = torch.full((B,), npages, dtype=torch.int32, device=cuda)
    q = torch.randn(B, Hq, D, generator=g, device=cuda).to(torch.bfloat16)
    return q, kp, vp, pt, pu, npg, total


@pytest.mark.parametrize("splits", [6, 0])
def test_noalloc_matches_workspace_entry_point_twice(splits, cuda):
    from helm_b200 import ops
    from helm_b200 import _native as N
    B, Hq, Hkv, npages = 3, 32, 4, 24
    q, kp, vp, pt, pu, npg, total = _inputs(cuda, B, Hq, Hkv, npages, seed=17)
    common = dict(num_kv_heads=Hkv, page_size=64, page_stride=Hkv * 64 * 128, head_stride=64 * 128,
                  num_pool_pages=total)
    ref = ops.paged_decode_attention(q, kp, vp, pt, pu, npg, num_splits=splits, out_dtype=torch.float32,
                                     **common)
    fn = _noalloc_fn()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    for call in range(2):
        out = torch.full((B, Hq, 128), float("nan"), dtype=torch.float32, device=cuda)
        p = ops.make_attn_params(q, kp, vp, pt, pu, npg, out=out, num_splits=splits, **common)
        assert p.workspace is None  # nothing supplied: the entry point must not need it
        code = fn(ctypes.byref(p), stream)
        N.check("helm_paged_attn_decode_noalloc", code)
        torch.cuda.synchronize(cuda)
        err = float((out - ref).abs().max()) / max(1.0, float(ref.abs().max()))
        assert err <= ATTN_TOL_16BIT, f"call {call}: {err:.3e}"
        assert torch.isfinite(out).all()


def test_noalloc_rejects_too_many_explicit_splits(cuda):
    from helm_b200 import ops
    from helm_b200 import _native as N
    B, Hq, Hkv, npages = 4, 64, 8, 200
    q, kp, vp, pt, pu, npg, total = _inputs(cuda, B, Hq, Hkv, npages, seed=3)
    out = torch.empty(B, Hq, 128, dtype=torch.bfloat16, device=cuda)
    # 200 splits x 4*64*130*4 bytes = 26.6 MB of records > the 8 MiB static scratch
    p = ops.make_attn_params(q, kp, vp, pt, pu, npg, num_kv_heads=Hkv, page_size=64, page_stride=Hkv * 64 * 128,
                             head_stride=64 * 128, num_pool_pages=total, out=out, num_splits=200)
    code = _noalloc_fn()(ctypes.byref(p), torch.cuda.current_stream(cuda).cuda_stream)
    assert code == N.ERR_WORKSPACE
    assert b"static scratch" in N.lib().helm_last_error()


def test_noalloc_caps_the_automatic_split_count(cuda):
    """num_splits = 0 on a call whose automatic split count needs more records than the static
    array holds: the entry point lowers the split count to what fits, and its result equals the
    workspace entry point's with that same split count, bit for bit, on two calls in a row."""
    from helm_b200 import ops
    from helm_b200 import _native as N
    B, Hq, Hkv, npages = 1, 64, 1, 300          # GQA group 64: the split path
    q, kp, vp, pt, pu, npg, total = _inputs(cuda, B, Hq, Hkv, npages, seed=29)
    common = dict(num_kv_heads=Hkv, page_size=64, page_stride=Hkv * 64 * 128, head_stride=64 * 128,
                  num_pool_pages=total)
    probe = ops.make_attn_params(q, kp, vp, pt, pu, npg, out=torch.empty(B, Hq, 128, device=cuda), num_splits=0,
                                 **common)
    S = ctypes.c_int32(0)
    N.lib().helm_paged_attn_workspace_bytes(ctypes.byref(probe), ctypes.byref(S))
    per_split = B * Hq * (128 + 2) * 4
    cap = 8 << 20
    if S.value * per_split <= cap:
        pytest.skip(f"{S.value} automatic splits fit the static array on this GPU")
    capped = cap // per_split
    ref = ops.paged_decode_attention(q, kp, vp, pt, pu, npg, num_splits=capped, out_dtype=torch.float32, **common)
    fn = _noalloc_fn()
    stream = torch.cuda.current_stream(cuda).cuda_stream
    for call in range(2):
        out = torch.full((B, Hq, 128), float("nan"), dtype=torch.float32, device=cuda)
        p = ops.make_attn_params(q, kp, vp, pt, pu, npg, out=out, num_splits=0, **common)
        N.check("helm_paged_attn_decode_noalloc", fn(ctypes.byref(p), stream))
        torch.cuda.synchronize(cuda)
        assert torch.equal(out, ref), f"call {call}"
