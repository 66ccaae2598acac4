"""perform_streaming_attention on the GPU: the reference suite's cases
(tests/unit/runtime/test_streaming_attention.py in HELM) ported to CUDA tensors, plus
allocator-backed pages with mixed GPU/CPU residency (staged through device slots)."""
import math

import pytest
import torch

from helm_b200.runtime import KVAllocator, KVCacheManager, KVPage, perform_streaming_attention
from tests.attn_util import assert_attn_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _page(k, v, page_id=0, start_token=0):
    used = k.size(2)
    return KVPage(page_id=page_id, layer_id=0, start_token=start_token, used_tokens=used, capacity_tokens=used,
                  k_tensor=k.clone(), v_tensor=v.clone(), device=k.device, state="GPU")


def _eager(q, k, v, scale=None):
    if scale is None:
        scale = 1.0 / math.sqrt(q.size(-1))
    w = torch.softmax(torch.matmul(q.double(), k.double().transpose(-2, -1)) * scale, dim=-1)
    return torch.matmul(w, v.double())


def _r(*s, dtype=torch.float32):
    return torch.randn(*s, device=DEV).to(dtype)


def test_single_two_three_pages_match_eager():
    torch.manual_seed(0)
    q, k, v = _r(1, 2, 1, 8), _r(1, 2, 4, 8), _r(1, 2, 4, 8)
    assert torch.allclose(perform_streaming_attention(q, [_page(k, v)]).double(), _eager(q, k, v), atol=1e-4)
    k1, v1, k2, v2 = _r(1, 2, 4, 8), _r(1, 2, 4, 8), _r(1, 2, 3, 8), _r(1, 2, 3, 8)
    out = perform_streaming_attention(q, [_page(k1, v1, 0, 0), _page(k2, v2, 1, 4)])
    assert torch.allclose(out.double(), _eager(q, torch.cat([k1, k2], 2), torch.cat([v1, v2], 2)), atol=1e-4)
    q = _r(1, 1, 1, 16)
    ks = [_r(1, 1, n, 16) for n in (3, 5, 2)]
    vs = [_r(1, 1, n, 16) for n in (3, 5, 2)]
    out = perform_streaming_attention(q, [_page(a, b, i) for i, (a, b) in enumerate(zip(ks, vs))])
    assert torch.allclose(out.double(), _eager(q, torch.cat(ks, 2), torch.cat(vs, 2)), atol=1e-4)


def test_edge_cases():
    q = _r(1, 2, 1, 8)
    out = perform_streaming_attention(q, [])
    assert out.shape == (1, 2, 1, 8) and torch.all(out == 0)
    k, v = _r(1, 2, 4, 8), _r(1, 2, 4, 8)
    empty = _page(k, v)
    empty.used_tokens = 0
    out = perform_streaming_attention(q, [empty])
    assert torch.allclose(out, torch.zeros_like(out), atol=1e-6)
    empty2 = _page(torch.zeros(1, 2, 4, 8, device=DEV), torch.zeros(1, 2, 4, 8, device=DEV))
    empty2.used_tokens = 0
    real = _page(k, v, page_id=1)
    assert torch.allclose(perform_streaming_attention(q, [empty2, real]), perform_streaming_attention(q, [real]),
                          atol=1e-5)


def test_scale_dtype_shape():
    q, k, v = _r(1, 1, 1, 4), _r(1, 1, 3, 4), _r(1, 1, 3, 4)
    assert torch.allclose(perform_streaming_attention(q, [_page(k, v)], scale=0.25).double(),
                          _eager(q, k, v, 0.25), atol=1e-4)
    q, k, v = _r(1, 1, 1, 16), _r(1, 1, 4, 16), _r(1, 1, 4, 16)
    assert torch.allclose(perform_streaming_attention(q, [_page(k, v)]),
                          perform_streaming_attention(q, [_page(k, v)], scale=1.0 / math.sqrt(16)), atol=1e-5)
    for dt in (torch.float32, torch.float16, torch.bfloat16):
        q, k, v = _r(1, 2, 1, 8, dtype=dt), _r(1, 2, 4, 8, dtype=dt), _r(1, 2, 4, 8, dtype=dt)
        assert perform_streaming_attention(q, [_page(k, v)]).dtype == dt
    q, k, v = _r(2, 4, 1, 16), _r(1, 4, 6, 16), _r(1, 4, 6, 16)
    assert perform_streaming_attention(q, [_page(k, v)]).shape == (2, 4, 1, 16)


def test_gqa_single_and_multi_page():
    q = _r(1, 4, 1, 8)
    ks, vs = [_r(1, 2, 4, 8), _r(1, 2, 3, 8)], [_r(1, 2, 4, 8), _r(1, 2, 3, 8)]
    out = perform_streaming_attention(q, [_page(ks[0], vs[0], 0, 0), _page(ks[1], vs[1], 1, 4)])
    ref = _eager(q, torch.cat(ks, 2).repeat_interleave(2, 1), torch.cat(vs, 2).repeat_interleave(2, 1))
    assert out.shape == (1, 4, 1, 8) and torch.allclose(out.double(), ref, atol=1e-4)


def test_large_logits_no_nan():
    q = torch.ones(1, 1, 1, 64, device=DEV) * 100.0
    k = torch.ones(1, 1, 8, 64, device=DEV) * 100.0
    v = _r(1, 1, 8, 64)
    out = perform_streaming_attention(q, [_page(k, v)])
    assert torch.isfinite(out).all()


def test_cpu_query_raises():
    with pytest.raises(RuntimeError):
        perform_streaming_attention(torch.randn(1, 2, 1, 8), [])


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_allocator_pages_with_mixed_residency(dtype):
    """Pages from a KVAllocator, half evicted to pinned host memory: GPU pages read in place,
    host pages staged into device slots; result equals the all-resident eager attention."""
    torch.manual_seed(1)
    Hq, Hkv, D, P = 32, 8, 128, 64
    alloc = KVAllocator(num_layers=1, num_kv_heads=Hkv, head_dim=D, page_size=P, dtype=dtype)
    mgr = KVCacheManager(alloc, gpu_high_watermark_bytes=10 ** 12)
    k = _r(1, Hkv, 64 * 10 + 17, D, dtype=dtype)
    v = _r(1, Hkv, 64 * 10 + 17, D, dtype=dtype)
    mgr.append_prefill(0, k, v)
    pb = 2 * Hkv * P * D * torch.tensor([], dtype=dtype).element_size()
    mgr.evict_pages(5 * pb)
    pages = mgr.iterate_layer_pages(0)
    states = [p.state for p in pages]
    assert states.count("CPU") == 5 and states[-1] == "GPU"
    assert alloc.store(torch.device("cpu")).pinned
    q = _r(1, Hq, 1, D, dtype=dtype)
    out = perform_streaming_attention(q, pages)
    ref = _eager(q, k.repeat_interleave(4, 1), v.repeat_interleave(4, 1))
    assert_attn_close(out.float(), ref, dtype, "mixed residency")
    # the evicted copies are intact on the host
    assert torch.equal(pages[0].k_tensor[:, :, :64].to(DEV), k[:, :, :64])
