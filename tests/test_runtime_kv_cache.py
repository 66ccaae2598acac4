"""KVCacheManager / LayerKVCache: the reference suite's assertions (tests/unit/runtime/test_kv_cache.py
and test_batch_kv_offload.py in HELM) against helm_b200.runtime, plus residency counters."""
import pytest
import torch

from helm_b200.runtime import KVAllocator, KVCacheManager, LayerKVCache
from tests.trace_replay import FAKE, OnFake

NUM_HEADS, HEAD_DIM, PAGE_SIZE, NUM_LAYERS = 2, 8, 4, 4


@pytest.fixture()
def allocator():
    return KVAllocator(num_layers=NUM_LAYERS, num_kv_heads=NUM_HEADS, head_dim=HEAD_DIM, page_size=PAGE_SIZE,
                       dtype=torch.float32)


@pytest.fixture()
def cache(allocator):
    mgr = KVCacheManager(allocator, gpu_high_watermark_bytes=0)
    mgr.initialize_layer_caches(num_layers=NUM_LAYERS)
    return mgr


def _kv(n):
    return torch.randn(1, NUM_HEADS, n, HEAD_DIM), torch.randn(1, NUM_HEADS, n, HEAD_DIM)


def test_layer_cache_append_and_tail(allocator):
    layer = LayerKVCache(layer_id=0)
    p1, p2 = allocator.allocate(torch.device("cpu")), allocator.allocate(torch.device("cpu"))
    layer.append_page(p1)
    assert layer.tail_page is p1 and len(layer.pages) == 1
    layer.append_page(p2)
    assert layer.tail_page is p2


def test_initialize_and_seq_len(cache):
    assert cache.num_layers() == NUM_LAYERS and cache.layers_keys() == list(range(NUM_LAYERS))
    assert cache.seq_len() == 0


@pytest.mark.parametrize("n,pages", [(3, 1), (9, 3), (PAGE_SIZE, 1), (8, 2)])
def test_prefill_page_counts(cache, n, pages):
    k, v = _kv(n)
    cache.append_prefill(0, k, v)
    assert len(cache.layers[0].pages) == pages and cache.layers[0].total_tokens == n


def test_prefill_data_and_start_tokens(cache):
    k, v = _kv(8)
    cache.append_prefill(0, k, v)
    p0, p1 = cache.layers[0].pages
    assert torch.equal(p0.k_tensor[:, :, :4], k[:, :, :4]) and torch.equal(p1.v_tensor[:, :, :4], v[:, :, 4:])
    assert (p0.start_token, p1.start_token) == (0, 4)


def test_prefill_auto_creates_layer(cache):
    del cache.layers[3]
    cache.append_prefill(3, *_kv(2))
    assert 3 in cache.layers


def test_decode_appends(cache):
    cache.append_prefill(0, *_kv(2))
    cache.append_decode(0, *_kv(1))
    assert len(cache.layers[0].pages) == 1 and cache.layers[0].tail_page.used_tokens == 3
    c2 = KVCacheManager(cache.allocator, 0)
    c2.append_prefill(0, *_kv(PAGE_SIZE))
    c2.append_decode(0, *_kv(1))
    assert len(c2.layers[0].pages) == 2 and c2.layers[0].tail_page.used_tokens == 1
    c3 = KVCacheManager(cache.allocator, 0)
    for _ in range(PAGE_SIZE + 2):
        c3.append_decode(0, *_kv(1))
    assert len(c3.layers[0].pages) == 2 and c3.layers[0].total_tokens == PAGE_SIZE + 2 and c3.seq_len() == 6


def test_iterate_layer_pages(cache):
    cache.append_prefill(0, *_kv(3))
    pages = cache.iterate_layer_pages(0)
    assert isinstance(pages, list) and len(pages) == 1
    assert cache.iterate_layer_pages(99) == []
    pages.clear()
    assert len(cache.layers[0].pages) == 1


def test_report_bytes(cache):
    cache.append_prefill(0, *_kv(3))
    r = cache.report_bytes_per_tier()
    assert r["gpu_active_bytes"] == 0 and r["cpu_active_bytes"] == 2 * NUM_HEADS * PAGE_SIZE * HEAD_DIM * 4


def test_clear_returns_pages(cache):
    free_before = len(cache.allocator.cpu_free_pool)
    cache.append_prefill(0, *_kv(PAGE_SIZE))
    cache.clear()
    assert cache.num_layers() == 0 and cache.seq_len() == 0
    assert len(cache.allocator.cpu_free_pool) >= free_before


def test_evict_without_gpu_pages_is_noop(cache):
    cache.append_prefill(0, *_kv(8))
    cache.evict_pages(99999)
    assert all(p.state == "CPU" for p in cache.layers[0].pages)


def test_eviction_with_standin_device_and_tail_protection(allocator):
    """Zero watermark with 'GPU' pages (stand-in device): every full non-tail page leaves."""
    mgr = KVCacheManager(allocator, gpu_high_watermark_bytes=0)
    k, v = _kv(13)
    mgr.append_prefill(0, k.as_subclass(OnFake), v.as_subclass(OnFake))
    states = [p.state for p in mgr.layers[0].pages]
    assert states == ["CPU", "CPU", "CPU", "GPU"]
    assert mgr.layers[0].tail_page.state == "GPU"
    # the evicted data is intact on the host
    assert torch.equal(mgr.layers[0].pages[1].k_tensor[:, :, :4], k[:, :, 4:8])
    assert not mgr.all_gpu_resident(0)


def test_all_gpu_resident_counter_matches_scan(allocator):
    mgr = KVCacheManager(allocator, gpu_high_watermark_bytes=10 ** 9)
    k, v = _kv(9)
    mgr.append_prefill(1, k.as_subclass(OnFake), v.as_subclass(OnFake))
    assert mgr.all_gpu_resident(1) and mgr.all_gpu_resident(5)
    mgr.evict_pages(1)
    scan = all(not (p.used_tokens > 0 and p.state != "GPU") for p in mgr.layers[1].pages)
    assert mgr.all_gpu_resident(1) == scan is False


def test_batch_managers_are_independent(allocator):
    kvcms = [KVCacheManager(allocator, 0) for _ in range(3)]
    kvcms[0].append_prefill(0, *_kv(4))
    assert 0 in kvcms[0].layers and 0 not in kvcms[1].layers and 0 not in kvcms[2].layers
    kvcms[1].append_prefill(0, *_kv(8))
    kvcms[2].append_prefill(0, *_kv(4))
    kvcms[1].append_decode(0, *_kv(1))
    assert [m.layers[0].total_tokens for m in kvcms] == [4, 9, 4]
    used = allocator.report_usage()["active_cpu_pages"]
    assert used > 0
    for m in kvcms:
        m.clear()
    assert allocator.report_usage()["active_cpu_pages"] == 0 and all(len(m.layers) == 0 for m in kvcms)


def test_contiguous_api_on_cpu(allocator):
    """build/prefill/write/get/advance/migrate of the contiguous buffers (kv_cache.py:206-289)."""
    m = KVCacheManager(allocator, 10 ** 9)
    assert m.build_contiguous(2, NUM_HEADS, HEAD_DIM, capacity=2048, device=torch.device("cpu"),
                              dtype=torch.float32)
    k, v = _kv(5)
    for lid in range(2):
        m.append_prefill(lid, k, v)
        m.prefill_contiguous(lid, k, v)
    assert m.cont_seq_len == 5 and m.cont_prefill_len == 5
    for step in range(3):
        for lid in range(2):
            kk, vv = _kv(1)
            m.write_decode_contiguous(lid, kk, vv)
            K, V = m.get_kv_contiguous(lid)
            assert K.shape[2] == 5 + step + 1 and torch.equal(K[:, :, -1:], kk)
        m.advance_contiguous()
    m.migrate_contiguous_to_pages()
    assert not m.use_contiguous and m.layers[0].total_tokens == 8 and m.layers[1].total_tokens == 8
    m.reset_contiguous()
    assert not m.use_contiguous
