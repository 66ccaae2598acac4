"""KVAllocator: the reference suite's assertions (tests/unit/runtime/test_kv_allocator.py in HELM)
run against helm_b200.runtime.KVAllocator, plus slab-specific checks."""
import pytest
import torch

from helm_b200.runtime import KVAllocator

CPU = torch.device("cpu")


def _alloc(**kw):
    d = dict(num_layers=2, num_kv_heads=2, head_dim=8, page_size=4, dtype=torch.float32)
    d.update(kw)
    return KVAllocator(**d)


def test_allocate_cpu_state():
    page = _alloc().allocate(CPU)
    assert page.state == "CPU" and page.device.type == "cpu"


def test_allocate_resets_metadata():
    a = _alloc()
    page = a.allocate(CPU)
    page.layer_id, page.start_token, page.used_tokens = 99, 500, 3
    a.free(page)
    p2 = a.allocate(CPU)
    assert (p2.layer_id, p2.start_token, p2.used_tokens) == (-1, 0, 0)


def test_allocate_triggers_batch_reserve():
    a = _alloc()
    assert a.cpu_total_pages == 0
    a.allocate(CPU)
    assert a.cpu_total_pages == 16


def test_page_shape_and_dtype():
    a = KVAllocator(num_layers=2, num_kv_heads=3, head_dim=16, page_size=8)
    page = a.allocate(CPU)
    assert page.k_tensor.shape == (1, 3, 8, 16) and page.v_tensor.shape == (1, 3, 8, 16)
    assert _alloc(dtype=torch.float16).allocate(CPU).k_tensor.dtype == torch.float16


def test_page_ids_are_unique_and_sequential():
    a = _alloc()
    ids = [a.allocate(CPU).page_id for _ in range(20)]
    assert len(set(ids)) == 20
    # batch of 16 created in order, popped LIFO
    assert ids[:16] == list(range(15, -1, -1))


def test_free_returns_to_pool_and_lifo_reuse():
    a = _alloc()
    p1 = a.allocate(CPU)
    before = len(a.cpu_free_pool)
    a.free(p1)
    assert p1.state == "FREE" and len(a.cpu_free_pool) == before + 1
    assert a.allocate(CPU) is p1


def test_reserve_batch_accumulates():
    a = _alloc()
    a.reserve_batch(3, CPU)
    a.reserve_batch(4, CPU)
    assert a.cpu_total_pages == 7 and len(a.cpu_free_pool) == 7


def test_move_page_same_device_returns_same_and_keeps_data():
    a = _alloc()
    page = a.allocate(CPU)
    page.used_tokens = 2
    page.k_tensor[:, :, :2, :] = 42.0
    page.v_tensor[:, :, :2, :] = 99.0
    result = a.move_page(page, CPU)
    assert result is page
    assert torch.all(result.k_tensor[:, :, :2, :] == 42.0) and torch.all(result.v_tensor[:, :, :2, :] == 99.0)


def test_report_usage_keys_and_consistency():
    a = _alloc()
    a.allocate(CPU)
    r = a.report_usage()
    for key in ("gpu_pool_size", "cpu_pool_size", "active_gpu_pages", "active_cpu_pages", "gpu_free_pages",
                "cpu_free_pages", "gpu_reserved_bytes", "cpu_reserved_bytes", "gpu_used_bytes", "cpu_used_bytes"):
        assert key in r
    assert r["active_cpu_pages"] == 1
    assert r["cpu_used_bytes"] <= r["cpu_reserved_bytes"]
    assert r["cpu_reserved_bytes"] == 16 * 2 * 2 * 4 * 8 * 4


def test_pages_are_views_of_one_slab():
    """All CPU pages of the allocator share one slab; slots are distinct and consecutive
    allocations read ascending slots."""
    a = _alloc()
    pages = [a.allocate(CPU) for _ in range(5)]
    st = a.store(CPU)
    assert [p.slot for p in pages] == [0, 1, 2, 3, 4]
    pages[3].k_tensor.fill_(7.0)
    assert torch.all(st.slab[3, 0] == 7.0)
    assert pages[3].k_tensor.data_ptr() == st.slab[3, 0].data_ptr()


def test_slab_growth_keeps_page_data():
    a = _alloc()
    pages = [a.allocate(CPU) for _ in range(16)]
    for i, p in enumerate(pages):
        p.k_tensor.fill_(float(i))
    more = [a.allocate(CPU) for _ in range(40)]  # forces growth
    assert a.store(CPU).capacity >= 56
    for i, p in enumerate(pages):
        assert torch.all(p.k_tensor == float(i))
    assert len({p.slot for p in pages + more}) == 56


# ---- CUDA (the reference's skipped-on-CPU tests) -------------------------------------------

@pytest.mark.gpu
def test_allocate_gpu_state():
    page = _alloc().allocate(torch.device("cuda:0"))
    assert page.state == "GPU" and page.device.type == "cuda"
    assert page.k_tensor.is_cuda


@pytest.mark.gpu
def test_move_page_cpu_to_gpu_copies_data_and_frees_old():
    a = _alloc()
    page = a.allocate(CPU)
    page.layer_id, page.start_token, page.used_tokens = 2, 8, 3
    page.k_tensor[:, :, :3, :] = 7.0
    page.v_tensor[:, :, :3, :] = 8.0
    free_before = len(a.cpu_free_pool)
    new = a.move_page(page, torch.device("cuda:0"))
    assert new.device.type == "cuda" and (new.layer_id, new.start_token, new.used_tokens) == (2, 8, 3)
    assert torch.allclose(new.k_tensor[:, :, :3, :].cpu(), torch.full((1, 2, 3, 8), 7.0))
    assert torch.allclose(new.v_tensor[:, :, :3, :].cpu(), torch.full((1, 2, 3, 8), 8.0))
    assert len(a.cpu_free_pool) == free_before + 1


@pytest.mark.gpu
def test_move_page_gpu_to_cpu_leaves_dead_page_and_async_copy_is_visible():
    a = _alloc()
    g = a.allocate(torch.device("cuda:0"))
    g.used_tokens = 4
    g.k_tensor.fill_(3.0)
    g.v_tensor.fill_(5.0)
    total = a.gpu_total_pages
    new = a.move_page(g, CPU)
    assert g.state == "DEAD" and g.k_tensor.numel() == 0 and a.gpu_total_pages == total - 1
    assert torch.all(new.k_tensor[:, :, :4] == 3.0) and torch.all(new.v_tensor[:, :, :4] == 5.0)


@pytest.mark.gpu
def test_move_page_empty_tokens_no_copy():
    a = _alloc()
    page = a.allocate(CPU)
    new = a.move_page(page, torch.device("cuda:0"))
    assert new.device.type == "cuda" and new.used_tokens == 0
