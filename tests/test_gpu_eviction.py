"""Batched asynchronous eviction on the GPU (KVAllocator.move_page -> PageStore.defer_move ->
helm_move_pages on the transfer stream).

Pages evicted to pinned host memory must hold exactly the data that was prefilled into them, even
when (a) the host slab grows while copies are queued or in flight, (b) the device slots the copies
read are handed to new pages and overwritten right after the eviction, and (c) the evicted pages
are attended over (staged back) in the same step.  The page bookkeeping is compared with a run of
the same calls on the CPU stand-in device, which copies synchronously (the reference's order,
helm/runtime/kv_allocator.py:104-116)."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
Hkv, D, P = 2, 128, 64


def _fill(mgr, layers, tokens, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    data = {}
    for l in layers:
        K = torch.randn((1, Hkv, tokens, D), generator=g, device=DEV).to(torch.bfloat16)
        V = torch.randn((1, Hkv, tokens, D), generator=g, device=DEV).to(torch.bfloat16)
        mgr.append_prefill(l, K, V)
        data[l] = (K.cpu(), V.cpu())
    return data


def _check_pages(mgr, data):
    n_cpu = 0
    for l, (K, V) in data.items():
        for p in mgr.iterate_layer_pages(l):
            t0, u = p.start_token, p.used_tokens
            assert torch.equal(p.k_tensor[0, :, :u].cpu(), K[0, :, t0:t0 + u]), (l, p)
            assert torch.equal(p.v_tensor[0, :, :u].cpu(), V[0, :, t0:t0 + u]), (l, p)
            n_cpu += p.state == "CPU"
    return n_cpu


def test_evicted_pages_survive_host_growth_and_slot_reuse():
    from helm_b200.runtime import KVAllocator, KVCacheManager
    alloc = KVAllocator(num_layers=4, num_kv_heads=Hkv, head_dim=D, page_size=P, dtype=torch.bfloat16)
    page_bytes = 2 * Hkv * P * D * 2
    # room for 12 evictable pages on the GPU: later pages push the oldest ones out
    mgr = KVCacheManager(alloc, gpu_high_watermark_bytes=12 * page_bytes)
    data = _fill(mgr, [0, 1], 20 * P + 17, seed=1)
    host = alloc.store(torch.device("cpu"))
    assert host.growths >= 1                      # the host slab grew while evictions were queued
    # new pages reuse the evicted pages' device slots and overwrite them immediately
    data.update(_fill(mgr, [2, 3], 9 * P + 5, seed=2))
    torch.cuda.synchronize()
    n_cpu = _check_pages(mgr, data)
    assert n_cpu > 20
    rep = alloc.report_usage()
    assert rep["active_cpu_pages"] == n_cpu


def test_attention_right_after_eviction_reads_the_evicted_data():
    """Evict, then attend over the layer in the same stream order without any host sync: the
    staging copy must wait for the queued eviction copies."""
    from helm_b200.runtime import KVAllocator, KVCacheManager, perform_streaming_attention
    from oracle.attention import eager_attention
    alloc = KVAllocator(num_layers=1, num_kv_heads=Hkv, head_dim=D, page_size=P, dtype=torch.bfloat16)
    page_bytes = 2 * Hkv * P * D * 2
    mgr = KVCacheManager(alloc, gpu_high_watermark_bytes=1 << 40)
    data = _fill(mgr, [0], 24 * P, seed=3)
    mgr.evict_pages(10 * page_bytes)              # queued, not yet issued
    host = alloc.store(torch.device("cpu"))
    assert len(host.pending_moves) == 10
    g = torch.Generator(device=DEV).manual_seed(4)
    q = torch.randn((1, 8, 1, D), generator=g, device=DEV).to(torch.bfloat16)
    out = perform_streaming_attention(q, mgr.iterate_layer_pages(0))
    K, V = data[0]
    ref = eager_attention(q[0, :, 0].cpu().float().numpy(), K[0].float().numpy(), V[0].float().numpy(),
                          1 / math.sqrt(D))
    err = float((out[0, :, 0].float().cpu().double() - torch.from_numpy(ref)).abs().max())
    assert err <= 2e-3 * max(1.0, float(abs(ref).max())) + 2 ** -8 * float(abs(ref).max())
    assert sum(p.state == "CPU" for p in mgr.iterate_layer_pages(0)) == 10


def test_gpu_bookkeeping_equals_the_synchronous_cpu_run():
    """The same calls through the batched GPU path and the synchronous CPU stand-in device give
    identical page ids, states, token ranges and report dicts."""
    from helm_b200.runtime import KVAllocator, KVCacheManager
    from tests.trace_replay import OnFake

    def run(fake, storage_dev):
        alloc = KVAllocator(num_layers=3, num_kv_heads=Hkv, head_dim=D, page_size=P, dtype=torch.bfloat16)
        mgr = KVCacheManager(alloc, gpu_high_watermark_bytes=5 * 2 * Hkv * P * D * 2)
        g = torch.Generator().manual_seed(7)
        for l, n in ((0, 9 * P + 3), (1, 4 * P), (2, 7 * P + 60)):
            K = torch.randn((1, Hkv, n, D), generator=g).to(torch.bfloat16).to(storage_dev)
            V = torch.randn((1, Hkv, n, D), generator=g).to(torch.bfloat16).to(storage_dev)
            if fake:
                K, V = K.as_subclass(OnFake), V.as_subclass(OnFake)
            mgr.append_prefill(l, K, V)
        pages = [(p.page_id, p.layer_id, p.start_token, p.used_tokens, p.state)
                 for l in range(3) for p in mgr.iterate_layer_pages(l)]
        return pages, alloc.report_usage()

    gpu = run(False, DEV)
    cpu = run(True, torch.device("cpu"))
    assert gpu == cpu
