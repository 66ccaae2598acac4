"""GPU tests of the KV slot append kernel (host- and device-directed modes)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _pool(n, Hkv, P, D, dtype, dev):
    return torch.zeros(n, 2, Hkv, P, D, dtype=dtype, device=dev)


@pytest.mark.parametrize("src_dtype,kv_dtype", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.float16),
                                                (torch.float16, torch.float32)])
def test_host_directed_writes_slot_and_table(src_dtype, kv_dtype, cuda):
    from helm_b200 import ops
    B, Hkv, P, D = 3, 2, 8, 16
    pool = _pool(10, Hkv, P, D, kv_dtype, cuda)
    k = torch.randn(B, Hkv, D, dtype=torch.float32).to(src_dtype).to(cuda)
    v = torch.randn(B, Hkv, D, dtype=torch.float32).to(src_dtype).to(cuda)
    dest = torch.tensor([[4, 0, 0], [7, 2, 5], [1, 1, 7]], dtype=torch.int32, device=cuda)
    pt = torch.zeros(B, 4, dtype=torch.int32, device=cuda)
    pu = torch.zeros(B, 4, dtype=torch.int32, device=cuda)
    npg = torch.tensor([0, 3, 1], dtype=torch.int32, device=cuda)
    ops.kv_append(k, v, pool[:, 0], pool[:, 1], page_stride=2 * Hkv * P * D, head_stride=P * D,
                  num_pool_pages=10, page_size=P, dest=dest, page_table=pt, page_used=pu, num_pages=npg)
    for b, (pid, li, slot) in enumerate(dest.tolist()):
        assert torch.equal(pool[pid, 0, :, slot], k[b].to(kv_dtype))
        assert torch.equal(pool[pid, 1, :, slot], v[b].to(kv_dtype))
        assert pt[b, li].item() == pid and pu[b, li].item() == slot + 1
    assert npg.tolist() == [1, 3, 2]


def test_device_directed_appends_across_page_boundary(cuda):
    from helm_b200 import ops
    B, Hkv, P, D = 2, 1, 4, 8
    pool = _pool(8, Hkv, P, D, torch.float32, cuda)
    pt = torch.tensor([[0, -1, -1], [1, -1, -1]], dtype=torch.int32, device=cuda)
    pu = torch.tensor([[3, 0, 0], [4, 0, 0]], dtype=torch.int32, device=cuda)
    npg = torch.tensor([1, 1], dtype=torch.int32, device=cuda)
    spare = torch.tensor([[5, 6], [2, 3]], dtype=torch.int32, device=cuda)
    nxt = torch.zeros(2, dtype=torch.int32, device=cuda)
    flag = torch.zeros(1, dtype=torch.int32, device=cuda)
    toks = []
    for step in range(6):
        k = torch.full((B, Hkv, D), float(step + 1), device=cuda)
        toks.append(k)
        ops.kv_append(k, -k, pool[:, 0], pool[:, 1], page_stride=2 * Hkv * P * D, head_stride=P * D,
                      num_pool_pages=8, page_size=P, page_table=pt, page_used=pu, num_pages=npg,
                      spare_pages=spare, spare_next=nxt, error_flag=flag)
    # seq 0: slot 3 of page 0, then 4 slots of page 5, then 1 slot of page 6
    assert pt[0].tolist() == [0, 5, 6] and pu[0].tolist() == [4, 4, 1] and npg[0].item() == 3
    assert pool[0, 0, 0, 3, 0].item() == 1.0 and pool[5, 0, 0, 3, 0].item() == 5.0
    assert pool[6, 1, 0, 0, 0].item() == -6.0
    # seq 1: page 1 full -> page 2 (4 tokens) -> page 3 (2 tokens)
    assert pt[1].tolist() == [1, 2, 3] and pu[1].tolist() == [4, 4, 2]
    assert flag.item() == 0
    # spare list exhausted for seq 0 after two more pages' worth -> error flag, no write
    for step in range(8):
        k = torch.zeros((B, Hkv, D), device=cuda)
        ops.kv_append(k, k, pool[:, 0], pool[:, 1], page_stride=2 * Hkv * P * D, head_stride=P * D,
                      num_pool_pages=8, page_size=P, page_table=pt, page_used=pu, num_pages=npg,
                      spare_pages=spare, spare_next=nxt, error_flag=flag)
    from helm_b200 import _native as N
    assert flag.item() & N.DEVERR_APPEND_FULL


@pytest.mark.parametrize("src_dtype", [torch.bfloat16, torch.float32])
def test_kv_write_pages_chunks_and_table(src_dtype, cuda):
    """helm_kv_write_pages: a prompt's K/V (strided as the patched forward hands them over) cut
    into 64-token chunks written to scattered pool slots in one launch, the last chunk partial,
    plus the device page-table row; bytewise against torch indexing."""
    from helm_b200 import ops
    Hkv, D, P, S = 4, 128, 64, 64 * 9 + 23
    g = torch.Generator(device=cuda).manual_seed(9)
    kv = torch.randn((1, S, 2 * Hkv, D), generator=g, device=cuda).to(src_dtype)
    K = kv[:, :, :Hkv].transpose(1, 2)            # [1, Hkv, S, D], token stride 2*Hkv*D
    V = kv[:, :, Hkv:].transpose(1, 2)
    pool = torch.zeros((40, 2, Hkv, P, D), dtype=torch.bfloat16, device=cuda)
    slots = torch.randperm(40, generator=torch.Generator().manual_seed(3))[:10].tolist()
    pages = [(sl, 64 * i, min(64, S - 64 * i)) for i, sl in enumerate(slots)]
    pt = torch.full((16,), -1, dtype=torch.int32, device=cuda)
    pu = torch.zeros(16, dtype=torch.int32, device=cuda)
    npg = torch.tensor([2], dtype=torch.int32, device=cuda)
    ops.kv_write_pages(K, V, pool[:, 0], pool[:, 1], pages, page_stride=2 * Hkv * P * D, head_stride=P * D,
                       num_pool_pages=40, page_size=P, table=(pt, pu, npg, 2))
    torch.cuda.synchronize()
    for sl, t0, n in pages:
        assert torch.equal(pool[sl, 0, :, :n], K[0, :, t0:t0 + n].to(torch.bfloat16))
        assert torch.equal(pool[sl, 1, :, :n], V[0, :, t0:t0 + n].to(torch.bfloat16))
    assert pt[2:12].tolist() == slots and pt[:2].tolist() == [-1, -1]
    assert pu[2:12].tolist() == [n for _, _, n in pages]
    assert int(npg.item()) == 12
    untouched = [i for i in range(40) if i not in slots]
    assert torch.count_nonzero(pool[untouched]).item() == 0


def test_append_prefill_uses_one_launch_per_call(cuda):
    """KVCacheManager.append_prefill on a CUDA allocator: every page's data lands in its slot (one
    helm_kv_write_pages launch per flush), for a fresh pool and for one with recycled slots."""
    from helm_b200.runtime import KVAllocator, KVCacheManager
    alloc = KVAllocator(num_layers=2, num_kv_heads=2, head_dim=128, page_size=64, dtype=torch.bfloat16)
    mgr = KVCacheManager(alloc, gpu_high_watermark_bytes=1 << 40)
    g = torch.Generator(device=cuda).manual_seed(1)
    K = torch.randn((1, 2, 64 * 5 + 7, 128), generator=g, device=cuda).to(torch.bfloat16)
    V = torch.randn((1, 2, 64 * 5 + 7, 128), generator=g, device=cuda).to(torch.bfloat16)
    mgr.append_prefill(0, K, V)
    mgr.clear()                                   # pages back to the pools: slots get reused
    mgr.append_prefill(1, K[:, :, :200], V[:, :, :200])
    mgr.append_prefill(1, K[:, :, 200:], V[:, :, 200:])
    torch.cuda.synchronize()
    pages = mgr.iterate_layer_pages(1)
    assert sum(p.used_tokens for p in pages) == K.shape[2]
    for p in pages:
        t0, u = p.start_token, p.used_tokens
        assert torch.equal(p.k_tensor[0, :, :u], K[0, :, t0:t0 + u])
        assert torch.equal(p.v_tensor[0, :, :u], V[0, :, t0:t0 + u])
