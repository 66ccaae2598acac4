"""The fused decode prologue (helm_decode_prologue) and RMSNorm (helm_rmsnorm) against the HF
functions they replace: Qwen3RMSNorm for q_norm / k_norm / layer norms and apply_rotary_pos_emb,
computed in float64 from the same inputs; the pool rows written by the prologue's append equal
those of a helm_kv_append of the reference k / v."""
import math

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _rope_tables(B, D, pos, theta=1e6, dtype=torch.bfloat16):
    inv = 1.0 / theta ** (torch.arange(0, D, 2, dtype=torch.float64) / D)
    f = torch.tensor(pos, dtype=torch.float64)[:, None] * inv[None]
    emb = torch.cat([f, f], -1)
    return emb.cos().to(dtype).to(DEV), emb.sin().to(dtype).to(DEV)     # [B, D]


def _ref(x, w, eps, cos, sin):
    """float64: per-head RMSNorm (w None: none), then x*cos + rotate_half(x)*sin."""
    x = x.double()
    if w is not None:
        x = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w.double()
    D = x.shape[-1]
    rot = torch.cat([-x[..., D // 2:], x[..., :D // 2]], -1)
    return x * cos.double()[:, None] + rot * sin.double()[:, None]


@pytest.mark.parametrize("norm", [True, False])
@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
def test_prologue_host_directed(norm, dtype):
    from helm_b200 import ops
    torch.manual_seed(0)
    B, Hq, Hkv, D, P, pages = 3, 16, 4, 128, 64, 10
    q = torch.randn(B, Hq, D, device=DEV).to(dtype)
    k = torch.randn(B, Hkv, D, device=DEV).to(dtype)
    v = torch.randn(B, Hkv, D, device=DEV).to(dtype)
    wq = (1 + 0.1 * torch.randn(D, device=DEV)).to(dtype) if norm else None
    wk = (1 + 0.1 * torch.randn(D, device=DEV)).to(dtype) if norm else None
    cos, sin = _rope_tables(B, D, [5, 700, 16000], dtype=dtype)
    pool = torch.zeros(pages, 2, Hkv, P, D, device=DEV, dtype=dtype)
    dest = np.array([[2, 0, 5], [7, 1, 63], [0, 2, 0]], dtype=np.int32)
    q_out = torch.empty_like(q)
    ops.decode_prologue(q, k, v, q_out, pool[:, 0], pool[:, 1], q_norm_w=wq, k_norm_w=wk, eps=1e-6, cos=cos,
                        sin=sin, page_stride=2 * Hkv * P * D, head_stride=P * D, num_pool_pages=pages, page_size=P,
                        dest_host=dest)
    torch.cuda.synchronize()
    tol = 2e-2 if dtype == torch.bfloat16 else 4e-3
    q_ref = _ref(q, wq, 1e-6, cos, sin)
    assert float((q_out.double() - q_ref).abs().max()) <= tol * max(1.0, float(q_ref.abs().max()))
    k_ref = _ref(k, wk, 1e-6, cos, sin)
    for b in range(B):
        pid, _, slot = dest[b]
        got_k = pool[pid, 0, :, slot].double()
        assert float((got_k - k_ref[b]).abs().max()) <= tol * max(1.0, float(k_ref.abs().max()))
        assert torch.equal(pool[pid, 1, :, slot], v[b])


def test_prologue_device_directed_and_q_only():
    from helm_b200 import ops
    torch.manual_seed(1)
    B, Hq, Hkv, D, P, pages = 2, 8, 2, 128, 64, 8
    dt = torch.bfloat16
    q = torch.randn(B, Hq, D, device=DEV).to(dt)
    k = torch.randn(B, Hkv, D, device=DEV).to(dt)
    v = torch.randn(B, Hkv, D, device=DEV).to(dt)
    cos, sin = _rope_tables(B, D, [64, 3], dtype=dt)
    pool = torch.zeros(pages, 2, Hkv, P, D, device=DEV, dtype=dt)
    table = torch.tensor([[1, 0, 0], [3, 4, 0]], dtype=torch.int32, device=DEV)
    used = torch.tensor([[64, 0, 0], [64, 3, 0]], dtype=torch.int32, device=DEV)
    npg = torch.tensor([1, 2], dtype=torch.int32, device=DEV)
    spare = torch.tensor([[6, 7], [5, 2]], dtype=torch.int32, device=DEV)
    nxt = torch.zeros(2, dtype=torch.int32, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    q_out = torch.empty_like(q)
    kw = dict(page_stride=2 * Hkv * P * D, head_stride=P * D, num_pool_pages=pages, page_size=P, page_table=table,
              page_used=used, num_pages=npg, spare_pages=spare, spare_next=nxt, error_flag=err)
    ops.decode_prologue(q, k, v, q_out, pool[:, 0], pool[:, 1], cos=cos, sin=sin, **kw)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    # sequence 0: tail full -> spare page 6, slot 0; sequence 1: page 4 slot 3
    assert npg.tolist() == [2, 2] and table[0, 1].item() == 6 and used[0, 1].item() == 1 and used[1, 1].item() == 4
    k_ref = _ref(k, None, 0.0, cos, sin)
    assert float((pool[6, 0, :, 0].double() - k_ref[0]).abs().max()) <= 2e-2 * float(k_ref.abs().max())
    assert torch.equal(pool[4, 1, :, 3], v[1])
    # q only (a rank without the tail page): nothing appended, q identical
    snap = pool.clone()
    q2 = torch.empty_like(q)
    ops.decode_prologue(q, k, v, q2, pool[:, 0], pool[:, 1], cos=cos, sin=sin, do_append=False, **kw)
    torch.cuda.synchronize()
    assert torch.equal(q2, q_out) and torch.equal(pool, snap) and npg.tolist() == [2, 2]


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("rows,dim", [(1, 4096), (3, 5120), (257, 128), (5, 17)])
def test_rmsnorm_matches_hf(rows, dim, dtype):
    import transformers.models.qwen3.modeling_qwen3 as m
    from helm_b200 import ops
    torch.manual_seed(rows + dim)
    norm = m.Qwen3RMSNorm(dim, eps=1e-6).to(DEV, dtype)
    with torch.no_grad():
        norm.weight.copy_(1 + 0.1 * torch.randn(dim))
    x = (3 * torch.randn(rows, dim, device=DEV)).to(dtype)
    ref = norm(x)
    got = ops.rmsnorm(x, norm.weight, norm.variance_epsilon)
    ulp = 2.0 ** -7 if dtype == torch.bfloat16 else 2.0 ** -10
    diff = (got.float() - ref.float()).abs()
    assert float((diff / ref.float().abs().clamp_min(1e-3)).max()) <= 2.5 * ulp
