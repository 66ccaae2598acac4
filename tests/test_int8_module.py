"""Int8Linear / patch_int8_linears / quantize_weight (helm_b200.kernels)."""
import pytest
import torch
import torch.nn as nn

from helm_b200 import kernels as K


def test_quantize_weight_bounds_and_error():
    torch.manual_seed(0)
    w = torch.randn(64, 128) * torch.linspace(0.01, 3, 64)[:, None]
    w[5] = 0
    q, s = K.quantize_weight(w, torch.float32)
    assert q.dtype == torch.int8 and q.abs().max() <= 127 and s.shape == (64,)
    deq = q.float() * s[:, None]
    assert torch.all((deq - w).abs() <= s[:, None] / 2 + 1e-6)
    assert torch.all(q[5] == 0) and s[5] == 1.0


def test_patch_on_cpu_model_patches_nothing_and_module_refuses_cpu():
    m = nn.Sequential(nn.Linear(32, 16), nn.ReLU(), nn.Linear(16, 8))
    assert K.patch_int8_linears(m) == 0
    lin = K.Int8Linear.from_linear(nn.Linear(32, 16).to(torch.bfloat16))
    assert lin.weight.dtype == torch.int8 and lin.scale.dtype == torch.bfloat16
    with pytest.raises(RuntimeError):
        lin(torch.randn(1, 32, dtype=torch.bfloat16))


def test_availability_probes():
    assert K.is_available()
    assert K.load_error() is None


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 4, 8, 40, 200])
def test_int8_linear_module_matches_dequantised_linear(M):
    torch.manual_seed(1)
    lin = nn.Linear(1024, 384, bias=True).cuda().to(torch.bfloat16)
    q = K.Int8Linear.from_linear(lin)
    x = torch.randn(M, 1024, device="cuda", dtype=torch.bfloat16)
    ref = x.double() @ (q.weight.double() * q.scale.double()[:, None]).T + q.bias.double()
    y = q(x)
    assert y.shape == (M, 384) and y.dtype == torch.bfloat16
    assert float((y.double() - ref).abs().max()) <= 1e-2 * float(ref.abs().max())


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 8, 64, 200])
def test_fused_glu_and_qkv_modules(M):
    """Int8GLU (one launch with silu(gate) * up in the epilogue, or the dequantised GEMM for prefill
    sizes) and Int8QKV (one launch, three strided views) against float64 on the same int8 weights."""
    torch.manual_seed(2)
    gate = nn.Linear(512, 320, bias=False).cuda().to(torch.bfloat16)
    up = nn.Linear(512, 320, bias=False).cuda().to(torch.bfloat16)
    glu = K.Int8GLU(gate, up)
    x = torch.randn(M, 512, device="cuda", dtype=torch.bfloat16)
    qg, sg = K.quantize_weight(gate.weight)
    qu, su = K.quantize_weight(up.weight)
    g = x.double() @ (qg.double() * sg.double()[:, None]).T
    u = x.double() @ (qu.double() * su.double()[:, None]).T
    ref = torch.nn.functional.silu(g) * u
    y = glu(x)
    assert y.shape == (M, 320) and y.dtype == torch.bfloat16
    assert float((y.double() - ref).abs().max()) <= 2e-2 * float(ref.abs().max())
    q, k, v = (nn.Linear(512, n, bias=True).cuda().to(torch.bfloat16) for n in (256, 64, 64))
    fused = K.Int8QKV(q, k, v)
    outs = fused(x)
    for lin, o, view in zip((q, k, v), outs, fused.views()):
        assert torch.equal(o, view(x)) if M <= 64 else o.shape == view(x).shape
        qw, sw = K.quantize_weight(lin.weight)
        r = x.double() @ (qw.double() * sw.double()[:, None]).T + lin.bias.double()
        assert float((o.double() - r).abs().max()) <= 1e-2 * float(r.abs().max())


@pytest.mark.gpu
def test_patch_tiny_qwen3_and_decode_with_offload():
    """INT8 linears + paged decode attention in one model (the config-4 combination)."""
    import transformers
    from helm_b200.runtime import KVOffloadConfig, KVOffloadManager
    from tests.test_gpu_offload_model import _pipeline_logits, _reference_logits
    cfg = transformers.Qwen3Config(vocab_size=320, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                   num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                                   max_position_embeddings=4096)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    model = transformers.Qwen3ForCausalLM(cfg).cuda().to(torch.bfloat16).eval()
    n = K.patch_int8_linears(model)
    assert n == 2 * 7 + 1  # q, k, v, o, gate, up, down per layer, and the lm_head
    assert isinstance(model.model.layers[0].self_attn.q_proj, K.Int8Linear)
    assert isinstance(model.model.layers[0].self_attn._helm_qkv, K.Int8QKV)
    assert isinstance(model.model.layers[0].mlp._helm_glu, K.Int8GLU)
    assert isinstance(model.lm_head, K.Int8Linear)
    torch.manual_seed(4)
    ids = torch.randint(0, 320, (2, 140), device="cuda")
    ref = _reference_logits(model, ids)[:, 99:]     # int8 model, torch attention
    mgr = KVOffloadManager(model, KVOffloadConfig.from_model(model, cont_capacity=0), batch_size=2)
    try:
        ours = _pipeline_logits(model, ids, 100)
    finally:
        mgr.restore()
    err = float((ours.float() - ref.float()).abs().max())
    assert err <= 0.06 * max(1.0, float(ref.float().abs().max()))
