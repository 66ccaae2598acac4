"""Pins the float64 formulas the decode-prologue GPU tests compare against (per-head RMSNorm, then
x*cos + rotate_half(x)*sin) to the installed transformers functions the patched forward replaces
(Qwen3RMSNorm, apply_rotary_pos_emb, the Qwen3 rotary tables).  CPU only."""
import torch

from tests.test_gpu_prologue import _ref, _rope_tables


def test_rope_and_norm_formula_match_transformers(monkeypatch):
    import transformers.models.qwen3.modeling_qwen3 as m
    import tests.test_gpu_prologue as tp
    monkeypatch.setattr(tp, "DEV", torch.device("cpu"))
    torch.manual_seed(0)
    B, H, D = 3, 4, 128
    x = torch.randn(B, H, D, dtype=torch.float64)
    w = 1 + 0.1 * torch.randn(D, dtype=torch.float64)
    pos = [5, 700, 16000]
    cos, sin = _rope_tables(B, D, pos, dtype=torch.float64)
    # transformers: RMSNorm module then apply_rotary_pos_emb on [B, H, 1, D] with cos/sin [B, 1, D]
    norm = m.Qwen3RMSNorm(D, eps=1e-6).double()
    with torch.no_grad():
        norm.weight.copy_(w)
    xn = norm(x)
    q_hf, _ = m.apply_rotary_pos_emb(xn[:, :, None], xn[:, :, None], cos[:, None], sin[:, None])
    ours = _ref(x, w, 1e-6, cos, sin)
    # the HF module computes its statistics in fp32 even for float64 inputs: agreement to fp32
    assert torch.allclose(ours, q_hf[:, :, 0].detach(), rtol=1e-5, atol=1e-5)
    # and the tables equal the model's own rotary embedding at those positions (it forms the angles
    # position * inv_freq in fp32: about 1e-7 relative, 2e-3 absolute at position 16000)
    cfg = m.Qwen3Config(hidden_size=256, num_attention_heads=2, num_key_value_heads=1, head_dim=D, rope_theta=1e6,
                        max_position_embeddings=40960)
    rot = m.Qwen3RotaryEmbedding(cfg)
    c_hf, s_hf = rot(x, torch.tensor([pos]).T)
    assert torch.allclose(cos, c_hf[:, 0].double(), atol=3e-3)
    assert torch.allclose(sin, s_hf[:, 0].double(), atol=3e-3)
