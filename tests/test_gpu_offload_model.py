"""End-to-end drop-in test: tiny random-init HF decoders (Qwen3, Qwen2, Llama) driven like HELM's
PipelineRuntime (explicit causal / decode masks, one token per step) with KVOffloadManager's
patched attention, against the unpatched model's logits on the full sequence.

Covers the three decode paths (contiguous buffers, all-GPU pages, mixed residency with
eviction to pinned host memory), batch > 1, page-boundary crossings and reset().  The bar is set by
bf16's own noise: the patched model's logits against an fp32 run of the same model may differ by
at most 1.25 x what the unpatched bf16 model's logits do (plus 0.2 % of the logit scale)."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _tiny(arch, dtype=torch.bfloat16):
    import transformers
    kw = dict(vocab_size=320, hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=8,
              num_key_value_heads=2, max_position_embeddings=4096, rms_norm_eps=1e-6)
    if arch == "qwen3":
        cfg = transformers.Qwen3Config(head_dim=128, rope_theta=1e6, **kw)
        cls = transformers.Qwen3ForCausalLM
    elif arch == "qwen2":
        cfg = transformers.Qwen2Config(**kw)
        cls = transformers.Qwen2ForCausalLM
    else:
        cfg = transformers.LlamaConfig(head_dim=128, **kw)
        cls = transformers.LlamaForCausalLM
    torch.manual_seed(0)
    cfg._attn_implementation = "sdpa"
    model = cls(cfg).to(DEV, dtype).eval()
    return model


def _causal(n, dtype):
    m = torch.full((n, n), torch.finfo(dtype).min, device=DEV, dtype=dtype)
    return torch.triu(m, diagonal=1)[None, None]


@torch.no_grad()
def _reference_logits(model, ids):
    """Unpatched model on the full sequence: logits at every position."""
    n = ids.shape[1]
    pos = torch.arange(n, device=DEV)[None]
    return model(input_ids=ids, attention_mask=_causal(n, model.dtype), position_ids=pos, use_cache=False).logits


@torch.no_grad()
def _pipeline_logits(model, ids, prompt_len):
    """Prefill prompt_len tokens, then decode the rest one token at a time (teacher forced)."""
    dtype = model.dtype
    pos = torch.arange(prompt_len, device=DEV)[None]
    out = [model(input_ids=ids[:, :prompt_len], attention_mask=_causal(prompt_len, dtype), position_ids=pos,
                 use_cache=False).logits[:, -1]]
    for t in range(prompt_len, ids.shape[1]):
        mask = torch.zeros((1, 1, 1, t + 1), device=DEV, dtype=dtype)
        lg = model(input_ids=ids[:, t:t + 1], attention_mask=mask, position_ids=torch.tensor([[t]], device=DEV),
                   use_cache=False).logits
        out.append(lg[:, -1])
    return torch.stack(out, dim=1)  # logits predicting tokens prompt_len .. n


def _check(ours, ref, what, ref32=None):
    """ours vs the unpatched bf16 model (ref).  With ref32 (the same model run in fp32) the bar is
    relative to bf16's own noise: our error against fp32 may exceed the unpatched bf16 model's error
    against fp32 by at most 25 % plus 0.2 % of the logit scale."""
    err = float((ours.float() - ref.float()).abs().max())
    scale = max(1.0, float(ref.float().abs().max()))
    assert err <= 0.03 * scale, f"{what}: max logit error {err:.4f} (scale {scale:.2f})"
    agree = (ours.argmax(-1) == ref.argmax(-1)).float().mean().item()
    assert agree >= 0.95, f"{what}: argmax agreement {agree:.2f}"
    if ref32 is not None:
        noise = float((ref.float() - ref32).abs().max())
        ours32 = float((ours.float() - ref32).abs().max())
        assert ours32 <= 1.25 * noise + 2e-3 * scale, \
            f"{what}: error vs fp32 {ours32:.4f} > 1.25 x the bf16 model's own {noise:.4f} + 0.2% of {scale:.2f}"


def _fp32_logits(model, ids):
    import copy
    m32 = copy.deepcopy(model).float()
    out = _reference_logits(m32, ids).float()
    del m32
    return out


@pytest.mark.parametrize("mode", ["paged", "contiguous", "offload", "paged_fused_norms"])
def test_qwen3_decode_paths_match_unpatched(mode):
    from helm_b200.runtime import KVOffloadConfig, KVOffloadManager
    model = _tiny("qwen3")
    B, S, steps = 2, 100, 70
    torch.manual_seed(1)
    ids = torch.randint(0, 320, (B, S + steps), device=DEV)
    ref = _reference_logits(model, ids)[:, S - 1:]
    ref32 = _fp32_logits(model, ids)[:, S - 1:]
    cfg = KVOffloadConfig.from_model(model, page_size=64, cont_capacity=4096 if mode == "contiguous" else 0,
                                     gpu_watermark_bytes=(2 * 2 * 64 * 128 * 2 * 2) if mode == "offload" else 10 ** 12)
    mgr = KVOffloadManager(model, cfg, batch_size=B, fused_norms=mode == "paged_fused_norms")
    try:
        ours = _pipeline_logits(model, ids, S)
        _check(ours, ref, mode, ref32)
        rep = mgr.report()
        if mode == "offload":
            assert rep["active_cpu_pages"] > 0
            assert any(p.state == "CPU" for p in mgr.kvcms[0].layers[0].pages)
        if mode == "contiguous":
            assert mgr.kvcms[0].use_contiguous and mgr.kvcms[0].cont_seq_len == S + steps
        else:
            assert mgr.kvcms[1].layers[1].total_tokens == S + steps
        assert int(mgr.batch.error_flag.item()) == 0
        # reset and run again: identical results
        mgr.reset()
        again = _pipeline_logits(model, ids, S)
        assert torch.equal(again, ours)
    finally:
        mgr.restore()


@pytest.mark.parametrize("arch", ["qwen2", "llama"])
def test_other_architectures(arch):
    from helm_b200.runtime import KVOffloadConfig, KVOffloadManager
    model = _tiny(arch)
    torch.manual_seed(2)
    ids = torch.randint(0, 320, (1, 150), device=DEV)
    ref = _reference_logits(model, ids)[:, 99:]
    ref32 = _fp32_logits(model, ids)[:, 99:]
    mgr = KVOffloadManager(model, KVOffloadConfig.from_model(model, cont_capacity=0), batch_size=1)
    try:
        _check(_pipeline_logits(model, ids, 100), ref, arch, ref32)
    finally:
        mgr.restore()


def test_unbatched_managers_use_per_item_path():
    """_decode_batched with managers that are not a registered batch (no device tables)."""
    import math
    from helm_b200.runtime import KVAllocator, KVCacheManager
    from helm_b200.runtime.kv_offload import _decode_batched
    torch.manual_seed(3)
    Hq, Hkv, D = 16, 4, 128
    alloc = KVAllocator(num_layers=1, num_kv_heads=Hkv, head_dim=D, page_size=64, dtype=torch.bfloat16)
    kvcms = [KVCacheManager(alloc, gpu_high_watermark_bytes=10 ** 12) for _ in range(2)]
    hist = []
    for m in kvcms:
        k = torch.randn(1, Hkv, 90, D, device=DEV, dtype=torch.bfloat16)
        v = torch.randn(1, Hkv, 90, D, device=DEV, dtype=torch.bfloat16)
        m.append_prefill(0, k, v)
        hist.append((k, v))
    q = torch.randn(2, Hq, 1, D, device=DEV, dtype=torch.bfloat16)
    k1 = torch.randn(2, Hkv, 1, D, device=DEV, dtype=torch.bfloat16)
    v1 = torch.randn(2, Hkv, 1, D, device=DEV, dtype=torch.bfloat16)
    out = _decode_batched(kvcms, q, k1, v1, 0, 1.0 / math.sqrt(D))
    for b in range(2):
        K = torch.cat([hist[b][0], k1[b:b + 1]], 2).repeat_interleave(4, 1).double()
        V = torch.cat([hist[b][1], v1[b:b + 1]], 2).repeat_interleave(4, 1).double()
        ref = torch.softmax(q[b:b + 1].double() @ K.transpose(-1, -2) / math.sqrt(D), -1) @ V
        assert float((out[b:b + 1].double() - ref).abs().max()) < 2e-2
