"""CUDA-graph decode (helm_b200.runtime.graph.DecodeGraph) against eager decode through the same
KVOffloadManager patches: identical greedy tokens and matching logits over steps that cross page
boundaries, host bookkeeping (page lists, token counts, device tables) consistent with the device,
and eager decode continuing correctly after close()."""
import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def _tiny(seed=0):
    import transformers
    cfg = transformers.Qwen3Config(vocab_size=320, hidden_size=256, intermediate_size=512, num_hidden_layers=3,
                                   num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                                   max_position_embeddings=4096, rms_norm_eps=1e-6, rope_theta=1e6)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    return transformers.Qwen3ForCausalLM(cfg).to(DEV, torch.bfloat16).eval()


def _prefill(model, ids):
    n = ids.shape[1]
    mask = torch.full((n, n), torch.finfo(torch.bfloat16).min, device=DEV, dtype=torch.bfloat16).triu_(1)
    return model(input_ids=ids, attention_mask=mask[None, None], position_ids=torch.arange(n, device=DEV)[None].expand(
        ids.shape[0], n), use_cache=False, logits_to_keep=1).logits


def _eager_step(model, tok, pos):
    m = torch.zeros((tok.shape[0], 1, 1, pos + 1), device=DEV, dtype=torch.bfloat16)
    p = torch.full((tok.shape[0], 1), pos, device=DEV, dtype=torch.long)
    return model(input_ids=tok, attention_mask=m, position_ids=p, use_cache=False, logits_to_keep=1).logits


@torch.no_grad()
@pytest.mark.parametrize("B,fused_norms", [(1, False), (2, False), (2, True)])
def test_graph_decode_matches_eager(B, fused_norms):
    from helm_b200.runtime import KVOffloadConfig, KVOffloadManager
    from helm_b200.runtime.graph import DecodeGraph
    model = _tiny()
    S, steps = 120, 80          # 120 -> 200 tokens: crosses the 128 and 192 page boundaries
    ids = torch.randint(0, 320, (B, S), device=DEV, generator=torch.Generator(device=DEV).manual_seed(1))
    cfg = KVOffloadConfig.from_model(model, page_size=64, cont_capacity=0, gpu_watermark_bytes=1 << 40)

    # eager reference run
    mgr = KVOffloadManager(model, cfg, batch_size=B)
    tok = _prefill(model, ids)[:, -1:].argmax(-1)
    ref_tokens, ref_logits = [], []
    for t in range(steps):
        lg = _eager_step(model, tok, S + t)
        ref_logits.append(lg.float())
        tok = lg[:, -1:].argmax(-1)
        ref_tokens.append(tok)
    mgr.restore()

    # graph run from the same prefill
    mgr = KVOffloadManager(model, cfg, batch_size=B, fused_norms=fused_norms)
    try:
        tok = _prefill(model, ids)[:, -1:].argmax(-1)
        g = DecodeGraph(mgr, model)
        agree = 0
        for t in range(steps):
            lg = g.step(tok if t == 0 else ref_tokens[t - 1])     # teacher-forced on the eager tokens
            err = float((lg.float() - ref_logits[t]).abs().max())
            assert err <= 0.05 * max(1.0, float(ref_logits[t].abs().max())), f"step {t}: {err}"
            same = torch.equal(lg[:, -1:].argmax(-1), ref_tokens[t])
            agree += same
            if not fused_norms:   # same kernels as the eager run: the same greedy tokens
                assert same, f"step {t}: tokens differ"
        assert agree >= 0.9 * steps
        tok = ref_tokens[-1]
        torch.cuda.synchronize()
        assert int(mgr.batch.error_flag.item()) == 0
        # host bookkeeping = device tables
        for m_i, m in enumerate(mgr.kvcms):
            for l in range(3):
                layer = m.layers[l]
                assert layer.total_tokens == S + steps
                assert sum(p.used_tokens for p in layer.pages) == S + steps
                n = len(layer.pages)
                assert int(mgr.batch.npages[l, m_i]) == n
                assert mgr.batch.table[l, m_i, :n].tolist() == [p.slot for p in layer.pages]
                assert mgr.batch.used[l, m_i, :n].tolist() == [p.used_tokens for p in layer.pages]
        g.close()
        # eager decode continues on the same cache
        lg = _eager_step(model, tok, S + steps)
        assert torch.isfinite(lg.float()).all()
        assert mgr.kvcms[0].layers[0].total_tokens == S + steps + 1
    finally:
        mgr.restore()


@torch.no_grad()
def test_graph_decode_rejects_unsupported():
    from helm_b200.runtime import KVOffloadConfig, KVOffloadManager
    from helm_b200.runtime.graph import DecodeGraph
    model = _tiny()
    mgr = KVOffloadManager(model, KVOffloadConfig.from_model(model, cont_capacity=4096), batch_size=1)
    try:
        with pytest.raises(RuntimeError):
            DecodeGraph(mgr, model)
    finally:
        mgr.restore()


@torch.no_grad()
def test_graph_decode_survives_slab_growth():
    """The device slab is reallocated between two steps (as a growth for other pages would): the
    next step recaptures against the new slab, and the decode stays equal to the eager one."""
    from helm_b200.runtime import KVOffloadConfig, KVOffloadManager
    from helm_b200.runtime.graph import DecodeGraph
    model = _tiny()
    B, S, steps = 2, 60, 30
    ids = torch.randint(0, 320, (B, S), device=DEV, generator=torch.Generator(device=DEV).manual_seed(3))
    cfg = KVOffloadConfig.from_model(model, page_size=64, cont_capacity=0, gpu_watermark_bytes=1 << 40)
    mgr = KVOffloadManager(model, cfg, batch_size=B)
    tok = _prefill(model, ids)[:, -1:].argmax(-1)
    ref = []
    for t in range(steps):
        lg = _eager_step(model, tok, S + t)
        ref.append(lg.float())
        tok = lg[:, -1:].argmax(-1)
    mgr.restore()
    mgr = KVOffloadManager(model, cfg, batch_size=B)
    try:
        tok = _prefill(model, ids)[:, -1:].argmax(-1)
        g = DecodeGraph(mgr, model)
        store = mgr.allocator.store(DEV)
        for t in range(steps):
            if t == 10:
                old = store.slab.data_ptr()
                store.reserve(store.capacity + 4096)
                assert store.slab.data_ptr() != old
            lg = g.step(tok)
            assert torch.isfinite(lg.float()).all(), f"step {t}"
            assert float((lg.float() - ref[t]).abs().max()) <= 0.05 * max(1.0, float(ref[t].abs().max()))
            tok = lg[:, -1:].argmax(-1)
        assert int(mgr.batch.error_flag.item()) == 0
        g.close()
    finally:
        mgr.restore()
