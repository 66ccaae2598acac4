"""Sharded decode through the drop-in runtime on 2 GPUs: a tiny random-init Qwen3 model driven by
KVOffloadManager(shard_group=KVShardGroup(...)) -- each rank stores its share of every prompt's
pages, only the last rank appends the new tokens, the fused decode prologue runs on every rank
(q only where no tail page lives) and the per-rank attention records are exchanged -- against the
unpatched model's logits on the full sequence; every rank returns identical logits.  Spawns its
own two ranks; skipped with fewer than 2 GPUs."""
import datetime
import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, exchange, result_q):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        import transformers
        from helm_b200.runtime import KVOffloadConfig, KVOffloadManager
        from helm_b200.runtime.sharded import KVShardGroup
        cfg = transformers.Qwen3Config(vocab_size=320, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                                       num_attention_heads=8, num_key_value_heads=2, head_dim=128,
                                       max_position_embeddings=4096, rms_norm_eps=1e-6, rope_theta=1e6)
        cfg._attn_implementation = "sdpa"
        torch.manual_seed(0)
        model = transformers.Qwen3ForCausalLM(cfg).to(dev, torch.bfloat16).eval()
        B, S, steps = 2, 150, 40
        ids = torch.randint(0, 320, (B, S + steps), generator=torch.Generator().manual_seed(1)).to(dev)
        dt = torch.bfloat16

        def causal(n):
            return torch.full((n, n), torch.finfo(dt).min, device=dev, dtype=dt).triu_(1)[None, None]

        with torch.no_grad():
            n = S + steps
            ref = model(input_ids=ids, attention_mask=causal(n), position_ids=torch.arange(n, device=dev)[None],
                        use_cache=False).logits[:, S - 1:].float()
            group = KVShardGroup(B * cfg.num_attention_heads, cfg.head_dim, dev, exchange=exchange)
            mgr = KVOffloadManager(model, KVOffloadConfig.from_model(model, page_size=64, cont_capacity=0,
                                                                     gpu_watermark_bytes=1 << 40),
                                   batch_size=B, shard_group=group)
            out = [model(input_ids=ids[:, :S], attention_mask=causal(S), position_ids=torch.arange(S, device=dev)[None],
                         use_cache=False).logits[:, -1]]
            for t in range(S, n):
                m = torch.zeros((B, 1, 1, t + 1), device=dev, dtype=dt)
                out.append(model(input_ids=ids[:, t:t + 1], attention_mask=m,
                                 position_ids=torch.full((B, 1), t, device=dev), use_cache=False).logits[:, -1])
            ours = torch.stack(out[:-1], 1).float()
            torch.cuda.synchronize()
            err = float((ours - ref[:, :-1]).abs().max())
            scale = max(1.0, float(ref.abs().max()))
            agree = float((ours.argmax(-1) == ref[:, :-1].argmax(-1)).float().mean())
            gathered = [torch.empty_like(ours) for _ in range(world)]
            dist.all_gather(gathered, ours.contiguous())
            same = all(torch.equal(g, gathered[0]) for g in gathered)
            tokens = [mgr.kvcms[b].layers[0].total_tokens for b in range(B)]
            flag = int(mgr.batch.error_flag.item()) | int(group.error_flag.item())
            mgr.restore()
            group.close()
        result_q.put((rank, err / scale, agree, same, tokens, flag))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["fused", "nccl"])
def test_two_gpu_sharded_model_decode(exchange):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, exchange, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
    results = sorted(q.get(timeout=5) for _ in range(2))
    for p in procs:
        assert p.exitcode == 0
    S, steps = 150, 40
    for rank, rel, agree, same, tokens, flag in results:
        assert flag == 0, f"rank {rank}: device error flag {flag}"
        assert rel <= 0.06, f"rank {rank}: logit error {rel:.4f} of scale"
        assert agree >= 0.9, f"rank {rank}: argmax agreement {agree:.2f}"
        assert same, f"rank {rank}: ranks disagree"
        # rank 0 holds the first floor(pages/2) whole pages of the prompt; rank 1 the rest and every
        # decoded token
        npg = -(-S // 64)
        lo = (npg // 2) * 64
        expect = lo if rank == 0 else S - lo + steps
        assert tokens == [expect, expect], f"rank {rank}: cached tokens {tokens}"
