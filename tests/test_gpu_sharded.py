"""KV sequence sharding on 2, 4 and 8 GPUs: the exchange fused into the attention kernel, the P2P
record exchange (helm_gather_merge over CUDA IPC) and the NCCL exchange, against the single-GPU
attention over the whole sequence, with bit-identical outputs on every rank.  Spawns its own ranks;
each world size is skipped when the box has fewer GPUs."""
import math
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
    import datetime
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    try:
        from helm_b200 import ops
        from helm_b200.runtime.sharded import KVShardGroup, shard_bounds
        Hq, Hkv, D, P = 32, 4, 128, 64
        npgs = [50, 1, 17]                               # sequence 1 has no pages on rank 0
        B = len(npgs)
        total = sum(npgs)
        g = torch.Generator().manual_seed(7)            # same data on every rank
        kp = torch.randn(total, Hkv, P, D, generator=g).to(torch.bfloat16).to(dev)
        vp = torch.randn(total, Hkv, P, D, generator=g).to(torch.bfloat16).to(dev)
        perm = torch.randperm(total, generator=g).to(torch.int32)
        width = max(npgs)
        pt = torch.zeros((B, width), dtype=torch.int32)
        pu = torch.zeros((B, width), dtype=torch.int32)
        lpt = torch.zeros((B, width), dtype=torch.int32)
        lpu = torch.zeros((B, width), dtype=torch.int32)
        lnp = torch.zeros((B,), dtype=torch.int32)
        i = 0
        for b, n in enumerate(npgs):
            pt[b, :n] = perm[i:i + n]
            pu[b, :n] = P
            pu[b, n - 1] = 29
            i += n
            lo, hi = shard_bounds(n, rank, world)
            lpt[b, :hi - lo] = pt[b, lo:hi]
            lpu[b, :hi - lo] = pu[b, lo:hi]
            lnp[b] = hi - lo
        common = dict(num_kv_heads=Hkv, page_size=P, page_stride=Hkv * P * D, head_stride=P * D,
                      num_pool_pages=total)
        rows = B * Hq
        group = KVShardGroup(rows, D, dev, exchange=exchange)
        errs = []
        for call in range(5):
            q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16).to(dev)
            full = ops.paged_decode_attention(q, kp, vp, pt.to(dev), pu.to(dev),
                                              torch.tensor(npgs, dtype=torch.int32, device=dev),
                                              out_dtype=torch.float32, **common)
            if exchange == "fused":
                out = ops.paged_decode_attention(q, kp, vp, lpt.to(dev), lpu.to(dev), lnp.to(dev),
                                                 out_dtype=torch.float32, exchange=group.xparams_ptr,
                                                 error_flag=group.error_flag, **common)
            elif exchange == "split":
                ws = torch.empty(1 << 20, device=dev)
                parts = ops.paged_decode_attention(q, kp, vp, lpt.to(dev), lpu.to(dev), lnp.to(dev),
                                                   records_only=True, workspace=ws, **common)
                out = torch.empty(rows, D, device=dev, dtype=torch.float32)
                group.gather_merge(parts, out=out)
            else:
                rec = torch.empty(rows, D + 2, device=dev)
                ops.paged_decode_attention(q, kp, vp, lpt.to(dev), lpu.to(dev), lnp.to(dev), out_record=rec,
                                           **common)
                out = torch.empty(rows, D, device=dev, dtype=torch.float32)
                group.gather_merge(rec, out=out)
            torch.cuda.synchronize(dev)
            errs.append(float((out.reshape(B, Hq, D) - full).abs().max()))
            # every rank must hold the identical merged output (rank-order merge)
            outs = [torch.empty_like(out) for _ in range(world)]
            dist.all_gather(outs, out.contiguous())
            same = all(torch.equal(o, outs[0]) for o in outs)
            if not same:
                errs.append(float("inf"))
        flag = int(group.error_flag.item())
        group.close()
        result_q.put((rank, max(errs), flag))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("exchange", ["fused", "split", "p2p", "nccl"])
def test_sharded_exchange_matches_single_gpu(exchange, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, exchange, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=240)
    results = sorted(q.get(timeout=5) for _ in range(world))
    for p in procs:
        assert p.exitcode == 0
    for rank, err, flag in results:
        assert flag == 0, f"rank {rank}: device error flag {flag}"
        assert err < 1e-4, f"rank {rank}: {err}"
