"""KV sequence sharding on 2 GPUs: the P2P record exchange (helm_gather_merge over CUDA IPC) and
the NCCL exchange, against the single-GPU attention over the whole sequence.  Spawns its own two
ranks; skipped with fewer than 2 GPUs."""
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
        B, Hq, Hkv, D, P, npg = 3, 32, 4, 128, 64, 50
        g = torch.Generator().manual_seed(7)            # same data on every rank
        kp = torch.randn(B * npg, Hkv, P, D, generator=g).to(torch.bfloat16)
        vp = torch.randn(B * npg, Hkv, P, D, generator=g).to(torch.bfloat16)
        pt = torch.randperm(B * npg, generator=g).to(torch.int32).reshape(B, npg)
        pu = torch.full((B, npg), P, dtype=torch.int32)
        pu[:, -1] = 29
        kp, vp = kp.to(dev), vp.to(dev)
        common = dict(num_kv_heads=Hkv, page_size=P, page_stride=Hkv * P * D, head_stride=P * D,
                      num_pool_pages=B * npg)
        rows = B * Hq
        group = KVShardGroup(rows, D, dev, exchange=exchange)
        lo, hi = shard_bounds(npg, rank, world)
        errs = []
        for call in range(5):
            q = torch.randn(B, Hq, D, generator=g).to(torch.bfloat16).to(dev)
            full = ops.paged_decode_attention(q, kp, vp, pt.to(dev), pu.to(dev),
                                              torch.full((B,), npg, dtype=torch.int32, device=dev),
                                              out_dtype=torch.float32, **common)
            rec = torch.empty(rows, D + 2, device=dev)
            ops.paged_decode_attention(q, kp, vp, pt[:, lo:hi].contiguous().to(dev),
                                       pu[:, lo:hi].contiguous().to(dev),
                                       torch.full((B,), hi - lo, dtype=torch.int32, device=dev),
                                       out_record=rec, **common)
            out = torch.empty(rows, D, device=dev, dtype=torch.float32)
            group.gather_merge(rec, out=out)
            torch.cuda.synchronize(dev)
            errs.append(float((out.reshape(B, Hq, D) - full).abs().max()))
        flag = int(group.error_flag.item())
        group.close()
        result_q.put((rank, max(errs), flag))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("exchange", ["p2p", "nccl"])
def test_two_gpu_exchange_matches_single_gpu(exchange):
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
        p.join(timeout=240)
    results = sorted(q.get(timeout=5) for _ in range(2))
    for p in procs:
        assert p.exitcode == 0
    for rank, err, flag in results:
        assert flag == 0, f"rank {rank}: device error flag {flag}"
        assert err < 1e-4, f"rank {rank}: {err}"
