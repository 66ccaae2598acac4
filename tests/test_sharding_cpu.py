"""Host logic of KV sequence sharding, on CPU: the page partition, the prompt token ranges each rank
stores, the record exchange protocol over a world-size-2 gloo group (each rank's partial record over
its share of the pages, all-gathered and merged in rank order = attention over the whole sequence,
identical on every rank), and failure detection when a rank never joins the exchange (the waiting
rank's collective ends with an error after a short timeout; no GPU involved)."""
import datetime
import os
import socket
import time

import numpy as np
import pytest
import torch

from helm_b200.runtime.sharded import shard_bounds
from helm_b200.runtime.kv_offload import _shard_tokens
from oracle.attention import Page, lse_merge, partial_record, streaming_attention


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shard_bounds_partition(world):
    for n in range(0, 260):
        prev = 0
        sizes = []
        for r in range(world):
            lo, hi = shard_bounds(n, r, world)
            assert lo == prev and hi >= lo
            sizes.append(hi - lo)
            prev = hi
        assert prev == n
        assert max(sizes) - min(sizes) <= 1


def test_shard_bounds_rejects_bad_rank():
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)
    with pytest.raises(ValueError):
        shard_bounds(10, 0, 0)


class _Shard:
    def __init__(self, rank, world):
        self.rank, self.world = rank, world


@pytest.mark.parametrize("world", [2, 4, 8])
def test_prompt_token_ranges_are_whole_pages(world):
    P = 64
    for n_tok in [1, 63, 64, 65, 1000, 4096, 4097]:
        got = [_shard_tokens(n_tok, P, _Shard(r, world)) for r in range(world)]
        assert got[0][0] == 0 and got[-1][1] == n_tok
        for (lo, hi), (lo2, _) in zip(got, got[1:]):
            assert hi == lo2
        for lo, hi in got[:-1]:
            assert lo % P == 0 and (hi - lo) % P == 0   # only the last rank may hold a partial page
    assert _shard_tokens(100, P, None) == (0, 100)


# ----------------------------------------------------------------------------
# two gloo ranks
# ----------------------------------------------------------------------------
def _pages(seed, npg, Hkv, P, D):
    rng = np.random.default_rng(seed)
    pages = []
    for i in range(npg):
        used = P if i < npg - 1 else 29
        pages.append(Page(rng.standard_normal((Hkv, P, D)).astype(np.float32),
                          rng.standard_normal((Hkv, P, D)).astype(np.float32), used))
    q = rng.standard_normal((4 * Hkv, D)).astype(np.float32)
    return q, pages


def _exchange_worker(rank, world, port, q_out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=30))
    try:
        Hkv, P, D = 2, 16, 32
        results = []
        for seed, npg in [(0, 7), (1, 1), (2, 2), (3, 13)]:
            q, pages = _pages(seed, npg, Hkv, P, D)
            lo, hi = shard_bounds(npg, rank, world)
            mine = pages[lo:hi]
            if mine:
                k = np.concatenate([p.k[:, :p.used] for p in mine], axis=1)
                v = np.concatenate([p.v[:, :p.used] for p in mine], axis=1)
                rec = partial_record(q, k, v, 1.0 / np.sqrt(D))
            else:
                rec = partial_record(q, None, None, 1.0 / np.sqrt(D))
            t = torch.from_numpy(rec)
            gathered = [torch.empty_like(t) for _ in range(world)]
            dist.all_gather(gathered, t)
            out, _ = lse_merge(np.stack([g.numpy() for g in gathered]))   # rank order
            full = streaming_attention(q, pages)
            results.append((float(np.abs(out - full).max()), out.tobytes()))
        q_out.put((rank, results))
    finally:
        dist.destroy_process_group()


def test_gloo_two_rank_exchange_matches_whole_sequence():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_exchange_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for (e0, b0), (e1, b1) in zip(res[0], res[1]):
        assert e0 < 1e-12 and e1 < 1e-12
        assert b0 == b1          # identical merged output on both ranks


def _dropout_worker(rank, world, port, q_out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=3))
    if rank == 1:
        # this rank leaves between steps: it never enters the next exchange
        q_out.put((rank, "left"))
        q_out.close()
        q_out.join_thread()     # flush the queue before the hard exit
        os._exit(0)
    t = torch.zeros(4, dtype=torch.float64)
    gathered = [torch.empty_like(t) for _ in range(world)]
    t0 = time.time()
    try:
        dist.all_gather(gathered, t)
        q_out.put((rank, "no error"))
    except Exception as e:  # the waiting rank learns of the failure on the host
        q_out.put((rank, f"error after {time.time() - t0:.1f}s: {type(e).__name__}"))
    q_out.close()
    q_out.join_thread()
    os._exit(0)


def test_gloo_rank_dropout_is_detected():
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dropout_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(2))
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "left"
    assert res[0].startswith("error after"), res[0]
