"""Failure detection on the GPU without a fault: the bounded waits of the cross-GPU exchanges run out.

One process, one GPU.  The exchange is given a world of two ranks whose "peer" receive buffer is a
second local buffer that nothing reads, so the words and flags of rank 1 never arrive.  With a
1 ms wait bound the kernels give up, set HELM_DEVERR_TIMEOUT in the caller's error word and
return; the context stays usable, which the test checks with a normal call afterwards.  Nothing
here traps or hangs: every wait is bounded, and the bound is what is being tested.
"""
import ctypes
import time

import pytest
import torch

from tests.attn_util import assert_attn_close

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)
B, Hq, Hkv, D, P, NPG = 2, 16, 2, 128, 64, 12
WAIT_NS = 1_000_000    # 1 ms


def _pool(seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    total = B * NPG
    kp = torch.randn(total, Hkv, P, D, generator=g, device=DEV).to(torch.bfloat16)
    vp = torch.randn(total, Hkv, P, D, generator=g, device=DEV).to(torch.bfloat16)
    pt = torch.arange(total, dtype=torch.int32, device=DEV).reshape(B, NPG)
    pu = torch.full((B, NPG), P, dtype=torch.int32, device=DEV)
    npg = torch.full((B,), NPG, dtype=torch.int32, device=DEV)
    q = torch.randn(B, Hq, D, generator=g, device=DEV).to(torch.bfloat16)
    return q, kp, vp, pt, pu, npg, total


def _check_usable(q, kp, vp, pt, pu, npg, total):
    """A plain call after the timeout still computes the right attention."""
    from helm_b200 import ops
    from oracle import attention as OA
    out = ops.paged_decode_attention(q, kp, vp, pt, pu, npg, num_kv_heads=Hkv, page_size=P,
                                     page_stride=Hkv * P * D, head_stride=P * D, num_pool_pages=total,
                                     out_dtype=torch.float32)
    ref = OA.paged_attention_torch(q.cpu(), kp.cpu(), vp.cpu(), pt.cpu(), pu.cpu(), npg.cpu())
    assert_attn_close(out.cpu(), ref, torch.bfloat16, "after timeout")


def test_fused_exchange_wait_runs_out():
    from helm_b200 import _native as N
    from helm_b200 import ops
    lib = N.lib()
    q, kp, vp, pt, pu, npg, total = _pool(11)
    rows = B * Hq
    xr, xf, xc = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    assert lib.helm_shard_exchange_bytes(2, rows, D, ctypes.byref(xr), ctypes.byref(xf), ctypes.byref(xc)) > 0
    recv_mine = torch.zeros(xr.value, dtype=torch.uint8, device=DEV)
    recv_peer = torch.zeros(xr.value, dtype=torch.uint8, device=DEV)    # nobody ever reads or fills it
    counters = torch.zeros(max(xc.value, 4), dtype=torch.uint8, device=DEV)
    x = N.ShardExchange()
    x.rank, x.world = 0, 2
    x.peer_recv[0], x.peer_recv[1] = recv_mine.data_ptr(), recv_peer.data_ptr()
    x.recv_local = recv_mine.data_ptr()
    x.counters = counters.data_ptr()
    x.wait_ns = WAIT_NS
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    out = torch.full((B, Hq, D), 7.0, dtype=torch.bfloat16, device=DEV)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    ops.paged_decode_attention(q, kp, vp, pt, pu, npg, num_kv_heads=Hkv, page_size=P, page_stride=Hkv * P * D,
                               head_stride=P * D, num_pool_pages=total, out=out, error_flag=err,
                               exchange=ctypes.pointer(x))
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(err.item()) & N.DEVERR_TIMEOUT
    assert elapsed < 1.0, f"the 1 ms bound took {elapsed:.3f} s"
    assert torch.count_nonzero(out).item() == 0     # rows whose exchange gave up are zero
    _check_usable(q, kp, vp, pt, pu, npg, total)


def test_gather_merge_wait_runs_out():
    from helm_b200 import _native as N
    lib = N.lib()
    rows = B * Hq
    rb, fb, cb = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    assert lib.helm_gather_merge_state_bytes(2, rows, D, ctypes.byref(rb), ctypes.byref(fb), ctypes.byref(cb)) > 0
    mine = torch.zeros(rb.value + fb.value, dtype=torch.uint8, device=DEV)
    peer = torch.zeros(rb.value + fb.value, dtype=torch.uint8, device=DEV)
    counters = torch.zeros(max(cb.value, 4), dtype=torch.uint8, device=DEV)
    record = torch.randn(rows, D + 2, device=DEV)
    record[:, D] = 0.0
    record[:, D + 1] = 1.0
    out = torch.full((rows, D), 7.0, device=DEV)
    err = torch.zeros(1, dtype=torch.int32, device=DEV)
    p = N.GatherMergeParams()
    p.rank, p.world, p.rows, p.D = 0, 2, rows, D
    p.record = record.data_ptr()
    p.peer_recv[0], p.peer_recv[1] = mine.data_ptr(), peer.data_ptr()
    p.peer_flags[0], p.peer_flags[1] = mine.data_ptr() + rb.value, peer.data_ptr() + rb.value
    p.recv_local, p.flags_local = mine.data_ptr(), mine.data_ptr() + rb.value
    p.counters = counters.data_ptr()
    p.out, p.out_dtype = out.data_ptr(), N.F32
    p.error_flag = err.data_ptr()
    p.wait_ns = WAIT_NS
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    N.check("helm_gather_merge", lib.helm_gather_merge(ctypes.byref(p), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    elapsed = time.perf_counter() - t0
    assert int(err.item()) & N.DEVERR_TIMEOUT
    assert elapsed < 1.0, f"the 1 ms bound took {elapsed:.3f} s"
    _check_usable(*_pool(12))
