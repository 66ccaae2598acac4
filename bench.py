#!/usr/bin/env python
"""Benchmark of the B200 decode hot path.

Default workload (the metric's long-context decode): a Qwen3-32B-shaped
attention stack -- 64 layers, 64 query / 8 KV heads, head_dim 128, bf16, batch 4, 131072 cached
tokens per sequence in 64-token pages, KV sharded by sequence over the N GPUs (one process per
GPU).  One step = one decode step of the stack: for every layer, append the new token's K/V (on
the rank holding the sequence tail, device-directed) and run the paged attention over the rank's
shard -- at N = 1 the automatic plan (the split kernel with about one resident wave of CTAs, then
the LSE merge); for N > 1 the persistent kernel, which itself exchanges the per-head (m, l, o)
records with the other ranks over NVLink and merges them (`--exchange split` runs the split
kernel and a separate merge-and-exchange launch instead).  Synthetic data (seeded normal K/V
through KVCacheManager.append_prefill); the KV working set (137 GB / N) is far larger than L2, so
no flush is needed.  The step is captured in a CUDA graph; `e2e` reruns it through the runtime's
_decode_batched with pinned-host inputs and outputs.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl helm|reference]
                  [--workload config5|config1|config2|config3|config4|prefill|kernels]

Other workloads (single JSON line each): config1 -- the reference's mixed-residency fp32 case
through perform_streaming_attention; config2 -- the INT8 GEMV shapes; config3 -- a Qwen3-8B-shaped
decode step through KVOffloadManager (CUDA graph); config4 -- a Qwen3-14B-shaped INT8 decode step
with half of the KV in pinned host memory; prefill -- the config-2 weights at M = 4096 through the
tcgen05 INT8 GEMM; kernels -- every kernel family once, with its achieved GB/s or TFLOP/s.

Rank 0 prints one JSON line.  `--impl reference` times the reference's own CPU algorithm on the
host cores instead (oracle/cpu_baseline.py; the compiled reference GEMV for config2).
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

import torch

REPO = os.path.dirname(os.path.abspath(__file__))
if REPO not in sys.path:
    sys.path.insert(0, REPO)

METRIC = "paged decode-attn HBM GB/s (% of peak); decode tok/s at 1/2/4/8 B200"
CFG = dict(layers=64, batch=4, q_heads=64, kv_heads=8, head_dim=128, page=64, ctx=131072)
WORKLOAD = ("config5: Qwen3-32B-shaped attention stack, 64 layers, 64q/8kv heads, d128, bf16, "
            "batch 4, 131072-token paged KV (64-token pages), KV sequence-sharded")


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="helm", choices=["helm", "reference"])
    ap.add_argument("--workload", default="config5",
                    choices=["config5", "config2", "config1", "config3", "config4", "prefill", "kernels"],
                    help="config5: the sharded decode-attention stack (default); config2: INT8 GEMV shapes; "
                         "config1: the reference's single-layer mixed-residency fp32 case; config3: a "
                         "Qwen3-8B-shaped decode step through KVOffloadManager; config4: a Qwen3-14B-shaped "
                         "INT8 decode step with half the KV on the host; prefill: the config-2 weights at M=4096 "
                         "through the tcgen05 INT8 GEMM (and dequantise + cuBLAS beside it); kernels: every "
                         "kernel family once, with its achieved GB/s or TFLOP/s")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-sub-records", action="store_true",
                    help="config5 at N=1: skip the config-2 and config-1 sub-records of the line")
    ap.add_argument("--e2e-steps", type=int, default=None)
    ap.add_argument("--exchange", default="fused", choices=["fused", "split", "p2p", "nccl"],
                    help="cross-GPU record exchange for N > 1")
    # Smaller stacks for ncu captures only; the reported workload is config 5 unless these are set.
    ap.add_argument("--layers", type=int, default=None)
    ap.add_argument("--ctx", type=int, default=None)
    # One config-2 GEMV shape / row count only (ncu captures of a single shape); the reported
    # workload is all nine calls unless these are set.
    ap.add_argument("--shape", default=None, help="config2 only: N,K of a single shape")
    ap.add_argument("--rows", type=int, default=None, help="config2 only: a single M")
    ap.add_argument("--kernel", default=None, help="kernels only: a single case by name")
    args = ap.parse_args()
    if args.layers is not None:
        CFG["layers"] = args.layers
    if args.ctx is not None:
        CFG["ctx"] = args.ctx
    return args


# DRAM traffic of one attention launch, from the ncu capture summarised in
# profiles/attn_tc_persistent_config5.txt (small case of the same kernel): reads per algorithmic
# byte, and the record/output writes of a batch-4, 64-head call.
ATTN_READ_PER_ALG_BYTE = 269.749504 / 268.664832
ATTN_WRITE_BYTES = 5.910784e6
# The same for the split path (attention + merge launches of one call, 9 splits), from
# profiles/attn_tc_kernel_config5.md.
ATTN_SPLIT_READ_PER_ALG_BYTE = 269.597696 / 268.566528
# records written by the attention and read back by the merge, per split and record row (D + 2
# floats): 1.132 MB written + 1.212 MB read for 9 splits x 256 rows in that capture
ATTN_SPLIT_RECORD_BYTES = (1.132e6 + 1.212e6) / (9 * 256 * 130)


def peaks():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ----------------------------------------------------------------------------
# nvidia-smi clock sampler (runs during the timed region)
# ----------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.lines = []

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.idx)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except Exception:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append((time.time(), line.strip()))

    def stop(self, t_from=None, t_to=None):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.t.join(timeout=2)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ts, ln in self.lines:
            if (t_from is not None and ts < t_from) or (t_to is not None and ts > t_to):
                continue
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def gpu_selector(dev, local):
    """nvidia-smi -i argument for this process's GPU (its UUID when torch exposes it)."""
    try:
        u = str(torch.cuda.get_device_properties(dev).uuid)
        return u if u.startswith("GPU-") else "GPU-" + u
    except Exception:
        vis = os.environ.get("CUDA_VISIBLE_DEVICES")
        return vis.split(",")[local] if vis else str(local)


# ----------------------------------------------------------------------------
# distributed helpers
# ----------------------------------------------------------------------------
def dist_setup(n):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if world != n:
        raise SystemExit(f"--gpus {n} but WORLD_SIZE={world}: launch with torchrun --nproc-per-node {n}")
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, local, world


def init_pg(world, local, backend="nccl"):
    import datetime
    import torch.distributed as dist
    if world > 1 and not dist.is_initialized():
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local) if backend == "nccl" else None)
    return dist


def max_over_ranks(x: float, world: int, dev) -> float:
    if world == 1:
        return x
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


# ----------------------------------------------------------------------------
# reference arm: the reference's CPU algorithm on the host cores
# ----------------------------------------------------------------------------
def run_reference(args, rank):
    if rank != 0:
        return
    from oracle.cpu_baseline import time_decode_attention
    c = CFG
    warm = min(args.warmup, 1)
    calls = max(1, min(args.steps, 3))
    t, n, threads = time_decode_attention(c["q_heads"], c["kv_heads"], c["head_dim"], c["page"], c["ctx"],
                                          torch.bfloat16, path=2, min_seconds=0.0 if warm == 0 else 5.0,
                                          max_calls=calls)
    step_s = t * c["layers"] * c["batch"]
    tok_s = c["batch"] / step_s
    sample = (f"reference all-CPU path (kv_cache.py:376-380, ported op-for-op) on 1 of {c['layers']} layers x "
              f"1 of {c['batch']} sequences at {c['ctx']} tokens, median of {n} calls, x{c['layers'] * c['batch']}")
    line = {"impl": "reference", "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": n, "warmup": warm, "ms_per_step": step_s * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "config": {"workload": WORKLOAD, "parallelism": "host cores", "global_batch": c["batch"],
                       "seq_len": c["ctx"]},
            "cpu_baseline": {"value": tok_s, "unit": "tok/s", "cores": threads, "kind": "port", "sample": sample},
            "e2e": {"value": tok_s, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# helm arm
# ----------------------------------------------------------------------------
CHUNK_PAGES = 64   # K/V are generated per chunk of 64 pages of one (layer, sequence)


def kv_chunk(l, b, c, Hkv, D, P, dev):
    """K and V [1, Hkv, CHUNK_PAGES*P, D] bf16 of chunk c (global pages c*64 .. c*64+63) of layer l,
    sequence b: seeded by (l, b, c) alone, so any rank -- and the checker -- rebuilds any chunk."""
    g = torch.Generator(device=dev).manual_seed(((l * 4096 + b) * 65536 + c) * 2 + 1)
    K = torch.randn((1, Hkv, CHUNK_PAGES * P, D), generator=g, device=dev, dtype=torch.bfloat16)
    V = torch.randn((1, Hkv, CHUNK_PAGES * P, D), generator=g, device=dev, dtype=torch.bfloat16)
    return K, V


class Stack:
    """The sharded attention stack on one rank, held by the drop-in runtime: a KVAllocator whose
    device slab holds every page, one KVCacheManager per sequence (prefilled through
    append_prefill) and the batch's device page tables (DecodeBatch).  K/V come from kv_chunk (the
    rank's share of every sequence); q and the appended tokens are the same on every rank."""

    def __init__(self, rank, world, dev, spare_pages, exchange="fused"):
        from helm_b200 import ops
        from helm_b200.runtime import KVAllocator, KVCacheManager
        from helm_b200.runtime.paged import DecodeBatch
        from helm_b200.runtime.sharded import shard_bounds
        self.ops = ops
        c = CFG
        self.rank, self.world, self.dev = rank, world, dev
        self.L, self.B, self.Hq, self.Hkv, self.D, self.P = (c["layers"], c["batch"], c["q_heads"], c["kv_heads"],
                                                             c["head_dim"], c["page"])
        plo, phi = shard_bounds(c["ctx"] // self.P, rank, world)
        self.npg = phi - plo
        self.local_ctx = self.npg * self.P
        self.tail = rank == world - 1
        self.spare = spare_pages if self.tail else 0
        self.alloc = KVAllocator(num_layers=self.L, num_kv_heads=self.Hkv, head_dim=self.D, page_size=self.P,
                                 dtype=torch.bfloat16)
        self.alloc.reserve_capacity(dev, self.L * self.B * (self.npg + self.spare) + 4 * self.L * self.B + 64)
        self.kvcms = [KVCacheManager(self.alloc, gpu_high_watermark_bytes=1 << 62) for _ in range(self.B)]
        self.batch = DecodeBatch(self.kvcms, self.L, dev, width=self.npg + self.spare + 8)
        self.plo, self.phi = plo, phi
        for l in range(self.L):
            for b in range(self.B):
                for c in range(plo // CHUNK_PAGES, (phi + CHUNK_PAGES - 1) // CHUNK_PAGES):
                    K, V = kv_chunk(l, b, c, self.Hkv, self.D, self.P, dev)
                    t0 = max(plo - c * CHUNK_PAGES, 0) * self.P
                    t1 = (min(phi, (c + 1) * CHUNK_PAGES) - c * CHUNK_PAGES) * self.P
                    self.kvcms[b].append_prefill(l, K[:, :, t0:t1], V[:, :, t0:t1])
                self.batch.sync_row(l, b)
        del K, V
        g = torch.Generator(device=dev).manual_seed(1234)   # q and new tokens: identical on every rank
        self.store = self.alloc.store(dev)
        self.n_pool = self.store.capacity
        # spare pages for the device-directed appends of the graph-captured step (tail rank)
        spare_ids = torch.zeros((self.L, self.B, max(self.spare, 1)), dtype=torch.int32)
        for l in range(self.L):
            for b in range(self.B):
                for j in range(self.spare):
                    spare_ids[l, b, j] = self.alloc.allocate(dev).slot
        self.spare_ids = spare_ids.to(dev)
        self.spare_next = torch.zeros((self.L, self.B), dtype=torch.int32, device=dev)
        self.error_flag = self.batch.error_flag
        self.q = torch.randn((self.L, self.B, self.Hq, self.D), generator=g, device=dev).to(torch.bfloat16)
        self.k_new = torch.randn((self.L, self.B, self.Hkv, self.D), generator=g, device=dev).to(torch.bfloat16)
        self.v_new = torch.randn((self.L, self.B, self.Hkv, self.D), generator=g, device=dev).to(torch.bfloat16)
        self.out = torch.empty((self.L, self.B, self.Hq, self.D), dtype=torch.bfloat16, device=dev)
        rows = self.B * self.Hq
        self.rec = torch.empty((self.L, rows, self.D + 2), dtype=torch.float32, device=dev)
        self.shard = None
        if world > 1:
            from helm_b200.runtime.sharded import KVShardGroup
            self.shard = KVShardGroup(rows, self.D, dev, exchange=exchange)
        self.fused = self.shard is not None and self.shard.fused
        self.records_only = self.shard is not None and self.shard.records_only
        self.k_base, self.v_base = self.store.base_ptrs()
        self.page_stride = self.store.page_elems
        self.head_stride = self.store.head_stride
        self._build_params()

    def _build_params(self):
        ops = self.ops
        from helm_b200 import _native as N
        self.lib = N.lib()
        self.attn_params, self.append_params = [], []
        ws_need = 0
        bt = self.batch
        for l in range(self.L):
            p = ops.make_attn_params(
                self.q[l], self.k_base, self.v_base, bt.table[l], bt.used[l], bt.npages[l],
                num_kv_heads=self.Hkv, page_size=self.P, page_stride=self.page_stride,
                head_stride=self.head_stride, num_pool_pages=self.n_pool, max_pages=bt.width,
                out=self.out[l] if (self.world == 1 or self.fused) else None,
                out_record=self.rec[l] if (self.world > 1 and not self.fused and not self.records_only) else None,
                error_flag=self.error_flag)
            if self.fused:
                p.exchange = self.shard.xparams_ptr
            S = ctypes.c_int32(0)
            need = self.lib.helm_paged_attn_workspace_bytes(ctypes.byref(p), ctypes.byref(S))
            p.num_splits = S.value
            ws_need = max(ws_need, need)
            self.attn_params.append(p)
            if self.tail:
                a = ops.make_append_params(
                    self.k_new[l], self.v_new[l], self.k_base, self.v_base, page_stride=self.page_stride,
                    head_stride=self.head_stride, num_pool_pages=self.n_pool, page_size=self.P,
                    page_table=bt.table[l], page_used=bt.used[l], num_pages=bt.npages[l],
                    spare_pages=self.spare_ids[l], spare_next=self.spare_next[l], error_flag=self.error_flag)
                self.append_params.append(a)
        self.splits = self.attn_params[0].num_splits
        self.ws = torch.zeros(max(ws_need // 4, 1), dtype=torch.float32, device=self.dev)
        for p in self.attn_params:
            p.workspace = self.ws.data_ptr()
            p.workspace_bytes = self.ws.numel() * 4
        per_layer = (1 if self.tail else 0) + 1 + (1 if (self.splits > 1 and not self.records_only) else 0) + \
            (1 if (self.world > 1 and not self.fused) else 0)
        self.launches_per_step = self.L * per_layer

    def attn_bytes(self, tokens_per_seq):
        """Algorithmic bytes of one attention launch: K+V of every cached token read once per
        (sequence, kv head) plus q in and the output out."""
        kv = 2 * self.Hkv * self.D * 2 * tokens_per_seq * self.B
        qo = self.B * self.Hq * self.D * (2 + (2 if self.world == 1 else 4))
        return kv + qo

    def attend(self, l, stream):
        """One layer's attention call (the kernel the roofline measures)."""
        from helm_b200 import _native as N
        N.check("helm_paged_attn_decode",
                self.lib.helm_paged_attn_decode(ctypes.byref(self.attn_params[l]), stream.cuda_stream))

    def step(self, stream):
        """One decode step over all layers on the device-resident state (device-directed append
        on the tail rank, attention, and for N > 1 the record exchange + merge)."""
        from helm_b200 import _native as N
        sp = stream.cuda_stream
        for l in range(self.L):
            if self.tail:
                N.check("helm_kv_append", self.lib.helm_kv_append(ctypes.byref(self.append_params[l]), sp))
            N.check("helm_paged_attn_decode", self.lib.helm_paged_attn_decode(ctypes.byref(self.attn_params[l]), sp))
            if self.world > 1 and not self.fused:
                self.exchange(l, self.out[l].view(self.B * self.Hq, self.D))

    def exchange(self, l, out):
        """The separate exchange of layer l's attention result (p2p / split / nccl modes): the merged
        record, or in records-only mode the split records left in the workspace."""
        if self.records_only:
            rows, S = self.B * self.Hq, self.splits
            parts = self.ws[:S * rows * (self.D + 2)].view(S, rows, self.D + 2)
            return self.shard.gather_merge(parts, out=out)
        return self.shard.gather_merge(self.rec[l], out=out)


def run_helm(args, rank, local, world):
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    dist = init_pg(world, local)
    c = CFG
    total_steps = args.warmup + args.steps + 16
    spare = (total_steps + c["page"] - 1) // c["page"] + 1
    st = Stack(rank, world, dev, spare, exchange=args.exchange)
    stream = torch.cuda.current_stream(dev)
    torch.cuda.synchronize(dev)

    clocks = ClockSampler(gpu_selector(dev, local))
    clocks.start()
    # Eager warm-up (also initialises NCCL before graph capture).
    for _ in range(args.warmup):
        st.step(stream)
    torch.cuda.synchronize(dev)
    barrier(world)

    # One decode step (all layers) captured once and replayed: no host work between kernels.
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        st.step(torch.cuda.current_stream(dev))
    torch.cuda.synchronize(dev)
    graph.replay()  # warm replay (appends one more token, like a warm-up step)
    torch.cuda.synchronize(dev)
    barrier(world)

    # ---------------- device-timed region ----------------
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize(dev)
    t_load0 = time.time()
    t0.record(stream)
    for s in range(args.steps):
        graph.replay()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    t_load1 = time.time()
    barrier(world)
    ms = t0.elapsed_time(t1)
    ms_max = max_over_ranks(ms, world, dev)
    ms_step = ms_max / args.steps
    # correctness of what was timed: eager warm-up steps + the warm replay + the timed replays each
    # appended one token per (layer, sequence)
    check = check_stack(st, stream, world, dev, appended=args.warmup + 1 + args.steps)

    # Attention-call durations for the roofline: back-to-back calls over every layer, each
    # bracketed by CUDA events on the launching stream (no other work in between).
    attn_ms = []
    for rep in range(2):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(st.L)]
        for l in range(st.L):
            evs[l][0].record(stream)
            st.attend(l, stream)
            evs[l][1].record(stream)
        torch.cuda.synchronize(dev)
        if rep:
            attn_ms += [a.elapsed_time(b) for a, b in evs]
    attn_avg_ms = sum(attn_ms) / len(attn_ms)
    breakdown = component_breakdown(st, stream, world, dev)
    err = int(st.error_flag.item())
    del graph

    # ---------------- end-to-end through the public op API ----------------
    e2e_steps = args.e2e_steps if args.e2e_steps is not None else args.steps
    e2e = run_e2e(st, stream, e2e_steps, world, dev) if e2e_steps > 0 else None
    clk = clocks.stop(t_load0, time.time())
    clk["window_s"] = round(time.time() - t_load0, 3)
    clk["timed_region_s"] = round(t_load1 - t_load0, 3)

    if rank == 0:
        hbm_peak, peak_kind = peaks()
        tokens_per_seq = st.local_ctx + ((args.warmup + 1 + args.steps) if st.tail else 0)
        bytes_launch = st.attn_bytes(tokens_per_seq)
        achieved = bytes_launch / (attn_avg_ms * 1e-3) / 1e9
        step_bytes_all = bytes_launch * st.L * world
        tok_s = c["batch"] / (ms_step * 1e-3)
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline()
        line = {
            "metric": METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic",
            "timing": "CUDA graph of one decode step (all layers) replayed K times; CUDA events, max over ranks",
            "setup": {"prefill": "append_prefill per (layer, sequence) through KVCacheManager",
                      "pool_gb": round(st.store.slab.numel() * 2 / 1e9, 1)},
            "config": {"workload": WORKLOAD if (c["layers"], c["ctx"]) == (64, 131072) else
                       f"REDUCED (profiling only): {c['layers']} layers, ctx {c['ctx']}",
                       "global_batch": c["batch"], "seq_len": c["ctx"],
                       "layers": c["layers"], "parallelism": f"kv-seq-shard{world}",
                       "l2": "inputs larger than L2 (KV %.1f GB per GPU)" % (st.store.slab.numel() * 2 / 1e9),
                       "num_splits": st.splits},
            "hbm_gbs": step_bytes_all / (ms_step * 1e-3) / 1e9 / world,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak,
                         "traffic": (ATTN_SPLIT_READ_PER_ALG_BYTE * bytes_launch + ATTN_SPLIT_RECORD_BYTES *
                                     st.splits * st.B * st.Hq * (st.D + 2)
                                     if (world == 1 and st.splits > 0) else
                                     ATTN_READ_PER_ALG_BYTE * bytes_launch + ATTN_WRITE_BYTES
                                     if (world == 1 and st.splits < 0) else None),
                         "traffic_source": ("ncu dram__bytes_read/write.sum of the attention + merge launches of a "
                                            "268.7 MB call, reads scaled by the bytes streamed "
                                            "(profiles/attn_tc_kernel_config5.md)" if st.splits > 0 else
                                            "ncu dram__bytes_read/write.sum of a 268.7 MB launch, reads scaled "
                                            "by the units streamed (profiles/attn_tc_persistent_config5.txt)"),
                         "peak_kind": peak_kind,
                         "kernel": (f"attn_tc_kernel ({st.splits} splits, records only) + gather_merge_kernel "
                                    "(merge + exchange)" if st.records_only else
                                    f"attn_tc_kernel ({st.splits} splits) + lse_merge_wide_kernel (one "
                                    "helm_paged_attn_decode call)" if st.splits > 0 else
                                    "attn_tc_persistent_kernel (one helm_paged_attn_decode call = one launch)"),
                         "bytes_per_launch": bytes_launch, "avg_launch_ms": attn_avg_ms},
            "breakdown_ms_per_layer": breakdown,
            "check": check,
            "cpu_baseline": cpu,
            "e2e": e2e,
            "gpu_launches": st.launches_per_step * args.steps,
            "clocks": clk,
            "device_error_flag": err,
        }
    barrier(world)
    if st.shard is not None:
        st.shard.close()
    if world == 1 and not args.no_sub_records:
        # configs 2 and 1 (the INT8 GEMV shapes and the reference's fp32 single-layer case), timed in
        # the same run after the config-5 pool is released, nested in the one line as sub-records
        del st
        torch.cuda.empty_cache()
        subs = {}
        for name, fn in (("config2", config2_line), ("config1", config1_line)):
            subs[name] = fn(args, rank, world, dev)
        if rank == 0:
            line["sub_records"] = subs
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.destroy_process_group()


def check_stack(st, stream, world, dev, appended):
    """Correctness of the sharded stack, outside the timed region.  Every rank makes one more
    attention call of the last layer (exchange included) into an fp32 output; the outputs of all
    ranks must be bit-identical, and rank 0 recomputes 2 sequences x 2 kv heads of it in float64
    on the host from the seeds: every cached token (kv_chunk of every global page) plus the
    `appended` decode tokens (the step appends the same k_new / v_new each time), softmax
    attention as in the reference's all-CPU path (kv_cache.py:376-380).  Returns the check record
    on rank 0."""
    from helm_b200 import _native as N
    l = st.L - 1
    out32 = torch.empty((st.B, st.Hq, st.D), dtype=torch.float32, device=dev)
    p = N.PagedAttnParams()
    ctypes.memmove(ctypes.byref(p), ctypes.byref(st.attn_params[l]), ctypes.sizeof(p))
    p.out = out32.data_ptr()
    p.out_dtype = N.F32
    p.out_record = None
    if world > 1 and not st.fused:
        p.out = None
        p.out_record = None if st.records_only else st.rec[l].data_ptr()
    N.check("helm_paged_attn_decode", st.lib.helm_paged_attn_decode(ctypes.byref(p), stream.cuda_stream))
    if world > 1 and not st.fused:
        st.exchange(l, out32.view(st.B * st.Hq, st.D))
    torch.cuda.synchronize(dev)
    identical = True
    if world > 1:
        import torch.distributed as dist
        got = [torch.empty_like(out32) for _ in range(world)]
        dist.all_gather(got, out32)
        identical = all(torch.equal(got[0], t) for t in got[1:])
    if st.rank != 0:
        return None
    gq = st.Hq // st.Hkv
    scale = 1.0 / math.sqrt(st.D)
    n_chunks = (CFG["ctx"] // st.P + CHUNK_PAGES - 1) // CHUNK_PAGES
    max_err, max_ref = 0.0, 0.0
    seqs, heads = sorted({0, st.B - 1}), sorted({0, st.Hkv - 1})
    for b in seqs:
        ks = {g: [] for g in heads}
        vs = {g: [] for g in heads}
        for c in range(n_chunks):
            K, V = kv_chunk(l, b, c, st.Hkv, st.D, st.P, dev)
            n_tok = min(CHUNK_PAGES * st.P, CFG["ctx"] - c * CHUNK_PAGES * st.P)
            for g in heads:
                ks[g].append(K[0, g, :n_tok].cpu())
                vs[g].append(V[0, g, :n_tok].cpu())
        for g in heads:
            k_all = torch.cat(ks[g] + [st.k_new[l, b, g].cpu()[None]] * appended).double()
            v_all = torch.cat(vs[g] + [st.v_new[l, b, g].cpu()[None]] * appended).double()
            q = st.q[l, b, g * gq:(g + 1) * gq].cpu().double()
            w = torch.softmax((q @ k_all.T) * scale, dim=-1)
            ref = w @ v_all
            got = out32[b, g * gq:(g + 1) * gq].cpu().double()
            max_err = max(max_err, float((got - ref).abs().max()))
            max_ref = max(max_ref, float(ref.abs().max()))
    rel = max_err / max_ref if max_ref > 0 else max_err
    return {"rel_err": rel, "max_abs_err": max_err, "max_ref": max_ref, "bar": 2e-3, "ok": rel <= 2e-3,
            "ranks_bit_identical": identical,
            "sample": (f"last layer, sequences {seqs} x kv heads {heads} ({len(seqs) * len(heads) * gq} query "
                       f"heads), all {CFG['ctx'] + appended} cached tokens, fp32 kernel output vs float64 "
                       f"softmax attention on the host")}


def component_breakdown(st, stream, world, dev, reps=3):
    """Per-layer device time of each part of a decode step (append, attention, exchange + merge),
    from CUDA events around each launch in an eager pass; max over ranks of the mean."""
    from helm_b200 import _native as N
    sums = [0.0, 0.0, 0.0]
    n = 0
    for rep in range(reps):
        evs = [[torch.cuda.Event(enable_timing=True) for _ in range(4)] for _ in range(st.L)]
        barrier(world)
        for l in range(st.L):
            e = evs[l]
            e[0].record(stream)
            if st.tail:
                N.check("helm_kv_append", st.lib.helm_kv_append(ctypes.byref(st.append_params[l]), stream.cuda_stream))
            e[1].record(stream)
            st.attend(l, stream)
            e[2].record(stream)
            if world > 1 and not st.fused:
                st.exchange(l, st.out[l].view(st.B * st.Hq, st.D))
            e[3].record(stream)
        torch.cuda.synchronize(dev)
        if rep == 0:
            continue
        for e in evs:
            sums[0] += e[0].elapsed_time(e[1])
            sums[1] += e[1].elapsed_time(e[2])
            sums[2] += e[2].elapsed_time(e[3])
            n += 1
    out = {k: max_over_ranks(v / n, world, dev) for k, v in zip(("append", "attention", "exchange_merge"), sums)}
    return {k: round(v, 4) for k, v in out.items()}


def run_e2e(st, stream, steps, world, dev):
    """The same decode steps through the drop-in runtime API: per layer
    helm_b200.runtime.kv_offload._decode_batched (the call the patched attention forward makes)
    with the step's inputs (q and the new K/V of every layer) copied from pinned host memory and
    the outputs read back every step."""
    from helm_b200.runtime.kv_offload import _decode_batched
    L, B = st.L, st.B
    # the graph-captured steps advanced the device tables on their own: resync them from the host
    st.batch.synced = [[None] * st.B for _ in range(st.L)]
    q_h = st.q.cpu().pin_memory()
    k_h = st.k_new.cpu().pin_memory()
    v_h = st.v_new.cpu().pin_memory()
    out_h = torch.empty(st.out.shape, dtype=st.out.dtype).pin_memory()
    q_d = torch.empty_like(st.q)
    k_d = torch.empty_like(st.k_new)
    v_d = torch.empty_like(st.v_new)
    out_d = torch.empty_like(st.out)
    h2d = q_h.numel() * 2 + k_h.numel() * 2 * 2
    d2h = out_h.numel() * 2
    scale = 1.0 / math.sqrt(st.D)
    shard = st.shard

    def one_step():
        q_d.copy_(q_h, non_blocking=True)
        k_d.copy_(k_h, non_blocking=True)
        v_d.copy_(v_h, non_blocking=True)
        for l in range(L):
            out_d[l] = _decode_batched(st.kvcms, q_d[l].unsqueeze(2), k_d[l].unsqueeze(2), v_d[l].unsqueeze(2),
                                       l, scale, shard=shard)[:, :, 0]
        out_h.copy_(out_d, non_blocking=True)

    one_step()  # warm
    torch.cuda.synchronize(dev)
    barrier(world)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0.record(stream)
    for _ in range(steps):
        one_step()
    t1.record(stream)
    torch.cuda.synchronize(dev)
    ms = max_over_ranks(t0.elapsed_time(t1), world, dev) / steps
    return {"value": CFG["batch"] / (ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": h2d,
            "d2h_bytes_per_step": d2h, "ms_per_step": ms,
            "api": "helm_b200.runtime.kv_offload._decode_batched per layer (KVCacheManager/KVAllocator state)"}


# ----------------------------------------------------------------------------
# config 2: INT8 weight-only GEMV (the linears feeding attention)
# ----------------------------------------------------------------------------
C2_SHAPES = [(12288, 4096), (4096, 12288), (6144, 4096)]   # (N, K)
C2_ROWS = [1, 4, 8]
C2_METRIC = "int8 weight-only linear: algorithmic HBM GB/s (config2 shapes, M in 1/4/8)"
C2_WORKLOAD = ("config2: y = (x . Wq^T) * s, W int8 [N,K] uniform[-127,127], s fp16 U(0.001,0.02), x fp16 N(0,1); "
               "(N,K) in (12288,4096) (4096,12288) (6144,4096); M in 1,4,8")


def c2_bytes(M, Nn, K):
    """Algorithmic bytes of one call: int8 weight + fp16 scale + fp16 x in + fp16 y out."""
    return Nn * K + Nn * 2 + M * K * 2 + M * Nn * 2


def c2_inputs(Nn, K, M, dev, copies):
    g = torch.Generator().manual_seed(0)
    w = [torch.randint(-127, 128, (Nn, K), generator=g, dtype=torch.int8).to(dev) for _ in range(copies)]
    s = (torch.rand(Nn, generator=g) * 0.019 + 0.001).to(torch.float16).to(dev)
    x = torch.randn(M, K, generator=g).to(torch.float16).to(dev)
    return w, s, x


def run_config2(args, rank, local, world):
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    init_pg(world, local)
    line = config2_line(args, rank, world, dev)
    if rank == 0:
        print(json.dumps(line), flush=True)
    barrier(world)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def config2_line(args, rank, world, dev):
    """Device time of helm_int8_linear at every config-2 shape: a CUDA graph of one call per weight
    copy (copies rotate through > 4x L2, so every call streams its weight from HBM), replayed;
    CUDA events on the launching stream.  Replicas only: every rank runs the same work.  Returns
    the JSON record (rank 0; None elsewhere)."""
    from helm_b200 import _native as N
    from helm_b200 import ops
    from helm_b200.kernels import Int8Linear
    stream = torch.cuda.current_stream(dev)
    local = dev.index
    lib = N.lib()
    l2 = torch.cuda.get_device_properties(dev).L2_cache_size
    clocks = ClockSampler(gpu_selector(dev, local))
    clocks.start()
    cases, tot_bytes, tot_ms = [], 0, 0.0
    t_load0 = time.time()
    e2e_bytes_in = e2e_bytes_out = 0
    e2e_ms = 0.0
    shapes = [tuple(int(v) for v in args.shape.split(","))] if args.shape else C2_SHAPES
    for (Nn, K) in shapes:
        copies = max(4, -(-4 * l2 // (Nn * K)))
        for M in ([args.rows] if args.rows else C2_ROWS):
            w, s, x = c2_inputs(Nn, K, M, dev, copies)
            wp = [ops.int8_pack_weight(wi) for wi in w]   # the layout Int8Linear keeps
            y = torch.empty((M, Nn), dtype=torch.float16, device=dev)

            def time_calls(fn, weights):
                def calls():
                    for wi in weights:
                        N.check("helm_int8_linear", fn(
                            x.data_ptr(), ops.dtype_code(x.dtype), wi.data_ptr(), s.data_ptr(),
                            ops.dtype_code(s.dtype), None, y.data_ptr(), M, Nn, K,
                            torch.cuda.current_stream(dev).cuda_stream))
                for _ in range(max(args.warmup, 3)):
                    calls()
                torch.cuda.synchronize(dev)
                graph = torch.cuda.CUDAGraph()
                with torch.cuda.graph(graph):
                    calls()
                graph.replay()
                torch.cuda.synchronize(dev)
                reps = max(1, args.steps // 10)
                t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                barrier(world)
                t0.record(stream)
                for _ in range(reps):
                    graph.replay()
                t1.record(stream)
                torch.cuda.synchronize(dev)
                return max_over_ranks(t0.elapsed_time(t1), world, dev) / (reps * copies)
            ms = time_calls(lib.helm_int8_linear_packed, [p.data for p in wp])
            ms_rowmajor = time_calls(lib.helm_int8_linear, w)
            nbytes = c2_bytes(M, Nn, K)
            tot_bytes += nbytes
            tot_ms += ms
            # end to end through the public module: x from pinned host memory, y read back
            mod = Int8Linear(K, Nn, bias=False, device=dev, dtype=torch.float16)
            mod.weight = w[0]
            mod.scale = s
            x_h = x.cpu().pin_memory()
            y_h = torch.empty((M, Nn), dtype=torch.float16).pin_memory()
            n_e2e = 50
            for _ in range(3):
                y_h.copy_(mod(x_h.to(dev, non_blocking=True)), non_blocking=True)
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(n_e2e):
                y_h.copy_(mod(x_h.to(dev, non_blocking=True)), non_blocking=True)
            e1.record(stream)
            torch.cuda.synchronize(dev)
            e2e_ms += e0.elapsed_time(e1) / n_e2e
            e2e_bytes_in += x_h.numel() * 2
            e2e_bytes_out += y_h.numel() * 2
            cases.append({"N": Nn, "K": K, "M": M, "us": round(ms * 1e3, 3), "gbs": round(nbytes / (ms * 1e-3) / 1e9, 1),
                          "copies": copies, "rowmajor_us": round(ms_rowmajor * 1e3, 3),
                          "rowmajor_gbs": round(nbytes / (ms_rowmajor * 1e-3) / 1e9, 1)})
            del w, wp, x, y, mod
    prefill = c2_prefill_gemm(args, dev, world) if not (args.shape or args.rows) else None
    clk = clocks.stop(t_load0, time.time())
    if rank == 0:
        hbm_peak, peak_kind = peaks()
        agg = tot_bytes / (tot_ms * 1e-3) / 1e9
        cpu = None
        if world == 1 and not args.no_cpu_baseline:
            cpu = cpu_baseline_config2()
        line = {
            "metric": C2_METRIC, "value": agg * world, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": tot_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8 x fp16 -> fp32", "data": "synthetic",
            "timing": ("per shape: CUDA graph of one helm_int8_linear_packed call per weight copy (the packed layout "
                       "Int8Linear keeps), replayed; CUDA events; a step = the 9 calls; rowmajor_* = the same calls "
                       "on row-major weights (helm_int8_linear)"),
            "config": {"workload": C2_WORKLOAD if not (args.shape or args.rows) else
                       f"REDUCED (profiling only): shape {args.shape or 'all'}, M {args.rows or 'all'}",
                       "parallelism": f"replicas{world}",
                       "l2": "weight copies rotate through > 4x L2 per shape"},
            "cases": cases,
            "roofline": {"bound": "hbm", "achieved": agg, "peak": hbm_peak, "unit": "GB/s", "frac": agg / hbm_peak,
                         "traffic": None, "peak_kind": peak_kind, "kernel": "int8 GEMV (int8_tma_kernel, packed weights: helm_int8_linear_packed)",
                         "bytes_per_launch": tot_bytes / len(cases), "avg_launch_ms": tot_ms / len(cases)},
            "cpu_baseline": cpu,
            "e2e": {"value": tot_bytes / (e2e_ms * 1e-3) / 1e9 * world, "unit": "GB/s",
                    "h2d_bytes_per_step": e2e_bytes_in, "d2h_bytes_per_step": e2e_bytes_out, "ms_per_step": e2e_ms,
                    "api": "helm_b200.kernels.Int8Linear.forward per call, x from pinned host, y read back"},
            "gpu_launches": len(cases) * 1,
            "prefill_gemm": prefill,
            "clocks": clk,
        }
        return line
    return None


def bf16_peak():
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), "measured (burst)"
    except Exception:
        return 1590.0, "fallback"


def c2_prefill_gemm(args, dev, world, M=4096):
    """The same three weights at a prefill-sized M: the tcgen05 INT8 GEMM (helm_int8_gemm_packed,
    what Int8Linear runs for more than 64 rows) against dequantising the weight and calling cuBLAS
    (torch.nn.functional.linear), both timed with CUDA events over CUDA graphs of repeated calls."""
    import torch.nn.functional as F
    from helm_b200 import ops
    stream = torch.cuda.current_stream(dev)
    peak, kind = bf16_peak()
    out = []
    for (Nn, K) in C2_SHAPES:
        g = torch.Generator(device=dev).manual_seed(5)
        w = torch.randint(-127, 128, (Nn, K), generator=g, device=dev, dtype=torch.int8)
        s = (torch.rand(Nn, generator=g, device=dev) * 0.019 + 0.001).to(torch.bfloat16)
        x = torch.randn(M, K, generator=g, device=dev).to(torch.bfloat16)
        pk = ops.int8_pack_weight(w)
        y = torch.empty((M, Nn), dtype=torch.bfloat16, device=dev)

        def ours():
            ops.int8_linear(x, pk, s, out=y, gemm=True)

        def dequant_cublas():
            F.linear(x, w.to(torch.bfloat16) * s[:, None])

        res = {"N": Nn, "K": K, "M": M}
        for name, fn in (("tcgen05", ours), ("dequant_cublas", dequant_cublas)):
            for _ in range(3):
                fn()
            torch.cuda.synchronize(dev)
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph):
                for _ in range(10):
                    fn()
            graph.replay()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(3):
                graph.replay()
            e1.record(stream)
            torch.cuda.synchronize(dev)
            ms = e0.elapsed_time(e1) / 30
            tf = 2.0 * M * Nn * K / (ms * 1e-3) / 1e12
            res[name] = {"us": round(ms * 1e3, 2), "tflops": round(tf, 1), "frac": round(tf / peak, 3)}
            del graph
        out.append(res)
        del w, x, pk, y
    return {"bound": "tensor", "peak_tflops": peak, "peak_kind": kind, "cases": out,
            "how": "bf16 x, int8 weights; CUDA graph of 10 calls replayed 3 times; 2*M*N*K flops"}


# ----------------------------------------------------------------------------
# Per-kernel roofline table (--workload kernels)
# ----------------------------------------------------------------------------
def _graph_time_ms(fn, reps, stream, warm=3):
    """Device time of one call: `reps` calls captured in a CUDA graph, replayed once between CUDA
    events (eager calls between events when the call cannot be captured)."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    try:
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            for _ in range(reps):
                fn()
        graph.replay()
        torch.cuda.synchronize()
        e0.record(stream)
        graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
        del graph
        return e0.elapsed_time(e1) / reps, "cuda graph"
    except RuntimeError:
        torch.cuda.synchronize()
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / reps, "eager"


def kernel_cases(dev):
    """(name, kernels, bound, algorithmic bytes or flops, setup, description) for every kernel family
    of the library.  Each setup allocates its inputs and returns (call, check): inputs of the
    bandwidth-bound cases are larger than L2 (126 MB), so repeated calls stream from HBM; the
    decode-step kernels (append, prologue, exchange) move a few KB per call and are latency-bound by
    nature."""
    import ctypes
    import numpy as np
    from helm_b200 import _native as N
    from helm_b200 import ops
    bf = torch.bfloat16
    cases = []

    def pool(B, Hkv, D, P, ctx, dtype, seed):
        g = torch.Generator(device=dev).manual_seed(seed)
        npg = ctx // P
        slab = torch.randn((B * npg, 2, Hkv, P, D), generator=g, device=dev).to(dtype)
        pt = torch.arange(B * npg, dtype=torch.int32, device=dev).reshape(B, npg)
        pu = torch.full((B, npg), P, dtype=torch.int32, device=dev)
        nn = torch.full((B,), npg, dtype=torch.int32, device=dev)
        return slab, pt, pu, nn

    def attn_case(B, Hq, Hkv, D, P, ctx, dtype, splits, seed, copies=1):
        def setup():
            pools = [pool(B, Hkv, D, P, ctx, dtype, seed + i) for i in range(copies)]
            q = torch.randn((B, Hq, D), device=dev).to(dtype)
            out = torch.empty((B, Hq, D), dtype=q.dtype, device=dev)
            err = torch.zeros(1, dtype=torch.int32, device=dev)
            kw = dict(num_kv_heads=Hkv, page_size=P, page_stride=2 * Hkv * P * D, head_stride=P * D,
                      num_pool_pages=pools[0][0].shape[0], out=out, error_flag=err, num_splits=splits)
            it = [0]

            def call():
                slab, pt, pu, nn = pools[it[0] % copies]
                it[0] += 1
                ops.paged_decode_attention(q, slab[:, 0], slab[:, 1], pt, pu, nn, **kw)
            return call, lambda: int(err.item()) == 0 and bool(torch.isfinite(out).all())
        es = torch.empty((), dtype=dtype).element_size()
        return 2 * B * Hkv * ctx * D * es + 2 * B * Hq * D * es, setup

    b, s = attn_case(4, 64, 8, 128, 64, 16384, bf, -1, 1)
    cases.append(("attn_persistent", "attn_tc_persistent_kernel", "hbm", b, s,
                  "bf16, B 4, 64q/8kv, d128, 16384 tokens (256 pages) per sequence: one config-5 layer at N=8; "
                  "num_splits=-1"))
    b, s = attn_case(4, 64, 8, 128, 64, 16384, bf, 0, 1)
    cases.append(("attn_split", "attn_tc_kernel + lse_merge_wide_kernel", "hbm", b, s,
                  "the same call on the automatic plan (split path, 8 splits per sequence)"))
    b, s = attn_case(4, 32, 8, 128, 64, 16384, torch.float32, 0, 2)
    cases.append(("attn_warp_fp32", "attn_warp_kernel + lse_merge_kernel", "hbm", b, s,
                  "fp32 pages (config-1 heads), B 4, 32q/8kv, d128, 16384 tokens per sequence"))
    b, s = attn_case(1, 32, 8, 128, 64, 4096, torch.float32, 0, 10, copies=8)
    cases.append(("attn_config1", "attn_warp_kernel + lse_merge_kernel", "latency", b, s,
                  "config 1 all resident: fp32, B 1, 32q/8kv, d128, 4096 tokens, 8 instances rotating (268 MB)"))
    b, s = attn_case(4, 48, 2, 96, 64, 65536, bf, 0, 3)
    cases.append(("attn_warp_group24", "attn_warp_kernel (3 head chunks) + lse_merge_kernel", "hbm", b, s,
                  "bf16, B 4, 48q/2kv (GQA group 24), d96, 65536 tokens per sequence"))
    b, s = attn_case(4, 16, 4, 80, 64, 65536, bf, 0, 4)
    cases.append(("attn_generic", "attn_generic_kernel + lse_merge_kernel", "hbm", b, s,
                  "bf16, B 4, 16q/4kv, d80 (not a multiple of 32), 65536 tokens per sequence"))

    def merge_setup():
        S, rows, D = 16, 16384, 128
        part = torch.randn((S, rows, D + 2), device=dev)
        part[:, :, D] = torch.randn((S, rows), device=dev)
        part[:, :, D + 1] = torch.rand((S, rows), device=dev) + 0.5
        out = torch.empty((rows, D), device=dev)
        return (lambda: ops.lse_merge(part, out=out)), (lambda: bool(torch.isfinite(out).all()))
    cases.append(("lse_merge", "lse_merge_kernel", "hbm", 16 * 16384 * 130 * 4 + 16384 * 128 * 4, merge_setup,
                  "16 split records of 16384 rows x (128 + 2) fp32 into 16384 x 128 fp32"))

    def append_setup(prologue):
        B, Hq, Hkv, D, P = 4, 64, 8, 128, 64
        slab = torch.zeros((B * 4, 2, Hkv, P, D), dtype=bf, device=dev)
        kn = torch.randn((B, Hkv, D), device=dev).to(bf)
        vn = torch.randn((B, Hkv, D), device=dev).to(bf)
        dest = np.ascontiguousarray(np.array([[4 * b_ + 1, 1, 17] for b_ in range(B)], dtype=np.int32))
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        kw = dict(page_stride=2 * Hkv * P * D, head_stride=P * D, num_pool_pages=B * 4, page_size=P,
                  dest_host=dest, error_flag=err)
        if not prologue:
            return (lambda: ops.kv_append(kn, vn, slab[:, 0], slab[:, 1], **kw)), (lambda: int(err.item()) == 0)
        qi = torch.randn((B, Hq, D), device=dev).to(bf)
        qo = torch.empty_like(qi)
        qw = (torch.rand(D, device=dev) + 0.5).to(bf)
        kwn = (torch.rand(D, device=dev) + 0.5).to(bf)
        ang = torch.rand((B, D), device=dev)
        cos, sin = ang.cos().to(bf), ang.sin().to(bf)
        return (lambda: ops.decode_prologue(qi, kn, vn, qo, slab[:, 0], slab[:, 1], q_norm_w=qw, k_norm_w=kwn,
                                            cos=cos, sin=sin, **kw)), (lambda: int(err.item()) == 0)
    cases.append(("kv_append", "kv_append_kernel", "latency", 2 * 4 * 8 * 128 * (2 + 2), lambda: append_setup(False),
                  "one decode token of B 4 x 8 kv heads x d128, bf16, host-directed destinations"))
    cases.append(("decode_prologue", "decode_prologue_kernel", "latency",
                  4 * (64 + 2 * 8) * 128 * 2 * 2 + 2 * 4 * 128 * 2, lambda: append_setup(True),
                  "q/k RMSNorm + RoPE + q write + K/V append, B 4, 64q/8kv, d128, bf16"))

    def norm_setup():
        x = torch.randn((16384, 5120), device=dev).to(bf)
        w = (torch.rand(5120, device=dev) + 0.5).to(bf)
        y = torch.empty_like(x)
        return (lambda: ops.rmsnorm(x, w, 1e-6, out=y)), (lambda: bool(torch.isfinite(y).all()))
    cases.append(("rmsnorm", "rmsnorm_kernel", "hbm", 2 * 16384 * 5120 * 2 + 5120 * 2, norm_setup,
                  "16384 rows x 5120, bf16 (a prefill-sized norm)"))

    def prefill_setup():
        Hkv, D, P, S = 8, 128, 64, 32768
        K = torch.randn((1, Hkv, S, D), device=dev).to(bf)
        V = torch.randn((1, Hkv, S, D), device=dev).to(bf)
        slab = torch.empty((S // P, 2, Hkv, P, D), dtype=bf, device=dev)
        perm = np.random.default_rng(0).permutation(S // P)
        pages = [(int(perm[i]), i * P, P) for i in range(S // P)]
        err = torch.zeros(1, dtype=torch.int32, device=dev)

        def call():
            ops.kv_write_pages(K, V, slab[:, 0], slab[:, 1], pages, page_stride=2 * Hkv * P * D, head_stride=P * D,
                               num_pool_pages=S // P, page_size=P, error_flag=err)
        return call, lambda: int(err.item()) == 0 and torch.equal(slab[int(perm[3]), 0, 2], K[0, 2, 3 * P:4 * P])
    cases.append(("kv_write_pages", "prefill_pages_kernel", "hbm", 2 * 2 * 8 * 32768 * 128 * 2, prefill_setup,
                  "one 32768-token prompt, 8 kv heads, d128, bf16, into 512 scattered pool slots"))

    PB = 2 * 8 * 64 * 128 * 2          # one config-5 page (K and V of 8 heads), 256 KiB

    def host_setup(to_host):
        n = 1024
        dslab = torch.randn((n, PB // 2), device=dev).to(bf)
        hslab = torch.empty((n, PB // 2), dtype=bf, pin_memory=True)
        ids = np.random.default_rng(1).permutation(n).astype(np.int32)
        if to_host:
            return (lambda: ops.move_pages(hslab, ids, dslab, np.arange(n, dtype=np.int32), PB)), (lambda: True)
        return (lambda: ops.copy_pages(dslab, 0, hslab, ids, PB)), (lambda: True)
    cases.append(("move_pages", "move_pages_kernel", "host link", 1024 * PB, lambda: host_setup(True),
                  "1024 config-5 pages (256 KiB) device -> pinned host, scattered destinations"))
    cases.append(("copy_pages", "gather_pages_kernel", "host link", 1024 * PB, lambda: host_setup(False),
                  "1024 config-5 pages pinned host -> device, scattered sources"))

    def gemv_setup(Nn, K, M, glu):
        g = torch.Generator(device=dev).manual_seed(5)
        copies = max(1, -(-4 * 126 * 2 ** 20 // (Nn * K))) if M <= 64 else 1   # weights rotate through > 4x L2
        pks = [ops.int8_pack_weight(torch.randint(-127, 128, (Nn, K), generator=g, device=dev, dtype=torch.int8))
               for _ in range(copies)]
        sc = (torch.rand(Nn, generator=g, device=dev) * 0.019 + 0.001).to(bf)
        x = torch.randn((M, K), generator=g, device=dev).to(bf)
        y = torch.empty((M, Nn // 2 if glu else Nn), dtype=bf, device=dev)
        it = [0]

        def call():
            pk = pks[it[0] % copies]
            it[0] += 1
            if glu:
                ops.int8_linear_glu(x, pk, sc, out=y)
            else:
                ops.int8_linear(x, pk, sc, out=y, gemm=M > 64)
        return call, lambda: ops.int8_linear_error() == 0
    cases.append(("int8_gemv", "int8_tma_kernel", "hbm", c2_bytes(8, 12288, 4096),
                  lambda: gemv_setup(12288, 4096, 8, False), "packed INT8 (12288, 4096), M 8, bf16 x"))
    cases.append(("int8_gemv_glu", "int8_tma_kernel (gated)", "hbm",
                  2 * 17408 * 5120 + 2 * 17408 * 2 + 8 * 5120 * 2 + 8 * 17408 * 2,
                  lambda: gemv_setup(2 * 17408, 5120, 8, True),
                  "config-4 MLP gate/up: packed INT8 (2 x 17408, 5120), M 8, silu(g) * u epilogue"))
    cases.append(("int8_gemm", "int8_gemm_tc_kernel", "tensor", 2 * 4096 * 6144 * 4096,
                  lambda: gemv_setup(6144, 4096, 4096, False), "packed INT8 (6144, 4096), M 4096 tokens, bf16 x"))

    def gm_setup():
        rows, D = 256, 128
        rb, fb, cb = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        N.lib().helm_gather_merge_state_bytes(1, rows, D, ctypes.byref(rb), ctypes.byref(fb), ctypes.byref(cb))
        st = torch.zeros(rb.value + fb.value, dtype=torch.uint8, device=dev)
        cnt = torch.zeros(max(cb.value, 4), dtype=torch.uint8, device=dev)
        rec = torch.randn((rows, D + 2), device=dev)
        rec[:, D + 1] = 1.0
        out = torch.empty((rows, D), device=dev)
        err = torch.zeros(1, dtype=torch.int32, device=dev)
        p = N.GatherMergeParams()
        p.rank, p.world, p.rows, p.D = 0, 1, rows, D
        p.record = rec.data_ptr()
        p.peer_recv[0], p.peer_flags[0] = st.data_ptr(), st.data_ptr() + rb.value
        p.recv_local, p.flags_local = st.data_ptr(), st.data_ptr() + rb.value
        p.counters = cnt.data_ptr()
        p.out, p.out_dtype, p.error_flag = out.data_ptr(), N.F32, err.data_ptr()
        p.wait_ns = 10_000_000
        keep = (st, cnt, rec, out, err, p)

        def call():
            N.check("helm_gather_merge", N.lib().helm_gather_merge(ctypes.byref(keep[5]),
                                                                  torch.cuda.current_stream(dev).cuda_stream))
        return call, lambda: int(err.item()) == 0
    cases.append(("gather_merge", "gather_merge_kernel", "latency", 2 * 256 * 130 * 4 + 256 * 128 * 4, gm_setup,
                  "one rank's exchange of 256 rows x (128 + 2) at world 1 (push into its own slot, merge): the "
                  "kernel's local half; the NVLink half runs only under multi-rank launches"))
    return cases


def run_kernels(args, rank, local, world):
    """Every kernel family once, at a size that shows its bound, timed with CUDA events over CUDA
    graphs; one JSON line with a row per kernel (achieved GB/s or TFLOP/s against the measured peak).
    `--kernel NAME` limits it to one case (ncu captures)."""
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.current_stream(dev)
    hbm, hkind = peaks()
    tf_peak, tkind = bf16_peak()
    rows = []
    for name, kern, bound, work, setup, what in kernel_cases(dev):
        if args.kernel and name != args.kernel:
            continue
        call, check = setup()
        reps = 3 if bound == "host link" else max(5, min(args.steps, 50))
        ms, how = _graph_time_ms(call, reps, stream, warm=max(3, args.warmup))
        ok = bool(check())
        row = {"case": name, "kernel": kern, "bound": bound, "what": what, "us": round(ms * 1e3, 2),
               "timing": how, "ok": ok}
        if bound == "tensor":
            tf = work / (ms * 1e-3) / 1e12
            row.update(flops=work, tflops=round(tf, 1), frac=round(tf / tf_peak, 3))
        else:
            gbs = work / (ms * 1e-3) / 1e9
            row.update(bytes=work, gbs=round(gbs, 1), frac=round(gbs / hbm, 3) if bound != "host link" else None)
        rows.append(row)
        del call, check
        torch.cuda.empty_cache()
    if rank == 0:
        hb = [r for r in rows if r["bound"] == "hbm"]
        agg = sum(r["bytes"] for r in hb) / max(1e-12, sum(r["us"] for r in hb) * 1e-6) / 1e9 if hb else None
        print(json.dumps({"metric": "per-kernel achieved GB/s (TFLOP/s for the GEMM), algorithmic bytes / CUDA-event "
                                    "time", "value": agg, "unit": "GB/s (HBM-bound cases, aggregate)",
                          "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "higher_is_better": True,
                          "scaling": "weak", "vs_baseline": None, "dtype": "per case", "data": "synthetic",
                          "config": {"workload": "one call of every kernel family (REDUCED sizes, profiling table)",
                                     "l2": "bandwidth-bound inputs > 126 MB"},
                          "peaks": {"hbm_gbs": hbm, "hbm_kind": hkind, "bf16_tflops": tf_peak, "bf16_kind": tkind},
                          "cases": rows, "cpu_baseline": None, "e2e": None}), flush=True)


def c2_reference_time(min_seconds=2.0):
    """The reference's own AVX2 fp16 GEMV (helm/kernels/fp16_gemv.cpp, built into oracle/_ref) on the
    fp16-dequantised config-2 weights, every shape and M; median seconds per call."""
    from oracle.build_ref import load
    from oracle.cpu_baseline import host_threads
    mod = load()
    threads = host_threads()
    torch.set_num_threads(threads)
    out, tot_bytes, tot_s = [], 0, 0.0
    for (Nn, K) in C2_SHAPES:
        g = torch.Generator().manual_seed(0)
        w = torch.randint(-127, 128, (Nn, K), generator=g, dtype=torch.int8)
        s = (torch.rand(Nn, generator=g) * 0.019 + 0.001).to(torch.float16)
        wf = (w.float() * s.float()[:, None]).to(torch.float16).contiguous()
        for M in C2_ROWS:
            x = torch.randn(M, K, generator=g).to(torch.float16)
            mod.helm_fp16_linear(x, wf)
            ts = []
            t_end = time.perf_counter() + min_seconds
            while time.perf_counter() < t_end or len(ts) < 3:
                t0 = time.perf_counter()
                mod.helm_fp16_linear(x, wf)
                ts.append(time.perf_counter() - t0)
            t = statistics.median(ts)
            tot_bytes += c2_bytes(M, Nn, K)
            tot_s += t
            out.append({"N": Nn, "K": K, "M": M, "us": round(t * 1e6, 1)})
    return tot_bytes, tot_s, out, threads


def cpu_baseline_config2():
    tot_bytes, tot_s, cases, threads = c2_reference_time(min_seconds=1.0)
    return {"value": tot_bytes / tot_s / 1e9, "unit": "GB/s", "cores": threads, "kind": "reference",
            "sample": ("reference helm_fp16_linear (fp16_gemv.cpp, compiled from the reference source) on the "
                       "fp16-dequantised weights, the 9 config-2 calls, median of >= 1 s each; value = the int8 "
                       "path's algorithmic bytes / the reference's time for the same GEMVs"),
            "cases": cases}


def run_reference_config2(args, rank):
    if rank != 0:
        return
    tot_bytes, tot_s, cases, threads = c2_reference_time(min_seconds=1.0)
    v = tot_bytes / tot_s / 1e9
    line = {"impl": "reference", "metric": C2_METRIC, "value": v, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": 1, "warmup": 1, "ms_per_step": tot_s * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "fp16 x fp16 -> fp32", "data": "synthetic",
            "config": {"workload": C2_WORKLOAD, "parallelism": "host cores"}, "cases": cases,
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads, "kind": "reference",
                             "sample": "helm_fp16_linear on the dequantised weights, 9 calls, median >= 1 s each"},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# config 1: the reference's own CPU case -- one layer, 4096 fp32 tokens, half of the pages on the host
# ----------------------------------------------------------------------------
C1 = dict(Hq=32, Hkv=8, D=128, P=64, ctx=4096, offloaded=32)
C1_METRIC = "single-layer paged decode attention: algorithmic GB/s (config1, fp32, 32 of 64 pages host-resident)"
C1_WORKLOAD = ("config1: batch 1, 32q/8kv heads, d128, 4096 fp32 tokens in 64-token pages, first 32 pages offloaded "
               "to pinned host memory, scale 1/sqrt(128), seed 0")
C1_BYTES = 2 * C1["Hkv"] * C1["ctx"] * C1["D"] * 4 + C1["Hq"] * C1["D"] * 4 * 2


def _c1_manager(dev, seed):
    from helm_b200.runtime import KVAllocator, KVCacheManager
    c = C1
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(1, c["Hq"], 1, c["D"], generator=g)
    k = torch.randn(1, c["Hkv"], c["ctx"], c["D"], generator=g)
    v = torch.randn(1, c["Hkv"], c["ctx"], c["D"], generator=g)
    alloc = KVAllocator(num_layers=1, num_kv_heads=c["Hkv"], head_dim=c["D"], page_size=c["P"], dtype=torch.float32)
    mgr = KVCacheManager(alloc, gpu_high_watermark_bytes=1 << 62)
    mgr.append_prefill(0, k.to(dev), v.to(dev))
    return q.to(dev), alloc, mgr


def run_config1(args, rank, local, world):
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    init_pg(world, local)
    line = config1_line(args, rank, world, dev)
    if rank == 0:
        print(json.dumps(line), flush=True)
    barrier(world)


def config1_line(args, rank, world, dev):
    """perform_streaming_attention (the drop-in call) on the reference's config 1: pages 0-31 evicted
    to pinned host memory through KVCacheManager.evict_pages, pages 32-63 resident; every call stages
    the host pages into device slots and attends over all 64.  Also the kernel alone on 8 all-resident
    instances (rotating through > 2x L2), from prebuilt device page tables in a CUDA graph.  Returns
    the JSON record (rank 0; None elsewhere)."""
    from helm_b200 import ops
    from helm_b200.runtime import perform_streaming_attention
    stream = torch.cuda.current_stream(dev)
    local = dev.index
    c = C1
    clocks = ClockSampler(gpu_selector(dev, local))
    clocks.start()
    t_load0 = time.time()
    # --- the drop-in call with half of the pages on the host ---
    q, alloc, mgr = _c1_manager(dev, 0)
    page_bytes = 2 * c["Hkv"] * c["P"] * c["D"] * 4
    mgr.evict_pages(c["offloaded"] * page_bytes)
    pages = mgr.iterate_layer_pages(0)
    n_cpu = sum(p.state == "CPU" for p in pages)
    for _ in range(max(args.warmup, 3)):
        perform_streaming_attention(q, pages)
    torch.cuda.synchronize(dev)
    steps = max(args.steps, 10)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        out = perform_streaming_attention(q, pages)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    mixed_ms = e0.elapsed_time(e1) / steps
    # e2e: q from pinned host memory, the output read back every call
    q_h = q.cpu().pin_memory()
    o_h = torch.empty(q.shape, dtype=q.dtype).pin_memory()
    e0.record(stream)
    for _ in range(steps):
        o_h.copy_(perform_streaming_attention(q_h.to(dev, non_blocking=True), pages), non_blocking=True)
    e1.record(stream)
    torch.cuda.synchronize(dev)
    e2e_ms = e0.elapsed_time(e1) / steps
    # --- the kernel alone: 8 all-resident instances, prebuilt tables, CUDA graph ---
    inst = []
    for i in range(8):
        qi, alloc_i, mgr_i = _c1_manager(dev, 100 + i)
        store = alloc_i.store(dev)
        pl = mgr_i.iterate_layer_pages(0)
        pt = torch.tensor([[p.slot for p in pl]], dtype=torch.int32, device=dev)
        pu = torch.tensor([[p.used_tokens for p in pl]], dtype=torch.int32, device=dev)
        npg = torch.tensor([len(pl)], dtype=torch.int32, device=dev)
        kb, vb = store.base_ptrs()
        inst.append((qi.view(1, c["Hq"], c["D"]).contiguous(), store, pt, pu, npg, alloc_i, mgr_i))
    outs = [torch.empty(1, c["Hq"], c["D"], device=dev) for _ in inst]

    def calls():
        for (qi, store, pt, pu, npg, _, _), o in zip(inst, outs):
            ops.paged_decode_attention(qi, store.slab[:, 0], store.slab[:, 1], pt, pu, npg, num_kv_heads=c["Hkv"],
                                       page_size=c["P"], page_stride=store.page_elems, head_stride=store.head_stride,
                                       num_pool_pages=store.capacity, out=o)
    for _ in range(3):
        calls()
    torch.cuda.synchronize(dev)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        calls()
    graph.replay()
    torch.cuda.synchronize(dev)
    reps = max(args.steps // 5, 5)
    e0.record(stream)
    for _ in range(reps):
        graph.replay()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    kern_ms = e0.elapsed_time(e1) / (reps * len(inst))
    del graph
    clk = clocks.stop(t_load0, time.time())
    if rank == 0:
        hbm_peak, peak_kind = peaks()
        gbs = C1_BYTES / (mixed_ms * 1e-3) / 1e9
        kgbs = C1_BYTES / (kern_ms * 1e-3) / 1e9
        cpu = None
        if not args.no_cpu_baseline:
            from oracle.cpu_baseline import time_decode_attention
            t2, n2, threads = time_decode_attention(c["Hq"], c["Hkv"], c["D"], c["P"], c["ctx"], torch.float32,
                                                    path=2, min_seconds=3.0, max_calls=30)
            t3, n3, _ = time_decode_attention(c["Hq"], c["Hkv"], c["D"], c["P"], c["ctx"], torch.float32,
                                              path=3, min_seconds=3.0, max_calls=30)
            cpu = {"value": C1_BYTES / t2 / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
                   "sample": (f"reference all-CPU path (kv_cache.py:376-380) ported, config 1, median of {n2} calls "
                              f"({t2 * 1e3:.2f} ms); its Path-3 loop (kv_cache.py:387-442): {t3 * 1e3:.2f} ms")}
        line = {
            "metric": C1_METRIC, "value": gbs, "unit": "GB/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": mixed_ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "timing": "perform_streaming_attention per call (host pages staged every call), CUDA events",
            "config": {"workload": C1_WORKLOAD, "parallelism": "single GPU",
                       "l2": "mixed path: host pages cross PCIe every call; kernel-only: 8 instances (268 MB)"},
            "pages_on_host": n_cpu, "h2d_bytes_per_call": n_cpu * page_bytes,
            "kernel_only": {"ms": kern_ms, "gbs": kgbs, "frac": kgbs / hbm_peak,
                            "how": "all 64 pages resident, 8 instances rotating, CUDA graph"},
            "roofline": {"bound": "hbm", "achieved": kgbs, "peak": hbm_peak, "unit": "GB/s", "frac": kgbs / hbm_peak,
                         "traffic": None, "peak_kind": peak_kind,
                         "kernel": "paged attention (fp32 pages: attn_generic_kernel path), kernel-only timing",
                         "bytes_per_launch": C1_BYTES, "avg_launch_ms": kern_ms},
            "cpu_baseline": cpu,
            "e2e": {"value": C1_BYTES / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step":
                    q_h.numel() * 4 + n_cpu * page_bytes, "d2h_bytes_per_step": o_h.numel() * 4, "ms_per_step": e2e_ms,
                    "api": "helm_b200.runtime.perform_streaming_attention, q from pinned host, output read back"},
            "gpu_launches": None,
            "clocks": clk,
        }
        return line
    return None


def run_reference_config1(args, rank):
    if rank != 0:
        return
    from oracle.cpu_baseline import time_decode_attention
    c = C1
    t2, n2, threads = time_decode_attention(c["Hq"], c["Hkv"], c["D"], c["P"], c["ctx"], torch.float32, path=2,
                                            min_seconds=3.0, max_calls=max(args.steps, 20))
    v = C1_BYTES / t2 / 1e9
    line = {"impl": "reference", "metric": C1_METRIC, "value": v, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": n2, "warmup": 1, "ms_per_step": t2 * 1e3, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": C1_WORKLOAD, "parallelism": "host cores"},
            "cpu_baseline": {"value": v, "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": f"reference all-CPU path ported, median of {n2} calls"},
            "e2e": {"value": v, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------------------
# config 3: a Qwen3-8B-shaped decode step through KVOffloadManager (bf16, batch 1, 16384 tokens)
# ----------------------------------------------------------------------------
C3 = dict(layers=36, hidden=4096, heads=32, kv_heads=8, head_dim=128, inter=12288, vocab=151936, ctx=16384)
C3_METRIC = "decode tok/s, Qwen3-8B-shaped model through KVOffloadManager (config3, bf16, batch 1, 16384-token paged KV)"
C3_WORKLOAD = ("config3: random-init Qwen3-8B-shaped decoder (36 layers, hidden 4096, 32/8 heads, d128, SwiGLU "
               "12288, vocab 151936), bf16, batch 1, 16384-token paged KV (64-token pages, cont_capacity=0)")


def c3_step_bytes(model, ctx):
    """Algorithmic HBM bytes of one decode step: every weight except the embedding table read once
    (one embedding row), plus K+V of every cached token of every layer."""
    c = C3
    tensors = list(model.named_parameters()) + [(n, b) for n, b in model.named_buffers() if "rotary" not in n]
    w = sum(t.numel() * t.element_size() for n, t in tensors if "embed_tokens" not in n)
    kv = 2 * c["layers"] * c["kv_heads"] * c["head_dim"] * 2 * ctx
    return w + c["hidden"] * 2 + kv


def run_config3(args, rank, local, world):
    """Decode steps of a random-init Qwen3-8B-shaped HF model whose attention forwards are patched by
    KVOffloadManager (paged mode): prefill 16384 random tokens, then greedy decode one token per
    step, the token fed back on the device.  `value` times K steps with CUDA events (the host-side
    runtime included: this path is not graph-captured); `e2e` also reads every token back to the host."""
    import transformers
    from helm_b200.runtime import KVOffloadConfig, KVOffloadManager
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    init_pg(world, local)
    stream = torch.cuda.current_stream(dev)
    c = C3
    cfg = transformers.Qwen3Config(vocab_size=c["vocab"], hidden_size=c["hidden"], intermediate_size=c["inter"],
                                   num_hidden_layers=c["layers"], num_attention_heads=c["heads"],
                                   num_key_value_heads=c["kv_heads"], head_dim=c["head_dim"], rope_theta=1e6,
                                   max_position_embeddings=40960, rms_norm_eps=1e-6, tie_word_embeddings=False)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    with torch.device(dev):
        model = transformers.Qwen3ForCausalLM(cfg).eval()
    torch.set_default_dtype(prev)
    # config 3 keeps the whole KV on the device (the reference's default watermark, 512 tokens per
    # layer, is sized for consumer GPUs and would stream the rest over PCIe every step)
    mgr = KVOffloadManager(model, KVOffloadConfig.from_model(model, page_size=64, cont_capacity=0,
                                                             gpu_watermark_bytes=1 << 40), batch_size=1,
                           fused_norms=True)
    ctx = c["ctx"]
    g = torch.Generator(device=dev).manual_seed(0)
    ids = torch.randint(0, c["vocab"], (1, ctx), generator=g, device=dev)
    clocks = ClockSampler(gpu_selector(dev, local))
    clocks.start()
    t_load0 = time.time()
    with torch.no_grad():
        mask = torch.full((ctx, ctx), torch.finfo(torch.bfloat16).min, device=dev, dtype=torch.bfloat16).triu_(1)
        logits = model(input_ids=ids, attention_mask=mask[None, None], position_ids=torch.arange(ctx, device=dev)[None],
                       use_cache=False, logits_to_keep=1).logits
        del mask
        tok = logits[:, -1:].argmax(-1)
        pos = ctx

        def step(tok, pos):
            m = torch.zeros((1, 1, 1, pos + 1), device=dev, dtype=torch.bfloat16)
            lg = model(input_ids=tok, attention_mask=m, position_ids=torch.tensor([[pos]], device=dev),
                       use_cache=False, logits_to_keep=1).logits
            return lg[:, -1:].argmax(-1)
        for _ in range(max(args.warmup, 3)):
            tok = step(tok, pos)
            pos += 1
        torch.cuda.synchronize(dev)
        steps = min(max(args.steps, 10), 100)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            tok = step(tok, pos)
            pos += 1
        e1.record(stream)
        torch.cuda.synchronize(dev)
        eager_ms = e0.elapsed_time(e1) / steps
        # the same decode with the whole step captured in a CUDA graph (DecodeGraph)
        from helm_b200.runtime.graph import DecodeGraph
        dg = DecodeGraph(mgr, model)
        for _ in range(max(args.warmup, 3)):
            tok = dg.step(tok)[:, -1:].argmax(-1)
            pos += 1
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(steps):
            tok = dg.step(tok)[:, -1:].argmax(-1)
            pos += 1
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / steps
        ctx_mid = pos - steps // 2
        # e2e: the token read back to the host every step (what a serving loop does)
        e0.record(stream)
        for _ in range(steps):
            tok = dg.step(tok)[:, -1:].argmax(-1)
            pos += 1
            tok_host = int(tok.item())
        e1.record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms = e0.elapsed_time(e1) / steps
        dg.close()
        # the same model with INT8 weight-only linears (patch_int8_linears), same cache
        bf16_bytes = c3_step_bytes(model, ctx_mid)
        from helm_b200.kernels import patch_int8_linears
        n_int8 = patch_int8_linears(model)
        torch.cuda.empty_cache()
        dg = DecodeGraph(mgr, model)
        for _ in range(3):
            tok = dg.step(tok)[:, -1:].argmax(-1)
            pos += 1
        torch.cuda.synchronize(dev)
        e0.record(stream)
        for _ in range(steps):
            tok = dg.step(tok)[:, -1:].argmax(-1)
            pos += 1
        e1.record(stream)
        torch.cuda.synchronize(dev)
        int8_ms = e0.elapsed_time(e1) / steps
        dg.close()
        int8_bytes = c3_step_bytes(model, pos - steps // 2)
    clk = clocks.stop(t_load0, time.time())
    err = int(mgr.batch.error_flag.item()) if getattr(mgr, "batch", None) is not None else 0
    rep = mgr.report()
    mgr.restore()
    if rank == 0:
        hbm_peak, peak_kind = peaks()
        tok_s = 1.0 / (ms * 1e-3)
        ach = bf16_bytes / (ms * 1e-3) / 1e9
        line = {
            "metric": C3_METRIC, "value": tok_s, "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16", "data": "synthetic (random-init weights, random token ids)",
            "timing": ("DecodeGraph: the whole decode step (model.forward with the KVOffloadManager patches, "
                       "fused decode prologue and fused RMSNorm) captured in one CUDA graph and replayed per "
                       "token, host bookkeeping mirrored after each replay; CUDA events"),
            "eager": {"ms_per_step": eager_ms, "tok_s": 1.0 / (eager_ms * 1e-3),
                      "how": "the same model.forward called eagerly per token"},
            "config": {"workload": C3_WORKLOAD, "model": "Qwen3-8B-shaped (random init)", "global_batch": 1,
                       "seq_len": ctx, "parallelism": "single GPU", "l2": "weights 15 GB + KV per step >> L2"},
            "roofline": {"bound": "hbm", "achieved": ach, "peak": hbm_peak, "unit": "GB/s", "frac": ach / hbm_peak,
                         "traffic": None, "peak_kind": peak_kind,
                         "kernel": "whole decode step (weights + KV of every layer read once)",
                         "bytes_per_step": bf16_bytes},
            "int8_linears": {"replaced": n_int8, "ms_per_step": int8_ms, "tok_s": 1.0 / (int8_ms * 1e-3),
                             "algorithmic_gbs": int8_bytes / (int8_ms * 1e-3) / 1e9},
            "cpu_baseline": None,
            "e2e": {"value": 1.0 / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": 8,
                    "d2h_bytes_per_step": 8, "ms_per_step": e2e_ms,
                    "api": "DecodeGraph.step (model.forward with KVOffloadManager patches); the token read back every step"},
            "gpu_launches": None, "clocks": clk, "device_error_flag": err, "kv_report": rep,
        }
        print(json.dumps(line, default=str), flush=True)
    del model
    barrier(world)


def run_reference_config3(args, rank):
    if rank != 0:
        return
    print(json.dumps({"impl": "reference", "unavailable": "config 3 is a full 8B-parameter model decode; the "
                      "reference's CPU path is infeasible at this size on the host cores (its per-layer CPU "
                      "attention is timed by --workload config1 and config5)"}), flush=True)


# ----------------------------------------------------------------------------
# config 4: Qwen3-14B-shaped, INT8 linears, batch 8, 32768 tokens per sequence, half the KV on the host
# ----------------------------------------------------------------------------
C4 = dict(layers=40, hidden=5120, heads=40, kv_heads=8, head_dim=128, inter=17408, vocab=151936, ctx=32768, batch=8)
C4_METRIC = ("decode tok/s, Qwen3-14B-shaped INT8 model through KVOffloadManager (config4, batch 8, 32768-token "
             "paged KV per sequence, oldest 50% of the pages in pinned host memory)")


def run_config4(args, rank, local, world):
    """Decode steps of a random-init Qwen3-14B-shaped model with INT8 weight-only linears
    (patch_int8_linears) through KVOffloadManager: every sequence holds 32768 cached tokens, filled
    with seeded K/V through KVCacheManager.append_prefill under a GPU watermark of half the KV, so
    the reference's eviction policy moves the oldest half of every sequence's pages to pinned host
    memory; each decode step then stages those host pages back through the device (the reference's
    mixed-residency path), layer by layer.  With N > 1 the pages are sharded by sequence position
    over the ranks (KVShardGroup) and every rank holds 1/N of them."""
    import transformers
    from helm_b200.kernels import patch_int8_linears
    from helm_b200.runtime import KVOffloadConfig, KVOffloadManager
    from helm_b200.runtime.sharded import KVShardGroup, shard_bounds
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    init_pg(world, local)
    stream = torch.cuda.current_stream(dev)
    c = C4
    B, L, ctx = c["batch"], c["layers"], c["ctx"]
    cfg = transformers.Qwen3Config(vocab_size=c["vocab"], hidden_size=c["hidden"], intermediate_size=c["inter"],
                                   num_hidden_layers=L, num_attention_heads=c["heads"],
                                   num_key_value_heads=c["kv_heads"], head_dim=c["head_dim"], rope_theta=1e6,
                                   max_position_embeddings=40960, rms_norm_eps=1e-6, tie_word_embeddings=False)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(0)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    with torch.device(dev):
        model = transformers.Qwen3ForCausalLM(cfg).eval()
    torch.set_default_dtype(prev)
    n_int8 = patch_int8_linears(model)
    torch.cuda.empty_cache()
    P, Hkv, D = 64, c["kv_heads"], c["head_dim"]
    page_bytes = 2 * Hkv * P * D * 2
    plo, phi = shard_bounds(ctx // P, rank, world)
    local_pages = phi - plo
    kv_bytes = L * B * local_pages * page_bytes
    group = KVShardGroup(B * c["heads"], D, dev) if world > 1 else None
    mgr = KVOffloadManager(model, KVOffloadConfig.from_model(model, page_size=P, cont_capacity=0,
                                                             gpu_watermark_bytes=kv_bytes // 2),
                           batch_size=B, shard_group=group, fused_norms=True)
    alloc = mgr.allocator
    alloc.reserve_capacity(dev, L * B * (local_pages // 2 + 8) + B * local_pages + 1024)
    alloc.reserve_capacity(torch.device("cpu"), L * B * (local_pages // 2 + 8))
    g = torch.Generator(device=dev).manual_seed(100 + rank)
    t_fill = time.time()
    with torch.no_grad():
        for l in range(L):
            for b in range(B):
                K = torch.randn((1, Hkv, local_pages * P, D), generator=g, device=dev, dtype=torch.bfloat16)
                V = torch.randn((1, Hkv, local_pages * P, D), generator=g, device=dev, dtype=torch.bfloat16)
                mgr.kvcms[b].append_prefill(l, K, V)
        del K, V
        torch.cuda.synchronize(dev)
        t_fill = time.time() - t_fill
        rep0 = mgr.report()
        host_pages = rep0["active_cpu_pages"]
        clocks = ClockSampler(gpu_selector(dev, local))
        clocks.start()
        t_load0 = time.time()
        gt = torch.Generator(device=dev).manual_seed(7)

        def step(pos):
            ids = torch.randint(0, c["vocab"], (B, 1), generator=gt, device=dev)
            m = torch.zeros((B, 1, 1, pos + 1), device=dev, dtype=torch.bfloat16)
            return model(input_ids=ids, attention_mask=m, position_ids=torch.full((B, 1), pos, device=dev),
                         use_cache=False, logits_to_keep=1).logits
        pos = ctx
        for _ in range(max(1, min(args.warmup, 2))):
            step(pos)
            pos += 1
        torch.cuda.synchronize(dev)
        barrier(world)
        steps = max(2, min(args.steps, 5))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            lg = step(pos)
            pos += 1
        e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = max_over_ranks(e0.elapsed_time(e1), world, dev) / steps
        # e2e: the next tokens read back to the host every step
        e0.record(stream)
        for _ in range(steps):
            lg = step(pos)
            pos += 1
            tok_host = lg[:, -1].argmax(-1).cpu()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        e2e_ms = max_over_ranks(e0.elapsed_time(e1), world, dev) / steps
    clk = clocks.stop(t_load0, time.time())
    err = int(mgr.batch.error_flag.item())
    rep = mgr.report()
    mgr.restore()
    if group is not None:
        group.close()
    if rank == 0:
        hbm_peak, peak_kind = peaks()
        w_bytes = sum(t.numel() * t.element_size() for n, t in list(model.named_parameters()) +
                      list(model.named_buffers()) if "embed_tokens" not in n and "rotary" not in n)
        host_bytes = host_pages * page_bytes          # streamed from the host every step
        dev_kv = (L * B * local_pages - host_pages) * page_bytes
        hbm_bytes = w_bytes + dev_kv + 2 * host_bytes   # staged pages are written, then read, on the device
        line = {
            "metric": C4_METRIC, "value": B / (ms * 1e-3) * 1.0, "unit": "tok/s", "n_gpus": world, "steps": steps,
            "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "bf16 activations, int8 weights", "data": "synthetic (random-init "
            "weights, seeded K/V, random token ids)",
            "timing": "eager model.forward per token (mixed residency: host pages staged every layer), CUDA events",
            "config": {"workload": "config4: random-init Qwen3-14B-shaped decoder (40 layers, hidden 5120, 40/8 "
                                   "heads, d128, SwiGLU 17408), INT8 weight-only linears, batch 8, 32768-token paged "
                                   "KV per sequence, oldest 50% of pages in pinned host memory",
                       "model": "Qwen3-14B-shaped (random init)", "global_batch": B, "seq_len": ctx,
                       "parallelism": f"kv-seq-shard{world}", "l2": "weights 14 GB + KV >> L2"},
            "int8_linears": n_int8, "fill_seconds": round(t_fill, 1),
            "pages_on_host": host_pages, "host_bytes_per_step": host_bytes,
            "pcie_gbs": host_bytes / (ms * 1e-3) / 1e9,
            "roofline": {"bound": "host link (PCIe) for the offloaded half; HBM for the rest",
                         "achieved": hbm_bytes / (ms * 1e-3) / 1e9, "peak": hbm_peak, "unit": "GB/s",
                         "frac": hbm_bytes / (ms * 1e-3) / 1e9 / hbm_peak, "traffic": None, "peak_kind": peak_kind,
                         "bytes_per_step": hbm_bytes},
            "cpu_baseline": None,
            "e2e": {"value": B / (e2e_ms * 1e-3), "unit": "tok/s", "h2d_bytes_per_step": 8 * B + host_bytes,
                    "d2h_bytes_per_step": 8 * B, "ms_per_step": e2e_ms,
                    "api": "model.forward with KVOffloadManager patches (INT8 linears); tokens read back each step"},
            "gpu_launches": None, "clocks": clk, "device_error_flag": err, "kv_report": rep,
        }
        print(json.dumps(line, default=str), flush=True)
    del model
    barrier(world)
    if world > 1:
        import torch.distributed as dist
        dist.destroy_process_group()


def cpu_baseline():
    from oracle.cpu_baseline import time_decode_attention
    c = CFG
    t, n, threads = time_decode_attention(c["q_heads"], c["kv_heads"], c["head_dim"], c["page"], c["ctx"],
                                          torch.bfloat16, path=2, min_seconds=8.0, max_calls=3)
    step_s = t * c["layers"] * c["batch"]
    return {"value": c["batch"] / step_s, "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": (f"reference all-CPU attention path (kv_cache.py:376-380, torch CPU, ported) on 1 layer x "
                       f"1 sequence at {c['ctx']} tokens, median of {n} calls ({t * 1e3:.0f} ms), "
                       f"extrapolated x{c['layers'] * c['batch']} to one decode step")}


def main():
    args = parse()
    rank, local, world = dist_setup(args.gpus)
    if args.workload == "config2":
        if args.impl == "reference":
            run_reference_config2(args, rank)
        else:
            run_config2(args, rank, local, world)
        return
    if args.workload == "kernels":
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "a per-kernel table of this library's CUDA "
                                  "kernels has no reference counterpart (the reference has no GPU kernels)"}))
            return
        if rank == 0:
            run_kernels(args, rank, local, world)
        return
    if args.workload == "prefill":
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "the reference has no INT8 GEMM (its linear is "
                                  "the fp16 CPU GEMV, timed by --workload config2)"}))
            return
        dev = torch.device("cuda", local)
        torch.cuda.set_device(dev)
        res = c2_prefill_gemm(args, dev, world)
        if rank == 0:
            flops = sum(2.0 * c["M"] * c["N"] * c["K"] for c in res["cases"])
            ms = sum(c["tcgen05"]["us"] for c in res["cases"]) / 1e3
            tf = flops / (ms * 1e-3) / 1e12
            print(json.dumps({"metric": "int8 weight-only prefill GEMM TFLOP/s (config-2 weights, M=4096)",
                              "value": tf, "unit": "TFLOP/s", "n_gpus": world, "steps": 30, "warmup": 3,
                              "ms_per_step": ms, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                              "dtype": "bf16 x int8 -> fp32", "data": "synthetic",
                              "config": {"workload": "the three config-2 weights at M=4096 tokens"},
                              "roofline": {"bound": "tensor", "achieved": tf, "peak": res["peak_tflops"],
                                           "unit": "TFLOP/s", "frac": tf / res["peak_tflops"], "traffic": None,
                                           "peak_kind": res["peak_kind"], "kernel": "int8_gemm_tc_kernel"},
                              "cases": res["cases"], "cpu_baseline": None, "e2e": None}), flush=True)
        return
    if args.workload == "config1":
        if args.impl == "reference":
            run_reference_config1(args, rank)
        else:
            run_config1(args, rank, local, world)
        return
    if args.workload == "config3":
        if args.impl == "reference":
            run_reference_config3(args, rank)
        else:
            run_config3(args, rank, local, world)
        return
    if args.workload == "config4":
        if args.impl == "reference":
            if rank == 0:
                print(json.dumps({"impl": "reference", "unavailable": "config 4 is a full 14B-parameter model "
                                  "decode with 43 GB of KV; the reference's CPU path is infeasible at this size"}))
        else:
            run_config4(args, rank, local, world)
        return
    if args.impl == "reference":
        run_reference(args, rank)
        return
    run_helm(args, rank, local, world)


if __name__ == "__main__":
    main()
