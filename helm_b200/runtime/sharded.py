"""KV sequence sharding over the GPUs of one node (one process per GPU).

No counterpart in HELM (its runtime is single-process).  Rank g of G holds
pages [g*n/G, (g+1)*n/G) of every sequence and layer; the last rank holds the
tail and receives new tokens.  Per layer every rank runs the paged attention
over its pages into a merged record (o, m, l) per (sequence, query head), and
KVShardGroup.gather_merge exchanges those records and merges them so every
rank ends with the same attention output.

Three exchanges are provided:
* "fused" (default): inside the attention kernel itself (helm_paged_attn_decode
  with params.exchange): the CTA that completes a (sequence, kv head) pair
  stores the pair's record into every other rank's receive buffer over NVLink
  (CUDA IPC mappings) as 64-bit (value, epoch) words, waits for the other
  ranks' words and merges them -- the collective overlaps the tail of the
  attention, and no extra launch runs;
* "p2p": helm_gather_merge, the same exchange as a separate kernel after the
  attention (used when the attention cannot run the persistent kernel);
* "split": the attention's split path in records-only mode (its split records
  stay in the workspace), then helm_gather_merge merging those records and
  exchanging them in one launch: the lower fixed cost of the split path, two
  launches per layer;
* "nccl": torch.distributed.all_gather_into_tensor + helm_lse_merge.
"""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch

from .. import _native as N
from .. import ops


def shard_bounds(n: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous share [lo, hi) of n items (pages) for `rank`: floor(n*g/G) .. floor(n*(g+1)/G)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} / world {world}")
    return (n * rank) // world, (n * (rank + 1)) // world


class KVShardGroup:
    def __init__(self, rows: int, head_dim: int, device, group=None, exchange: str = "fused",
                 wait_s: float = 0.0):
        """rows = B*Hq records of head_dim dims per exchange.  wait_s bounds each device-side wait
        for the peers' records (0: the library default, 2 s); a wait that runs out sets
        HELM_DEVERR_TIMEOUT in the error word and leaves the affected rows zero."""
        import torch.distributed as dist
        self.group = group
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rows, self.D = rows, head_dim
        self.device = torch.device(device)
        self.exchange = exchange
        self.error_flag = torch.zeros(1, dtype=torch.int32, device=self.device)
        self._bases = []
        self.params = None
        self.xparams_ptr = None
        if self.world > N.MAX_RANKS:
            raise ValueError(f"KVShardGroup: at most {N.MAX_RANKS} ranks")
        if exchange == "nccl" or self.world == 1:
            self.gathered = torch.empty((self.world, rows, head_dim + 2), dtype=torch.float32, device=self.device)
            return
        if exchange not in ("p2p", "fused", "split"):
            raise ValueError(f"unknown exchange {exchange!r}")
        lib = N.lib()
        # state of the separate exchange kernel (helm_gather_merge) ...
        rb, fb, cb = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        if lib.helm_gather_merge_state_bytes(self.world, rows, head_dim, ctypes.byref(rb), ctypes.byref(fb),
                                             ctypes.byref(cb)) < 0:
            N.check("helm_gather_merge_state_bytes", N.ERR_INVALID_ARGUMENT)
        # ... and of the exchange fused into the attention kernel
        xr, xf, xc = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
        if lib.helm_shard_exchange_bytes(self.world, rows, head_dim, ctypes.byref(xr), ctypes.byref(xf),
                                         ctypes.byref(xc)) < 0:
            N.check("helm_shard_exchange_bytes", N.ERR_INVALID_ARGUMENT)
        # receive slots + flags in one allocation each (shared with the peers), counters local
        self.buf = torch.zeros(rb.value + fb.value, dtype=torch.uint8, device=self.device)
        self.counters = torch.zeros(max(cb.value, 4), dtype=torch.uint8, device=self.device)
        self.xbuf = torch.zeros(xr.value + xf.value, dtype=torch.uint8, device=self.device)
        self.xcounters = torch.zeros(max(xc.value, 4), dtype=torch.uint8, device=self.device)
        torch.cuda.synchronize(self.device)
        mine = []
        for t in (self.buf, self.xbuf):
            handle = (ctypes.c_char * 64)()
            off = ctypes.c_int64()
            N.check("helm_ipc_export", lib.helm_ipc_export(t.data_ptr(), handle, ctypes.byref(off)))
            mine.append((bytes(handle), off.value))
        infos = [None] * self.world
        dist.all_gather_object(infos, mine, group=group)
        ptrs = [[0, 0] for _ in range(self.world)]
        for r in range(self.world):
            for i, t in enumerate((self.buf, self.xbuf)):
                if r == self.rank:
                    ptrs[r][i] = t.data_ptr()
                    continue
                h = (ctypes.c_char * 64).from_buffer_copy(infos[r][i][0])
                out_ptr, base = ctypes.c_void_p(), ctypes.c_void_p()
                N.check("helm_ipc_import", lib.helm_ipc_import(h, infos[r][i][1], ctypes.byref(out_ptr),
                                                               ctypes.byref(base)))
                self._bases.append(base.value)
                ptrs[r][i] = out_ptr.value
        p = N.GatherMergeParams()
        p.rank, p.world, p.rows, p.D = self.rank, self.world, rows, head_dim
        x = N.ShardExchange()
        x.rank, x.world = self.rank, self.world
        for r in range(self.world):
            p.peer_recv[r] = ptrs[r][0]
            p.peer_flags[r] = ptrs[r][0] + rb.value
            x.peer_recv[r] = ptrs[r][1]
        p.recv_local = self.buf.data_ptr()
        p.flags_local = self.buf.data_ptr() + rb.value
        p.counters = self.counters.data_ptr()
        p.error_flag = self.error_flag.data_ptr()
        p.wait_ns = x.wait_ns = int(wait_s * 1e9)
        x.recv_local = self.xbuf.data_ptr()
        x.counters = self.xcounters.data_ptr()
        self.params = p
        self.xparams = x
        self.xparams_ptr = ctypes.pointer(x)
        dist.barrier(group=group)

    @property
    def fused(self) -> bool:
        """True when the attention call itself should do the exchange."""
        return self.exchange == "fused" and self.params is not None and self.world > 1

    @property
    def records_only(self) -> bool:
        """True when the attention call should leave its split records for gather_merge to merge."""
        return self.exchange == "split" and self.params is not None and self.world > 1

    def gather_merge(self, record: torch.Tensor, out: Optional[torch.Tensor] = None,
                     out_record: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
        """Exchanges this rank's record [rows, D+2] (fp32), or its S split records [S, rows, D+2]
        (merged first, in the same launch), and writes the merged result to out [rows, D] and/or
        out_record [rows, D+2] on every rank."""
        parts = record.dim() == 3
        if (record.shape[-2:] != (self.rows, self.D + 2) or record.dim() not in (2, 3)
                or record.dtype != torch.float32 or not record.is_contiguous()):
            raise ValueError("gather_merge: record must be contiguous fp32 [rows, D+2] or [S, rows, D+2]")
        if self.world == 1:
            return ops.lse_merge(record if parts else record.unsqueeze(0), out=out, out_record=out_record)
        if self.params is None:
            import torch.distributed as dist
            if parts:
                merged = torch.empty((self.rows, self.D + 2), dtype=torch.float32, device=self.device)
                ops.lse_merge(record, out_record=merged)
                record = merged
            dist.all_gather_into_tensor(self.gathered, record, group=self.group)
            return ops.lse_merge(self.gathered, out=out, out_record=out_record)
        p = self.params
        p.record = record.data_ptr()
        p.num_partials = record.shape[0] if parts else 0
        p.partial_stride = self.rows * (self.D + 2) if parts else 0
        p.out = None if out is None else out.data_ptr()
        p.out_dtype = ops.dtype_code(out.dtype) if out is not None else N.F32
        p.out_record = None if out_record is None else out_record.data_ptr()
        N.check("helm_gather_merge", N.lib().helm_gather_merge(ctypes.byref(p),
                                                               torch.cuda.current_stream(self.device).cuda_stream))
        return out

    def close(self) -> None:
        """Unmaps the peers' buffers (call on every rank, after the last exchange)."""
        import torch.distributed as dist
        if self._bases:
            torch.cuda.synchronize(self.device)
            if dist.is_initialized():
                dist.barrier(group=self.group)
            lib = N.lib()
            for base in self._bases:
                lib.helm_ipc_close(base)
            self._bases = []
            if dist.is_initialized():
                dist.barrier(group=self.group)
        self.params = None
        self.xparams_ptr = None
