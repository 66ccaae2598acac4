"""Restatement of HELM's KV page bookkeeping.  TEST INFRASTRUCTURE ONLY.

Pure Python, no tensors: devices are the strings 'cuda' and 'cpu'; a page's
data is tracked as a checksum pair (sum of its used K values, sum of its used
V values) computed from the values written into it.  It follows
helm/runtime/kv_allocator.py:6-163 and helm/runtime/kv_cache.py:30-193 step
by step (cited per method).  Pinned by tests/golden/bookkeeping_traces.json
(recorded from the reference itself).
"""
from __future__ import annotations

from typing import Dict, List, Optional


class Page:
    __slots__ = ("page_id", "layer_id", "start_token", "used_tokens", "capacity", "device", "state", "k", "v")

    def __init__(self, page_id, device, capacity):
        self.page_id = page_id
        self.layer_id = -1
        self.start_token = 0
        self.used_tokens = 0
        self.capacity = capacity
        self.device = device
        self.state = "FREE"
        self.k: List[float] = []   # per-token sums of the K values written
        self.v: List[float] = []


class Allocator:
    def __init__(self, Hkv, P, D, elem_bytes):
        self.Hkv, self.P, self.D, self.elem = Hkv, P, D, elem_bytes
        self.gpu_free: List[Page] = []
        self.cpu_free: List[Page] = []
        self.gpu_total = 0
        self.cpu_total = 0
        self.next_id = 0

    def _create(self, device):                      # kv_allocator.py:22-48
        p = Page(self.next_id, device, self.P)
        self.next_id += 1
        if device == "cuda":
            self.gpu_total += 1
        else:
            self.cpu_total += 1
        return p

    def reserve_batch(self, n, device):             # kv_allocator.py:50-57
        for _ in range(n):
            (self.gpu_free if device == "cuda" else self.cpu_free).append(self._create(device))

    def allocate(self, device):                     # kv_allocator.py:59-78
        if device == "cuda":
            if not self.gpu_free:
                self.reserve_batch(8, device)
            p = self.gpu_free.pop()
            p.state = "GPU"
        else:
            if not self.cpu_free:
                self.reserve_batch(16, device)
            p = self.cpu_free.pop()
            p.state = "CPU"
        p.layer_id, p.start_token, p.used_tokens, p.device = -1, 0, 0, device
        return p

    def free(self, p):                              # kv_allocator.py:80-93
        p.state, p.layer_id, p.start_token, p.used_tokens = "FREE", -1, 0, 0
        (self.gpu_free if p.device == "cuda" else self.cpu_free).append(p)

    def move_page(self, p, target):                 # kv_allocator.py:95-144
        if p.device == target:
            return p
        n = self.allocate(target)
        used = p.used_tokens
        n.k = list(p.k[:used])
        n.v = list(p.v[:used])
        n.layer_id, n.start_token, n.used_tokens, n.device = p.layer_id, p.start_token, used, target
        if p.device == "cuda" and target != "cuda":
            p.k, p.v = [], []
            p.state = "DEAD"
            self.gpu_total -= 1
        else:
            self.free(p)
        return n

    def report_usage(self):                         # kv_allocator.py:146-163
        bpp = 2 * (self.Hkv * self.P * self.D * self.elem)
        gu = self.gpu_total - len(self.gpu_free)
        cu = self.cpu_total - len(self.cpu_free)
        return {"gpu_pool_size": self.gpu_total, "cpu_pool_size": self.cpu_total, "active_gpu_pages": gu,
                "active_cpu_pages": cu, "gpu_free_pages": len(self.gpu_free), "cpu_free_pages": len(self.cpu_free),
                "gpu_reserved_bytes": self.gpu_total * bpp, "cpu_reserved_bytes": self.cpu_total * bpp,
                "gpu_used_bytes": gu * bpp, "cpu_used_bytes": cu * bpp}


class Layer:
    def __init__(self, lid):
        self.layer_id = lid
        self.pages: List[Page] = []
        self.tail: Optional[Page] = None
        self.total_tokens = 0


class Manager:
    def __init__(self, alloc: Allocator, watermark):
        self.a = alloc
        self.layers: Dict[int, Layer] = {}
        self.watermark = watermark

    def page_bytes(self, p):
        return 0 if p.state == "DEAD" else 2 * self.a.Hkv * self.a.P * self.a.D * self.a.elem

    def init_layers(self, n):                       # kv_cache.py:51-53
        for i in range(n):
            self.layers[i] = Layer(i)

    def append_prefill(self, lid, k_tok, v_tok, device):   # kv_cache.py:55-85
        """k_tok / v_tok: per-token checksums of the chunk."""
        if lid not in self.layers:
            self.layers[lid] = Layer(lid)
        L = self.layers[lid]
        n = len(k_tok)
        for s in range(0, n, self.a.P):
            c = min(self.a.P, n - s)
            p = self.a.allocate(device)
            p.layer_id, p.start_token, p.used_tokens = lid, L.total_tokens, c
            p.k = list(k_tok[s:s + c])
            p.v = list(v_tok[s:s + c])
            L.pages.append(p)
            L.tail = p
            L.total_tokens += c
            self.enforce()

    def append_decode(self, lid, k1, v1, device, skip=False):   # kv_cache.py:87-113
        if lid not in self.layers:
            self.layers[lid] = Layer(lid)
        L = self.layers[lid]
        if L.tail is None or L.tail.used_tokens == L.tail.capacity:
            p = self.a.allocate(device)
            p.layer_id, p.start_token, p.used_tokens = lid, L.total_tokens, 0
            p.k, p.v = [], []
            L.pages.append(p)
            L.tail = p
        p = L.tail
        p.k = p.k[:p.used_tokens] + [k1]
        p.v = p.v[:p.used_tokens] + [v1]
        p.used_tokens += 1
        L.total_tokens += 1
        if not skip:
            self.enforce()

    def evict(self, nbytes):                        # kv_cache.py:121-159
        if nbytes <= 0:
            return
        cand = []
        for L in self.layers.values():
            for p in L.pages:
                if p.state == "GPU" and p.device == "cuda" and p is not L.tail and p.used_tokens == p.capacity:
                    cand.append((L, p))
        cand.sort(key=lambda t: t[1].start_token)
        done = 0
        for L, p in cand:
            if done >= nbytes:
                break
            n = self.a.move_page(p, "cpu")
            L.pages[L.pages.index(p)] = n
            if L.tail is p:
                L.tail = n
            done += 2 * self.a.Hkv * self.a.P * self.a.D * self.a.elem

    def enforce(self):                              # kv_cache.py:161-172
        b = 0
        for L in self.layers.values():
            for p in L.pages:
                if p.state == "GPU" and p.device == "cuda" and p is not L.tail and p.used_tokens == p.capacity:
                    b += 2 * self.a.Hkv * self.a.P * self.a.D * self.a.elem
        if b > self.watermark:
            self.evict(b - self.watermark)

    def clear(self):                                # kv_cache.py:183-193
        for L in self.layers.values():
            for p in L.pages:
                if p.state != "DEAD":
                    self.a.free(p)
            L.pages.clear()
            L.tail = None
            L.total_tokens = 0
        self.layers.clear()

    def seq_len(self):
        return self.layers[0].total_tokens if 0 in self.layers else 0

    def bytes_per_tier(self):                       # kv_cache.py:294-310
        g = c = 0
        for L in self.layers.values():
            for p in L.pages:
                if p.state == "DEAD":
                    continue
                if p.state == "GPU":
                    g += self.page_bytes(p)
                elif p.state == "CPU":
                    c += self.page_bytes(p)
        return {"gpu_active_bytes": g, "cpu_active_bytes": c}
