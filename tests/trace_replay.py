"""Replays the bookkeeping traces of tests/golden/bookkeeping_traces.json on (a) the oracle
restatement and (b) the helm_b200 runtime classes, producing snapshots in the fixture's format.

The product replay runs on the CPU with a stand-in 'cuda' device (FAKE below): pages allocated
for it are GPU pages to the bookkeeping (state 'GPU', device.type 'cuda') but are stored in host
memory, the same device substitution the fixture generator applied to the reference."""
from __future__ import annotations

import numpy as np
import torch

from oracle import bookkeeping as OB

DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


class FakeCuda:
    type = "cuda"
    index = 0
    _helm_storage = torch.device("cpu")

    def __repr__(self):
        return "fakecuda"


FAKE = FakeCuda()


class OnFake(torch.Tensor):
    """A CPU tensor that reports the stand-in device."""

    @property
    def device(self):
        return FAKE


def _draws(rng, a, n):
    k = rng.standard_normal((1, a["Hkv"], n, a["D"])).astype(np.float32)
    v = rng.standard_normal((1, a["Hkv"], n, a["D"])).astype(np.float32)
    return torch.from_numpy(k).to(DT[a["dtype"]]), torch.from_numpy(v).to(DT[a["dtype"]])


def replay_product(spec):
    from helm_b200.runtime import KVAllocator, KVCacheManager
    a = spec["alloc"]
    alloc = KVAllocator(num_layers=a["num_layers"], num_kv_heads=a["Hkv"], head_dim=a["D"], page_size=a["P"],
                        dtype=DT[a["dtype"]])
    kvcms = [KVCacheManager(alloc, gpu_high_watermark_bytes=w) for w in spec["watermarks"]]
    rng = np.random.default_rng(spec["seed"])
    snaps = []
    for op in spec["ops"]:
        kind = op[0]
        if kind in ("prefill", "decode"):
            _, mi, lid, n = op[:4]
            extra = op[4] if len(op) > 4 else {}
            k, v = _draws(rng, a, n)
            k, v = k.as_subclass(OnFake), v.as_subclass(OnFake)
            if kind == "prefill":
                kvcms[mi].append_prefill(lid, k, v)
            else:
                kvcms[mi].append_decode(lid, k, v, skip_residency=extra.get("skip", False))
        elif kind == "evict":
            kvcms[op[1]].evict_pages(op[2])
        elif kind == "clear":
            kvcms[op[1]].clear()
        elif kind == "init_layers":
            kvcms[op[1]].initialize_layer_caches(op[2])
        elif kind == "reserve":
            alloc.reserve_batch(op[1], FAKE if op[2] == "cuda" else torch.device("cpu"))
        snaps.append(snapshot_product(alloc, kvcms))
    return snaps


def snapshot_product(alloc, kvcms):
    snap = {"usage": alloc.report_usage(),
            "gpu_free_ids": [p.page_id for p in alloc.gpu_free_pool],
            "cpu_free_ids": [p.page_id for p in alloc.cpu_free_pool],
            "next_page_id": alloc._next_page_id, "managers": []}
    for m in kvcms:
        layers = {}
        for lid, layer in m.layers.items():
            pages = []
            for p in layer.pages:
                if p.state == "DEAD":
                    ck = None
                else:
                    u = p.used_tokens
                    ck = [float(p.k_tensor[:, :, :u].double().sum()), float(p.v_tensor[:, :, :u].double().sum())]
                pages.append([p.page_id, p.layer_id, p.start_token, p.used_tokens, p.capacity_tokens, p.state,
                              p.device.type, ck])
            layers[str(lid)] = {"pages": pages, "total_tokens": layer.total_tokens,
                                "tail": layer.tail_page.page_id if layer.tail_page is not None else None}
        snap["managers"].append({"layers": layers, "bytes": m.report_bytes_per_tier(), "seq_len": m.seq_len()})
    return snap


def replay_oracle(spec):
    a = spec["alloc"]
    elem = torch.tensor([], dtype=DT[a["dtype"]]).element_size()
    alloc = OB.Allocator(a["Hkv"], a["P"], a["D"], elem)
    ms = [OB.Manager(alloc, w) for w in spec["watermarks"]]
    rng = np.random.default_rng(spec["seed"])
    snaps = []
    for op in spec["ops"]:
        kind = op[0]
        if kind in ("prefill", "decode"):
            _, mi, lid, n = op[:4]
            extra = op[4] if len(op) > 4 else {}
            k, v = _draws(rng, a, n)
            kt = k.double().sum(dim=(0, 1, 3)).tolist()
            vt = v.double().sum(dim=(0, 1, 3)).tolist()
            if kind == "prefill":
                ms[mi].append_prefill(lid, kt, vt, "cuda")
            else:
                ms[mi].append_decode(lid, kt[0], vt[0], "cuda", skip=extra.get("skip", False))
        elif kind == "evict":
            ms[op[1]].evict(op[2])
        elif kind == "clear":
            ms[op[1]].clear()
        elif kind == "init_layers":
            ms[op[1]].init_layers(op[2])
        elif kind == "reserve":
            alloc.reserve_batch(op[1], op[2])
        snaps.append(snapshot_oracle(alloc, ms))
    return snaps


def snapshot_oracle(alloc, ms):
    snap = {"usage": alloc.report_usage(), "gpu_free_ids": [p.page_id for p in alloc.gpu_free],
            "cpu_free_ids": [p.page_id for p in alloc.cpu_free], "next_page_id": alloc.next_id, "managers": []}
    for m in ms:
        layers = {}
        for lid, L in m.layers.items():
            pages = []
            for p in L.pages:
                ck = None if p.state == "DEAD" else [float(sum(p.k[:p.used_tokens])), float(sum(p.v[:p.used_tokens]))]
                pages.append([p.page_id, p.layer_id, p.start_token, p.used_tokens, p.capacity, p.state, p.device, ck])
            layers[str(lid)] = {"pages": pages, "total_tokens": L.total_tokens,
                                "tail": L.tail.page_id if L.tail is not None else None}
        snap["managers"].append({"layers": layers, "bytes": m.bytes_per_tier(), "seq_len": m.seq_len()})
    return snap


def split_checksums(snap):
    """(snapshot without page checksums, list of checksums) for exact-vs-tolerant comparison."""
    import copy
    s = copy.deepcopy(snap)
    cks = []
    for m in s["managers"]:
        for L in m["layers"].values():
            for p in L["pages"]:
                cks.append(p[7])
                p[7] = None
    return s, cks
