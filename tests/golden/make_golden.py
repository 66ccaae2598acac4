"""Generates the golden fixtures in tests/golden/ from the HELM reference itself.

Run where the reference checkout is importable (its root in HELM_REFERENCE_ROOT, else the
default below):  python tests/golden/make_golden.py

Fixtures written (all small; the GPU host never needs the reference):
  attention_cases.npz   -- outputs, for the seeded cases of cases.py, of the
                           reference perform_streaming_attention
                           (helm/runtime/kv_cache.py:318-442, CPU pages, its
                           Path 2), incl. GQA / ragged / empty pages / fp16.
  attention_config1.npz -- BASELINE config 1 (seed 0, torch.randn draws of
                           q [1,32,1,128], k/v [1,8,4096,128], 64 pages of 64):
                           reference output + sha256 of the inputs.
  bookkeeping_traces.json -- op sequences replayed on the reference
                           KVAllocator / KVCacheManager (kv_allocator.py,
                           kv_cache.py:55-172) with a stand-in 'cuda' device so
                           eviction runs on CPU: page lists, states, ids,
                           report_usage() and report_bytes_per_tier() after
                           every op.
  fp16_gemv.npz         -- the reference AVX2 helm_fp16_linear
                           (helm/kernels/fp16_gemv.cpp:105-157) applied to
                           fp16-dequantised INT8 weights, M = 1.
"""
from __future__ import annotations

import json
import math
import os
import pathlib
import sys

import numpy as np
import torch

HERE = pathlib.Path(__file__).resolve().parent
REPO = HERE.parent.parent
if not os.environ.get("HELM_REFERENCE_ROOT"):
    raise SystemExit("make_golden.py: set HELM_REFERENCE_ROOT to the root of a HELM checkout (the directory "
                     "that contains helm/runtime/kv_cache.py)")
REF = pathlib.Path(os.environ["HELM_REFERENCE_ROOT"])
sys.path.insert(0, str(REF))
sys.path.insert(0, str(REPO))

from helm.runtime import kv_allocator as ref_alloc  # noqa: E402
from helm.runtime import kv_cache as ref_cache  # noqa: E402
from tests.golden.cases import (ATTN_CASES, attn_case_inputs, config1_inputs,  # noqa: E402
                                sha256_tensors, trace_specs)

DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def _ref_page(k, v, page_id, start, used, cap, state="CPU"):
    return ref_cache.KVPage(page_id=page_id, layer_id=0, start_token=start, used_tokens=used,
                            capacity_tokens=cap, k_tensor=k.clone(), v_tensor=v.clone(),
                            device=k.device, state=state)


def make_attention_cases():
    arrays = {}
    meta = []
    for case in ATTN_CASES:
        name, seed, Hq, Hkv, D, cap, useds, dt, scale = case
        q, ks, vs = attn_case_inputs(case)
        tq = torch.from_numpy(q).to(DT[dt])
        tk = torch.from_numpy(ks).to(DT[dt])
        tv = torch.from_numpy(vs).to(DT[dt])
        pages, start = [], 0
        for i, u in enumerate(useds):
            pages.append(_ref_page(tk[i:i + 1], tv[i:i + 1], i, start, u, cap))
            start += u
        out = ref_cache.perform_streaming_attention(tq, pages, scale=scale)
        arrays[f"{name}/out"] = out.float().numpy()
        meta.append({"name": name, "seed": seed, "out_dtype": str(out.dtype).replace("torch.", "")})
    np.savez_compressed(HERE / "attention_cases.npz", **arrays)
    (HERE / "attention_cases.json").write_text(json.dumps(meta, indent=1))


def make_config1():
    q, k, v = config1_inputs()
    pages = []
    for i in range(64):
        sl = slice(64 * i, 64 * (i + 1))
        pages.append(_ref_page(k[:, :, sl], v[:, :, sl], i, 64 * i, 64, 64, "CPU"))
    out = ref_cache.perform_streaming_attention(q, pages)
    np.savez_compressed(HERE / "attention_config1.npz", out=out.numpy(),
                        sha256=np.array(sha256_tensors(q, k, v)))


# ---------------------------------------------------------------------------
# Bookkeeping traces with a stand-in CUDA device.
# ---------------------------------------------------------------------------

class FakeCuda:
    """Device stand-in: .type == 'cuda', equal only to itself."""
    type = "cuda"
    index = 0

    def __repr__(self):
        return "fakecuda"


FAKE = FakeCuda()
_APPEND = {"on": False}


def _install_fake_device():
    orig_alloc = ref_alloc.KVAllocator.allocate
    orig_move = ref_alloc.KVAllocator.move_page

    def _create_page(self, device):
        shape = (1, self.num_kv_heads, self.page_size, self.head_dim)
        page = ref_cache.KVPage(page_id=self._next_page_id, layer_id=-1, start_token=0, used_tokens=0,
                                capacity_tokens=self.page_size,
                                k_tensor=torch.empty(shape, dtype=self.dtype),
                                v_tensor=torch.empty(shape, dtype=self.dtype), device=device, state="FREE")
        self._next_page_id += 1
        if device.type == "cuda":
            self.gpu_total_pages += 1
        else:
            self.cpu_total_pages += 1
        return page

    def allocate(self, device):
        if _APPEND["on"] and getattr(device, "type", None) == "cpu":
            device = FAKE
        return orig_alloc(self, device)

    def move_page(self, page, target_device):
        saved = _APPEND["on"]
        _APPEND["on"] = False
        try:
            return orig_move(self, page, target_device)
        finally:
            _APPEND["on"] = saved

    ref_alloc.KVAllocator._create_page = _create_page
    ref_alloc.KVAllocator.allocate = allocate
    ref_alloc.KVAllocator.move_page = move_page


def _snapshot(alloc, kvcms):
    snap = {"usage": alloc.report_usage(),
            "gpu_free_ids": [p.page_id for p in alloc.gpu_free_pool],
            "cpu_free_ids": [p.page_id for p in alloc.cpu_free_pool],
            "next_page_id": alloc._next_page_id,
            "managers": []}
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


def run_trace(spec):
    """Replays spec['ops'] on fresh reference objects; returns the snapshots after every op."""
    a = spec["alloc"]
    alloc = ref_alloc.KVAllocator(num_layers=a["num_layers"], num_kv_heads=a["Hkv"], head_dim=a["D"],
                                  page_size=a["P"], dtype=DT[a["dtype"]])
    kvcms = [ref_cache.KVCacheManager(alloc, gpu_high_watermark_bytes=w) for w in spec["watermarks"]]
    rng = np.random.default_rng(spec["seed"])
    snaps = []
    for op in spec["ops"]:
        kind = op[0]
        if kind in ("prefill", "decode"):
            _, mi, lid, n = op[:4]
            extra = op[4] if len(op) > 4 else {}
            k = torch.from_numpy(rng.standard_normal((1, a["Hkv"], n, a["D"])).astype(np.float32)).to(DT[a["dtype"]])
            v = torch.from_numpy(rng.standard_normal((1, a["Hkv"], n, a["D"])).astype(np.float32)).to(DT[a["dtype"]])
            _APPEND["on"] = True
            try:
                if kind == "prefill":
                    kvcms[mi].append_prefill(lid, k, v)
                else:
                    kvcms[mi].append_decode(lid, k, v, skip_residency=extra.get("skip", False))
            finally:
                _APPEND["on"] = False
        elif kind == "evict":
            kvcms[op[1]].evict_pages(op[2])
        elif kind == "clear":
            kvcms[op[1]].clear()
        elif kind == "init_layers":
            kvcms[op[1]].initialize_layer_caches(op[2])
        elif kind == "reserve":
            alloc.reserve_batch(op[1], FAKE if op[2] == "cuda" else torch.device("cpu"))
        else:
            raise ValueError(kind)
        snaps.append(_snapshot(alloc, kvcms))
    return snaps


def make_bookkeeping():
    _install_fake_device()
    out = []
    for spec in trace_specs():
        out.append({"spec": spec, "snapshots": run_trace(spec)})
    (HERE / "bookkeeping_traces.json").write_text(json.dumps(out))


def make_fp16_gemv():
    from oracle import build_ref
    build_ref.build()
    mod = build_ref.load()
    rng = np.random.default_rng(31)
    arrays = {}
    for N_, K_ in ((256, 512), (96, 1024)):
        w = rng.integers(-127, 128, size=(N_, K_), dtype=np.int8)
        s = rng.uniform(0.001, 0.02, size=(N_,)).astype(np.float16)
        x = rng.standard_normal((1, K_)).astype(np.float16)
        w_deq = torch.from_numpy(w.astype(np.float32) * s.astype(np.float32)[:, None]).half()
        y = mod.helm_fp16_linear(torch.from_numpy(x), w_deq, None)
        key = f"{N_}x{K_}"
        arrays[f"{key}/w"] = w
        arrays[f"{key}/s"] = s
        arrays[f"{key}/x"] = x
        arrays[f"{key}/y"] = y.numpy()
    np.savez_compressed(HERE / "fp16_gemv.npz", **arrays)


if __name__ == "__main__":
    torch.set_num_threads(8)
    make_attention_cases()
    make_config1()
    make_bookkeeping()
    make_fp16_gemv()
    print("golden fixtures written to", HERE)
