"""The CPU oracle against the reference's own outputs (tests/golden), on the CPU."""
import json
import pathlib

import numpy as np
import pytest
import torch

from oracle import attention as OA
from oracle import cpu_baseline as CB
from tests.golden.cases import ATTN_CASES, attn_case_inputs, config1_inputs, sha256_tensors

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def _case_pages(case):
    name, seed, Hq, Hkv, D, cap, useds, dt, scale = case
    q, k, v = attn_case_inputs(case)
    dtype = DT[dt]
    qr = torch.from_numpy(q).to(dtype).double().numpy().reshape(Hq, D)
    kr = torch.from_numpy(k).to(dtype).double().numpy()
    vr = torch.from_numpy(v).to(dtype).double().numpy()
    return qr, kr, vr, useds, dtype


@pytest.mark.parametrize("case", ATTN_CASES, ids=[c[0] for c in ATTN_CASES])
def test_oracle_streaming_attention_matches_reference(case):
    name, seed, Hq, Hkv, D, cap, useds, dt, scale = case
    golden = np.load(GOLDEN / "attention_cases.npz")[f"{name}/out"].reshape(Hq, D)
    qr, kr, vr, useds, dtype = _case_pages(case)
    pages = [OA.Page(kr[i], vr[i], u) for i, u in enumerate(useds)]
    ref = OA.streaming_attention(qr, pages, scale)
    # the reference output is rounded to the case dtype
    out = torch.from_numpy(ref).to(dtype).double().numpy()
    tol = 1e-5 if dtype == torch.float32 else 0.0
    err = np.abs(out - golden).max() / max(1.0, np.abs(golden).max()) if golden.size else 0.0
    ulp = {torch.float32: 0, torch.float16: 2 ** -10, torch.bfloat16: 2 ** -7}[dtype]
    assert err <= tol + ulp, f"{name}: {err}"


@pytest.mark.parametrize("case", ATTN_CASES, ids=[c[0] for c in ATTN_CASES])
def test_oracle_path3_and_split_merge_agree(case):
    """The Path-3 online-softmax restatement and the split-record + LSE merge both equal the
    float64 one-shot attention."""
    name, seed, Hq, Hkv, D, cap, useds, dt, scale = case
    qr, kr, vr, useds, dtype = _case_pages(case)
    pages = [OA.Page(kr[i], vr[i], u, resident=(i % 2 == 1)) for i, u in enumerate(useds)]
    ref = OA.streaming_attention(qr, pages, scale)
    p3 = OA.online_softmax_path3(qr, pages, scale)
    assert np.abs(p3 - ref).max() <= 1e-4 * max(1.0, np.abs(ref).max())
    sc = (1.0 / np.sqrt(D)) if scale is None else scale
    recs = []
    for i, pg in enumerate(pages):
        act = pg.used > 0
        recs.append(OA.partial_record(qr, pg.k[:, :pg.used] if act else None, pg.v[:, :pg.used] if act else None, sc))
    recs.append(OA.partial_record(qr, None, None, sc))  # an empty split
    out, merged = OA.lse_merge(np.stack(recs))
    assert np.abs(out - ref).max() <= 1e-10 * max(1.0, np.abs(ref).max())


def test_oracle_config1_matches_reference():
    g = np.load(GOLDEN / "attention_config1.npz")
    q, k, v = config1_inputs()
    if sha256_tensors(q, k, v) != str(g["sha256"]):
        pytest.skip("torch.randn stream differs on this host")
    pages = [OA.Page(k[0, :, 64 * i:64 * (i + 1)].numpy(), v[0, :, 64 * i:64 * (i + 1)].numpy(), 64,
                     resident=i >= 32) for i in range(64)]
    ref = OA.streaming_attention(q[0, :, 0].numpy(), pages)
    assert np.abs(ref - g["out"].reshape(32, 128)).max() <= 1e-5
    p3 = OA.online_softmax_path3(q[0, :, 0].numpy(), pages)
    assert np.abs(p3 - g["out"].reshape(32, 128)).max() <= 1e-5


def test_cpu_baseline_port_matches_reference_outputs():
    """The timed CPU port (bench.py's baseline) reproduces the reference outputs."""
    for case in ATTN_CASES:
        name, seed, Hq, Hkv, D, cap, useds, dt, scale = case
        q, k, v = attn_case_inputs(case)
        dtype = DT[dt]
        tq = torch.from_numpy(q).to(dtype)
        pages = [(torch.from_numpy(k[i:i + 1]).to(dtype), torch.from_numpy(v[i:i + 1]).to(dtype), u)
                 for i, u in enumerate(useds)]
        golden = np.load(GOLDEN / "attention_cases.npz")[f"{name}/out"]
        for fn in (CB.path2_attention, CB.path3_attention):
            out = fn(tq, pages, scale).float().numpy()
            ulp = {torch.float32: 1e-5, torch.float16: 2 ** -10, torch.bfloat16: 2 ** -7}[dtype]
            assert np.abs(out - golden).max() <= ulp * max(1.0, np.abs(golden).max()), (name, fn.__name__)


def test_int8_oracle_matches_reference_fp16_gemv():
    from oracle.int8_linear import int8_linear_ref
    g = np.load(GOLDEN / "fp16_gemv.npz")
    for key in ("256x512", "96x1024"):
        w, s, x, y = g[f"{key}/w"], g[f"{key}/s"], g[f"{key}/x"], g[f"{key}/y"]
        ref = int8_linear_ref(x, w, s)
        assert np.abs(ref - y).max() <= 1e-2 * np.abs(ref).max()
