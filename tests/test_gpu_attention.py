"""GPU parity of the paged decode attention kernels (through the C ABI).

Oracles: the reference's own outputs (tests/golden, made from HELM's
perform_streaming_attention) and the float64 restatement in oracle/attention.py.
"""
import json
import math
import os
import pathlib

import numpy as np
import pytest
import torch

from oracle import attention as OA
from tests.attn_util import assert_attn_close, attn_error, pool_from_pages
from tests.golden.cases import ATTN_CASES, attn_case_inputs

pytestmark = pytest.mark.gpu

GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
DT = {"float32": torch.float32, "float16": torch.float16, "bfloat16": torch.bfloat16}


def _ops():
    from helm_b200 import ops
    return ops


def run_pages(q, kp, vp, tables, useds, nums, *, P, scale=None, num_splits=0, out_dtype=None,
              error_flag=None):
    """q [B, Hq, D] cuda; kp/vp pool [n, Hkv, P, D]; tables/useds lists of per-sequence lists."""
    ops = _ops()
    B = q.shape[0]
    width = max(1, max(len(t) for t in tables))
    pt = torch.zeros((B, width), dtype=torch.int32)
    pu = torch.zeros((B, width), dtype=torch.int32)
    for b in range(B):
        pt[b, :len(tables[b])] = torch.tensor(tables[b], dtype=torch.int32)
        pu[b, :len(useds[b])] = torch.tensor(useds[b], dtype=torch.int32)
    dev = q.device
    Hkv = kp.shape[1]
    D = kp.shape[-1]
    return ops.paged_decode_attention(
        q, kp, vp, pt.to(dev), pu.to(dev), torch.tensor(nums, dtype=torch.int32, device=dev),
        num_kv_heads=Hkv, page_size=P, page_stride=Hkv * P * D, head_stride=P * D, num_pool_pages=kp.shape[0],
        scale=scale, num_splits=num_splits, out_dtype=out_dtype, error_flag=error_flag)


@pytest.mark.parametrize("case", ATTN_CASES, ids=[c[0] for c in ATTN_CASES])
@pytest.mark.parametrize("splits", [1, 0])
def test_golden_cases(case, splits, cuda):
    """Each reference test scenario: our kernel vs the reference's own output and the oracle."""
    name, seed, Hq, Hkv, D, cap, useds, dt, scale = case
    golden = np.load(GOLDEN / "attention_cases.npz")[f"{name}/out"]
    q, k, v = attn_case_inputs(case)
    dtype = DT[dt]
    kp, vp, ids = pool_from_pages(k, v, dtype, cuda, shuffle_seed=seed)
    qd = torch.from_numpy(q).to(dtype).reshape(1, Hq, D).to(cuda)
    out = run_pages(qd, kp, vp, [ids.tolist()], [useds], [len(useds)], P=cap, scale=scale, num_splits=splits)
    assert out.dtype == dtype and out.shape == (1, Hq, D)
    # vs the reference output (same dtype): may differ by one output rounding step
    gold = torch.from_numpy(golden).reshape(1, Hq, D)
    err_gold = attn_error(out, gold)
    tol_gold = 1e-4 if dtype == torch.float32 else 2 * (2.0 ** -8 if dtype == torch.bfloat16 else 2.0 ** -11) + 2e-3
    assert err_gold <= tol_gold, f"{name}: vs reference output {err_gold:.2e}"
    # vs float64 oracle on the same (rounded) inputs, fp32 output
    kr = torch.from_numpy(k).to(dtype).double().numpy()
    vr = torch.from_numpy(v).to(dtype).double().numpy()
    qr = torch.from_numpy(q).to(dtype).double().numpy().reshape(Hq, D)
    pages = [OA.Page(kr[i], vr[i], u) for i, u in enumerate(useds)]
    ref = torch.from_numpy(OA.streaming_attention(qr, pages, scale)).reshape(1, Hq, D)
    out32 = run_pages(qd, kp, vp, [ids.tolist()], [useds], [len(useds)], P=cap, scale=scale,
                      num_splits=splits, out_dtype=torch.float32)
    assert_attn_close(out32, ref, dtype, name)
    if all(u == 0 for u in useds):
        assert torch.all(out == 0)


def test_config1_matches_reference(cuda):
    """BASELINE config 1 (seed 0, fp32, 64 pages of 64, half of them 'offloaded'): the kernel
    output vs the reference's own output."""
    from tests.golden.cases import config1_inputs, sha256_tensors
    g = np.load(GOLDEN / "attention_config1.npz")
    q, k, v = config1_inputs()
    if sha256_tensors(q, k, v) != str(g["sha256"]):
        pytest.skip("torch.randn stream differs on this host; config-1 inputs not reproducible")
    kpages = k.reshape(1, 8, 64, 64, 128)[0].permute(1, 0, 2, 3).contiguous()  # [64 pages, 8, 64, 128]
    vpages = v.reshape(1, 8, 64, 64, 128)[0].permute(1, 0, 2, 3).contiguous()
    out = run_pages(q.reshape(1, 32, 128).to(cuda), kpages.to(cuda), vpages.to(cuda), [list(range(64))],
                    [[64] * 64], [64], P=64)
    ref = torch.from_numpy(g["out"]).reshape(1, 32, 128)
    assert float((out.cpu() - ref).abs().max()) <= 1e-4


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("gq", [1, 4, 5, 8, 16])
@pytest.mark.parametrize("splits", [1, 3, 0, -1])
def test_random_pool_tensor_core_path(dtype, gq, splits, cuda):
    """B=3 sequences of ragged lengths over a shuffled pool (P=64, D=128): the TMA/tensor-core path."""
    torch.manual_seed(1000 + gq)
    Hkv, D, P = 2, 128, 64
    Hq = Hkv * gq
    lens = [1, 700, 64 * 9]
    npages = [math.ceil(n / P) for n in lens]
    total = sum(npages) + 5
    kp = torch.randn(total, Hkv, P, D).to(dtype)
    vp = torch.randn(total, Hkv, P, D).to(dtype)
    perm = torch.randperm(total).tolist()
    tables, useds, i = [], [], 0
    for n, npg in zip(lens, npages):
        tables.append(perm[i:i + npg])
        useds.append([P] * (npg - 1) + [n - P * (npg - 1)])
        i += npg
    q = torch.randn(3, Hq, D).to(dtype)
    out = run_pages(q.to(cuda), kp.to(cuda), vp.to(cuda), tables, useds, npages, P=P, num_splits=splits,
                    out_dtype=torch.float32)
    ref = OA.paged_attention_torch(q, kp, vp, torch.tensor([t + [0] * (max(npages) - len(t)) for t in tables]),
                                   torch.tensor([u + [0] * (max(npages) - len(u)) for u in useds]),
                                   torch.tensor(npages))
    assert_attn_close(out, ref, dtype, f"gq={gq} splits={splits}")


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("D", [32, 64, 96, 160, 192, 256])
@pytest.mark.parametrize("gq", [1, 3, 12, 24])
@pytest.mark.parametrize("splits", [0, 2])
def test_warp_kernel_head_dims_and_groups(dtype, D, gq, splits, cuda):
    """The CUDA-core warp kernel over head dims that are multiples of 32 and GQA groups of any size
    (served in chunks of up to 8 heads per CTA), P = 16 pages, ragged lengths."""
    torch.manual_seed(2000 + D + gq)
    Hkv, P = 2, 16
    Hq = Hkv * gq
    lens = [1, 100, 250]
    npages = [math.ceil(n / P) for n in lens]
    total = sum(npages) + 3
    kp = torch.randn(total, Hkv, P, D).to(dtype)
    vp = torch.randn(total, Hkv, P, D).to(dtype)
    perm = torch.randperm(total).tolist()
    tables, useds, i = [], [], 0
    for n, npg in zip(lens, npages):
        tables.append(perm[i:i + npg])
        useds.append([P] * (npg - 1) + [n - P * (npg - 1)])
        i += npg
    q = torch.randn(3, Hq, D).to(dtype)
    out = run_pages(q.to(cuda), kp.to(cuda), vp.to(cuda), tables, useds, npages, P=P, num_splits=splits,
                    out_dtype=torch.float32)
    ref = OA.paged_attention_torch(q, kp, vp, torch.tensor([t + [0] * (max(npages) - len(t)) for t in tables]),
                                   torch.tensor([u + [0] * (max(npages) - len(u)) for u in useds]),
                                   torch.tensor(npages))
    assert_attn_close(out, ref, dtype, f"D={D} gq={gq} splits={splits}")


def test_warp_kernel_matches_generic_kernel(cuda, monkeypatch):
    """A group of 24 at D = 96 on the warp kernel (three head chunks) and on the generic kernel."""
    torch.manual_seed(9)
    Hkv, D, P, gq = 2, 96, 64, 24
    kp = torch.randn(30, Hkv, P, D, dtype=torch.bfloat16, device=cuda)
    vp = torch.randn(30, Hkv, P, D, dtype=torch.bfloat16, device=cuda)
    q = torch.randn(2, Hkv * gq, D, dtype=torch.bfloat16, device=cuda)
    tables = [list(range(0, 15)), list(range(29, 14, -1))]
    useds = [[64] * 14 + [9], [64] * 15]
    a = run_pages(q, kp, vp, tables, useds, [15, 15], P=P, out_dtype=torch.float32)
    monkeypatch.setenv("HELM_B200_FORCE_GENERIC", "1")
    b = run_pages(q, kp, vp, tables, useds, [15, 15], P=P, out_dtype=torch.float32)
    assert float((a - b).abs().max()) < 1e-4


def test_tensor_core_path_matches_generic_path(cuda, monkeypatch):
    torch.manual_seed(7)
    Hkv, D, P, gq = 8, 128, 64, 8
    kp = torch.randn(40, Hkv, P, D, dtype=torch.bfloat16, device=cuda)
    vp = torch.randn(40, Hkv, P, D, dtype=torch.bfloat16, device=cuda)
    q = torch.randn(2, Hkv * gq, D, dtype=torch.bfloat16, device=cuda)
    tables = [list(range(0, 20)), list(range(39, 19, -1))]
    useds = [[64] * 19 + [3], [64] * 20]
    a = run_pages(q, kp, vp, tables, useds, [20, 20], P=P, out_dtype=torch.float32)
    monkeypatch.setenv("HELM_B200_FORCE_GENERIC", "1")
    b = run_pages(q, kp, vp, tables, useds, [20, 20], P=P, out_dtype=torch.float32)
    assert float((a - b).abs().max()) < 1e-4


def test_stale_nan_rows_do_not_leak(cuda):
    """Rows past page_used hold NaN: the output must stay finite and equal to the clean result."""
    torch.manual_seed(3)
    Hkv, D, P = 4, 128, 64
    kp = torch.randn(6, Hkv, P, D, dtype=torch.bfloat16, device=cuda)
    vp = torch.randn(6, Hkv, P, D, dtype=torch.bfloat16, device=cuda)
    q = torch.randn(1, Hkv * 4, D, dtype=torch.bfloat16, device=cuda)
    clean = run_pages(q, kp, vp, [[0, 1, 2]], [[64, 64, 10]], [3], P=P, out_dtype=torch.float32)
    kp[2, :, 10:] = float("nan")
    vp[2, :, 10:] = float("nan")
    dirty = run_pages(q, kp, vp, [[0, 1, 2]], [[64, 64, 10]], [3], P=P, out_dtype=torch.float32)
    assert torch.isfinite(dirty).all()
    assert float((clean - dirty).abs().max()) == 0.0


def test_empty_sequences_and_pages(cuda):
    Hkv, D, P = 2, 128, 64
    kp = torch.randn(4, Hkv, P, D, dtype=torch.bfloat16, device=cuda)
    vp = torch.randn(4, Hkv, P, D, dtype=torch.bfloat16, device=cuda)
    q = torch.randn(3, 8, D, dtype=torch.bfloat16, device=cuda)
    out = run_pages(q, kp, vp, [[], [1, 2], [3]], [[], [0, 0], [5]], [0, 2, 1], P=P)
    assert torch.all(out[0] == 0) and torch.all(out[1] == 0)
    assert torch.isfinite(out).all() and out[2].abs().sum() > 0


def test_bad_page_id_sets_error_flag(cuda):
    """An out-of-range page id is skipped and reported through the device error flag."""
    from helm_b200 import _native as N
    Hkv, D, P = 2, 128, 64
    kp = torch.randn(4, Hkv, P, D, dtype=torch.bfloat16, device=cuda)
    vp = torch.randn(4, Hkv, P, D, dtype=torch.bfloat16, device=cuda)
    q = torch.randn(1, 8, D, dtype=torch.bfloat16, device=cuda)
    for force_generic in (False, True):
        if force_generic:
            os.environ["HELM_B200_FORCE_GENERIC"] = "1"
        try:
            flag = torch.zeros(1, dtype=torch.int32, device=cuda)
            out = run_pages(q, kp, vp, [[0, 9]], [[64, 64]], [2], P=P, error_flag=flag, num_splits=1)
            ref = run_pages(q, kp, vp, [[0]], [[64]], [1], P=P, num_splits=1)
        finally:
            os.environ.pop("HELM_B200_FORCE_GENERIC", None)
        assert int(flag.item()) & N.DEVERR_PAGE_ID
        assert torch.equal(out, ref)


@pytest.mark.parametrize("S,D", [(5, 128), (74, 128), (1100, 64), (9, 256), (6, 65)])
def test_lse_merge_matches_oracle(S, D, cuda):
    """Split-parallel merge (even D) and the dim-per-thread merge (odd D), including more partials
    than one shared-memory chunk (1100) and the config-1 split count (74)."""
    from helm_b200 import ops
    rng = np.random.default_rng(5 + S + D)
    rows = 12
    recs = np.zeros((S, rows, D + 2))
    recs[..., :D] = rng.standard_normal((S, rows, D))
    recs[..., D] = rng.standard_normal((S, rows)) * 4
    recs[..., D + 1] = rng.uniform(0.5, 3.0, (S, rows))
    recs[1, 3, D] = -np.inf  # empty partials
    recs[1, 3, D + 1] = 0
    recs[1, 3, :D] = 0
    recs[:, 7, D] = -np.inf
    recs[:, 7, D + 1] = 0
    recs[:, 7, :D] = 0
    ref_out, ref_rec = OA.lse_merge(recs)
    t = torch.from_numpy(recs.astype(np.float32)).to(cuda)
    rec = torch.empty(rows, D + 2, device=cuda)
    out = ops.lse_merge(t, out_record=rec, out=torch.empty(rows, D, device=cuda))
    assert np.allclose(out.cpu().numpy(), ref_out, atol=1e-5, rtol=1e-5)
    r = rec.cpu().numpy()
    fin = np.isfinite(ref_rec[:, D])
    assert np.allclose(r[fin], ref_rec[fin], atol=1e-4, rtol=1e-5)
    assert np.all(np.isneginf(r[~fin, D])) and np.all(out.cpu().numpy()[7] == 0)


def test_split_records_merge_to_single_pass(cuda):
    """Records of a split run merged with helm_lse_merge equal the one-pass result."""
    from helm_b200 import ops
    torch.manual_seed(11)
    Hkv, D, P = 8, 128, 64
    kp = torch.randn(64, Hkv, P, D, dtype=torch.bfloat16, device=cuda)
    vp = torch.randn(64, Hkv, P, D, dtype=torch.bfloat16, device=cuda)
    q = torch.randn(2, 64, D, dtype=torch.bfloat16, device=cuda)
    tables = [list(range(32)), list(range(32, 64))]
    useds = [[64] * 32, [64] * 31 + [1]]
    one = run_pages(q, kp, vp, tables, useds, [32, 32], P=P, num_splits=1, out_dtype=torch.float32)
    # two half-length page lists -> two merged records -> lse_merge
    recs = []
    for half in range(2):
        tb = [t[16 * half:16 * (half + 1)] for t in tables]
        ub = [u[16 * half:16 * (half + 1)] for u in useds]
        rec = torch.empty(2 * 64, D + 2, device=cuda)
        pt = torch.tensor(tb, dtype=torch.int32, device=cuda)
        pu = torch.tensor(ub, dtype=torch.int32, device=cuda)
        ops.paged_decode_attention(q, kp, vp, pt, pu, torch.tensor([16, 16], dtype=torch.int32, device=cuda),
                                   num_kv_heads=Hkv, page_size=P, page_stride=Hkv * P * D, head_stride=P * D,
                                   num_pool_pages=64, num_splits=3, out_record=rec)
        recs.append(rec)
    merged = ops.lse_merge(torch.stack(recs).contiguous(), out=torch.empty(128, D, device=cuda))
    assert float((merged.reshape(2, 64, D) - one).abs().max()) < 1e-5


def test_full_size_config5_layer(cuda):
    """One full config-5 layer (B=4, 64/8 heads, 131072 tokens, bf16) on a shuffled pool: every
    (sequence, kv head) checked against the float64 oracle on a subsample of query heads."""
    torch.manual_seed(5)
    B, Hq, Hkv, D, P, ctx = 4, 64, 8, 128, 64, 131072
    npg = ctx // P
    total = B * npg
    kp = torch.empty(total, Hkv, P, D, dtype=torch.bfloat16, device=cuda)
    vp = torch.empty(total, Hkv, P, D, dtype=torch.bfloat16, device=cuda)
    for i in range(0, total, 1024):
        kp[i:i + 1024].normal_()
        vp[i:i + 1024].normal_()
    perm = torch.randperm(total, device=cuda).to(torch.int32).reshape(B, npg)
    used = torch.full((B, npg), P, dtype=torch.int32, device=cuda)
    q = torch.randn(B, Hq, D, dtype=torch.bfloat16, device=cuda)
    from helm_b200 import ops
    out = ops.paged_decode_attention(q, kp, vp, perm, used, torch.full((B,), npg, dtype=torch.int32, device=cuda),
                                     num_kv_heads=Hkv, page_size=P, page_stride=Hkv * P * D, head_stride=P * D,
                                     num_pool_pages=total, out_dtype=torch.float32)
    for b in range(B):
        ids = perm[b].long()
        for g in (0, 5):
            k = kp[ids, g].reshape(-1, D).double()
            v = vp[ids, g].reshape(-1, D).double()
            qq = q[b, g * 8:(g + 1) * 8].double()
            p = torch.softmax(qq @ k.T / math.sqrt(D), dim=-1)
            ref = (p @ v).cpu()
            err = attn_error(out[b, g * 8:(g + 1) * 8], ref)
            assert err <= 2e-3, (b, g, err)


@pytest.mark.parametrize("lens", [[0, 1, 64 * 3 + 5, 64 * 40, 17], [64 * 7], [1, 1, 1], [0, 0], [5000, 0, 3000, 64]])
@pytest.mark.parametrize("gq", [8, 5, 16])
def test_persistent_kernel_matches_split_kernel(lens, gq, cuda):
    """The persistent (work-balanced, fused-merge) launch against the split-grid launch and the
    oracle, with ragged / empty sequences; twice in a row (the arrival counters are reset)."""
    torch.manual_seed(sum(lens) + gq)
    Hkv, D, P = 4, 128, 64
    npages = [math.ceil(n / P) for n in lens]
    total = max(1, sum(npages)) + 3
    kp = torch.randn(total, Hkv, P, D, device=cuda).to(torch.bfloat16)
    vp = torch.randn(total, Hkv, P, D, device=cuda).to(torch.bfloat16)
    perm = torch.randperm(total).tolist()
    tables, useds, i = [], [], 0
    for n, npg in zip(lens, npages):
        tables.append(perm[i:i + npg])
        useds.append([P] * (npg - 1) + [n - P * (npg - 1)] if npg else [])
        i += npg
    q = torch.randn(len(lens), Hkv * gq, D, device=cuda).to(torch.bfloat16)
    a1 = run_pages(q, kp, vp, tables, useds, npages, P=P, num_splits=-1, out_dtype=torch.float32)
    a2 = run_pages(q, kp, vp, tables, useds, npages, P=P, num_splits=-1, out_dtype=torch.float32)
    s1 = run_pages(q, kp, vp, tables, useds, npages, P=P, num_splits=1, out_dtype=torch.float32)
    s0 = run_pages(q, kp, vp, tables, useds, npages, P=P, num_splits=0, out_dtype=torch.float32)
    assert torch.equal(a1, a2)
    assert float((a1 - s1).abs().max()) < 1e-4
    assert float((s0 - s1).abs().max()) < 1e-4
    width = max(1, max(npages))
    ref = OA.paged_attention_torch(q.cpu(), kp.cpu(), vp.cpu(),
                                   torch.tensor([t + [0] * (width - len(t)) for t in tables]),
                                   torch.tensor([u + [0] * (width - len(u)) for u in useds]), torch.tensor(npages))
    assert_attn_close(a1, ref, torch.bfloat16, f"persistent lens={lens}")
    for b, n in enumerate(lens):
        if n == 0:
            assert torch.all(a1[b] == 0)


def test_persistent_out_record_merges_across_calls(cuda):
    """out_record of the persistent launch (num_splits=-1) and of the automatic plan, merged over
    two halves of a sequence, equals the one-call output (the multi-GPU merge contract)."""
    from helm_b200 import ops
    torch.manual_seed(21)
    Hkv, D, P, gq, B = 8, 128, 64, 8, 3
    kp = torch.randn(300, Hkv, P, D, device=cuda).to(torch.bfloat16)
    vp = torch.randn(300, Hkv, P, D, device=cuda).to(torch.bfloat16)
    q = torch.randn(B, Hkv * gq, D, device=cuda).to(torch.bfloat16)
    perm = torch.randperm(300, device=cuda).to(torch.int32)
    pt = perm[:B * 90].reshape(B, 90).contiguous()
    pu = torch.full((B, 90), P, dtype=torch.int32, device=cuda)
    full = ops.paged_decode_attention(q, kp, vp, pt, pu, torch.full((B,), 90, dtype=torch.int32, device=cuda),
                                      num_kv_heads=Hkv, page_size=P, page_stride=Hkv * P * D, head_stride=P * D,
                                      num_pool_pages=300, out_dtype=torch.float32)
    for splits in (-1, 0):
        recs = []
        for lo, hi in ((0, 37), (37, 90)):
            rec = torch.empty(B * Hkv * gq, D + 2, device=cuda)
            ops.paged_decode_attention(q, kp, vp, pt[:, lo:hi].contiguous(), pu[:, lo:hi].contiguous(),
                                       torch.full((B,), hi - lo, dtype=torch.int32, device=cuda), num_kv_heads=Hkv,
                                       page_size=P, page_stride=Hkv * P * D, head_stride=P * D, num_pool_pages=300,
                                       out_record=rec, num_splits=splits)
            recs.append(rec)
        merged = ops.lse_merge(torch.stack(recs).contiguous(), out=torch.empty(B * Hkv * gq, D, device=cuda))
        assert float((merged.reshape(B, -1, D) - full).abs().max()) < 1e-5, splits


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_records_only_and_gather_merge_of_split_records(dtype, cuda):
    """Records-only mode leaves the split records in the workspace; helm_lse_merge of them, and
    helm_gather_merge given them as partials (world 1: the merge + push + wait + merge path on
    one GPU), equal the normal call."""
    import ctypes
    from helm_b200 import _native as N
    from helm_b200 import ops
    torch.manual_seed(31)
    Hkv, D, P, gq, B = 4, 128, 64, 8, 3
    Hq = Hkv * gq
    kp = torch.randn(120, Hkv, P, D, device=cuda).to(dtype)
    vp = torch.randn(120, Hkv, P, D, device=cuda).to(dtype)
    q = torch.randn(B, Hq, D, device=cuda).to(dtype)
    pt = torch.randperm(120, device=cuda).to(torch.int32)[:B * 40].reshape(B, 40).contiguous()
    pu = torch.full((B, 40), P, dtype=torch.int32, device=cuda)
    pu[:, 39] = 11
    npg = torch.tensor([40, 7, 23], dtype=torch.int32, device=cuda)
    common = dict(num_kv_heads=Hkv, page_size=P, page_stride=Hkv * P * D, head_stride=P * D, num_pool_pages=120)
    full = ops.paged_decode_attention(q, kp, vp, pt, pu, npg, out_dtype=torch.float32, **common)
    ws = torch.empty(1 << 21, device=cuda)
    parts = ops.paged_decode_attention(q, kp, vp, pt, pu, npg, records_only=True, workspace=ws, **common)
    rows = B * Hq
    assert parts.shape[1:] == (rows, D + 2) and parts.shape[0] >= 1
    merged = ops.lse_merge(parts.contiguous(), out=torch.empty(rows, D, device=cuda))
    assert float((merged.reshape(B, Hq, D) - full).abs().max()) < 1e-5
    lib = N.lib()
    rb, fb, cb = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int64()
    assert lib.helm_gather_merge_state_bytes(1, rows, D, ctypes.byref(rb), ctypes.byref(fb), ctypes.byref(cb)) > 0
    st = torch.zeros(rb.value + fb.value, dtype=torch.uint8, device=cuda)
    cnt = torch.zeros(max(cb.value, 4), dtype=torch.uint8, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    for call in range(2):
        out = torch.full((rows, D), 7.0, device=cuda)
        p = N.GatherMergeParams()
        p.rank, p.world, p.rows, p.D = 0, 1, rows, D
        p.record = parts.data_ptr()
        p.num_partials, p.partial_stride = parts.shape[0], rows * (D + 2)
        p.peer_recv[0], p.peer_flags[0] = st.data_ptr(), st.data_ptr() + rb.value
        p.recv_local, p.flags_local = st.data_ptr(), st.data_ptr() + rb.value
        p.counters = cnt.data_ptr()
        p.out, p.out_dtype, p.error_flag = out.data_ptr(), N.F32, err.data_ptr()
        p.wait_ns = 100_000_000
        N.check("helm_gather_merge", lib.helm_gather_merge(ctypes.byref(p), torch.cuda.current_stream().cuda_stream))
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        assert float((out.reshape(B, Hq, D) - full).abs().max()) < 1e-5, call
