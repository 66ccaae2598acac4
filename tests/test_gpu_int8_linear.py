"""GPU parity of the INT8 weight-only linear (through the C ABI).

Oracles: float64 dequantise-then-matmul (oracle/int8_linear.py) and the
reference's own AVX2 fp16 GEMV applied to the fp16-dequantised weights
(tests/golden/fp16_gemv.npz).  Bar: max |y - ref| <= 1e-2 * max |ref|.
"""
import pathlib

import numpy as np
import pytest
import torch

from oracle.int8_linear import int8_linear_ref

pytestmark = pytest.mark.gpu
GOLDEN = pathlib.Path(__file__).resolve().parent / "golden"
TOL = 1e-2


def rel_err(y, ref):
    y = y.detach().double().cpu().numpy()
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


def _inputs(M, N, K, seed, xdtype=torch.float16):
    rng = np.random.default_rng(seed)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    s = rng.uniform(0.001, 0.02, size=(N,)).astype(np.float16)
    x = rng.standard_normal((M, K)).astype(np.float32)
    return w, s, torch.from_numpy(x).to(xdtype)


@pytest.mark.parametrize("shape", [(12288, 4096), (4096, 12288), (6144, 4096)])
@pytest.mark.parametrize("M", [1, 4, 8])
def test_config2_shapes(shape, M, cuda):
    from helm_b200 import ops
    N, K = shape
    w, s, x = _inputs(M, N, K, seed=N + K + M)
    y = ops.int8_linear(x.to(cuda), torch.from_numpy(w).to(cuda), torch.from_numpy(s).to(cuda))
    ref = int8_linear_ref(x.double().numpy(), w, s)
    assert y.shape == (M, N) and y.dtype == torch.float16
    assert rel_err(y, ref) <= TOL
    assert ops.int8_linear_error() == 0


@pytest.mark.parametrize("M", [1, 2, 3, 5, 9, 16, 17])
@pytest.mark.parametrize("xdtype", [torch.float16, torch.bfloat16])
def test_odd_shapes_bias_bf16(M, xdtype, cuda):
    from helm_b200 import ops
    N, K = 333, 528
    w, s, x = _inputs(M, N, K, seed=M, xdtype=xdtype)
    bias = torch.randn(N, dtype=torch.float32).to(xdtype)
    y = ops.int8_linear(x.to(cuda), torch.from_numpy(w).to(cuda), torch.from_numpy(s).float().to(cuda),
                        bias=bias.to(cuda))
    ref = int8_linear_ref(x.double().numpy(), w, s, bias.double().numpy())
    assert y.dtype == xdtype
    assert rel_err(y, ref) <= TOL


def test_leading_dims_preserved(cuda):
    from helm_b200 import ops
    w, s, x = _inputs(6, 64, 256, seed=3)
    y = ops.int8_linear(x.reshape(2, 3, 256).to(cuda), torch.from_numpy(w).to(cuda), torch.from_numpy(s).to(cuda))
    assert y.shape == (2, 3, 64)


@pytest.mark.parametrize("key", ["256x512", "96x1024"])
def test_matches_reference_fp16_gemv(key, cuda):
    """Against the reference AVX2 kernel run on the dequantised weights (fp16 W*s)."""
    from helm_b200 import ops
    g = np.load(GOLDEN / "fp16_gemv.npz")
    w, s, x, y_ref = g[f"{key}/w"], g[f"{key}/s"], g[f"{key}/x"], g[f"{key}/y"]
    y = ops.int8_linear(torch.from_numpy(x).to(cuda), torch.from_numpy(w).to(cuda), torch.from_numpy(s).to(cuda))
    assert rel_err(y, y_ref.astype(np.float64)) <= TOL


def test_rejects_bad_k(cuda):
    from helm_b200 import ops
    from helm_b200._native import HelmError
    w = torch.zeros(8, 24, dtype=torch.int8, device=cuda)
    with pytest.raises(HelmError):
        ops.int8_linear(torch.zeros(1, 24, dtype=torch.float16, device=cuda), w,
                        torch.ones(8, dtype=torch.float16, device=cuda))


@pytest.mark.parametrize("N,K", [(1024, 16384),   # few long rows: K split over a 4-CTA cluster
                                 (2048, 8192),    # 2-CTA cluster
                                 (20000, 4096),   # 32 rows per CTA, ragged last tile
                                 (77, 16), (130, 48), (64, 272), (96, 4112)])  # K tails below 256
@pytest.mark.parametrize("M", [1, 8, 9, 33, 64, 70])
@pytest.mark.parametrize("xdtype", [torch.float16, torch.bfloat16])
def test_split_and_tail_shapes(N, K, M, xdtype, cuda):
    """Every work split (rows per CTA, cluster K split, K tails, M past 8/16/32/64) against the
    float64 oracle; the tensor-core products are exact and accumulate in fp32, so the error is
    the output rounding: max |y - ref| <= 4e-3 * max |ref|."""
    from helm_b200 import ops
    w, s, x = _inputs(M, N, K, seed=N * 7 + K + M, xdtype=xdtype)
    bias = torch.randn(N, dtype=torch.float32).to(xdtype)
    y = ops.int8_linear(x.to(cuda), torch.from_numpy(w).to(cuda), torch.from_numpy(s).to(cuda),
                        bias=bias.to(cuda))
    ref = int8_linear_ref(x.double().numpy(), w, s, bias.double().numpy())
    assert y.shape == (M, N) and y.dtype == xdtype
    assert rel_err(y, ref) <= 4e-3 * (2.0 if xdtype == torch.bfloat16 else 1.0)
    assert ops.int8_linear_error() == 0


def test_repeated_calls_identical(cuda):
    """Deterministic: the K split and its reduction order are fixed, so two calls agree bit for bit."""
    from helm_b200 import ops
    w, s, x = _inputs(4, 1024, 16384, seed=5)
    wd, sd, xd = torch.from_numpy(w).to(cuda), torch.from_numpy(s).to(cuda), x.to(cuda)
    assert torch.equal(ops.int8_linear(xd, wd, sd), ops.int8_linear(xd, wd, sd))


def _glu_ref(x, wg, sg, bg, wu, su, bu):
    g = x @ (wg.astype(np.float64) * sg.astype(np.float64)[:, None]).T + bg
    u = x @ (wu.astype(np.float64) * su.astype(np.float64)[:, None]).T + bu
    return g / (1.0 + np.exp(-g)) * u


@pytest.mark.parametrize("I,K", [(64, 256), (1024, 1024), (2944, 528), (12288, 4096)])
@pytest.mark.parametrize("M", [1, 4, 9, 33, 64])
@pytest.mark.parametrize("xdtype", [torch.float16, torch.bfloat16])
def test_glu_matches_oracle(I, K, M, xdtype, cuda):
    """helm_int8_linear_glu (gate and up rows tile-interleaved, silu(gate) * up in the epilogue)
    against float64 gate / up projections; the error is the output rounding."""
    from helm_b200 import ops
    rng = np.random.default_rng(I + K + M)
    wg = rng.integers(-127, 128, size=(I, K), dtype=np.int8)
    wu = rng.integers(-127, 128, size=(I, K), dtype=np.int8)
    sg = rng.uniform(0.001, 0.02, size=(I,)).astype(np.float16)
    su = rng.uniform(0.001, 0.02, size=(I,)).astype(np.float16)
    bg = rng.standard_normal(I).astype(np.float32)
    bu = rng.standard_normal(I).astype(np.float32)
    x = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float32) / np.sqrt(K / 64)).to(xdtype)
    w = ops.interleave_glu_rows(torch.from_numpy(wg), torch.from_numpy(wu)).contiguous()
    s = ops.interleave_glu_rows(torch.from_numpy(sg), torch.from_numpy(su)).contiguous()
    b = ops.interleave_glu_rows(torch.from_numpy(bg), torch.from_numpy(bu)).to(xdtype)
    y = ops.int8_linear_glu(x.to(cuda), w.to(cuda), s.to(cuda), bias=b.to(cuda))
    bgx = torch.from_numpy(bg).to(xdtype).double().numpy()
    bux = torch.from_numpy(bu).to(xdtype).double().numpy()
    ref = _glu_ref(x.double().numpy(), wg, sg, bgx, wu, su, bux)
    assert y.shape == (M, I) and y.dtype == xdtype
    assert rel_err(y, ref) <= 4e-3 * (2.0 if xdtype == torch.bfloat16 else 1.0)
    assert ops.int8_linear_error() == 0


def test_glu_rejects_ragged_intermediate(cuda):
    from helm_b200 import ops
    from helm_b200._native import HelmError
    w = torch.zeros(48, 64, dtype=torch.int8, device=cuda)   # I = 24: not a multiple of 16
    with pytest.raises((HelmError, ValueError)):
        ops.int8_linear_glu(torch.zeros(1, 64, dtype=torch.float16, device=cuda), w,
                            torch.ones(48, dtype=torch.float16, device=cuda))


@pytest.mark.parametrize("N,K", [(12288, 4096), (4096, 12288), (6144, 4096), (333, 528), (77, 16), (96, 4112),
                                 (20000, 4096)])
@pytest.mark.parametrize("M", [1, 8, 9, 33, 64])
@pytest.mark.parametrize("xdtype", [torch.float16, torch.bfloat16])
def test_packed_equals_rowmajor(N, K, M, xdtype, cuda):
    """helm_int8_linear_packed on helm_int8_pack_weight's layout gives the row-major kernel's
    result bit for bit (same MMAs in the same order), including ragged N and K tails."""
    from helm_b200 import ops
    w, s, x = _inputs(M, N, K, seed=N + 3 * K + M, xdtype=xdtype)
    wd, sd, xd = torch.from_numpy(w).to(cuda), torch.from_numpy(s).to(cuda), x.to(cuda)
    bias = torch.randn(N, dtype=torch.float32).to(xdtype).to(cuda)
    pk = ops.int8_pack_weight(wd)
    assert torch.equal(pk.unpack(), wd)
    assert torch.equal(ops.int8_linear(xd, pk, sd, bias), ops.int8_linear(xd, wd, sd, bias))
    assert ops.int8_linear_error() == 0


@pytest.mark.parametrize("M", [1, 9, 64])
def test_packed_glu_equals_rowmajor(M, cuda):
    from helm_b200 import ops
    rng = np.random.default_rng(M)
    I, K = 1024, 2048
    w = torch.from_numpy(rng.integers(-127, 128, size=(2 * I, K), dtype=np.int8)).to(cuda)
    s = torch.from_numpy(rng.uniform(0.001, 0.02, size=(2 * I,)).astype(np.float16)).to(cuda)
    x = torch.randn(M, K, dtype=torch.bfloat16, device=cuda) / 8
    pk = ops.int8_pack_weight(w)
    assert torch.equal(ops.int8_linear_glu(x, pk, s), ops.int8_linear_glu(x, w, s))
