"""GPU parity of the tcgen05 INT8 weight-only GEMM (helm_int8_gemm_packed), the prefill-sized
(M > 64) path of the INT8 linear, against float64 dequantise-then-matmul (oracle/int8_linear.py).
The tensor-core products are exact (16-bit x values times integer weights) and accumulate in fp32,
so the error is the output rounding: max |y - ref| <= 4e-3 * max |ref| (8e-3 for bf16)."""
import numpy as np
import pytest
import torch

from oracle.int8_linear import int8_linear_ref

pytestmark = pytest.mark.gpu


def _inputs(M, N, K, seed, xdtype):
    rng = np.random.default_rng(seed)
    w = rng.integers(-127, 128, size=(N, K), dtype=np.int8)
    s = rng.uniform(0.001, 0.02, size=(N,)).astype(np.float16)
    x = (rng.standard_normal((M, K)) / np.sqrt(K / 64)).astype(np.float32)
    return w, s, torch.from_numpy(x).to(xdtype)


def _rel(y, ref):
    y = y.detach().double().cpu().numpy()
    return float(np.abs(y - ref).max() / max(np.abs(ref).max(), 1e-30))


@pytest.mark.parametrize("M,N,K", [(128, 128, 128), (65, 96, 256), (300, 333, 528), (1024, 4096, 4096),
                                   (257, 12288, 1024), (200, 1000, 4112)])
@pytest.mark.parametrize("xdtype", [torch.bfloat16, torch.float16])
@pytest.mark.parametrize("with_bias", [False, True])
def test_gemm_matches_oracle(M, N, K, xdtype, with_bias, cuda):
    from helm_b200 import ops
    w, s, x = _inputs(M, N, K, seed=M * 7 + N + K, xdtype=xdtype)
    bias = torch.randn(N, dtype=torch.float32).to(xdtype) if with_bias else None
    pk = ops.int8_pack_weight(torch.from_numpy(w).to(cuda))
    y = ops.int8_linear(x.to(cuda), pk, torch.from_numpy(s).to(cuda), None if bias is None else bias.to(cuda),
                        gemm=True)
    ref = int8_linear_ref(x.double().numpy(), w, s, None if bias is None else bias.double().numpy())
    assert y.shape == (M, N) and y.dtype == xdtype
    assert _rel(y, ref) <= 4e-3 * (2.0 if xdtype == torch.bfloat16 else 1.0)
    assert ops.int8_linear_error() == 0


def test_gemm_repeatable_and_module_prefill_path(cuda):
    """Two calls agree bit for bit; Int8Linear routes prefill-sized inputs to the GEMM."""
    import torch.nn as nn
    from helm_b200 import ops
    from helm_b200.kernels import Int8Linear
    torch.manual_seed(0)
    lin = nn.Linear(512, 384, bias=True).to(cuda).to(torch.bfloat16)
    m = Int8Linear.from_linear(lin)
    x = torch.randn(3, 70, 512, device=cuda, dtype=torch.bfloat16)
    a = ops.int8_linear(x, m.pk, m.scale, m.bias, gemm=True)
    b = ops.int8_linear(x, m.pk, m.scale, m.bias, gemm=True)
    assert torch.equal(a, b)
    assert torch.equal(m(x), a)
