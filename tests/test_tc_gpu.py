"""Parity of the prefill family (tcgen05 GEMM with fused dequant) against the CPU oracle on the GPU.

The prefill workload: x bf16 [2048, 4096], W 4-bit g64 [14336, 4096] -> y [2048, 14336], fp32 accumulation;
tolerance max|y - ref| <= 1e-2 * max|ref|. At the full size the oracle checks a sample of rows (the
kernel's rows are independent: row m of y depends on row m of x only), plus the whole output against a
dequantize + fp32 matmul on the GPU's own dequantized weights.
"""

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import TOL_REL, act, qweights, rel_err, to_torch, x_torch

pytestmark = pytest.mark.gpu


def _tc(cuda, M, N, K, bits, dtype, seed, choice=("tc",)):
    import torch
    from locals_b200 import kernels

    rng = np.random.default_rng(seed)
    wq, s, b = qweights(rng, N, K, bits, dtype)
    x = act(rng, M, K, dtype)
    tw, ts, tb = to_torch(wq, s, b, dtype, cuda)
    y = kernels.quantized_matmul(x_torch(x, dtype, cuda), tw, ts, tb, bits=bits, choice=choice)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    return x, (wq, s, b), y


@pytest.mark.parametrize("M,N,K,bits,dtype", [
    (128, 256, 512, 4, "bfloat16"),
    (256, 512, 1024, 4, "float16"),
    (200, 300, 640, 4, "bfloat16"),     # ragged M, N; K with a partial scale block (10 groups)
    (130, 224 * 3, 768, 4, "bfloat16"),
    (384, 256, 1024, 8, "bfloat16"),
    (128, 1040, 512, 8, "float16"),
])
def test_tc_small(cuda, M, N, K, bits, dtype):
    x, q, y = _tc(cuda, M, N, K, bits, dtype, seed=M + N + K)
    ref = O.round_to(O.qmm(x, *q, 64, bits), dtype)
    assert rel_err(y.float().cpu().numpy(), ref) <= TOL_REL


@pytest.mark.parametrize("bn", [256, 224, 128])
def test_tc_tilings_agree(cuda, bn):
    x, q, y = _tc(cuda, 256, 896, 1024, 4, "bfloat16", seed=5, choice=("tc", bn))
    ref = O.round_to(O.qmm(x, *q), "bfloat16")
    assert rel_err(y.float().cpu().numpy(), ref) <= TOL_REL


@pytest.mark.parametrize("choice", [("tc",), ("tcv", 256, 0, 0), ("tcv", 256, 0, 0, 1)])
def test_tc_config5_full(cuda, choice):
    # both prefill formulations: x on the MMA's M side (tc), and weights dequantized into tensor memory
    # with 256-token tiles on N (tcv)
    import torch
    from locals_b200 import kernels

    M, N, K = 2048, 14336, 4096
    x, q, y = _tc(cuda, M, N, K, 4, "bfloat16", seed=4, choice=choice)
    # sampled rows against the oracle
    rows = np.array([0, 1, 127, 128, 1000, 2047])
    ref = O.round_to(O.qmm(x[rows], *q), "bfloat16")
    assert rel_err(y[rows].float().cpu().numpy(), ref) <= TOL_REL
    # every row against an fp32 matmul of the GPU-dequantized weights
    tw, ts, tb = to_torch(*q, "bfloat16", cuda)
    wd = kernels.dequantize(tw, ts, tb, 64, 4).float()
    full = x_torch(x, "bfloat16", cuda).float() @ wd.T
    err = float((y.float() - full).abs().max() / full.abs().max())
    assert err <= TOL_REL
    torch.cuda.synchronize()


def test_auto_routes_prefill_to_tc(cuda):
    # M >= 128: the automatic choice takes the tensor-core family and matches the decode family
    from locals_b200 import kernels

    x, q, y = _tc(cuda, 256, 512, 1024, 4, "bfloat16", seed=8, choice=None)
    ref = O.round_to(O.qmm(x, *q), "bfloat16")
    assert rel_err(y.float().cpu().numpy(), ref) <= TOL_REL
