"""Parity of the dense prefill path (lq_qmm_dense: the weights dequantized once, then a dense tcgen05 GEMM -- the
reference's `_dense_matmul`, locals/kernels.py:999-1025) against the CPU oracle on the GPU.

Tolerance max|y - ref| <= 1e-2 * max|ref| (fp32 accumulation). At config 5's full size the oracle checks sampled rows
(rows of y are independent) and an fp32 matmul of the GPU-dequantized weights checks every row; the dense path and the
fused tc kernel compute the same products of the same bf16 weights, so they are also compared with each other.
"""

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import TOL_REL, act, qweights, rel_err, to_torch, x_torch

pytestmark = pytest.mark.gpu


def _run(cuda, M, N, K, bits, dtype, seed, choice=("dense",)):
    import torch
    from locals_b200 import kernels

    rng = np.random.default_rng(seed)
    wq, s, b = qweights(rng, N, K, bits, dtype)
    x = act(rng, M, K, dtype)
    tw, ts, tb = to_torch(wq, s, b, dtype, cuda)
    y = kernels.quantized_matmul(x_torch(x, dtype, cuda), tw, ts, tb, bits=bits, choice=choice)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    return x, (wq, s, b), (tw, ts, tb), y


@pytest.mark.parametrize("M,N,K,bits,dtype", [
    (128, 256, 512, 4, "bfloat16"),
    (256, 512, 1024, 4, "float16"),
    (200, 300, 640, 4, "bfloat16"),     # ragged M and N (a partial output tile)
    (130, 224 * 3, 768, 4, "bfloat16"),
    (1, 64, 256, 4, "bfloat16"),        # one token row
    (384, 256, 1024, 8, "bfloat16"),    # 8-bit weights (generic dequantize pass)
    (128, 1040, 512, 8, "float16"),
])
def test_dense_small(cuda, M, N, K, bits, dtype):
    x, q, _, y = _run(cuda, M, N, K, bits, dtype, seed=M + N + K)
    ref = O.round_to(O.qmm(x, *q, 64, bits), dtype)
    assert rel_err(y.float().cpu().numpy(), ref) <= TOL_REL


@pytest.mark.parametrize("bn", [256, 224, 128])
def test_dense_tilings_agree(cuda, bn):
    x, q, _, y = _run(cuda, 256, 896, 1024, 4, "bfloat16", seed=5, choice=("dense", bn))
    ref = O.round_to(O.qmm(x, *q), "bfloat16")
    assert rel_err(y.float().cpu().numpy(), ref) <= TOL_REL


def test_dense_dequantize_matches_mx_dequantize(cuda):
    # the dequantize pass writes what lq_dequantize (mx.dequantize) writes, within one rounding of the activation
    # dtype: the products fed to the GEMM are the fused kernel's
    import torch
    from locals_b200 import kernels

    x, q, (tw, ts, tb), y = _run(cuda, 512, 448, 2048, 4, "bfloat16", seed=3)
    yt = kernels.quantized_matmul(x_torch(x, "bfloat16", cuda), tw, ts, tb, bits=4, choice=("tc",))
    torch.cuda.synchronize()
    assert rel_err(y.float().cpu().numpy(), yt.float().cpu().numpy()) <= 2e-3


def test_dense_config5_full(cuda):
    import torch
    from locals_b200 import kernels

    M, N, K = 2048, 14336, 4096
    x, q, (tw, ts, tb), y = _run(cuda, M, N, K, 4, "bfloat16", seed=4, choice=None)  # the automatic choice
    rows = np.array([0, 1, 127, 128, 1000, 2047])
    ref = O.round_to(O.qmm(x[rows], *q), "bfloat16")
    assert rel_err(y[rows].float().cpu().numpy(), ref) <= TOL_REL
    wd = kernels.dequantize(tw, ts, tb, 64, 4).float()
    full = x_torch(x, "bfloat16", cuda).float() @ wd.T
    err = float((y.float() - full).abs().max() / full.abs().max())
    assert err <= TOL_REL
    torch.cuda.synchronize()


def test_dense_workspace_checked(cuda):
    import ctypes

    import torch
    from locals_b200 import _lib

    L = _lib.lib()
    M, N, K = 128, 256, 512
    rng = np.random.default_rng(1)
    wq, s, b = qweights(rng, N, K, 4, "bfloat16")
    tw, ts, tb = to_torch(wq, s, b, "bfloat16", cuda)
    x = x_torch(act(rng, M, K, "bfloat16"), "bfloat16", cuda)
    y = torch.empty((M, N), dtype=torch.bfloat16, device=cuda)
    need = L.lq_qmm_dense_workspace(N, K)
    assert need == N * K * 2
    ws = torch.empty(need, dtype=torch.uint8, device=cuda)
    args = [x.data_ptr(), tw.data_ptr(), ts.data_ptr(), tb.data_ptr(), y.data_ptr(), M, N, K, 4, 64, _lib.BF16]
    assert L.lq_qmm_dense(*args, ws.data_ptr(), ctypes.c_size_t(need - 2), None, None) == _lib.LQ_E_ARG
    assert L.lq_qmm_dense(*args, None, ctypes.c_size_t(need), None, None) == _lib.LQ_E_ARG
    assert L.lq_qmm_dense(*args, ws.data_ptr(), ctypes.c_size_t(need), None, None) == _lib.LQ_OK
    torch.cuda.synchronize()
