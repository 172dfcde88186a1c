"""Parity of the folded group-per-warp decode family (qmvq: codes fed raw to the MMA, scale and bias applied per group
in fp32, the reference's fragq formulation) against the CPU oracle, through the C ABI on the GPU.

The family takes dense 4-bit calls with M <= 16 and K % 256 == 0: the decode projections of configs 1 and 2 at their
real sizes, the fused q/k/v split, ragged N (a partial last 16-row fragment), K with a partial last 512-wide stage,
every fragment count a CTA may hold (including requests larger than the grid needs), both activation dtypes and one to
sixteen tokens.
Tolerance: max|y - ref| <= 1e-2 * max|ref| with fp32 accumulation (the reference's own kernel tests use
0.02 * (1 + max|ref|), tests/test_q35_kernels.py:60-93).
"""

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import TOL_REL, act, qweights, rel_err, to_torch, x_torch

pytestmark = pytest.mark.gpu


def _run(cuda, M, N, K, dtype, seed, choice=("qmvq", 0, 0, 0, 0)):
    import torch
    from locals_b200 import kernels

    rng = np.random.default_rng(seed)
    wq, s, b = qweights(rng, N, K, 4, dtype)
    x = act(rng, M, K, dtype)
    ref = O.round_to(O.qmm(x, wq, s, b, 64, 4), dtype)
    tw, ts, tb = to_torch(wq, s, b, dtype, cuda)
    y = kernels.quantized_matmul(x_torch(x, dtype, cuda), tw, ts, tb, bits=4, choice=choice)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    return y.float().cpu().numpy(), ref


@pytest.mark.parametrize("M,N,K,dtype", [
    (8, 4096, 4096, "float16"),      # config 1
    (1, 6144, 2560, "bfloat16"),     # config 2
    (4, 6144, 2560, "bfloat16"),
    (8, 6144, 2560, "bfloat16"),
    (16, 6144, 2560, "bfloat16"),
    (16, 4096, 4096, "float16"),
])
@pytest.mark.parametrize("sx", [1, 2])
def test_qmvq_configs(cuda, M, N, K, dtype, sx):
    y, ref = _run(cuda, M, N, K, dtype, seed=M * 13 + N + K, choice=("qmvq", 0, 0, 0, sx))
    assert rel_err(y, ref) <= TOL_REL


@pytest.mark.parametrize("M,N,K,dtype", [
    (3, 200, 512, "float16"),       # N not a multiple of 16: a partial last fragment
    (5, 136, 1024, "bfloat16"),
    (9, 72, 256, "bfloat16"),       # one stage, half of it past K
    (16, 520, 768, "float16"),      # K % 512 != 0: a partial last stage
    (2, 1040, 1792, "bfloat16"),
    (12, 3000, 2304, "bfloat16"),
    (1, 16, 256, "float16"),        # one fragment, one CTA
    (7, 20000, 512, "bfloat16"),    # more than 4 fragments a SM: several CTAs a SM
])
@pytest.mark.parametrize("sx", [1, 2])
def test_qmvq_ragged(cuda, M, N, K, dtype, sx):
    y, ref = _run(cuda, M, N, K, dtype, seed=N * 3 + K + M, choice=("qmvq", 0, 0, 0, sx))
    assert rel_err(y, ref) <= TOL_REL


# 97 fragments: FR requests 1-4 give grids of 97, 49, 33 and 25 CTAs (FR or FR - 1 fragments each); NS pins the ring
@pytest.mark.parametrize("choice", [("qmvq", 1, 0, 0, 0), ("qmvq", 2, 0, 0, 0), ("qmvq", 3, 0, 0, 0),
                                    ("qmvq", 4, 0, 0, 0), ("qmvq", 3, 1, 0, 0), ("qmvq", 2, 2, 0, 0), ("qmvq", 4, 3, 0, 0),
                                    # group x sums by the all-ones MMA or by adds
                                    ("qmvq", 0, 0, 0, 1), ("qmvq", 0, 0, 0, 2), ("qmvq", 3, 2, 0, 2),
                                    ("qmvq", 1, 0, 0, 1), ("qmvq", 4, 0, 0, 2),
                                    # K slices added over a cluster (2-5 CTAs along y)
                                    ("qmvq", 0, 0, 2, 0), ("qmvq", 0, 0, 3, 1), ("qmvq", 2, 0, 4, 0),
                                    ("qmvq", 4, 2, 5, 2)])
def test_qmvq_every_tiling(cuda, choice):
    y, ref = _run(cuda, 16, 1552, 2560, "bfloat16", seed=21, choice=choice)
    assert rel_err(y, ref) <= TOL_REL


def test_qmvq_split_outputs(cuda):
    # the fused q/k/v projection written straight into three outputs (locals/fuse.py:48-63)
    import torch
    from locals_b200 import kernels

    rng = np.random.default_rng(9)
    M, K, widths = 16, 2560, (4096, 1024, 1024)
    N = sum(widths)
    wq, s, b = qweights(rng, N, K, 4, "bfloat16")
    x = act(rng, M, K, "bfloat16")
    ref = O.round_to(O.qmm(x, wq, s, b, 64, 4), "bfloat16")
    tw, ts, tb = to_torch(wq, s, b, "bfloat16", cuda)
    outs = kernels.qmm_split(x_torch(x, "bfloat16", cuda), tw, ts, tb, widths, choice=("qmvq", 0, 0))
    torch.cuda.synchronize()
    got = np.concatenate([o.float().cpu().numpy() for o in outs], axis=1)
    assert rel_err(got, ref) <= TOL_REL


def test_qmvq_matches_qmvg(cuda):
    # the folded and the dequantizing family give the same answer within tolerance on the same call
    y0, ref = _run(cuda, 16, 6144, 2560, "bfloat16", seed=5, choice=("qmvg", 0, 0))
    y1, _ = _run(cuda, 16, 6144, 2560, "bfloat16", seed=5)
    assert rel_err(y1, y0) <= TOL_REL


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_qmvq_is_the_fp32_factoring(cuda, dtype):
    """The fold computes s * sum(q x) + b * sum(x) in fp32, the oracle's factoring of the reference's multi-row kernel
    (locals/qmv_multi.py:57-75), without rounding the weights: it lands within a few output ulps of the oracle."""
    y, ref = _run(cuda, 5, 1024, 4096, dtype, seed=77, choice=("qmvq", 0, 0, 0, 2))
    ulp = 2.0 ** -8 if dtype == "bfloat16" else 2.0 ** -11
    assert float(np.max(np.abs(y - ref))) <= 2 * ulp * float(np.max(np.abs(ref)))


@pytest.mark.parametrize("M,N,K,dtype", [
    (1, 2560, 9728, "bfloat16"),     # config 3's down projection
    (16, 2560, 9728, "bfloat16"),
    (4, 9728, 2560, "float16"),
    (8, 1000, 1280, "bfloat16"),     # a partial fragment and a partial last stage
    (3, 16, 256, "float16"),         # one fragment, one half stage
])
def test_qmvq_8bit(cuda, M, N, K, dtype):
    """8-bit codes: the high and low nibbles enter two MMAs, folded as s (16 acc_hi + acc_lo) + (b - 17 magic s) sum x."""
    import torch
    from locals_b200 import kernels

    rng = np.random.default_rng(M + N + K)
    wq, s, b = qweights(rng, N, K, 8, dtype)
    x = act(rng, M, K, dtype)
    ref = O.round_to(O.qmm(x, wq, s, b, 64, 8), dtype)
    tw, ts, tb = to_torch(wq, s, b, dtype, cuda)
    y = kernels.quantized_matmul(x_torch(x, dtype, cuda), tw, ts, tb, bits=8, choice=("qmvq", 0, 0, 0, 0))
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    assert rel_err(y.float().cpu().numpy(), ref) <= TOL_REL


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M,I,K,dtype", [
    (1, 9728, 2560, "bfloat16"),     # config 3's gate||up at one token
    (16, 9728, 2560, "bfloat16"),
    (5, 200, 512, "float16"),        # ragged rows
    (2, 768, 2048, "bfloat16"),      # config 4's expert shape
])
def test_qmvq_glu(cuda, bits, M, I, K, dtype):
    """Gate and up in one kernel with the SwiGLU epilogue (rounding points of locals/moe.py:284-289)."""
    import torch
    from locals_b200 import kernels

    rng = np.random.default_rng(bits * 7 + M + I)
    g = qweights(rng, I, K, bits, dtype)
    u = qweights(rng, I, K, bits, dtype)
    x = act(rng, M, K, dtype)
    href = O.swiglu(O.round_to(O.qmm(x, *g, 64, bits), dtype), O.round_to(O.qmm(x, *u, 64, bits), dtype), dtype)
    tg, tu = to_torch(*g, dtype, cuda), to_torch(*u, dtype, cuda)
    h = kernels.qmm_glu(x_torch(x, dtype, cuda), tg, tu, bits=bits, choice=("qmvq", 0, 0, 0, 0))
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    # four activation-dtype roundings before act * u: the reference bounds its own expert SwiGLU output by 2^-6 max
    # (tests/test_flint.py:80-111)
    assert rel_err(h.float().cpu().numpy(), href) <= 2.0 ** -6


@pytest.mark.parametrize("bits,M,N,K,ks", [
    (8, 1, 2560, 9728, 0),     # config 3's down projection: the library's choice splits K (5 slices)
    (8, 16, 2560, 9728, 8),
    (4, 3, 2560, 9728, 0),
    (4, 9, 1000, 4608, 3),     # a partial fragment, uneven slices
    (8, 2, 64, 768, 3),        # one stage a slice
])
def test_qmvq_k_slices(cuda, bits, M, N, K, ks):
    """K split over a thread-block cluster, the slices' sums added in rank order through distributed shared memory."""
    import torch
    from locals_b200 import kernels

    rng = np.random.default_rng(bits + M + N + K + ks)
    wq, s, b = qweights(rng, N, K, bits, "bfloat16")
    x = act(rng, M, K, "bfloat16")
    ref = O.round_to(O.qmm(x, wq, s, b, 64, bits), "bfloat16")
    tw, ts, tb = to_torch(wq, s, b, "bfloat16", cuda)
    y = kernels.quantized_matmul(x_torch(x, "bfloat16", cuda), tw, ts, tb, bits=bits, choice=("qmvq", 0, 0, ks, 0))
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    assert rel_err(y.float().cpu().numpy(), ref) <= TOL_REL


def test_qmvq_glu_k_slices(cuda):
    import torch
    from locals_b200 import kernels

    rng = np.random.default_rng(31)
    M, I, K = 4, 1024, 4096
    g = qweights(rng, I, K, 8, "bfloat16")
    u = qweights(rng, I, K, 8, "bfloat16")
    x = act(rng, M, K, "bfloat16")
    href = O.swiglu(O.round_to(O.qmm(x, *g, 64, 8), "bfloat16"), O.round_to(O.qmm(x, *u, 64, 8), "bfloat16"),
                    "bfloat16")
    tg, tu = to_torch(*g, "bfloat16", cuda), to_torch(*u, "bfloat16", cuda)
    h = kernels.qmm_glu(x_torch(x, "bfloat16", cuda), tg, tu, bits=8, choice=("qmvq", 0, 0, 4, 0))
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    assert rel_err(h.float().cpu().numpy(), href) <= 2.0 ** -6
