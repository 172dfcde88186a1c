"""Parity of the tensor-core decode family (tcv: weights dequantized into tensor memory, tokens on the
MMA's N side) against the CPU oracle, through the C ABI on the GPU.

Tolerance: max|y - ref| <= 1e-2 * max|ref| (fp32 accumulation of bf16/fp16 products of the dequantized
weights, which are rounded once to the activation dtype as the reference's dequantize does).
"""

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import TOL_REL, act, qweights, rel_err, to_torch, x_torch

pytestmark = pytest.mark.gpu


def _run(cuda, M, N, K, bits, dtype, seed, choice=("tcv", 0, 0, 0)):
    import torch
    from locals_b200 import kernels

    rng = np.random.default_rng(seed)
    wq, s, b = qweights(rng, N, K, bits, dtype)
    x = act(rng, M, K, dtype)
    ref = O.round_to(O.qmm(x, wq, s, b, 64, bits), dtype)
    tw, ts, tb = to_torch(wq, s, b, dtype, cuda)
    y = kernels.quantized_matmul(x_torch(x, dtype, cuda), tw, ts, tb, bits=bits, choice=choice)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    return y.float().cpu().numpy(), ref


# the decode workloads at their real sizes
@pytest.mark.parametrize("M,N,K,bits,dtype", [
    (1, 6144, 2560, 4, "bfloat16"),
    (16, 6144, 2560, 4, "bfloat16"),
    (8, 4096, 4096, 4, "float16"),
    (1, 9728, 2560, 8, "bfloat16"),
    (16, 2560, 9728, 8, "bfloat16"),
    (64, 2560, 9728, 8, "bfloat16"),
    (32, 4096, 4096, 4, "bfloat16"),
])
def test_tcv_configs(cuda, M, N, K, bits, dtype):
    y, ref = _run(cuda, M, N, K, bits, dtype, seed=M * 5 + N + bits)
    assert rel_err(y, ref) <= TOL_REL


# ragged shapes: N not a multiple of 128, M not a multiple of the token width, the smallest K, both
# dtypes, an odd number of K slices per CTA
@pytest.mark.parametrize("M,N,K,bits,dtype", [
    (3, 200, 512, 4, "float16"),
    (5, 136, 1024, 4, "bfloat16"),
    (9, 72, 256, 4, "bfloat16"),
    (17, 520, 768, 4, "float16"),
    (33, 96, 2048, 4, "bfloat16"),
    (64, 130, 512, 8, "float16"),
    (11, 64, 384, 8, "bfloat16"),
    (2, 1040, 2048, 8, "float16"),
    (48, 300, 1152, 8, "bfloat16"),
])
def test_tcv_ragged(cuda, M, N, K, bits, dtype):
    y, ref = _run(cuda, M, N, K, bits, dtype, seed=N * 3 + K + M)
    assert rel_err(y, ref) <= TOL_REL


# every split-K factor, forced ring wrap-around (2 weight slots), wider token tiles than needed
@pytest.mark.parametrize("choice", [("tcv", 16, 1, 0), ("tcv", 16, 2, 0), ("tcv", 16, 3, 0), ("tcv", 16, 5, 0),
                                    ("tcv", 16, 8, 0), ("tcv", 16, 1, 2), ("tcv", 16, 3, 2), ("tcv", 32, 2, 0),
                                    ("tcv", 64, 4, 3)])
def test_tcv_every_tiling(cuda, choice):
    y, ref = _run(cuda, 8, 768, 2560, 4, "bfloat16", seed=13, choice=choice)
    assert rel_err(y, ref) <= TOL_REL


# token tiles past 64 tokens: 128- and 256-token tiles on grid z, a ragged last tile, both dtypes
@pytest.mark.parametrize("M,N,K,bits,dtype,ntok", [
    (100, 520, 768, 4, "bfloat16", 0),
    (300, 384, 1024, 4, "float16", 0),
    (130, 272, 512, 8, "bfloat16", 0),
    (513, 256, 768, 4, "bfloat16", 256),
    (200, 300, 1024, 8, "float16", 128),
    (70, 136, 2048, 4, "bfloat16", 16),
])
def test_tcv_token_tiles(cuda, M, N, K, bits, dtype, ntok):
    y, ref = _run(cuda, M, N, K, bits, dtype, seed=M + N * 7 + K, choice=("tcv", ntok, 0, 0))
    assert rel_err(y, ref) <= TOL_REL


# the persistent form (one CTA per SM walking the tiles): ragged tiles, both dtypes and bit widths
@pytest.mark.parametrize("M,N,K,bits,dtype,ntok", [
    (300, 384, 1024, 4, "float16", 0),
    (513, 256, 768, 4, "bfloat16", 256),
    (200, 300, 1024, 8, "float16", 128),
    (70, 136, 2048, 4, "bfloat16", 16),
    (64, 2560, 9728, 8, "bfloat16", 0),
    (40, 1000, 512, 4, "bfloat16", 32),
])
def test_tcv_persistent(cuda, M, N, K, bits, dtype, ntok):
    y, ref = _run(cuda, M, N, K, bits, dtype, seed=M * 3 + N + K, choice=("tcv", ntok, 0, 0, 1))
    assert rel_err(y, ref) <= TOL_REL


def test_tcv_persistent_glu(cuda):
    import torch
    from locals_b200 import kernels

    rng = np.random.default_rng(31)
    M, K, I = 150, 1024, 384
    x = act(rng, M, K, "bfloat16")
    gq, gs, gb = qweights(rng, I, K, 4, "bfloat16")
    uq, us, ub = qweights(rng, I, K, 4, "bfloat16")
    href = O.swiglu(O.round_to(O.qmm(x, gq, gs, gb, 64, 4), "bfloat16"),
                    O.round_to(O.qmm(x, uq, us, ub, 64, 4), "bfloat16"), "bfloat16")
    h = kernels.qmm_glu(x_torch(x, "bfloat16", cuda), to_torch(gq, gs, gb, "bfloat16", cuda),
                        to_torch(uq, us, ub, "bfloat16", cuda), bits=4, choice=("tcv", 0, 0, 0, 1))
    torch.cuda.synchronize()
    assert rel_err(h.float().cpu().numpy(), href) <= 2.0 ** -6
    assert kernels.device_status() == 0


def test_tcv_split_and_glu(cuda):
    # the fused QKV split into three outputs and the fused gate/up SwiGLU on the tensor-core family
    import torch
    from locals_b200 import kernels

    rng = np.random.default_rng(21)
    M, K = 7, 1024
    widths = (256, 128, 128)
    N = sum(widths)
    wq, s, b = qweights(rng, N, K, 4, "bfloat16")
    x = act(rng, M, K, "bfloat16")
    ref = O.round_to(O.qmm(x, wq, s, b, 64, 4), "bfloat16")
    tw, ts, tb = to_torch(wq, s, b, "bfloat16", cuda)
    outs = kernels.qmm_split(x_torch(x, "bfloat16", cuda), tw, ts, tb, widths, bits=4, choice=("tcv", 0, 0, 0))
    got = np.concatenate([o.float().cpu().numpy() for o in outs], axis=1)
    assert rel_err(got, ref) <= TOL_REL

    for bits, I, M in ((4, 384, 7), (8, 200, 7), (4, 256, 200)):
        x = act(rng, M, K, "bfloat16")
        gq, gs, gb = qweights(rng, I, K, bits, "bfloat16")
        uq, us, ub = qweights(rng, I, K, bits, "bfloat16")
        g = O.round_to(O.qmm(x, gq, gs, gb, 64, bits), "bfloat16")
        u = O.round_to(O.qmm(x, uq, us, ub, 64, bits), "bfloat16")
        href = O.swiglu(g, u, "bfloat16")
        gate = to_torch(gq, gs, gb, "bfloat16", cuda)
        up = to_torch(uq, us, ub, "bfloat16", cuda)
        h = kernels.qmm_glu(x_torch(x, "bfloat16", cuda), gate, up, bits=bits, choice=("tcv", 0, 0, 0))
        torch.cuda.synchronize()
        # the intermediate h carries the rounding of gate/up before the activation: 2^-6 relative
        assert rel_err(h.float().cpu().numpy(), href) <= 2.0 ** -6
    assert kernels.device_status() == 0


def test_tcv_matches_qmv(cuda):
    # both decode families agree within tolerance on the same call (two consecutive calls each)
    import torch
    from locals_b200 import kernels

    rng = np.random.default_rng(3)
    wq, s, b = qweights(rng, 1024, 2560, 4, "bfloat16")
    x = x_torch(act(rng, 16, 2560, "bfloat16"), "bfloat16", cuda)
    tw, ts, tb = to_torch(wq, s, b, "bfloat16", cuda)
    ys = [kernels.quantized_matmul(x, tw, ts, tb, bits=4, choice=c).float()
          for c in (("tcv", 0, 0, 0), ("tcv", 0, 0, 0), ("qmv", 0, 0, 0, 0))]
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[1])
    assert rel_err(ys[0].cpu().numpy(), ys[2].cpu().numpy()) <= TOL_REL
