"""Parity of the group-per-warp decode family (qmvg) against the CPU oracle, through the C ABI on the GPU.

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


def _run(cuda, M, N, K, dtype, seed, choice=("qmvg", 0, 0)):
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
def test_qmvg_configs(cuda, M, N, K, dtype):
    y, ref = _run(cuda, M, N, K, dtype, seed=M * 13 + N + K)
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
def test_qmvg_ragged(cuda, M, N, K, dtype):
    y, ref = _run(cuda, M, N, K, dtype, seed=N * 3 + K + M)
    assert rel_err(y, ref) <= TOL_REL


# 97 fragments: FR requests 1-4 give grids of 97, 49, 33 and 25 CTAs (FR or FR - 1 fragments each); NS pins the ring
@pytest.mark.parametrize("choice", [("qmvg", 1, 0), ("qmvg", 2, 0), ("qmvg", 3, 0), ("qmvg", 4, 0), ("qmvg", 3, 1),
                                    ("qmvg", 2, 2), ("qmvg", 4, 3)])
def test_qmvg_every_tiling(cuda, choice):
    y, ref = _run(cuda, 16, 1552, 2560, "bfloat16", seed=21, choice=choice)
    assert rel_err(y, ref) <= TOL_REL


def test_qmvg_split_outputs(cuda):
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
    outs = kernels.qmm_split(x_torch(x, "bfloat16", cuda), tw, ts, tb, widths, choice=("qmvg", 0, 0))
    torch.cuda.synchronize()
    got = np.concatenate([o.float().cpu().numpy() for o in outs], axis=1)
    assert rel_err(got, ref) <= TOL_REL


def test_qmvg_matches_qmv(cuda):
    # both decode families give the same answer within tolerance on the same call
    y0, ref = _run(cuda, 16, 6144, 2560, "bfloat16", seed=5, choice=("qmv", 0, 0, 0, 0))
    y1, _ = _run(cuda, 16, 6144, 2560, "bfloat16", seed=5)
    assert rel_err(y1, y0) <= TOL_REL
