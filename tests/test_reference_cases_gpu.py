"""The reference's own kernel-test cases, on the GPU, against the CPU oracle.

The reference checks every kernel it may choose against MLX at run time (it stores no golden vectors); MLX cannot run
here, so the oracle's restatement of MLX's affine arithmetic stands in for it, and each case keeps the reference
test's shapes, row counts, dtypes and tolerance:

* tests/test_q35_kernels.py:60-93 -- (N, K) in {(512, 2048), (2048, 6144), (8224, 2048)} x M in {1, 2, 3, 5, 8, 11, 16},
  bf16 and fp16, every candidate tiling, |y - ref| <= 0.02 (1 + max|ref|). N = 8224 is not a multiple of any row tile.
* tests/test_nax_kernel.py:11-45 -- the small-M matrix-unit shapes (2560, 4096) ... (14336, 5120) at M = 1..32,
  |y - ref| <= 0.05 (1 + max|ref|) (the tuner's acceptance bound, locals/kernels.py:677); rows are their own (row i of
  a 12-row product equals the 1-row product of row i).
* tests/test_kernel_patching.py:154-175 -- the exactness bound for kernels that fold the scale per group in float:
  |y - exact| <= |mlx - exact|_max + 2^-7 max|exact|, exact = x . dequant(W)^T in float64, mlx = the restated MLX
  kernel (the oracle's s * sum(q x) + b * sum(x) in float32, rounded to the dtype).
* tests/test_moe_kernel.py:25-51 -- grouped experts D = 512, I = 384, E = 16, k = 4 at 1, 5 and 33 rows, x ~ N(0, 0.5),
  bf16 (0.02 (1 + max)) and fp16 (2e-3 (1 + max)) -- I = 384 is not a multiple of 256.

Weights are seeded N(0, 0.02) Gaussians quantized by the oracle (the reference uses MLX's own initialisation); the
north star's tighter bound max|y - ref| <= 1e-2 max|ref| is checked as well wherever the reference's bound is looser.
"""

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import TOL_REL, to_torch, x_torch

pytestmark = pytest.mark.gpu

Q35_SHAPES = [(512, 2048), (2048, 6144), (8224, 2048)]
Q35_ROWS = [1, 2, 3, 5, 8, 11, 16]
NAX_SHAPES = [(2560, 4096), (10240, 2560), (2560, 9216), (4096, 12288), (5120, 6144), (14336, 5120)]
NAX_ROWS = [1, 2, 5, 6, 8, 12, 15, 16, 17, 24, 31, 32]

_CACHE = {}


def _layer(N, K, dtype, seed, std=0.02):
    key = (N, K, dtype, seed, std)
    if key not in _CACHE:
        rng = np.random.default_rng(seed)
        w = (rng.standard_normal((N, K), dtype=np.float32) * std).astype(np.float32)
        _CACHE.clear()  # one large layer at a time
        _CACHE[key] = O.quantize(w, 64, 4, dtype)
    return _CACHE[key]


def _device_layer(wq, s, b, dtype, cuda):
    return to_torch(wq, s, b, dtype, cuda)


def _all_choices(M, K, N, dtype):
    import torch
    from locals_b200 import kernels

    tdt = torch.bfloat16 if dtype == "bfloat16" else torch.float16
    return [None] + kernels.candidates(M, K, N, 4, tdt)


def _run(x, tw, ts, tb, choice, cuda, dtype):
    from locals_b200 import kernels

    return kernels.quantized_matmul(x_torch(x, dtype, cuda), tw, ts, tb, bits=4, choice=choice)


def _check_status():
    import torch
    from locals_b200 import kernels

    torch.cuda.synchronize()
    assert kernels.device_status() == 0


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("N,K", Q35_SHAPES)
def test_q35_kernel_cases(cuda, N, K, dtype):
    wq, s, b = _layer(N, K, dtype, seed=N + K)
    tw, ts, tb = _device_layer(wq, s, b, dtype, cuda)
    rng = np.random.default_rng(K)
    xall = O.round_to(rng.standard_normal((max(Q35_ROWS), K), dtype=np.float32), dtype)
    refall = O.round_to(O.qmm(xall, wq, s, b, 64, 4), dtype)  # rows are independent: slice per M
    for M in Q35_ROWS:
        x, ref = xall[:M], refall[:M]
        m = float(np.abs(ref).max())
        for choice in _all_choices(M, K, N, dtype):
            y = _run(x, tw, ts, tb, choice, cuda, dtype).float().cpu().numpy()
            assert y.shape == (M, N)
            err = float(np.abs(y - ref).max())
            assert err <= 0.02 * (1 + m), (M, choice, err)
            assert err <= TOL_REL * m, (M, choice, err)
    _check_status()


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("N,K", NAX_SHAPES)
def test_nax_shape_cases(cuda, N, K, dtype):
    wq, s, b = _layer(N, K, dtype, seed=N + K, std=0.05)
    tw, ts, tb = _device_layer(wq, s, b, dtype, cuda)
    rng = np.random.default_rng(N)
    xall = O.round_to(rng.standard_normal((max(NAX_ROWS), K), dtype=np.float32), dtype)
    refall = O.round_to(O.qmm(xall, wq, s, b, 64, 4), dtype)
    for M in NAX_ROWS:
        x, ref = xall[:M], refall[:M]
        m = float(np.abs(ref).max())
        for choice in [None] + [c for c in _all_choices(M, K, N, dtype)[1:] if c[0] != "qmv"][:6]:
            y = _run(x, tw, ts, tb, choice, cuda, dtype).float().cpu().numpy()
            err = float(np.abs(y - ref).max())
            assert err <= 0.05 * (1 + m), (M, choice, err)
            assert err <= TOL_REL * m, (M, choice, err)
    _check_status()


def test_rows_of_a_batch_are_their_own(cuda):
    """Row i of a 12-row product equals the 1-row product of row i (tests/test_nax_kernel.py:36-45), for the
    library's automatic choice at both row counts."""
    N, K, dtype = 2560, 4096, "bfloat16"
    wq, s, b = _layer(N, K, dtype, seed=7, std=0.05)
    tw, ts, tb = _device_layer(wq, s, b, dtype, cuda)
    x = O.round_to(np.random.default_rng(3).standard_normal((12, K), dtype=np.float32), dtype)
    full = _run(x, tw, ts, tb, None, cuda, dtype).float().cpu().numpy()
    for i in (0, 5, 11):
        one = _run(x[i:i + 1], tw, ts, tb, None, cuda, dtype).float().cpu().numpy()
        assert float(np.abs(full[i:i + 1] - one).max()) <= 0.05 * (1.0 + float(np.abs(one).max()))
    _check_status()


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
def test_exactness_bound(cuda, dtype):
    """Every decode choice is no further from the exact product than the restated MLX kernel, give or take one
    rounding of the output (2^-7 max|exact|), at 1..16 rows, with and without whole tiles of rows."""
    for N, K in [(256, 512), (1040, 2048)]:
        rng = np.random.default_rng(N)
        wq, s, b = O.quantize((rng.standard_normal((N, K), dtype=np.float32) * 0.02).astype(np.float32), 64, 4, dtype)
        deq = O.dequantize(wq, s, b, 64, 4).astype(np.float64)
        tw, ts, tb = _device_layer(wq, s, b, dtype, cuda)
        for M in (1, 3, 8, 9, 16):
            x = O.round_to((np.random.default_rng(M).standard_normal((M, K), dtype=np.float32) * 0.5), dtype)
            exact = x.astype(np.float64) @ deq.T
            mlx = O.round_to(O.qmm(x, wq, s, b, 64, 4), dtype).astype(np.float64)
            room = float(np.abs(mlx - exact).max()) + 2.0 ** -7 * float(np.abs(exact).max())
            for choice in _all_choices(M, K, N, dtype):
                y = _run(x, tw, ts, tb, choice, cuda, dtype).double().cpu().numpy()
                assert float(np.abs(y - exact).max()) <= room, (N, K, M, choice)
    _check_status()


def _moe_arrays(E, D, I, dtype, seed):
    rng = np.random.default_rng(seed)
    mats = []
    for N, Kd in ((I, D), (I, D), (D, I)):
        ws = [O.quantize((rng.standard_normal((N, Kd), dtype=np.float32) * 0.02).astype(np.float32), 64, 4, dtype)
              for _ in range(E)]
        mats.append(ws)
    return mats


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("rows", [1, 5, 33])
def test_grouped_experts_case(cuda, dtype, rows):
    import torch
    from locals_b200 import moe

    D, I, E, k = 512, 384, 16, 4
    gate, up, down = _moe_arrays(E, D, I, dtype, seed=0)

    def stack(ws):
        return to_torch(np.stack([w[0] for w in ws]), np.stack([w[1] for w in ws]), np.stack([w[2] for w in ws]),
                        dtype, cuda)

    rng = np.random.default_rng(rows)
    x = O.round_to(rng.normal(0, 0.5, (rows, D)).astype(np.float32), dtype)
    inds = np.stack([rng.choice(E, k, replace=False) for _ in range(rows)]).astype(np.uint32)
    got = moe.switch_glu(x_torch(x, dtype, cuda), torch.from_numpy(inds.astype(np.int32)).to(cuda), stack(gate),
                         stack(up), stack(down)).float().cpu().numpy().reshape(rows, k, D)
    _check_status()
    want = np.zeros((rows, k, D), np.float32)
    for r in range(rows):
        for j in range(k):
            e = int(inds[r, j])
            xe = x[r:r + 1]
            h = O.swiglu(O.linear(xe, gate[e] + (4,), dtype), O.linear(xe, up[e] + (4,), dtype), dtype)
            want[r, j] = O.linear(h, down[e] + (4,), dtype)[0]
    tol = 0.02 if dtype == "bfloat16" else 2e-3
    assert float(np.abs(got - want).max()) <= tol * (1 + float(np.abs(want).max()))
