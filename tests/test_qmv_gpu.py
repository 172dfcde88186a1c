"""Parity of the decode family (qmv) against the CPU oracle, through the C ABI (ctypes) on the GPU.

Tolerance: max|y - ref| <= 1e-2 * max|ref| with fp32 accumulation; the reference's
own kernel tests use 0.02 * (1 + max|ref|) (tests/test_q35_kernels.py:60-93). Codes are bit-exact:
the GPU quantizer must reproduce the oracle's codes, scales and biases exactly.
"""

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import TOL_REL, act, qweights, rel_err, to_torch, x_torch

pytestmark = pytest.mark.gpu


def _run(cuda, M, N, K, bits, dtype, seed, choice=None):
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


# the decode workloads at their real sizes (fp16 4096x4096 at M=8; the fused QKV 6144x2560 bf16;
# the 8-bit MLP projections)
@pytest.mark.parametrize("M,N,K,bits,dtype", [
    (8, 4096, 4096, 4, "float16"),
    (1, 6144, 2560, 4, "bfloat16"),
    (4, 6144, 2560, 4, "bfloat16"),
    (8, 6144, 2560, 4, "bfloat16"),
    (16, 6144, 2560, 4, "bfloat16"),
    (1, 9728, 2560, 8, "bfloat16"),
    (16, 2560, 9728, 8, "bfloat16"),
    (64, 2560, 9728, 8, "bfloat16"),
])
def test_qmm_configs(cuda, M, N, K, bits, dtype):
    y, ref = _run(cuda, M, N, K, bits, dtype, seed=M * 7 + N + bits)
    assert rel_err(y, ref) <= TOL_REL


# ragged and odd shapes: N not a multiple of the row tile, M between token tiles, both dtypes, K
# with a partial last chunk (8-bit K % 512 != 0) and the smallest accepted K
@pytest.mark.parametrize("M,N,K,bits,dtype", [
    (3, 200, 512, 4, "float16"),
    (5, 136, 1024, 4, "bfloat16"),
    (9, 72, 256, 4, "bfloat16"),
    (17, 520, 768, 4, "float16"),
    (33, 96, 2048, 4, "bfloat16"),
    (64, 130, 512, 8, "float16"),
    (11, 64, 384, 8, "bfloat16"),
    (2, 1040, 2048, 8, "float16"),
    (100, 96, 512, 4, "bfloat16"),   # more rows than one pass: weights streamed per 64 rows
])
def test_qmm_ragged(cuda, M, N, K, bits, dtype):
    y, ref = _run(cuda, M, N, K, bits, dtype, seed=N * 3 + K + M)
    assert rel_err(y, ref) <= TOL_REL


@pytest.mark.parametrize("choice", [("qmv", 1, 1, 1, 1), ("qmv", 1, 2, 5, 0), ("qmv", 2, 1, 5, 2),
                                    ("qmv", 2, 4, 1, 0), ("qmv", 4, 2, 2, 0), ("qmv", 8, 2, 3, 1), ("qmv", 1, 4, 3, 0)])
def test_qmm_every_tiling(cuda, choice):
    # all tilings give the same answer within tolerance (the reference checks its candidates the same way)
    y, ref = _run(cuda, 8, 768, 2560, 4, "bfloat16", seed=11, choice=choice)
    assert rel_err(y, ref) <= TOL_REL


def test_rows_independent(cuda):
    # a row's result does not depend on the other rows of the batch (tests/test_nax_kernel.py:35-45)
    import torch
    from locals_b200 import kernels

    rng = np.random.default_rng(5)
    wq, s, b = qweights(rng, 512, 1024, 4, "bfloat16")
    tw, ts, tb = to_torch(wq, s, b, "bfloat16", cuda)
    x = x_torch(act(rng, 16, 1024, "bfloat16"), "bfloat16", cuda)
    full = kernels.quantized_matmul(x, tw, ts, tb)
    for m in (0, 7, 15):
        one = kernels.quantized_matmul(x[m:m + 1].contiguous(), tw, ts, tb)
        torch.testing.assert_close(one[0].float(), full[m].float(), rtol=0, atol=2e-2 * float(full.abs().max()))


@pytest.mark.parametrize("bits,dtype", [(4, "bfloat16"), (8, "bfloat16"), (4, "float16"), (8, "float16")])
def test_gpu_quantize_bit_exact(cuda, bits, dtype):
    import torch
    from locals_b200 import kernels

    rng = np.random.default_rng(bits)
    w = (rng.standard_normal((96, 512)) * 0.02).astype(np.float32)
    w[3, :64] = 0.0  # a zero group (q0 == 0 path)
    w[4, :64] = 0.125  # a constant group
    wq, s, b = O.quantize(w, 64, bits, dtype)
    tdt = torch.bfloat16 if dtype == "bfloat16" else torch.float16
    gq, gs, gb = kernels.quantize(torch.from_numpy(w).to(cuda), 64, bits, dtype=tdt)
    assert np.array_equal(gq.cpu().numpy().view(np.uint32), wq)
    assert np.array_equal(gs.float().cpu().numpy(), s)
    assert np.array_equal(gb.float().cpu().numpy(), b)
    # unpacked codes bit-exact
    assert np.array_equal(O.unpack(gq.cpu().numpy().view(np.uint32), 512, bits), O.unpack(wq, 512, bits))


@pytest.mark.parametrize("bits", [4, 8])
def test_gpu_dequantize(cuda, bits):
    import torch
    from locals_b200 import kernels

    rng = np.random.default_rng(9)
    wq, s, b = qweights(rng, 64, 512, bits, "bfloat16")
    tw, ts, tb = to_torch(wq, s, b, "bfloat16", cuda)
    got = kernels.dequantize(tw, ts, tb, 64, bits).float().cpu().numpy()
    ref = O.round_to(O.dequantize(wq, s, b, 64, bits), "bfloat16")
    # fma vs mul+add: at most one bf16 ulp apart
    assert np.max(np.abs(got - ref)) <= 2 ** -7 * np.max(np.abs(ref))
    torch.cuda.synchronize()


def test_fused_qkv_split(cuda):
    """The fused QKV decode projection: q/k/v concatenated [6144, 2560], output split into q [M,32,128], k/v [M,8,128]."""
    from locals_b200 import kernels
    from locals_b200.fuse import FusedQKV
    from locals_b200.kernels import QuantizedLinear

    rng = np.random.default_rng(1)
    M, D = 16, 2560
    parts = [qweights(rng, n, D, 4, "bfloat16") for n in (4096, 1024, 1024)]
    mods = [QuantizedLinear(*to_torch(*p, "bfloat16", cuda)) for p in parts]
    fused = FusedQKV(*mods, n_heads=32, n_kv_heads=8, head_dim=128)
    x = act(rng, M, D, "bfloat16")
    q, k, v = fused(x_torch(x, "bfloat16", cuda))
    assert q.shape == (M, 32, 128) and k.shape == (M, 8, 128) and v.shape == (M, 8, 128)
    for got, p in zip((q, k, v), parts):
        ref = O.round_to(O.qmm(x, *p), "bfloat16")
        assert rel_err(got.reshape(M, -1).float().cpu().numpy(), ref) <= TOL_REL
    # fusion exactness: the fused matmul equals the three separate ones (tests/test_kernel_patching.py:28-37)
    whole = kernels.quantized_matmul(x_torch(x, "bfloat16", cuda), fused.qkv.weight, fused.qkv.scales,
                                     fused.qkv.biases)
    assert np.array_equal(whole[:, :4096].float().cpu().numpy(), q.reshape(M, -1).float().cpu().numpy())


@pytest.mark.parametrize("M", [1, 4, 16, 64])
def test_fused_mlp_8bit(cuda, M):
    """The 8-bit MLP block: y = down(silu(gate x) * (up x)), 8-bit, gate/up fused with the SiLU.mul epilogue."""
    from locals_b200.fuse import FusedMLP
    from locals_b200.kernels import QuantizedLinear

    rng = np.random.default_rng(2)
    D, I = 2560, 9728
    g, u = qweights(rng, I, D, 8, "bfloat16"), qweights(rng, I, D, 8, "bfloat16")
    d = qweights(rng, D, I, 8, "bfloat16")
    mlp = FusedMLP(*[QuantizedLinear(*to_torch(*p, "bfloat16", cuda), bits=8) for p in (g, u, d)])
    x = act(rng, M, D, "bfloat16")
    h = mlp.hidden_act(x_torch(x, "bfloat16", cuda))
    href = O.swiglu(O.round_to(O.qmm(x, *g, 64, 8), "bfloat16"), O.round_to(O.qmm(x, *u, 64, 8), "bfloat16"),
                    "bfloat16")
    # h passes through four roundings to bf16 (g, u, sigmoid, g*sig) before act*u; a one-ulp difference in g
    # moves h by up to ~3 ulps. The reference bounds its own expert kernels' SwiGLU output the same way:
    # within 2^-6 * max of the fp32 reference (tests/test_flint.py:80-111).
    assert rel_err(h.float().cpu().numpy(), href) <= 2 ** -6
    y = mlp(x_torch(x, "bfloat16", cuda))
    yref = O.round_to(O.qmm(href, *d, 64, 8), "bfloat16")
    assert rel_err(y.float().cpu().numpy(), yref) <= TOL_REL
