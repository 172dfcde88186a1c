"""The residual add + RMS norm, the MoE combine + norm and row packing on the GPU against the CPU oracle.

h and y are bit-exact (elementwise adds rounded once); n may differ from the oracle by the rounding of a
differently ordered fp32 sum of squares: within 2^-6 relative of the value, and equal on >= 98% of values.
"""

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import TOL_REL, act, qweights, rel_err, to_torch, x_torch

pytestmark = pytest.mark.gpu


def _t(a, dtype, cuda):
    return x_torch(np.ascontiguousarray(a, np.float32), dtype, cuda)


def _close_n(got, ref):
    got, ref = np.asarray(got, np.float32), np.asarray(ref, np.float32)
    assert np.max(np.abs(got - ref) / (np.abs(ref) + 1e-3)) <= 2 ** -6
    assert np.mean(got == ref) >= 0.98


@pytest.mark.parametrize("rows,D,dtype", [(1, 2560, "bfloat16"), (16, 2560, "bfloat16"), (300, 4096, "float16"),
                                          (7, 8192, "bfloat16"), (5, 72, "float16"), (64, 2048, "bfloat16")])
def test_add_rms(cuda, rows, D, dtype):
    import torch
    from locals_b200 import kernels, norm

    rng = np.random.default_rng(rows + D)
    x = act(rng, rows, D, dtype)
    r = act(rng, rows, D, dtype)
    w = O.round_to((1 + 0.1 * rng.standard_normal(D)).astype(np.float32), dtype)
    h_ref, n_ref = O.add_rms(x, r, w, 1e-6, dtype)
    h, n = norm.add_rms(_t(x, dtype, cuda), _t(r, dtype, cuda), _t(w, dtype, cuda), 1e-6)
    torch.cuda.synchronize()
    assert np.array_equal(h.float().cpu().numpy(), h_ref)
    _close_n(n.float().cpu().numpy(), n_ref)
    assert kernels.device_status() == 0


@pytest.mark.parametrize("T,k,D,shared", [(1, 4, 2048, False), (16, 4, 2048, True), (100, 8, 2560, False)])
def test_combine_norm(cuda, T, k, D, shared):
    import torch
    from locals_b200 import kernels, moe

    dtype = "bfloat16"
    rng = np.random.default_rng(T * k + D)
    ys = act(rng, T * k, D, dtype)
    wt = rng.random((T, k)).astype(np.float32)
    res = act(rng, T, D, dtype)
    nw = O.round_to((1 + 0.1 * rng.standard_normal(D)).astype(np.float32), dtype)
    sh = act(rng, T, D, dtype) if shared else None
    # the kernel reads slot rows through pos: store them permuted and pass the inverse
    perm = rng.permutation(T * k)
    ys_perm = np.empty_like(ys)
    ys_perm[perm] = ys
    y_ref, n_ref = O.combine_norm(ys, wt, res, nw, 1e-5, dtype, shared=sh)
    y, n = moe.combine_norm(_t(ys_perm, dtype, cuda), torch.from_numpy(wt).to(cuda),
                            torch.from_numpy(perm.astype(np.int32)).to(cuda), _t(res, dtype, cuda),
                            _t(nw, dtype, cuda), 1e-5, None if sh is None else _t(sh, dtype, cuda))
    torch.cuda.synchronize()
    assert np.array_equal(y.float().cpu().numpy(), y_ref)
    _close_n(n.float().cpu().numpy(), n_ref)
    assert kernels.device_status() == 0


def test_packed_rows_linear(cuda):
    # a right-padded batch through a packed linear: valid rows as the unpacked call, padding rows zero
    import torch
    from locals_b200 import kernels

    rng = np.random.default_rng(9)
    B, L, K, N = 3, 5, 2560, 1024
    lengths = [5, 2, 3]
    wq, s, b = qweights(rng, N, K, 4, "bfloat16")
    lin = kernels.QuantizedLinear(*to_torch(wq, s, b, "bfloat16", cuda))
    x = x_torch(act(rng, B * L, K, "bfloat16"), "bfloat16", cuda).reshape(B, L, K)
    full = lin(x).float().cpu().numpy().reshape(B, L, N)
    with kernels.packed_rows(B, L, lengths, device=cuda):
        packed = lin(x).float().cpu().numpy().reshape(B, L, N)
    for bi, n in enumerate(lengths):
        assert rel_err(packed[bi, :n], full[bi, :n]) <= TOL_REL
        assert not packed[bi, n:].any()
    ref = O.round_to(O.qmm(x.float().cpu().numpy().reshape(B * L, K), wq, s, b, 64, 4), "bfloat16").reshape(B, L, N)
    for bi, n in enumerate(lengths):
        assert rel_err(packed[bi, :n], ref[bi, :n]) <= TOL_REL


def test_scatter_rows_bounds(cuda):
    import torch
    from locals_b200 import kernels

    ys = torch.arange(4 * 16, dtype=torch.float32, device=cuda).reshape(4, 16).to(torch.bfloat16)
    idx = torch.tensor([5, 0, 2, 7], dtype=torch.int32, device=cuda)
    y = kernels.scatter_rows(ys, idx, 8).float().cpu()
    want = torch.zeros(8, 16)
    want[idx.cpu().long()] = ys.float().cpu()
    assert torch.equal(y, want)
    assert kernels.device_status() == 0
