"""One-token MoE decode on the GPU: the gate/up projections of a token's k experts as one fragment-spread launch
(lq_moe_experts with P == k) and the down projections fused with the slot combine (lq_moe_down_combine), against the
CPU oracle and against the unfused grouped path.

Oracle per slot r (locals/moe.py:243-349): h_r = swiglu(T(gate_e x), T(up_e x)), y_r = T(down_e h_r),
y = T(sum_r w_r y_r) in float32 in slot order. Tolerance: max|y - ref| <= 1e-2 max|ref| (fp32 accumulation); the
fused kernel folds nothing differently from the unfused one except the accumulation order of each dot product.
"""

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import TOL_REL, qweights, rel_err, to_torch, x_torch

pytestmark = pytest.mark.gpu

_CACHE = {}


def _experts(E, D, I, dtype, cuda):
    key = (E, D, I, dtype)
    if key not in _CACHE:
        rng = np.random.default_rng(E + D + I)
        mats = []
        for N, Kd in ((I, D), (I, D), (D, I)):
            ws = [qweights(rng, N, Kd, 4, dtype) for _ in range(E)]
            stacked = to_torch(np.stack([w[0] for w in ws]), np.stack([w[1] for w in ws]),
                               np.stack([w[2] for w in ws]), dtype, cuda)
            mats.append((ws, stacked))
        _CACHE.clear()
        _CACHE[key] = mats
    return _CACHE[key]


def _oracle(x, inds, wts, mats, dtype):
    (g, _), (u, _), (d, _) = mats
    k = inds.shape[1]
    ys = np.zeros((k, d[0][0].shape[0]), np.float32)
    hs = []
    for r in range(k):
        e = int(inds[0, r])
        h = O.swiglu(O.linear(x, g[e] + (4,), dtype), O.linear(x, u[e] + (4,), dtype), dtype)
        hs.append(h[0])
        ys[r] = O.linear(h, d[e] + (4,), dtype)[0]
    y = O.round_to(O.combine(ys, wts), dtype)
    return np.stack(hs), y


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("E,D,I,k", [(64, 2048, 768, 4), (16, 512, 256, 4), (8, 768, 512, 2), (32, 1024, 512, 3)])
@pytest.mark.parametrize("sorted_grouping", [False, True])
def test_one_token_glu_and_down_combine(cuda, dtype, E, D, I, k, sorted_grouping):
    import torch
    from locals_b200 import kernels, moe

    mats = _experts(E, D, I, dtype, cuda)
    rng = np.random.default_rng(E * k + D)
    x = O.round_to(rng.standard_normal((1, D)).astype(np.float32), dtype)
    inds = rng.choice(E, k, replace=False).astype(np.int32)[None, :]
    wts = rng.random((1, k)).astype(np.float32)
    wts /= wts.sum()
    ref_h, ref_y = _oracle(x, inds, wts, mats, dtype)

    ti = torch.from_numpy(inds).to(cuda)
    tw = torch.from_numpy(wts).to(cuda)
    grouping = moe.group(ti, E) if sorted_grouping else moe.direct_grouping(ti)
    gate, up, down = mats[0][1], mats[1][1], mats[2][1]
    h = moe.experts(x_torch(x, dtype, cuda), grouping, [gate, up], I, max_rows=1, gather_k=k)
    y = moe.down_combine(h, grouping, tw, down)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    assert y is not None
    # h rows are in the grouping's order: row j is pair order[j]
    order = grouping[0].cpu().numpy()
    assert rel_err(h.float().cpu().numpy(), ref_h[order]) <= TOL_REL
    assert rel_err(y.float().cpu().numpy(), ref_y) <= TOL_REL
    # the unfused path (grouped down projection, then the combine kernel) agrees within the same bound
    ys = moe.experts(h, grouping, [down], D, max_rows=1)
    y2 = moe.combine(ys, tw, grouping[4])
    torch.cuda.synchronize()
    assert rel_err(y.float().cpu().numpy(), y2.float().cpu().numpy()) <= TOL_REL


def test_down_combine_declines_shapes_outside_it(cuda):
    """K % 256 != 0 (an intermediate of 384) or more than four slots: LQ_E_SHAPE, so the caller takes the two-call
    path; the MoE layer still computes the right answer through it."""
    import torch
    from locals_b200 import moe

    E, D, I, k = 16, 512, 384, 4
    mats = _experts(E, D, I, "bfloat16", cuda)
    ti = torch.tensor([[3, 1, 7, 12]], dtype=torch.int32, device=cuda)
    tw = torch.full((1, k), 0.25, dtype=torch.float32, device=cuda)
    h = torch.randn((k, I), device=cuda).to(torch.bfloat16)
    assert moe.down_combine(h, moe.direct_grouping(ti), tw, mats[2][1]) is None
    rng = np.random.default_rng(5)
    x = O.round_to(rng.standard_normal((1, D)).astype(np.float32), "bfloat16")
    wr = O.round_to((rng.standard_normal((E, D)) * 0.02).astype(np.float32), "float16")
    layer = moe.MoELayer(torch.from_numpy(wr).to(cuda, torch.float16), mats[0][1], mats[1][1], mats[2][1], top_k=k)
    xt = x_torch(x, "bfloat16", cuda)
    inds, wts = layer.route(xt)
    y = layer(xt)
    _, ref_y = _oracle(x, inds.cpu().numpy(), wts.cpu().numpy(), mats, "bfloat16")
    torch.cuda.synchronize()
    assert rel_err(y.float().cpu().numpy(), ref_y) <= TOL_REL
