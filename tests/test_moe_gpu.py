"""Parity of the routed-MoE kernels against the CPU oracle on the GPU (64 experts,
top-4, hidden 2048, expert intermediate 768, 4-bit g64, router Wr fp16, x bf16, softmax routing).

Selection parity compares per-token expert sets (tests/test_flint.py:59-66); tokens whose 4th and 5th
probabilities are closer than 1e-5 relative are reported as ambiguous, not silently passed.
"""

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import TOL_REL, act, qweights, rel_err, to_torch, x_torch

pytestmark = pytest.mark.gpu


def _router_inputs(rng, M, E, D):
    x = act(rng, M, D, "bfloat16")
    wr = O.round_to((rng.standard_normal((E, D)) * 0.02).astype(np.float32), "float16")
    return x, wr


def test_router_logits(cuda):
    import torch
    from locals_b200 import moe

    rng = np.random.default_rng(3)
    x, wr = _router_inputs(rng, 64, 64, 2048)
    got = moe.router_logits(x_torch(x, "bfloat16", cuda), torch.from_numpy(wr).to(cuda, torch.float16))
    ref = O.router(x, wr)
    # float32 dot products of exact 16-bit inputs: only the summation order differs
    # (the reference's router test: 1e-5 relative, tests/test_flint.py:69-77)
    np.testing.assert_allclose(got.cpu().numpy(), ref, rtol=1e-5, atol=1e-5 * np.abs(ref).max())


@pytest.mark.parametrize("mode", ["softmax", "sigmoid"])
def test_route_topk(cuda, mode):
    import torch
    from locals_b200 import moe

    rng = np.random.default_rng(4)
    logits = rng.standard_normal((512, 64)).astype(np.float32)
    logits[0] = 0.5  # all tied: experts 0..3
    logits[1, :] = -1.0
    logits[1, [5, 9]] = 2.0  # tie at the top: 5 before 9
    got_i, got_w = moe.route_topk(torch.from_numpy(logits).to(cuda), 4, moe.SOFTMAX if mode == "softmax" else moe.SIGMOID)
    ref_i, ref_w = O.topk(logits, 4, mode)
    gi = got_i.cpu().numpy().astype(np.uint32)
    assert np.array_equal(gi, ref_i)
    np.testing.assert_allclose(got_w.cpu().numpy(), ref_w, rtol=1e-5, atol=1e-6)


def test_route_topk_nan(cuda):
    # a NaN logit: still k distinct valid experts (tests/test_flint.py:114-130)
    import torch
    from locals_b200 import moe

    logits = np.random.default_rng(8).standard_normal((4, 64)).astype(np.float32)
    logits[:, 3] = np.nan
    i, w = moe.route_topk(torch.from_numpy(logits).to(cuda), 4, moe.SIGMOID)
    i = i.cpu().numpy()
    for row in i:
        assert len(set(row.tolist())) == 4 and row.max() < 64 and 3 not in row.tolist()


@pytest.mark.parametrize("P,E", [(4, 64), (2048, 64), (37, 8), (300, 512), (20000, 64), (9000, 1024)])
def test_group(cuda, P, E):
    import torch
    from locals_b200 import moe

    rng = np.random.default_rng(P + E)
    inds = rng.integers(0, E, P).astype(np.int32)
    order, starts, experts, nseg, pos = moe.group(torch.from_numpy(inds).to(cuda), E)
    r_order, r_starts, r_experts, r_nseg = O.group(inds.astype(np.uint32), E)
    n = int(nseg.cpu()[0])
    assert n == r_nseg
    assert np.array_equal(order.cpu().numpy(), r_order)
    assert np.array_equal(starts.cpu().numpy()[: n + 1], r_starts[: n + 1])
    assert np.array_equal(experts.cpu().numpy()[:n], r_experts[:n])
    assert np.array_equal(pos.cpu().numpy()[r_order], np.arange(P))


_EXPERT_CACHE = {}


def _experts(rng, E, D, I, cuda):
    key = (E, D, I)
    if key in _EXPERT_CACHE:
        return _EXPERT_CACHE[key]
    gate = [qweights(rng, I, D, 4, "bfloat16") for _ in range(E)]
    up = [qweights(rng, I, D, 4, "bfloat16") for _ in range(E)]
    down = [qweights(rng, D, I, 4, "bfloat16") for _ in range(E)]

    def stack(ws):
        return to_torch(np.stack([w[0] for w in ws]), np.stack([w[1] for w in ws]), np.stack([w[2] for w in ws]),
                        "bfloat16", cuda)

    _EXPERT_CACHE[key] = (gate, up, down, stack(gate), stack(up), stack(down))
    return _EXPERT_CACHE[key]


@pytest.mark.parametrize("M", [1, 8, 16, 64, 512])
def test_moe_layer(cuda, M):
    import torch
    from locals_b200 import moe

    rng = np.random.default_rng(3)
    E, K, D, I = 64, 4, 2048, 768
    x, wr = _router_inputs(rng, M, E, D)
    gate, up, down, tg, tu, td = _experts(rng, E, D, I, cuda)
    layer = moe.MoELayer(torch.from_numpy(wr).to(cuda, torch.float16), tg, tu, td, top_k=K)
    xt = x_torch(x, "bfloat16", cuda)
    inds, wts = layer.route(xt)
    y = layer(xt)
    torch.cuda.synchronize()
    from locals_b200 import kernels

    assert kernels.device_status() == 0
    # routing: same expert sets; ambiguous tokens reported
    logits = O.router(x, wr)
    r_inds, r_w = O.topk(logits, K, "softmax")
    probs = np.exp(logits - logits.max(1, keepdims=True))
    probs /= probs.sum(1, keepdims=True)
    srt = -np.sort(-probs, 1)
    ambiguous = np.where((srt[:, K - 1] - srt[:, K]) <= 1e-5 * srt[:, K - 1])[0]
    gi = inds.cpu().numpy()
    for t in range(M):
        if t in ambiguous:
            continue
        assert set(gi[t].tolist()) == set(r_inds[t].tolist()), t
    # outputs: oracle on the GPU's routing (so an ambiguous token does not mask an expert bug)
    ref = O.moe(x, gi.astype(np.uint32), wts.cpu().numpy(), [g + (4,) for g in gate], [u + (4,) for u in up],
                [d + (4,) for d in down], "bfloat16")
    assert rel_err(y.float().cpu().numpy(), ref) <= TOL_REL


@pytest.mark.parametrize("T", [1, 16, 512])
def test_route_fused(cuda, T):
    # router logits + top-k in one kernel: same expert sets as the two-kernel path, weights within 1e-5
    import torch
    from locals_b200 import moe

    rng = np.random.default_rng(T)
    x, wr = _router_inputs(rng, T, 64, 2048)
    xt, wt = x_torch(x, "bfloat16", cuda), torch.from_numpy(wr).to(cuda, torch.float16)
    i1, w1 = moe.route(xt, wt, 4)
    i2, w2 = moe.route_topk(moe.router_logits(xt, wt), 4)
    assert np.array_equal(i1.cpu().numpy(), i2.cpu().numpy())
    np.testing.assert_allclose(w1.cpu().numpy(), w2.cpu().numpy(), rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("T,E,k,mode", [(40, 64, 4, 0), (37, 20, 3, 1), (130, 128, 8, 0), (100, 64, 4, 1)])
def test_route_batched_equals_one_token(cuda, T, E, k, mode):
    """Batched routing (several tokens a warp: the cluster kernel up to 64 tokens, the tiled kernel above) keeps the
    one-warp dot's summation order, so each token's experts and weights are bit-identical to routing it alone."""
    import torch
    from locals_b200 import moe

    rng = np.random.default_rng(T + E)
    x, wr = _router_inputs(rng, T, E, 2048)
    xt, wt = x_torch(x, "bfloat16", cuda), torch.from_numpy(wr).to(cuda, torch.float16)
    ib, wb = moe.route(xt, wt, k, mode)
    for t in range(T):
        i1, w1 = moe.route(xt[t:t + 1].contiguous(), wt, k, mode)
        assert torch.equal(ib[t:t + 1], i1)
        assert torch.equal(wb[t:t + 1], w1)


@pytest.mark.parametrize("M", [1, 3])
def test_direct_grouping_matches_sort(cuda, M):
    # one segment a (token, slot) pair (no counting sort, the decode path for one token) computes what the sorted
    # grouping computes; at 3 tokens an expert may appear in two segments and is simply read twice
    import torch
    from locals_b200 import moe

    rng = np.random.default_rng(17 + M)
    E, K, D, I = 64, 4, 2048, 768
    x, wr = _router_inputs(rng, M, E, D)
    _, _, _, tg, tu, td = _experts(rng, E, D, I, cuda)
    xt = x_torch(x, "bfloat16", cuda)
    inds, wts = moe.route(xt, torch.from_numpy(wr).to(cuda, torch.float16), K)
    grouping = moe.group(inds, E)
    ys_sorted = moe.switch_glu_grouped(xt, inds, tg, tu, td, grouping=grouping)  # expert order
    y_sorted = moe.combine(ys_sorted, wts, grouping[4])
    ys_pairs = moe.switch_glu(xt, inds, tg, tu, td, grouping=grouping)  # pair order (M, k, D)
    y_pairs = moe.combine(ys_pairs.reshape(M * K, D), wts, None)
    ys_direct = moe.switch_glu(xt, inds, tg, tu, td, grouping=moe.direct_grouping(inds))
    y_direct = moe.combine(ys_direct.reshape(M * K, D), wts, None)
    assert torch.equal(y_pairs, y_sorted)  # the same rows, only reordered
    torch.cuda.synchronize()
    a, b = y_direct.float().cpu().numpy(), y_sorted.float().cpu().numpy()
    assert rel_err(a, b) <= 1e-3
