"""The one-token MoE layer in one launch (lq_moe_decode) on the GPU: its routing against lq_moe_route (bit-exact
experts and weights), its output against the CPU oracle's SwitchGLU + combine on the routed experts and against the
library's unfused one-token path (route + grouped gate/up + down_combine).

Oracle (locals/moe.py:577-591 for one token without the shared expert): per slot r with expert e,
h_r = swiglu(T(gate_e x), T(up_e x)), y_r = T(down_e h_r), y = T(sum_r w_r y_r) in float32 in slot order.
Tolerance: max|y - ref| <= 1e-2 max|ref| (fp32 accumulation; the fused kernel splits each down projection's K into
slices whose float32 partial sums are added in slice order)."""

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import TOL_REL, rel_err

pytestmark = pytest.mark.gpu


def _stack(torch, E, N, K, dtype, gen, dev):
    from locals_b200 import kernels

    w = torch.randn((E * N, K), generator=gen, device=dev, dtype=torch.float32) * 0.02
    wq, s, b = kernels.quantize(w, 64, 4, dtype=dtype)
    return wq.reshape(E, N, -1).contiguous(), s.reshape(E, N, -1).contiguous(), b.reshape(E, N, -1).contiguous()


def _host(m, e):
    return (m[0][e].cpu().numpy().view(np.uint32), m[1][e].float().cpu().numpy(), m[2][e].float().cpu().numpy(), 4)


def _layer(torch, E, D, I, dtype, seed, dev):
    gen = torch.Generator(device=dev)
    gen.manual_seed(seed)
    gate, up, down = _stack(torch, E, I, D, dtype, gen, dev), _stack(torch, E, I, D, dtype, gen, dev), \
        _stack(torch, E, D, I, dtype, gen, dev)
    wr = (torch.randn((E, D), generator=gen, device=dev) * 0.05).to(torch.float16)
    x = torch.randn((1, D), generator=gen, device=dev).to(dtype)
    return gate, up, down, wr, x


def _oracle(x, inds, wts, gate, up, down, E, dtype_name):
    used = set(int(e) for e in inds.reshape(-1))
    g = [(_host(gate, e) if e in used else None) for e in range(E)]
    u = [(_host(up, e) if e in used else None) for e in range(E)]
    d = [(_host(down, e) if e in used else None) for e in range(E)]
    return O.moe(x.float().cpu().numpy(), inds, wts, g, u, d, dtype_name)


CASES = [  # E, D, I, k, mode
    (64, 2048, 768, 4, 0),   # config 4
    (16, 512, 384, 4, 0),    # the reference's kernel-test experts (D 512, I 384, E 16, k 4)
    (20, 1024, 512, 3, 0),   # E not a multiple of the cluster: one CTA holds no router rows
    (64, 2048, 768, 8, 1),   # eight slots, sigmoid routing
    (256, 2048, 128, 2, 0),  # router rows too large to stage: read from global memory
]


@pytest.mark.parametrize("dtype", ["bfloat16", "float16"])
@pytest.mark.parametrize("E,D,I,k,mode", CASES)
def test_fused_decode_matches_route_oracle_and_unfused(cuda, dtype, E, D, I, k, mode):
    import torch
    from locals_b200 import kernels, moe

    tdt = torch.bfloat16 if dtype == "bfloat16" else torch.float16
    gate, up, down, wr, x = _layer(torch, E, D, I, tdt, E * 7 + D + k, cuda)
    inds = torch.empty((1, k), dtype=torch.int32, device=cuda)
    wts = torch.empty((1, k), dtype=torch.float32, device=cuda)
    y = moe.decode(x, wr, gate, up, down, k, mode, inds=inds, weights=wts)
    assert y is not None
    ri, rw = moe.route(x, wr, k, mode)
    unfused = moe.MoELayer(wr, gate, up, down, top_k=k, mode=mode, fused_decode=False)(x)
    torch.cuda.synchronize()
    assert kernels.device_status() == 0
    assert torch.equal(inds, ri)
    assert torch.equal(wts, rw)
    ref = _oracle(x, inds.cpu().numpy(), wts.cpu().numpy(), gate, up, down, E, dtype)
    assert rel_err(y.float().cpu().numpy(), ref) <= TOL_REL
    assert rel_err(y.float().cpu().numpy(), unfused.float().cpu().numpy()) <= TOL_REL


def test_fused_decode_repeats_and_leaves_workspace_zero(cuda):
    """Back-to-back launches on one workspace (the last CTA of each row block resets its counter): the same input
    gives the same bits every time, a different input its own answer, and the counters end at zero."""
    import torch
    from locals_b200 import moe

    E, D, I, k = 64, 2048, 768, 4
    gate, up, down, wr, x = _layer(torch, E, D, I, torch.bfloat16, 11, cuda)
    x2 = torch.randn_like(x, dtype=torch.float32).to(torch.bfloat16)
    work = moe.decode_workspace(E, k, D, I, cuda)
    ys = [moe.decode(v, wr, gate, up, down, k, workspace=work) for v in (x, x2, x, x2, x)]
    torch.cuda.synchronize()
    assert torch.equal(ys[0], ys[2]) and torch.equal(ys[0], ys[4])
    assert torch.equal(ys[1], ys[3])
    assert not torch.equal(ys[0], ys[1])
    assert int(work[:64].count_nonzero()) == 0
    layer = moe.MoELayer(wr, gate, up, down, top_k=k)
    assert torch.equal(layer(x), ys[0])


def test_fused_decode_in_a_cuda_graph(cuda):
    """Captured in a CUDA graph with PDL edges between layers (three layers in a row), replayed twice: the same bits
    as eager launches."""
    import torch
    from locals_b200 import moe

    E, D, I, k = 64, 2048, 768, 4
    layers = []
    for seed in (21, 22, 23):
        gate, up, down, wr, x = _layer(torch, E, D, I, torch.bfloat16, seed, cuda)
        layers.append(moe.MoELayer(wr, gate, up, down, top_k=k))

    def body(v):
        for la in layers:
            v = la(v)
        return v

    eager = body(x)
    st = torch.cuda.Stream(device=cuda)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(st):
        body(x)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=st):
            out = body(x)
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_fused_decode_declines_outside_its_shapes(cuda):
    """D % 128 != 0 or 8-bit experts: None (the layer then runs the unfused kernels)."""
    import torch
    from locals_b200 import moe

    gate, up, down, wr, x = _layer(torch, 8, 192, 128, torch.bfloat16, 3, cuda)
    assert moe.decode(x, wr, gate, up, down, 2) is None
    assert moe.decode(x, wr, gate, up, down, 2, bits=8) is None


def test_fused_decode_on_a_second_device(cuda):
    """The kernel's shared-memory limit belongs to the device it was set on: a process that decodes on GPU 0 and then on
    GPU 1 gets the same answers on both (skipped with one GPU)."""
    import torch
    from locals_b200 import moe

    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    E, D, I, k = 64, 2048, 768, 4
    ys = []
    for d in (0, 1):
        dev = torch.device("cuda", d)
        with torch.cuda.device(dev):
            gate, up, down, wr, x = _layer(torch, E, D, I, torch.bfloat16, 31, dev)
            y = moe.decode(x, wr, gate, up, down, k)
            torch.cuda.synchronize()
            assert y is not None
            ys.append(y.cpu())
    assert torch.equal(ys[0], ys[1])
