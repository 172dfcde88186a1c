"""8-bit KV decode attention on the GPU (lq_kv_attend) against the CPU oracle, over the reference test's cases
(tests/test_flint.py:277-299: 32 query heads on 4 key/value heads and 4 on 2, one to 2,100 keys, buffers larger
than their valid part, left padding) and the edges of the kernel: 1 and 16 query heads a key/value head, keys
split over many blocks and joined, rows with nothing to attend, no sinks, a dominant sink, fp16.

Bound: the reference test's max|got - ref| <= 2^-7 (1 + max|ref|) and the path's max|got - ref| <= 1e-2 max|ref|.
"""

import ctypes

import numpy as np
import pytest

from oracle import oracle as O
from tests.helpers import TOL_REL

pytestmark = pytest.mark.gpu

SCALE = 0.0884


def _make(cuda, B, H, KVH, cap, dtype, seed):
    import torch
    from locals_b200 import qkv

    g = torch.Generator(device=cuda)
    g.manual_seed(seed)
    q = torch.randn((B, H, 1, 128), generator=g, device=cuda).to(dtype)
    k = (torch.randn((B, KVH, cap, 128), generator=g, device=cuda) * 2).to(dtype)
    v = torch.randn((B, KVH, cap, 128), generator=g, device=cuda).to(dtype)
    sinks = (torch.randn((H,), generator=g, device=cuda) * 2).to(dtype)
    return q, qkv.quantize(k), qkv.quantize(v), sinks


def _np_triple(t):
    return (t[0].cpu().numpy().view(np.uint32), t[1].float().cpu().numpy(), t[2].float().cpu().numpy())


def _oracle(q, keys, values, n, sinks, start):
    return O.kv_attend(q.float().cpu().numpy()[:, :, 0], _np_triple(keys), _np_triple(values), n,
                       None if sinks is None else sinks.float().cpu().numpy(), SCALE,
                       None if start is None else start.cpu().numpy())


def _check(got, ref):
    got = got.float().cpu().numpy()[:, :, 0]
    assert np.all(np.isfinite(got))
    err, m = float(np.abs(got - ref).max()), float(np.abs(ref).max())
    assert err <= 2 ** -7 * (1 + m), (err, m)
    assert err <= TOL_REL * m or err == 0.0, (err, m)


@pytest.mark.parametrize("H,KVH", [(32, 4), (4, 2)])
@pytest.mark.parametrize("B,n,cap,pads", [(1, 1, 256, [0]), (1, 13, 256, [0]), (1, 2100, 2304, [0]),
                                          (3, 700, 768, [0, 37, 300])])
def test_reference_cases(cuda, H, KVH, B, n, cap, pads):
    import torch
    from locals_b200 import qkv

    q, keys, values, sinks = _make(cuda, B, H, KVH, cap, torch.bfloat16, n)
    start = torch.tensor(pads, dtype=torch.int32, device=cuda)
    got = qkv.attend(q, keys, values, n, sinks, SCALE, start)
    _check(got, _oracle(q, keys, values, n, sinks, start))


@pytest.mark.parametrize("B,H,KVH,n,cap,pads,dtype", [
    (2, 32, 2, 900, 1024, [0, 11], "bfloat16"),    # 16 query heads a kv head: both row halves of the MMA
    (2, 8, 8, 333, 400, [5, 0], "bfloat16"),       # one query head a kv head
    (1, 12, 4, 517, 521, [0], "float16"),          # 3 a kv head, capacity not a multiple of 16, fp16
    (2, 32, 4, 20000, 20013, [0, 5001], "bfloat16"),  # many blocks a row, joined
    (4, 64, 8, 4096, 4096, [0, 1, 2, 4095], "float16"),
])
def test_shapes(cuda, B, H, KVH, n, cap, pads, dtype):
    import torch
    from locals_b200 import qkv

    tdt = torch.bfloat16 if dtype == "bfloat16" else torch.float16
    q, keys, values, sinks = _make(cuda, B, H, KVH, cap, tdt, n + H)
    start = torch.tensor(pads, dtype=torch.int32, device=cuda)
    got = qkv.attend(q, keys, values, n, sinks, SCALE, start)
    _check(got, _oracle(q, keys, values, n, sinks, start))


def test_edges(cuda):
    import torch
    from locals_b200 import qkv

    q, keys, values, sinks = _make(cuda, 2, 32, 4, 1024, torch.bfloat16, 7)
    # no sinks, no start
    _check(qkv.attend(q, keys, values, 800, None, SCALE), _oracle(q, keys, values, 800, None, None))
    # a row whose start is past n attends to its sink alone (0), the other row as usual
    start = torch.tensor([0, 900], dtype=torch.int32, device=cuda)
    got = qkv.attend(q, keys, values, 800, sinks, SCALE, start)
    assert torch.count_nonzero(got[1]).item() == 0
    _check(got, _oracle(q, keys, values, 800, sinks, start))
    # n = 0: nothing attended anywhere
    got = qkv.attend(q, keys, values, 0, sinks, SCALE)
    assert torch.count_nonzero(got).item() == 0
    # a dominant sink
    big = torch.full_like(sinks, 60.0)
    _check(qkv.attend(q, keys, values, 800, big, SCALE), _oracle(q, keys, values, 800, big, None))
    # negative start reads from 0
    start = torch.tensor([-5, 3], dtype=torch.int32, device=cuda)
    _check(qkv.attend(q, keys, values, 1000, sinks, SCALE, start), _oracle(q, keys, values, 1000, sinks, start))


def test_workspace_checked(cuda):
    import torch
    from locals_b200 import _lib

    q, keys, values, sinks = _make(cuda, 1, 32, 4, 8192, torch.bfloat16, 3)
    L = _lib.lib()
    need = L.lq_kv_attend_workspace(1, 32, 4, 8192)
    assert need > 0
    out = torch.empty((1, 32, 1, 128), dtype=torch.bfloat16, device=cuda)
    ptrs = [t.data_ptr() for t in (q, keys[0], keys[1], keys[2], values[0], values[1], values[2])]
    ws = torch.empty(need, dtype=torch.uint8, device=cuda)
    args = ptrs + [None, 8192, None, ctypes.c_float(SCALE), 1, 32, 4, 8192, 128, _lib.BF16]
    assert L.lq_kv_attend(*args, ws.data_ptr(), need - 16, out.data_ptr(), None) == _lib.LQ_E_ARG
    assert L.lq_kv_attend(*args, ws.data_ptr(), need, out.data_ptr(), None) == _lib.LQ_OK
    torch.cuda.synchronize()
    _check(out, _oracle(q, keys, values, 8192, None, None))


def test_cache_prompt_then_decode(cuda):
    import torch
    from locals_b200 import qkv

    g = torch.Generator(device=cuda)
    g.manual_seed(11)
    B, KVH, H = 2, 4, 32
    cache = qkv.QuantizedKVCache8(left_padding=[0, 17])
    k = (torch.randn((B, KVH, 300, 128), generator=g, device=cuda) * 2).to(torch.bfloat16)
    v = torch.randn((B, KVH, 300, 128), generator=g, device=cuda).to(torch.bfloat16)
    cache.update_and_fetch(k, v)
    assert cache.keys[0].shape[2] == 512 and cache._idx == 300  # grown by a multiple of 256
    sinks = (torch.randn((H,), generator=g, device=cuda) * 2).to(torch.bfloat16)
    for step in range(3):
        k1 = (torch.randn((B, KVH, 1, 128), generator=g, device=cuda) * 2).to(torch.bfloat16)
        v1 = torch.randn((B, KVH, 1, 128), generator=g, device=cuda).to(torch.bfloat16)
        keys, values = cache.update_and_fetch(k1, v1)
        assert keys[0].shape[2] == 301 + step
        q = torch.randn((B, H, 1, 128), generator=g, device=cuda).to(torch.bfloat16)
        got = cache.attend(q, SCALE, sinks)
        _check(got, _oracle(q, cache.keys, cache.values, cache._idx, sinks, cache.left_padding))
    # the stored codes are MLX's quantization of what went in
    ref = qkv.quantize(k1)
    assert torch.equal(cache.keys[0][:, :, 302:303], ref[0]) and torch.equal(cache.keys[1][:, :, 302:303], ref[1])
