"""lq_kv_attend_noalloc on the GPU: the 8-bit KV decode attention for callers that cannot allocate device memory
at the point they attend (a plugin handed only raw device pointers, code running inside someone else's CUDA graph,
a runtime with a memory pool fixed at start-up). It keeps its per-block softmax parts in a fixed 4 MiB buffer inside
the library instead of a caller workspace.

Checked through the C ABI against lq_kv_attend (with a workspace from torch) on two calls in a row, the second with a
different shape, start offsets and query, so parts left in the shared buffer by the first call cannot leak into the
second; and a shape whose parts need more than the buffer is refused with LQ_E_SCRATCH before anything runs.
Bound: the path's max|got - ref| <= 1e-2 max|ref|. This file sorts last so a failure here stops a -x run only after
every other test has run; it also passes alone in a fresh process.
"""

import ctypes

import pytest

from tests.helpers import TOL_REL

pytestmark = pytest.mark.gpu

SCALE = 0.0884
STATIC_BYTES = 4 << 20


def _cache(cuda, B, H, KVH, cap, seed):
    import torch
    from locals_b200 import qkv

    g = torch.Generator(device=cuda)
    g.manual_seed(seed)
    q = torch.randn((B, H, 1, 128), generator=g, device=cuda).to(torch.bfloat16)
    keys = qkv.quantize((torch.randn((B, KVH, cap, 128), generator=g, device=cuda) * 2).to(torch.bfloat16))
    values = qkv.quantize(torch.randn((B, KVH, cap, 128), generator=g, device=cuda).to(torch.bfloat16))
    sinks = (torch.randn((H,), generator=g, device=cuda) * 2).float()
    return q, keys, values, sinks


def _args(q, keys, values, start, n, sinks, B, H, KVH, cap):
    ptrs = [t.data_ptr() for t in (q, keys[0], keys[1], keys[2], values[0], values[1], values[2])]
    from locals_b200 import _lib

    return ptrs + [start.data_ptr(), n, sinks.data_ptr(), ctypes.c_float(SCALE), B, H, KVH, cap, 128, _lib.BF16]


@pytest.mark.parametrize("first,second", [
    ((2, 32, 4, 5000, 5120, [0, 333]), (3, 16, 2, 2100, 2304, [7, 0, 1500])),
])
def test_noalloc_matches_workspace_entry_point(cuda, first, second):
    import torch
    from locals_b200 import _lib

    L = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    for i, (B, H, KVH, n, cap, pads) in enumerate((first, second)):
        q, keys, values, sinks = _cache(cuda, B, H, KVH, cap, 100 + i)
        start = torch.tensor(pads, dtype=torch.int32, device=cuda)
        args = _args(q, keys, values, start, n, sinks, B, H, KVH, cap)
        need = L.lq_kv_attend_workspace(B, H, KVH, n)
        assert 0 < need <= STATIC_BYTES  # the keys are split over blocks: the parts live in scratch
        ws = torch.empty(need, dtype=torch.uint8, device=cuda)
        ref = torch.empty((B, H, 1, 128), dtype=torch.bfloat16, device=cuda)
        got = torch.full((B, H, 1, 128), float("nan"), dtype=torch.bfloat16, device=cuda)
        assert L.lq_kv_attend(*args, ws.data_ptr(), need, ref.data_ptr(), stream) == _lib.LQ_OK
        assert L.lq_kv_attend_noalloc(*args, got.data_ptr(), stream) == _lib.LQ_OK
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        ref32, got32 = ref.float(), got.float()
        assert torch.isfinite(got32).all()
        err, m = (got32 - ref32).abs().max().item(), ref32.abs().max().item()
        assert err <= TOL_REL * m, (i, err, m)


def test_noalloc_on_a_second_device():
    """With two or more GPUs visible, the same check on device 1 after device 0 in one process: the buffer's address
    and the kernel's shared-memory attribute are per device, so device 1 must get its own (plain per-device calls, no
    peer memory)."""
    import torch
    from locals_b200 import _lib

    if torch.cuda.device_count() < 2:
        pytest.skip("one GPU visible")
    L = _lib.lib()
    B, H, KVH, n, cap, pads = 2, 32, 4, 5000, 5120, [0, 333]
    prev = torch.cuda.current_device()
    try:
        for d in (0, 1):
            dev = torch.device("cuda", d)
            torch.cuda.set_device(dev)
            q, keys, values, sinks = _cache(dev, B, H, KVH, cap, 200 + d)
            start = torch.tensor(pads, dtype=torch.int32, device=dev)
            args = _args(q, keys, values, start, n, sinks, B, H, KVH, cap)
            need = L.lq_kv_attend_workspace(B, H, KVH, n)
            ws = torch.empty(need, dtype=torch.uint8, device=dev)
            ref = torch.empty((B, H, 1, 128), dtype=torch.bfloat16, device=dev)
            got = torch.full((B, H, 1, 128), float("nan"), dtype=torch.bfloat16, device=dev)
            stream = torch.cuda.current_stream(dev).cuda_stream
            assert L.lq_kv_attend(*args, ws.data_ptr(), need, ref.data_ptr(), stream) == _lib.LQ_OK
            assert L.lq_kv_attend_noalloc(*args, got.data_ptr(), stream) == _lib.LQ_OK
            torch.cuda.synchronize(dev)
            assert _lib.device_status() == 0
            ref32, got32 = ref.float(), got.float()
            assert torch.isfinite(got32).all()
            err, m = (got32 - ref32).abs().max().item(), ref32.abs().max().item()
            assert err <= TOL_REL * m, (d, err, m)
    finally:
        torch.cuda.set_device(prev)


def test_noalloc_refuses_shapes_beyond_its_buffer(cuda):
    import torch
    from locals_b200 import _lib

    L = _lib.lib()
    B, H, KVH, n, cap = 443, 16, 1, 512, 512  # 443 (row, kv head) pairs split in two, 16 heads each: > 4 MiB of parts
    need = L.lq_kv_attend_workspace(B, H, KVH, n)
    assert need > STATIC_BYTES
    q, keys, values, sinks = _cache(cuda, B, H, KVH, cap, 7)
    start = torch.zeros((B,), dtype=torch.int32, device=cuda)
    out = torch.zeros((B, H, 1, 128), dtype=torch.bfloat16, device=cuda)
    args = _args(q, keys, values, start, n, sinks, B, H, KVH, cap)
    assert L.lq_kv_attend_noalloc(*args, out.data_ptr(), None) == _lib.LQ_E_SCRATCH
    assert L.lq_strerror(_lib.LQ_E_SCRATCH) == b"shape needs more than the 4 MiB static scratch buffer"
    torch.cuda.synchronize()
    assert torch.count_nonzero(out).item() == 0  # refused before any launch
