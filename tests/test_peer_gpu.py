"""The peer exchanges' flag meeting on one GPU, without a second rank: the second rank's buffer and sync block are
stand-ins in this GPU's memory. With the stand-in's flag already at the round, the call completes and both buffers hold
the block; with a flag that nothing sets, the bounded wait runs out after a second and leaves LQ_DEV_TIMEOUT in the
device status (no fault, no hang: the context stays usable). Only one kernel waits, so nothing on this GPU waits for
another kernel."""

import ctypes

import pytest

pytestmark = pytest.mark.gpu

ROUND = 16  # uint32 offset of the round counter in a sync block (flags at 0 .. 7)


def _call(torch, src, dst, sync, M, n, G, rank, N):
    from locals_b200 import _lib

    d = (ctypes.c_void_p * G)(*[t.data_ptr() for t in dst])
    s = (ctypes.c_void_p * G)(*[t.data_ptr() for t in sync])
    _lib.call("lq_peer_gather_cols", src.data_ptr(), M, n, rank * n, N, 2, d, G, rank, s,
              torch.cuda.current_stream().cuda_stream)


def test_flag_already_set_completes(cuda):
    import torch
    from locals_b200 import _lib, kernels

    nb = int(_lib.lib().lq_peer_sync_bytes())
    M, n = 4, 512
    src = torch.randn((M, n), device=cuda).to(torch.bfloat16)
    dst = [torch.zeros((M, 2 * n), dtype=torch.bfloat16, device=cuda) for _ in range(2)]
    sync = [torch.zeros(nb // 4, dtype=torch.int32, device=cuda) for _ in range(2)]
    for rnd in (1, 2):  # two calls in a row: the round advances, the CTA counter is back at zero
        sync[0][1] = rnd  # the stand-in peer (rank 1) has already reached this round
        _call(torch, src, dst, sync, M, n, 2, 0, 2 * n)
        torch.cuda.synchronize()
        assert kernels.device_status() == 0
        assert int(sync[0][ROUND]) == rnd          # this rank's round
        assert int(sync[1][0]) == rnd              # released into the peer's slot for rank 0
        for d in dst:
            assert torch.equal(d[:, :n], src)      # the block in both ranks' buffers


def test_missing_peer_times_out_with_status(cuda):
    import torch
    from locals_b200 import _lib, kernels

    nb = int(_lib.lib().lq_peer_sync_bytes())
    M, n = 2, 256
    src = torch.randn((M, n), device=cuda).to(torch.bfloat16)
    dst = [torch.zeros((M, 2 * n), dtype=torch.bfloat16, device=cuda) for _ in range(2)]
    sync = [torch.zeros(nb // 4, dtype=torch.int32, device=cuda) for _ in range(2)]
    kernels.device_status()  # (clear)
    _call(torch, src, dst, sync, M, n, 2, 1, 2 * n)  # as rank 1: waits for rank 0's flag, which nothing sets
    torch.cuda.synchronize()
    assert kernels.device_status() & 0x1  # LQ_DEV_TIMEOUT
    assert torch.equal(dst[0][:, n:], src)  # the stores were made before the wait
    x = torch.ones(8, device=cuda)  # the context is still usable
    assert float((x * 2).sum()) == 16.0
