"""The sharded modules on 2 and 4 GPUs (skipped when fewer GPUs are visible), exchanging over peer memory and with
NCCL: each sharded result is compared with the same computation on one GPU (the peer exchanges exactly, the
expert-parallel layer bit for bit)."""

import os
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, path):
    import torch.distributed as dist
    from datetime import timedelta

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60), device_id=dev)
    try:
        from locals_b200 import kernels, moe
        from locals_b200.kernels import QuantizedLinear
        from locals_b200.shard import ColumnShardedLinear, ExpertParallelMoE, ShardedMLP

        gen = torch.Generator(device=dev)
        gen.manual_seed(0)

        def layer(N, K, bits):
            return kernels.quantize(torch.randn((N, K), generator=gen, device=dev) * 0.02, 64, bits,
                                    dtype=torch.bfloat16)

        errs = {}
        lin = QuantizedLinear(*layer(1024, 2048, 4))
        x = torch.randn((8, 2048), generator=gen, device=dev).to(torch.bfloat16)
        ref = kernels.quantized_matmul(x, lin.weight, lin.scales, lin.biases)
        errs["linear"] = float((ColumnShardedLinear(lin)(x).float() - ref.float()).abs().max() / ref.float().abs().max())
        # prefill size: the dense GEMM with the all-gather in its own stores (peer buffers by CUDA IPC), twice in a
        # row (the two peer buffers), against the same dense path on one GPU; and the NCCL all-gather form
        big = QuantizedLinear(*layer(1024, 2048, 4))
        xp = torch.randn((256, 2048), generator=gen, device=dev).to(torch.bfloat16)
        refp = kernels.quantized_matmul(xp, big.weight, big.scales, big.biases, choice=("dense",)).float()
        fused = ColumnShardedLinear(big)
        y1 = fused(xp).float().clone()
        y2 = fused(xp * 2).float().clone()
        errs["gather_fused"] = float((y1 - refp).abs().max() / refp.abs().max())
        refp2 = kernels.quantized_matmul(xp * 2, big.weight, big.scales, big.biases, choice=("dense",)).float()
        errs["gather_fused_2"] = float((y2 - refp2).abs().max() / refp2.abs().max())
        errs["gather_nccl"] = float((ColumnShardedLinear(big, fused_gather=False)(xp).float() - refp).abs().max()
                                    / refp.abs().max())
        for pb in fused._peer.values():
            pb.close()
        # decode-size column gather over peer memory (lq_peer_gather_cols): exact, five calls in a row (both buffers of
        # each shape, the round flags advancing), two shapes interleaved as a sharded MLP uses them
        from locals_b200.shard import PeerGather

        pg = PeerGather()
        assert pg.ok
        bad = 0
        for it in range(5):
            for M_, n_ in ((1, 512), (16, 1024)):
                mine = torch.full((M_, n_), float(rank * 100 + it), device=dev).to(torch.bfloat16)
                mine[:, 0] = float(it)
                got = pg(mine)
                want = torch.cat([torch.full((M_, n_), float(p_ * 100 + it), device=dev) for p_ in range(world)], 1)
                want[:, ::n_] = float(it)
                want = want.to(torch.bfloat16).float()  # (the block as each rank holds it)
                bad += int((got.float() != want).sum())
        errs["peer_gather_mismatches"] = float(bad)
        pg.close()
        g, u, d = (QuantizedLinear(*layer(1024, 2048, 8), bits=8), QuantizedLinear(*layer(1024, 2048, 8), bits=8),
                   QuantizedLinear(*layer(2048, 1024, 8), bits=8))
        h = kernels.qmm_glu(x, (g.weight, g.scales, g.biases), (u.weight, u.scales, u.biases), bits=8)
        ref = kernels.quantized_matmul(h, d.weight, d.scales, d.biases, bits=8)
        errs["mlp"] = float((ShardedMLP(g, u, d)(x).float() - ref.float()).abs().max() / ref.float().abs().max())
        E, D, I = 16, 1024, 512

        def stack(N, Kd):
            parts = [layer(N, Kd, 4) for _ in range(E)]
            return tuple(torch.stack([p[i] for p in parts]).contiguous() for i in range(3))

        gate, up, down = stack(I, D), stack(I, D), stack(D, I)
        wr = (torch.randn((E, D), generator=gen, device=dev) * 0.05).to(torch.float16)
        xt = torch.randn((world * 8, D), generator=gen, device=dev).to(torch.bfloat16)
        full = moe.MoELayer(wr, gate, up, down, top_k=4)(xt)
        mine = xt[rank * 8:(rank + 1) * 8].contiguous()
        ep = ExpertParallelMoE(wr, gate, up, down, top_k=4)
        assert ep._pg is not None and ep._pg.ok  # the peer-memory exchanges (every rank on its own GPU)
        ref = full[rank * 8:(rank + 1) * 8]
        for _ in range(3):  # (the peer buffers in turn)
            got = ep(mine)
            # up to 16 tokens the folded grouped kernel runs each expert segment the same way whatever the other
            # segments: the same bits as the one-GPU layer (above, the mma.sync grouped kernel may split K differently
            # when a rank holds fewer experts: the tolerance below)
            if world * 8 <= 16:
                errs["moe_not_exact"] = max(errs.get("moe_not_exact", 0.0), float(not torch.equal(got, ref)))
            else:
                errs["moe_not_exact"] = 0.0
        errs["moe"] = float((got.float() - ref.float()).abs().max() / ref.float().abs().max())
        xt2 = torch.randn((world * 40, D), generator=gen, device=dev).to(torch.bfloat16)  # the gather path
        full2 = moe.MoELayer(wr, gate, up, down, top_k=4)(xt2)
        got2 = ep(xt2[rank * 40:(rank + 1) * 40].contiguous())
        errs["moe80"] = float((got2.float() - full2[rank * 40:(rank + 1) * 40].float()).abs().max()
                              / full2.float().abs().max())
        ep._pg.close()
        torch.cuda.synchronize()
        errs["status"] = kernels.device_status()
        out = [None] * world
        dist.all_gather_object(out, errs)
        if rank == 0:
            torch.save(out, path)
    finally:
        dist.destroy_process_group()


def _run(tmp_path, world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    import torch.multiprocessing as mp

    path = str(tmp_path / "errs.pt")
    mp.spawn(_worker, args=(world, _port(), path), nprocs=world, join=True)
    for errs in torch.load(path):
        assert errs.pop("status") == 0
        assert errs.pop("peer_gather_mismatches") == 0
        assert errs.pop("moe_not_exact") == 0
        for name, e in errs.items():
            assert e <= 1e-2, (name, e)


def test_sharded_two_gpus(tmp_path):
    _run(tmp_path, 2)


def test_sharded_four_gpus(tmp_path):
    """The same on four ranks (the peer exchanges with three peers each, four experts a rank)."""
    _run(tmp_path, 4)
