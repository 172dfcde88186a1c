"""The multi-GPU partitioning logic (locals_b200.shard) on two gloo ranks on the CPU.

The kernels need a GPU, so each rank's compute goes through oracle-backed hooks (shard.Ops); what is
tested is the product's own sharding: the row splits of MLX-format weights, the head-aligned q/k/v split,
the all-gather layout, the expert-parallel packing into fixed-capacity all-to-all blocks, the return path
and the slot-ordered combine. Each sharded result must equal the unsharded oracle computation exactly
(the same float32 arithmetic runs on the same rows, only on different ranks).
"""

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

DT = "bfloat16"


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _oracle_ops():
    from locals_b200.shard import Ops
    from oracle import oracle as O

    def npq(q):
        return (q[0].numpy().view(np.uint32), q[1].float().numpy(), q[2].float().numpy())

    def qmm(x, q, bits):
        return torch.from_numpy(O.round_to(O.qmm(x.float().numpy(), *npq(q), 64, bits), DT))

    def glu(x, gate, up, bits):
        g = O.round_to(O.qmm(x.float().numpy(), *npq(gate), 64, bits), DT)
        u = O.round_to(O.qmm(x.float().numpy(), *npq(up), 64, bits), DT)
        return torch.from_numpy(O.swiglu(g, u, DT))

    def route(x, wr, k, mode):
        i, w = O.topk(O.router(x.float().numpy(), wr.float().numpy()), k, "softmax" if mode == 0 else "sigmoid")
        return torch.from_numpy(i.astype(np.int32)), torch.from_numpy(w)

    def experts(rows, ids, gate, up, down, bits, max_rows):
        out = torch.zeros((rows.shape[0], down[0].shape[1]), dtype=torch.float32)
        for p in range(rows.shape[0]):
            e = int(ids[p])
            if e < 0:
                continue
            x = rows[p:p + 1].float().numpy()
            one = lambda m: (m[0][e].numpy().view(np.uint32), m[1][e].float().numpy(), m[2][e].float().numpy())
            g = O.round_to(O.qmm(x, *one(gate), 64, bits), DT)
            u = O.round_to(O.qmm(x, *one(up), 64, bits), DT)
            h = O.swiglu(g, u, DT)
            out[p] = torch.from_numpy(O.round_to(O.qmm(h, *one(down), 64, bits), DT)[0])
        return out

    def combine(ys, wts):
        return torch.from_numpy(O.round_to(O.combine(ys.float().numpy(), wts.numpy()), DT))

    return Ops(qmm, glu, route, experts, combine)


def _weights(seed):
    from oracle import oracle as O

    rng = np.random.default_rng(seed)

    def q(N, K, bits):
        wq, s, b = O.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float32), 64, bits, DT)
        return torch.from_numpy(wq.view(np.int32).copy()), torch.from_numpy(s), torch.from_numpy(b)

    return rng, q


def _worker(rank, world, port, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from locals_b200.kernels import QuantizedLinear
        from locals_b200.shard import ColumnShardedLinear, ExpertParallelMoE, ShardedMLP, ShardedQKV
        from oracle import oracle as O

        ops = _oracle_ops()
        rng, q = _weights(0)
        errs = {}
        # column-sharded linear
        lin = QuantizedLinear(*q(256, 512, 4))
        x = torch.from_numpy(O.round_to(rng.standard_normal((3, 512)).astype(np.float32), DT))
        y = ColumnShardedLinear(lin, ops=ops)(x)
        ref = ops.qmm(x, (lin.weight, lin.scales, lin.biases), 4)
        errs["linear"] = float((y - ref).abs().max())
        # q/k/v split at heads (4 query heads, 2 kv heads of 64)
        qm, km, vm = QuantizedLinear(*q(256, 256, 4)), QuantizedLinear(*q(128, 256, 4)), QuantizedLinear(*q(128, 256, 4))
        x2 = torch.from_numpy(O.round_to(rng.standard_normal((2, 256)).astype(np.float32), DT))
        qq, kk, vv = ShardedQKV(qm, km, vm, 4, 2, 64, ops=ops)(x2)
        errs["qkv"] = max(float((qq.reshape(2, -1) - ops.qmm(x2, (qm.weight, qm.scales, qm.biases), 4)).abs().max()),
                          float((vv.reshape(2, -1) - ops.qmm(x2, (vm.weight, vm.scales, vm.biases), 4)).abs().max()))
        # 8-bit MLP
        g, u, d = QuantizedLinear(*q(256, 256, 8), bits=8), QuantizedLinear(*q(256, 256, 8), bits=8), \
            QuantizedLinear(*q(256, 256, 8), bits=8)
        ym = ShardedMLP(g, u, d, ops=ops)(x2)
        h = ops.glu(x2, (g.weight, g.scales, g.biases), (u.weight, u.scales, u.biases), 8)
        errs["mlp"] = float((ym - ops.qmm(h, (d.weight, d.scales, d.biases), 8)).abs().max())
        # expert-parallel MoE: 8 experts, top-2, D 128, I 64; 3 tokens per rank
        E, K_, D, I = 8, 2, 128, 64

        def stack(N, Kd):
            parts = [q(N, Kd, 4) for _ in range(E)]
            return tuple(torch.stack([p[i] for p in parts]) for i in range(3))

        gate, up, down = stack(I, D), stack(I, D), stack(D, I)
        wr = torch.from_numpy(O.round_to((rng.standard_normal((E, D)) * 0.1).astype(np.float32), "float16"))
        xt = torch.from_numpy(O.round_to(rng.standard_normal((2 * 3, D)).astype(np.float32), DT))
        mine = xt[rank * 3:(rank + 1) * 3].contiguous()
        yt = ExpertParallelMoE(wr, gate, up, down, K_, ops=ops)(mine)
        inds, wts = ops.route(mine, wr, K_, 0)
        rows = mine.repeat_interleave(K_, 0)
        ids = inds.reshape(-1)
        ys = ops.experts(rows, ids, gate, up, down, 4, 0)
        errs["moe"] = float((yt - ops.combine(ys, wts)).abs().max())
        gathered = [None] * world
        dist.all_gather_object(gathered, errs)
        if rank == 0:
            torch.save(gathered, result_path)
    finally:
        dist.destroy_process_group()


def test_sharding_two_gloo_ranks(tmp_path):
    path = str(tmp_path / "errs.pt")
    mp.spawn(_worker, args=(2, _free_port(), path), nprocs=2, join=True)
    errs = torch.load(path)
    for rank_errs in errs:
        for name, e in rank_errs.items():
            assert e == 0.0, (name, e)
