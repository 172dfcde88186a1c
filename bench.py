"""Benchmark of the MLX affine quantized-matmul path on B200. Metric:
"4-bit qmm HBM GB/s at M=1-16 & TFLOP/s at M=2048; MoE tok/s vs MLX CPU".

Headline workload (the configuration the metric is quoted on): the fused QKV decode
projection, x bf16 [16, 2560] times a 4-bit g64 [6144, 2560] matrix, output split into q/k/v. One
step = that projection over a stack of L = 36 distinct layers (36 x 8.85 MB = 318 MB of weights: the
weights never sit in the 126 MB L2 between uses), captured in one CUDA graph. value = algorithmic bytes
(packed weights + scales + biases + x + outputs) / device time, GB/s.

e2e: the same step through the public API with host buffers: pinned x copied in, the captured layers,
the last layer's q/k/v copied out, all inside the timed region.

Extra keys report the other workloads (cfg1: fp16 4096x4096 qmm at M=8; cfg3: 8-bit MLP 2560->9728->2560;
cfg4: 64-expert top-4 MoE; cfg5: 2048x4096 . 14336x4096 prefill GEMM) measured the same way (CUDA events, warm-up, inputs larger
than L2 or rotated weight copies), and the CPU baseline (the C/OpenMP restatement of the reference's
arithmetic, all host cores, a bounded sample).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference] [--quick]
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "4-bit qmm HBM GB/s at M=1-16 & TFLOP/s at M=2048; MoE tok/s vs MLX CPU"
HEAD_M, HEAD_K, HEAD_N = 16, 2560, 6144
HEAD_WIDTHS = (4096, 1024, 1024)
L2_BYTES = 126 * 2 ** 20  # B200 L2
LAYERS = 36


def peaks():
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            p = json.load(f)
        return float(p["hbm_gbs"]), float(p["bf16_tflops"]), "measured"
    except (OSError, ValueError, KeyError):
        return 6650.0, 1590.0, "fallback"


def qmm_bytes(M, N, K, bits, out_cols=None):
    """Algorithmic bytes of one quantized matmul: packed weights + 16-bit scales and biases + x + y."""
    return N * K * bits // 8 + 2 * N * (K // 64) * 2 + M * K * 2 + M * (out_cols or N) * 2


def profile_traffic(name):
    """dram bytes per launch from a committed ncu summary (profiles/<name>.txt, line 'dram_bytes_per_launch: N')."""
    try:
        with open(os.path.join(ROOT, "profiles", name + ".txt")) as f:
            for line in f:
                if line.startswith("dram_bytes_per_launch:"):
                    return float(line.split(":")[1])
    except OSError:
        pass
    return None


class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_env():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return ws, rank, local


# --------------------------------------------------------------------------------------------------
# CPU reference arm and CPU baseline (the oracle port: the only place bench.py runs oracle/ code)
# --------------------------------------------------------------------------------------------------

def cpu_qkv_sample(seconds=10.0, rows=768):
    """The oracle's qmm on a sample of the headline workload (M=16 x K=2560, `rows` of the 6144 output
    rows) repeated for about `seconds`; returns (GB/s of algorithmic bytes, threads, sample text)."""
    import numpy as np

    from oracle import oracle as O

    rng = np.random.default_rng(1)
    w = (rng.standard_normal((rows, HEAD_K)) * 0.02).astype(np.float32)
    wq, s, b = O.quantize(w, 64, 4, "bfloat16")
    x = O.round_to(rng.standard_normal((HEAD_M, HEAD_K)).astype(np.float32), "bfloat16")
    threads = os.cpu_count() or 1
    O.qmm(x, wq, s, b, threads=threads)
    n, t0 = 0, time.perf_counter()
    while True:
        O.qmm(x, wq, s, b, threads=threads)
        n += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    by = qmm_bytes(HEAD_M, rows, HEAD_K, 4)
    return by * n / el / 1e9, threads, f"oracle qmm M=16 K=2560 on {rows} of 6144 rows x{n} calls ({el:.1f} s)"


def run_reference(args):
    ws, rank, _ = dist_env()
    if rank != 0:
        return 0
    gbs, threads, sample = cpu_qkv_sample(seconds=max(2.0, 3.0 * args.steps / 10))
    line = {"impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "higher_is_better": True, "dtype": "bf16 (4-bit codes)",
            "data": "synthetic", "config": {"workload": "fused QKV decode projection (cfg2), M=16",
                                            "x": [HEAD_M, HEAD_K], "w": [HEAD_N, HEAD_K], "bits": 4, "group": 64},
            "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                             "sample": sample},
            "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "note": "MLX (the reference's CPU backend) is not installable offline; the reference arm times the C/OpenMP "
                    "restatement of its arithmetic (oracle/lq_oracle.c)"}
    print(json.dumps(line), flush=True)
    return 0


# --------------------------------------------------------------------------------------------------
# GPU arm
# --------------------------------------------------------------------------------------------------

def make_layer(torch, N, K, bits, dtype, gen, dev):
    from locals_b200 import kernels

    w = torch.randn((N, K), generator=gen, device=dev, dtype=torch.float32) * 0.02
    return kernels.quantize(w, 64, bits, dtype=dtype)


def timed(torch, fn, steps, warmup, stream):
    """ms per step of fn() issued on `stream`, CUDA events on that stream, synchronized on both sides."""
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        e1.synchronize()
    return e0.elapsed_time(e1) / steps


def capture(torch, body, stream):
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        body()  # warm: first calls set kernel attributes outside the capture
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=stream):
            body()
    torch.cuda.synchronize()
    return g


def bench_qkv(torch, M, layers, steps, warmup, dev, stream, with_e2e=False, choice=None):
    """Fused QKV (config 2) over `layers` distinct weight copies; returns a dict of measurements. `choice` pins a
    kernel family (None: the library's own choice)."""
    from locals_b200 import kernels

    gen = torch.Generator(device=dev)
    gen.manual_seed(1)
    Ws = [make_layer(torch, HEAD_N, HEAD_K, 4, torch.bfloat16, gen, dev) for _ in range(layers)]
    x = (torch.randn((M, HEAD_K), generator=gen, device=dev)).to(torch.bfloat16)
    outs = {}

    def body():
        for i, (w, s, b) in enumerate(Ws):
            outs["qkv"] = kernels.qmm_split(x, w, s, b, HEAD_WIDTHS, choice=choice)

    g = capture(torch, body, stream)
    ms = timed(torch, g.replay, steps, warmup, stream)
    by = qmm_bytes(M, HEAD_N, HEAD_K, 4) * layers
    res = {"M": M, "ms_per_step": ms, "bytes_per_step": by, "gbs": by / (ms * 1e-3) / 1e9,
           "us_per_launch": ms * 1e3 / layers, "launches_per_step": layers}
    if with_e2e:
        hx = torch.empty((M, HEAD_K), dtype=torch.bfloat16, pin_memory=True)
        hx.copy_(x.cpu())
        hq = [torch.empty(o.shape, dtype=o.dtype, pin_memory=True) for o in outs["qkv"]]

        def e2e_step():
            x.copy_(hx, non_blocking=True)
            g.replay()
            for h, o in zip(hq, outs["qkv"]):
                h.copy_(o, non_blocking=True)

        ms_e2e = timed(torch, e2e_step, steps, warmup, stream)
        res["e2e_ms"] = ms_e2e
        res["e2e_gbs"] = by / (ms_e2e * 1e-3) / 1e9
        res["h2d"] = M * HEAD_K * 2
        res["d2h"] = sum(h.numel() * 2 for h in hq)
    del Ws
    return res


def bench_cfg1(torch, steps, warmup, dev, stream, copies=24):
    """Config 1: fp16 x [8, 4096] . 4-bit [4096, 4096]^T, rotated over `copies` weight copies (> L2)."""
    from locals_b200 import kernels

    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    Ws = [make_layer(torch, 4096, 4096, 4, torch.float16, gen, dev) for _ in range(copies)]
    x = torch.randn((8, 4096), generator=gen, device=dev).to(torch.float16)
    y = torch.empty((8, 4096), dtype=torch.float16, device=dev)

    def body():
        for w, s, b in Ws:
            kernels.quantized_matmul(x, w, s, b, out=y)

    g = capture(torch, body, stream)
    ms = timed(torch, g.replay, steps, warmup, stream)
    by = qmm_bytes(8, 4096, 4096, 4) * copies
    return {"gbs": by / (ms * 1e-3) / 1e9, "us_per_call": ms * 1e3 / copies}


def bench_mlp(torch, M, steps, warmup, dev, stream, layers=4):
    """Config 3: 8-bit MLP 2560 -> 9728 -> 2560 (gate||up + SiLU.mul fused, then down), `layers` copies."""
    from locals_b200.fuse import FusedMLP
    from locals_b200.kernels import QuantizedLinear

    gen = torch.Generator(device=dev)
    gen.manual_seed(2)
    mlps = []
    for _ in range(layers):
        g_ = QuantizedLinear(*make_layer(torch, 9728, 2560, 8, torch.bfloat16, gen, dev), bits=8)
        u_ = QuantizedLinear(*make_layer(torch, 9728, 2560, 8, torch.bfloat16, gen, dev), bits=8)
        d_ = QuantizedLinear(*make_layer(torch, 2560, 9728, 8, torch.bfloat16, gen, dev), bits=8)
        mlps.append(FusedMLP(g_, u_, d_))
    x = torch.randn((M, 2560), generator=gen, device=dev).to(torch.bfloat16)

    def body():
        for m in mlps:
            m(x)

    g = capture(torch, body, stream)
    ms = timed(torch, g.replay, steps, warmup, stream)
    by = (2 * 9728 * 2560 + 2560 * 9728) + 3 * 2 * 2 * (9728 * 40) + M * (2560 * 2 + 9728 * 4 + 2560 * 2)
    by *= layers
    return {"M": M, "gbs": by / (ms * 1e-3) / 1e9, "us_per_mlp": ms * 1e3 / layers,
            "tok_s": M * layers / (ms * 1e-3)}


def bench_moe(torch, M, steps, warmup, dev, stream):
    """Config 4: 64 experts, top-4, D 2048, I 768, 4-bit; router fp16, x bf16; tok/s of whole layers. Distinct layers
    (router and expert stacks) are rotated until the routed experts' weights of one pass exceed twice the L2 (each
    replay streams them from HBM): random packed codes with small positive scales (the timing does not depend on the
    values; the routing is random as the config's is)."""
    from locals_b200 import moe

    E, D, I, K = 64, 2048, 768, 4
    gen = torch.Generator(device=dev)
    gen.manual_seed(3)

    def stack(N, Kd):
        wq = torch.randint(-2 ** 31, 2 ** 31 - 1, (E, N, Kd // 8), generator=gen, device=dev, dtype=torch.int32)
        sc = (torch.rand((E, N, Kd // 64), generator=gen, device=dev) * 2e-3 + 5e-4).to(torch.bfloat16)
        return wq, sc, (-8.0 * sc.float()).to(torch.bfloat16)

    per_expert = 3 * I * D // 2 + 3 * 2 * 2 * I * D // 64
    x = torch.randn((M, D), generator=gen, device=dev).to(torch.bfloat16)
    layers, used, total = [], [], 0
    while not layers or (total < 2 * L2_BYTES and len(layers) < 32):
        gate, up, down = stack(I, D), stack(I, D), stack(D, I)
        wr = (torch.randn((E, D), generator=gen, device=dev) * 0.02).to(torch.float16)
        layer = moe.MoELayer(wr, gate, up, down, top_k=K)
        inds, _ = layer.route(x)
        u = int(torch.unique(inds).numel())
        layers.append(layer)
        used.append(u)
        total += u * per_expert

    def body():
        for la in layers:
            la(x)

    g = capture(torch, body, stream)
    ms = timed(torch, g.replay, steps, warmup, stream) / len(layers)
    by = sum(used) / len(layers) * per_expert + E * D * 2 + M * D * 2 * 2
    return {"M": M, "tok_s": M / (ms * 1e-3), "us_per_layer": ms * 1e3, "experts_used": round(sum(used) / len(used), 1),
            "layers_rotated": len(layers), "gbs": by / (ms * 1e-3) / 1e9}


def bench_norm(torch, steps, warmup, dev, stream, rows=8192, D=4096):
    """The fused residual add + RMS norm over rows x D bf16 (x, r read; h, n written; w cached): GB/s."""
    from locals_b200 import norm

    gen = torch.Generator(device=dev)
    gen.manual_seed(5)
    x = torch.randn((rows, D), generator=gen, device=dev).to(torch.bfloat16)
    r = torch.randn((rows, D), generator=gen, device=dev).to(torch.bfloat16)
    w = torch.randn((D,), generator=gen, device=dev).to(torch.bfloat16)
    g = capture(torch, lambda: norm.add_rms(x, r, w, 1e-6), stream)
    ms = timed(torch, g.replay, steps, warmup, stream)
    by = 4 * rows * D * 2 + D * 2
    return {"rows": rows, "D": D, "us": ms * 1e3, "GB/s": by / (ms * 1e-3) / 1e9}


def bench_kv(torch, steps, warmup, dev, stream, B=8, n=32768):
    """8-bit KV decode attention over a Flint full-attention layer's cache (32 query heads on 4 key/value heads,
    head dim 128, sinks) at n keys a row: GB/s of the cache read (272 bytes a key and kv head; > L2 at B*n = 2^18)."""
    from locals_b200 import qkv

    H, KVH = 32, 4
    gen = torch.Generator(device=dev)
    gen.manual_seed(6)
    keys = qkv.quantize((torch.randn((B, KVH, n, 128), generator=gen, device=dev) * 2).to(torch.bfloat16))
    values = qkv.quantize(torch.randn((B, KVH, n, 128), generator=gen, device=dev).to(torch.bfloat16))
    q = torch.randn((B, H, 1, 128), generator=gen, device=dev).to(torch.bfloat16)
    sinks = (torch.randn((H,), generator=gen, device=dev) * 2).to(torch.bfloat16)
    start = torch.zeros((B,), dtype=torch.int32, device=dev)
    g = capture(torch, lambda: qkv.attend(q, keys, values, n, sinks, 0.0884, start), stream)
    ms = timed(torch, g.replay, steps, warmup, stream)
    by = B * KVH * n * 272 + 2 * B * H * 128 * 2
    return {"B": B, "n": n, "us": ms * 1e3, "GB/s": by / (ms * 1e-3) / 1e9}


def bench_prefill(torch, steps, warmup, dev, stream):
    """Config 5: x bf16 [2048, 4096] . 4-bit [14336, 4096]^T -> TFLOP/s."""
    from locals_b200 import kernels

    gen = torch.Generator(device=dev)
    gen.manual_seed(4)
    w, s, b = make_layer(torch, 14336, 4096, 4, torch.bfloat16, gen, dev)
    x = torch.randn((2048, 4096), generator=gen, device=dev).to(torch.bfloat16)
    y = torch.empty((2048, 14336), dtype=torch.bfloat16, device=dev)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)

    def body():
        kernels.quantized_matmul(x, w, s, b, out=y)

    g = capture(torch, body, stream)
    tot = 0.0
    with torch.cuda.stream(stream):
        for _ in range(max(3, warmup)):
            g.replay()
        torch.cuda.synchronize()
        for _ in range(steps):
            flush.zero_()  # L2 flush between timed calls
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            g.replay()
            e1.record(stream)
            e1.synchronize()
            tot += e0.elapsed_time(e1)
    ms = tot / steps
    return {"tflops": 2 * 2048 * 14336 * 4096 / (ms * 1e-3) / 1e12, "ms": ms}



# --------------------------------------------------------------------------------------------------
# sharded configurations (all ranks; NCCL collectives; each rank's time on its own stream, max over ranks)
# --------------------------------------------------------------------------------------------------

def _timed_max(torch, fn, steps, warmup, stream, dist):
    """The step captured in a CUDA graph (NCCL collectives included, after an eager warm-up that sets up
    the communicator), timed on this rank's stream; the max over ranks. The graph is released here."""
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            fn()
    torch.cuda.synchronize()
    dist.barrier()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=stream):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    ms = timed(torch, g.replay, steps, 2, stream)
    del g
    t = torch.tensor([ms], device=torch.device("cuda", torch.cuda.current_device()))
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t[0])


def bench_sharded(torch, dist, ws, steps, warmup, dev, stream):
    """cfg3, cfg4, cfg5 split over the ranks (column shards + all-gather, expert parallelism), the exchanges over peer
    memory (CUDA IPC buffers, flags; NCCL only where ranks share a GPU), each step captured in a CUDA graph; returns
    rank-0 results."""
    from locals_b200 import moe
    from locals_b200.kernels import QuantizedLinear
    from locals_b200.shard import ExpertParallelMoE, ShardedMLP, ColumnShardedLinear

    out = {}
    gen = torch.Generator(device=dev)
    gen.manual_seed(2)
    mlps = []
    for _ in range(4):  # as the one-GPU config-3 bench: four distinct MLPs a step
        g_ = QuantizedLinear(*make_layer(torch, 9728, 2560, 8, torch.bfloat16, gen, dev), bits=8)
        u_ = QuantizedLinear(*make_layer(torch, 9728, 2560, 8, torch.bfloat16, gen, dev), bits=8)
        d_ = QuantizedLinear(*make_layer(torch, 2560, 9728, 8, torch.bfloat16, gen, dev), bits=8)
        mlps.append(ShardedMLP(g_, u_, d_))
        del g_, u_, d_
    out["cfg3_mlp_8bit_sharded"] = {}
    for M in (1, 16, 64):
        x = torch.randn((M, 2560), generator=gen, device=dev).to(torch.bfloat16)
        ms = _timed_max(torch, lambda: [m(x) for m in mlps], steps, warmup, stream, dist) / len(mlps)
        out["cfg3_mlp_8bit_sharded"][f"M={M}"] = {"us_per_mlp": round(ms * 1e3, 2), "tok/s": round(M / (ms * 1e-3), 1)}
    del mlps
    gen.manual_seed(3)
    E, D, I = 64, 2048, 768

    def stack(N, Kd):  # random packed codes, small positive scales (as the one-GPU config-4 bench)
        wq = torch.randint(-2 ** 31, 2 ** 31 - 1, (E, N, Kd // 8), generator=gen, device=dev, dtype=torch.int32)
        sc = (torch.rand((E, N, Kd // 64), generator=gen, device=dev) * 2e-3 + 5e-4).to(torch.bfloat16)
        return wq, sc, (-8.0 * sc.float()).to(torch.bfloat16)

    eps = []
    for _ in range(4):  # distinct layers a step (each rank holds its E/G experts of each)
        wr = (torch.randn((E, D), generator=gen, device=dev) * 0.02).to(torch.float16)
        eps.append(ExpertParallelMoE(wr, stack(I, D), stack(I, D), stack(D, I), top_k=4))
    out["cfg4_moe_ep"] = {}
    for M in (8, 64, 512):
        if M % ws:
            continue
        L = 4 if M <= 16 else 2
        x = torch.randn((M // ws, D), generator=gen, device=dev).to(torch.bfloat16)
        ms = _timed_max(torch, lambda: [e(x) for e in eps[:L]], steps, warmup, stream, dist) / L
        out["cfg4_moe_ep"][f"M={M}"] = {"us_per_layer": round(ms * 1e3, 2), "tok/s": round(M / (ms * 1e-3), 1),
                                        "layers_rotated": L}
    del eps
    gen.manual_seed(4)
    full = QuantizedLinear(*make_layer(torch, 14336, 4096, 4, torch.bfloat16, gen, dev))
    lin = ColumnShardedLinear(full)  # the GEMM stores its output tiles into every rank's buffer (fused all-gather)
    lin_nccl = ColumnShardedLinear(full, fused_gather=False)  # the same GEMM, then an NCCL all-gather
    del full
    x = torch.randn((2048, 4096), generator=gen, device=dev).to(torch.bfloat16)
    ms = _timed_max(torch, lambda: lin(x), max(3, steps // 4), warmup, stream, dist)
    ms_nccl = _timed_max(torch, lambda: lin_nccl(x), max(3, steps // 4), warmup, stream, dist)
    fl = 2 * 2048 * 14336 * 4096
    out["cfg5_prefill_sharded"] = {"ms": round(ms, 3), "TFLOP/s": round(fl / (ms * 1e-3) / 1e12, 1),
                                   "form": "dense GEMM with the all-gather in its epilogue (peer stores over NVLink)",
                                   "nccl_allgather_ms": round(ms_nccl, 3),
                                   "nccl_allgather_TFLOP/s": round(fl / (ms_nccl * 1e-3) / 1e12, 1)}
    return out


def sharded_speedups(extra, ws):
    """Per-N speed-up of each sharded configuration over the same workload on one GPU (rank 0's own runs in this
    process): time on one GPU / time on ws GPUs, and that over ws (the parallel efficiency)."""
    def put(key, t1, tn):
        if t1 and tn:
            extra[key]["speedup_vs_1gpu"] = round(t1 / tn, 3)
            extra[key]["efficiency"] = round(t1 / tn / ws, 3)

    try:
        put("cfg5_prefill_sharded", extra["cfg5_prefill"]["ms"], extra["cfg5_prefill_sharded"]["ms"])
    except KeyError:
        pass
    for M in (1, 16, 64):
        try:
            t1 = extra["cfg3_mlp_8bit"][f"M={M}"]["us_per_mlp"]
            d = extra["cfg3_mlp_8bit_sharded"][f"M={M}"]
            d["speedup_vs_1gpu"] = round(t1 / d["us_per_mlp"], 3)
            d["efficiency"] = round(t1 / d["us_per_mlp"] / ws, 3)
        except KeyError:
            pass
    for M in (8, 64, 512):
        try:
            t1 = extra["cfg4_moe"][f"M={M}"]["us_per_layer"]
            d = extra["cfg4_moe_ep"][f"M={M}"]
            d["speedup_vs_1gpu"] = round(t1 / d["us_per_layer"], 3)
            d["efficiency"] = round(t1 / d["us_per_layer"] / ws, 3)
        except KeyError:
            pass


def run_gpu(args):
    import torch

    ws, rank, local = dist_env()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if ws > 1:
        import torch.distributed as dist

        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from locals_b200 import _lib

    _lib.lib()
    stream = torch.cuda.Stream(device=dev)
    hbm, tfl, peak_kind = peaks()

    # ---- headline (per rank: its own stack of layers; weak scaling) ----
    head_layers = LAYERS
    with ClockSampler(local) as clk:
        if ws > 1:
            import torch.distributed as dist

            dist.barrier()
        torch.cuda.synchronize()
        head = bench_qkv(torch, HEAD_M, head_layers, args.steps, args.warmup, dev, stream, with_e2e=True)
        torch.cuda.synchronize()
        if ws > 1:
            dist.barrier()
    clocks = clk.summary()
    ms = head["ms_per_step"]
    ms_e2e = head["e2e_ms"]
    if ws > 1:
        t = torch.tensor([ms, ms_e2e], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms, ms_e2e = float(t[0]), float(t[1])
    total_bytes = head["bytes_per_step"] * ws
    value = total_bytes / (ms * 1e-3) / 1e9
    e2e_value = total_bytes / (ms_e2e * 1e-3) / 1e9
    per_launch_bytes = qmm_bytes(HEAD_M, HEAD_N, HEAD_K, 4)
    achieved = per_launch_bytes / (head["us_per_launch"] * 1e-6) / 1e9

    extra = {}
    if rank == 0 and not args.quick:
        extra["cfg2_fused_qkv"] = {}
        for M in (1, 4, 8, 16):
            r = bench_qkv(torch, M, head_layers, max(5, args.steps // 2), args.warmup, dev, stream)
            extra["cfg2_fused_qkv"][f"M={M}"] = {"GB/s": round(r["gbs"], 1), "frac_hbm": round(r["gbs"] / hbm, 3),
                                                 "us_per_call": round(r["us_per_launch"], 3)}
        # the two 4-bit decode families on the headline shape (the library's choice is one of them)
        extra["cfg2_decode_families_us"] = {}
        for fam in ("qmvg", "qmvq"):
            for M in (1, 4, 8, 16):
                r = bench_qkv(torch, M, head_layers, max(5, args.steps // 2), args.warmup, dev, stream,
                              choice=(fam, 0, 0))
                extra["cfg2_decode_families_us"][f"{fam} M={M}"] = round(r["us_per_launch"], 3)
        r = bench_cfg1(torch, max(5, args.steps // 2), args.warmup, dev, stream)
        extra["cfg1_qmm_fp16_m8"] = {"GB/s": round(r["gbs"], 1), "frac_hbm": round(r["gbs"] / hbm, 3),
                                     "us_per_call": round(r["us_per_call"], 3)}
        extra["cfg3_mlp_8bit"] = {}
        for M in (1, 4, 16, 64):
            r = bench_mlp(torch, M, max(5, args.steps // 2), args.warmup, dev, stream)
            extra["cfg3_mlp_8bit"][f"M={M}"] = {"GB/s": round(r["gbs"], 1), "frac_hbm": round(r["gbs"] / hbm, 3),
                                                "us_per_mlp": round(r["us_per_mlp"], 2), "tok/s": round(r["tok_s"], 1)}
        extra["cfg4_moe"] = {}
        for M in (1, 8, 16, 64, 512):
            r = bench_moe(torch, M, max(5, args.steps // 2), args.warmup, dev, stream)
            extra["cfg4_moe"][f"M={M}"] = {"tok/s": round(r["tok_s"], 1), "us_per_layer": round(r["us_per_layer"], 2),
                                           "experts_used": r["experts_used"], "GB/s": round(r["gbs"], 1),
                                           "layers_rotated": r["layers_rotated"]}
        r = bench_prefill(torch, 3, args.warmup, dev, stream)
        extra["cfg5_prefill"] = {"TFLOP/s": round(r["tflops"], 1), "frac_bf16": round(r["tflops"] / tfl, 3),
                                 "ms": round(r["ms"], 3)}
        r = bench_norm(torch, args.steps, args.warmup, dev, stream)
        extra["add_rms_norm_8192x4096"] = {"GB/s": round(r["GB/s"], 1), "frac_hbm": round(r["GB/s"] / hbm, 3),
                                           "us": round(r["us"], 2)}
        for B, n in ((8, 32768), (32, 8192)):
            r = bench_kv(torch, args.steps, args.warmup, dev, stream, B, n)
            extra[f"kv_attend_8bit_b{B}_n{n}"] = {"GB/s": round(r["GB/s"], 1), "frac_hbm": round(r["GB/s"] / hbm, 3),
                                                  "us": round(r["us"], 2)}

    if ws > 1 and not args.quick:
        extra.update(bench_sharded(torch, dist, ws, max(5, args.steps // 2), args.warmup, dev, stream))
        if rank == 0:
            sharded_speedups(extra, ws)

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        gbs, threads, sample = cpu_qkv_sample(seconds=10.0)
        cpu = {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample}

    if rank == 0:
        traffic = profile_traffic("qmvq_fused_qkv_m16")
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "bf16 (4-bit codes)", "data": "synthetic",
            "config": {"workload": "fused QKV decode projection (cfg2), M=16, x bf16 [16,2560], "
                                   "W 4-bit g64 [6144,2560] -> q[16,32,128] k,v[16,8,128]",
                       "layers_per_step": head_layers, "weights_per_step_MB": round(head["bytes_per_step"] / 1e6, 1),
                       "l2": "inputs larger than L2 (distinct weights per layer, 318 MB per step)",
                       "parallelism": (f"{ws} replicas of the config-2 layer stack (weak); configs 3-5 sharded "
                                       "over peer memory in the cfg*_sharded / cfg4_moe_ep keys") if ws > 1 else "1 GPU",
                       "graph": "CUDA graph of the step, PDL between launches"},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "traffic": traffic,
                         "kernel": "lq::qmvq_kernel<bf16,BITS=4,MT=2,FR=3,NMAT=1>", "peak_kind": peak_kind,
                         "algorithmic_bytes_per_launch": per_launch_bytes},
            "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": head["h2d"],
                    "d2h_bytes_per_step": head["d2h"]},
            "gpu_launches": head["launches_per_step"] * args.steps,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        line.update(extra)
        print(json.dumps(line), flush=True)
    if ws > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


# --------------------------------------------------------------------------------------------------
# single small cases for ncu captures (--case NAME): a few launches of one kernel family, nothing timed
# --------------------------------------------------------------------------------------------------

CASES = {
    "qkv16": "fused QKV decode, x bf16 [16,2560] . 4-bit [6144,2560]^T, 8 distinct layers (72 MB)",
    "qkv16_l2": "fused QKV decode at M=16 (the library's choice, qmvq) over 24 layers (218 MB > L2), for DRAM figures",
    "qkv1_l2": "fused QKV decode at M=1 (the library's choice, qmvq) over 24 layers (218 MB > L2)",
    "mlp64": "8-bit MLP gate||up + SiLU.mul and down at M=64, 4 layers",
    "mlp1": "8-bit MLP gate||up + SiLU.mul and down at M=1, 4 layers (320 MB > L2)",
    "tc": "prefill GEMM x bf16 [1024,4096] . 4-bit [7168,4096]^T",
    "moe1": "MoE layer at one token (the fused one-launch kernel), 64 experts top-4, D 2048, I 768, 16 distinct layers "
            "(170 MB of routed weights > L2)",
    "moe16": "MoE layer, 64 experts top-4, D 2048, I 768, M=16",
    "moe512": "MoE layer, 64 experts top-4, D 2048, I 768, M=512",
    "kv8": "8-bit KV decode attention, B=8, 32 query heads on 4 kv heads, 32768 keys (285 MB cache > L2)",
}


def run_case(name):
    import torch

    from locals_b200 import _lib, kernels, moe
    from locals_b200.fuse import FusedMLP
    from locals_b200.kernels import QuantizedLinear

    _lib.lib()
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(0)
    if name in ("qkv16", "qkv16_l2", "qkv1_l2"):
        L = 8 if name == "qkv16" else 24
        Ws = [make_layer(torch, HEAD_N, HEAD_K, 4, torch.bfloat16, gen, dev) for _ in range(L)]
        x = torch.randn((1 if name == "qkv1_l2" else 16, HEAD_K), generator=gen, device=dev).to(torch.bfloat16)
        for _ in range(3):
            for w, s, b in Ws:
                kernels.qmm_split(x, w, s, b, HEAD_WIDTHS)
    elif name in ("mlp64", "mlp1"):
        mlps = [FusedMLP(*[QuantizedLinear(*make_layer(torch, n, k, 8, torch.bfloat16, gen, dev), bits=8)
                           for n, k in ((9728, 2560), (9728, 2560), (2560, 9728))]) for _ in range(4)]
        x = torch.randn((64 if name == "mlp64" else 1, 2560), generator=gen, device=dev).to(torch.bfloat16)
        for _ in range(2):
            for m in mlps:
                m(x)
    elif name == "tc":
        w, s, b = make_layer(torch, 7168, 4096, 4, torch.bfloat16, gen, dev)
        x = torch.randn((1024, 4096), generator=gen, device=dev).to(torch.bfloat16)
        for _ in range(4):
            kernels.quantized_matmul(x, w, s, b)
    elif name == "moe1":
        E, D, I = 64, 2048, 768

        def stack(N, Kd):  # random packed codes, small positive scales (timing only)
            wq = torch.randint(-2 ** 31, 2 ** 31 - 1, (E, N, Kd // 8), generator=gen, device=dev, dtype=torch.int32)
            sc = (torch.rand((E, N, Kd // 64), generator=gen, device=dev) * 2e-3 + 5e-4).to(torch.bfloat16)
            return wq, sc, (-8.0 * sc.float()).to(torch.bfloat16)

        layers = [moe.MoELayer((torch.randn((E, D), generator=gen, device=dev) * 0.02).to(torch.float16),
                               stack(I, D), stack(I, D), stack(D, I), top_k=4) for _ in range(16)]
        x = torch.randn((1, D), generator=gen, device=dev).to(torch.bfloat16)
        for _ in range(3):
            for la in layers:
                la(x)
    elif name in ("moe16", "moe512"):
        E, D, I = 64, 2048, 768

        def stack(N, Kd):
            ws_ = [make_layer(torch, N, Kd, 4, torch.bfloat16, gen, dev) for _ in range(E)]
            return tuple(torch.stack([w[i] for w in ws_]).contiguous() for i in range(3))

        layer = moe.MoELayer((torch.randn((E, D), generator=gen, device=dev) * 0.02).to(torch.float16),
                             stack(I, D), stack(I, D), stack(D, I), top_k=4)
        x = torch.randn((16 if name == "moe16" else 512, D), generator=gen, device=dev).to(torch.bfloat16)
        for _ in range(3):
            layer(x)
    elif name == "kv8":
        from locals_b200 import qkv

        B, H, KVH, n = 8, 32, 4, 32768
        keys = qkv.quantize((torch.randn((B, KVH, n, 128), generator=gen, device=dev) * 2).to(torch.bfloat16))
        values = qkv.quantize(torch.randn((B, KVH, n, 128), generator=gen, device=dev).to(torch.bfloat16))
        q = torch.randn((B, H, 1, 128), generator=gen, device=dev).to(torch.bfloat16)
        sinks = (torch.randn((H,), generator=gen, device=dev) * 2).to(torch.bfloat16)
        for _ in range(3):
            qkv.attend(q, keys, values, n, sinks, 0.0884)
    else:
        raise SystemExit(f"unknown case {name}; known: {sorted(CASES)}")
    torch.cuda.synchronize()
    st = kernels.device_status()
    print(json.dumps({"case": name, "status": st}))
    return 0 if st == 0 else 1


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="lq", choices=["lq", "reference"])
    ap.add_argument("--quick", action="store_true", help="headline only (skip the other configs)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--case", default=None, help="run one small profiling case (see CASES) and exit")
    args = ap.parse_args()
    if args.case:
        return run_case(args.case)
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        return run_reference(args)
    return run_gpu(args)


if __name__ == "__main__":
    sys.exit(main())
