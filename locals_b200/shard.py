"""Multi-GPU sharding of the quantized-matmul path (one process per GPU, torch.distributed over NCCL).

The reference runs one model on one Apple GPU and has no distributed code; the partitioning here:

* ``ColumnShardedLinear`` -- a quantized linear split by output rows (columns of y): rank r keeps rows
  [r N/G, (r+1) N/G) of the packed weights, scales and biases (quantization groups run along K, so each
  row block is itself a valid MLX-format matrix, the argument of locals/fuse.py:3-6), computes its slice
  of y with the decode or prefill kernel and NCCL all-gathers the slices. Prefill-size calls (the dense
  dequantize + tcgen05 GEMM path) do their own all-gather: the GEMM writes its slice in place into this rank's
  full (M, N) buffer, one copy kernel of plain peer stores puts the slice into every other rank's buffer over
  NVLink (``PeerOutputs``: buffers mapped into every rank's process by CUDA IPC), and one small NCCL all-reduce
  orders completion -- no NCCL all-gather, no strided copy.
* ``ShardedQKV`` -- the fused q/k/v projection split at head boundaries: rank r keeps H/G query heads and
  KVH/G key/value heads; its local q/k/v come out of one kernel, then are all-gathered into full q, k, v.
* ``ShardedMLP`` -- gate||up split by intermediate rows (the SwiGLU is row-local), h all-gathered, the down
  projection split by output rows, y all-gathered.
* ``ExpertParallelMoE`` -- E/G experts and M/G tokens per rank. Each rank routes its own tokens, packs the
  (token, slot) pairs into fixed-capacity per-destination blocks (capacity = its pairs, so no host
  synchronisation and the step stays capturable in a CUDA graph), NCCL all-to-all dispatches rows and
  expert ids, the owner runs the grouped expert kernels on what it received, a second all-to-all returns
  the rows, and the source rank combines each token's slots in slot order (float32).

Every collective is issued by every rank in the same order. Compute goes through liblq.so kernels; the
``ops`` hook exists so CPU tests can check the partitioning and the collectives with gloo ranks.
"""

from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional, Sequence

import torch
import torch.distributed as dist

from .kernels import QuantizedLinear

# the fused GEMM + all-gather needs the dense prefill path and stores to at most this many ranks
FUSED_GATHER_MIN_M = 128
FUSED_GATHER_MAX_RANKS = 8


def _world(group) -> tuple:
    if not dist.is_available() or not dist.is_initialized():
        return 1, 0
    return dist.get_world_size(group), dist.get_rank(group)


@dataclass
class Ops:
    """Compute hooks: quantized matmul, SwiGLU matmul, and the MoE stages on one rank's data."""

    qmm: Callable          # (x, (w, s, b), bits) -> y
    glu: Callable          # (x, gate, up, bits) -> h
    route: Callable        # (x, router_w, k, mode) -> (inds int32 (T, k), weights f32 (T, k))
    experts: Callable      # (rows, local_ids, gate, up, down, bits, max_rows) -> out rows (pair order as given)
    combine: Callable      # (ys (T*k, D) in pair order, weights (T, k)) -> y (T, D), float32 sum in slot order


def kernel_ops() -> Ops:
    from . import kernels, moe

    def qmm(x, q, bits):
        return kernels.quantized_matmul(x, q[0], q[1], q[2], bits=bits)

    def glu(x, gate, up, bits):
        return kernels.qmm_glu(x, gate, up, bits=bits)

    def route(x, wr, k, mode):
        return moe.route_topk(moe.router_logits(x, wr), k, mode)

    def experts(rows, ids, gate, up, down, bits, max_rows):
        # rows (P, D) with local expert ids (P,) in [0, E) or -1 for padding; padding goes to bucket E,
        # which the grouped kernel skips (its output rows stay unwritten and are masked by the caller)
        E = gate[0].shape[0]
        ids_c = torch.where(ids < 0, torch.full_like(ids, E), ids).to(torch.int32)
        grouping = moe.group(ids_c, E + 1)
        order, pos = grouping[0], grouping[4]
        xs = moe.gather(rows, order, 1)
        h = moe.experts(xs, grouping, [gate, up], gate[0].shape[1], max_rows=max_rows, bits=bits)
        ys = moe.experts(h, grouping, [down], down[0].shape[1], max_rows=max_rows, bits=bits)
        return ys.index_select(0, pos.long())

    def combine(ys, wts):
        return moe.combine(ys.contiguous(), wts.contiguous(), None)

    return Ops(qmm, glu, route, experts, combine)


def _split_rows(t: torch.Tensor, parts: int, idx: int) -> torch.Tensor:
    n = t.shape[0]
    if n % parts:
        raise ValueError(f"{n} rows do not split into {parts} equal shards")
    step = n // parts
    return t[idx * step:(idx + 1) * step].contiguous()


def all_gather_cols(y_local: torch.Tensor, group=None) -> torch.Tensor:
    """(M, N/G) slices of every rank -> (M, N), rank r's slice at columns [r N/G, (r+1) N/G)."""
    G, _ = _world(group)
    if G == 1:
        return y_local
    M, Nl = y_local.shape
    buf = torch.empty((G * M, Nl), dtype=y_local.dtype, device=y_local.device)  # ranks stacked along dim 0
    dist.all_gather_into_tensor(buf, y_local.contiguous(), group=group)
    return buf.view(G, M, Nl).permute(1, 0, 2).reshape(M, G * Nl)


class PeerOutputs:
    """Two (M, N) output buffers of this rank (used in turn), mapped into every rank's process through CUDA IPC
    (handles exchanged over the process group), so a kernel on any rank can store into any rank's buffer. Creating
    one is a collective: every rank creates it with the same shape in the same order. A buffer handed out by
    ``next`` is overwritten two calls later: its readers must be queued on the stream before then."""

    def __init__(self, shape, dtype, device, group=None):
        import ctypes

        from . import _lib

        G, r = _world(group)
        self.G, self.rank = G, r
        M, N = shape
        self.block = torch.empty((2, M, N), dtype=dtype, device=device)  # one allocation: one IPC handle
        h = (ctypes.c_char * 64)()
        off = ctypes.c_size_t()
        _lib.call("lq_ipc_export", self.block.data_ptr(), h, ctypes.byref(off))
        handles = [None] * G
        dist.all_gather_object(handles, (bytes(h), int(off.value)), group=group)
        self.bases = []  # every rank's block, as an address valid in this process
        self._opened = []
        for p, (hb, o) in enumerate(handles):
            if p == r:
                self.bases.append(self.block.data_ptr())
                continue
            ptr = ctypes.c_void_p()
            _lib.call("lq_ipc_import", (ctypes.c_char * 64).from_buffer_copy(hb), o, ctypes.byref(ptr))
            self.bases.append(int(ptr.value))
            self._opened.append((int(ptr.value), o))
        self.step = M * N * self.block.element_size()
        self.i = 0

    def next(self):
        """(this rank's buffer, every rank's address of that buffer)."""
        j = self.i
        self.i ^= 1
        return self.block[j], [b + j * self.step for b in self.bases]

    def close(self) -> None:
        import ctypes

        from . import _lib

        for ptr, o in self._opened:
            _lib.lib().lq_ipc_close(ctypes.c_void_p(ptr), o)
        self._opened = []


def _distinct_gpus(group=None) -> bool:
    """True when every rank of the group drives its own GPU (a collective: every rank calls it). Ranks sharing a GPU
    must not meet on flags inside kernels (nothing makes their kernels run at the same time)."""
    G, _ = _world(group)
    props = torch.cuda.get_device_properties(torch.cuda.current_device())
    ids = [None] * G
    dist.all_gather_object(ids, str(getattr(props, "uuid", "")) or str(torch.cuda.current_device()), group=group)
    return len(set(ids)) == G


class PeerSync:
    """This rank's sync block of the peer gather (lq_peer_sync_bytes() bytes, zero-filled: the flags the other ranks
    store into, a round counter and a CTA counter), mapped into every rank's process through CUDA IPC. Creating one is
    a collective."""

    def __init__(self, device, group=None):
        import ctypes

        from . import _lib

        G, r = _world(group)
        self.block = torch.zeros(int(_lib.lib().lq_peer_sync_bytes()), dtype=torch.uint8, device=device)
        h = (ctypes.c_char * 64)()
        off = ctypes.c_size_t()
        _lib.call("lq_ipc_export", self.block.data_ptr(), h, ctypes.byref(off))
        handles = [None] * G
        dist.all_gather_object(handles, (bytes(h), int(off.value)), group=group)
        self.ptrs, self._opened = [], []
        for p, (hb, o) in enumerate(handles):
            if p == r:
                self.ptrs.append(self.block.data_ptr())
                continue
            ptr = ctypes.c_void_p()
            _lib.call("lq_ipc_import", (ctypes.c_char * 64).from_buffer_copy(hb), o, ctypes.byref(ptr))
            self.ptrs.append(int(ptr.value))
            self._opened.append((int(ptr.value), o))

    def close(self) -> None:
        import ctypes

        from . import _lib

        for ptr, o in self._opened:
            _lib.lib().lq_ipc_close(ctypes.c_void_p(ptr), o)
        self._opened = []


class PeerGather:
    """The all-gather of a column-sharded (M, N/G) result at decode sizes without NCCL (lq_peer_gather_cols): one
    kernel stores this rank's columns into every rank's (M, N) buffer over peer memory and meets the other ranks on
    flags. Needs every rank on its own GPU (checked once, a collective); otherwise ``ok`` is False and the caller
    uses the NCCL all-gather. Buffers are created per (M, N, dtype) on first use (a collective: every rank makes the same
    calls in the same order) and used in turn; a returned tensor is overwritten two gathers of that shape later."""

    def __init__(self, group=None):
        G, r = _world(group)
        self.G, self.rank, self.group = G, r, group
        self.ok = 1 < G <= FUSED_GATHER_MAX_RANKS and _distinct_gpus(group)
        self._bufs = {}
        self._sync = None

    def __call__(self, y_local: torch.Tensor) -> torch.Tensor:
        import ctypes

        from . import _lib

        y_local = y_local.contiguous()
        M, Nl = y_local.shape
        N = Nl * self.G
        y, addrs = self._buffer((M, N, y_local.dtype), (M, N), y_local.dtype, y_local.device)
        dst = (ctypes.c_void_p * self.G)(*addrs)
        sync = (ctypes.c_void_p * self.G)(*self._sync.ptrs)
        _lib.call("lq_peer_gather_cols", y_local.data_ptr(), M, Nl, self.rank * Nl, N, y_local.element_size(), dst,
                  self.G, self.rank, sync, torch.cuda.current_stream().cuda_stream)
        return y

    def _buffer(self, key, shape, dtype, device):
        if self._sync is None:
            self._sync = PeerSync(device, self.group)
        if key not in self._bufs:
            self._bufs[key] = PeerOutputs(shape, dtype, device, self.group)
        return self._bufs[key].next()

    def rows(self, x_local: torch.Tensor) -> torch.Tensor:
        """Every rank's (T, D) rows stacked in rank order (G T, D): the row all-gather, as one column block a rank."""
        x_local = x_local.contiguous()
        T, D = x_local.shape
        return self(x_local.view(1, T * D)).view(self.G * T, D)

    def scatter_rows(self, src: torch.Tensor, grouping, bucket: int, dst_rows: int) -> torch.Tensor:
        """Rows of src (the grouped expert kernels' output in a lq_moe_group_range grouping's order) to row order[j]
        of every rank's (dst_rows, D) buffer, the rows before the padding bucket only; returns this rank's buffer, which
        then holds every rank's rows."""
        import ctypes

        from . import _lib

        order, starts, experts, nseg, _ = grouping
        R, D = src.shape
        y, addrs = self._buffer(("rows", dst_rows, D, src.dtype), (dst_rows, D), src.dtype, src.device)
        dst = (ctypes.c_void_p * self.G)(*addrs)
        sync = (ctypes.c_void_p * self.G)(*self._sync.ptrs)
        _lib.call("lq_peer_scatter_rows", src.data_ptr(), order.data_ptr(), starts.data_ptr(), experts.data_ptr(),
                  nseg.data_ptr(), bucket, R, D * src.element_size(), dst_rows, dst, self.G, self.rank, sync,
                  torch.cuda.current_stream().cuda_stream)
        return y

    def close(self) -> None:
        for b in self._bufs.values():
            b.close()
        if self._sync is not None:
            self._sync.close()


def gather_ok(y_local: torch.Tensor) -> bool:
    """The peer gather's layout: 16-byte column blocks."""
    return y_local.is_cuda and (y_local.shape[1] * y_local.element_size()) % 16 == 0


class ColumnShardedLinear:
    def __init__(self, full: QuantizedLinear, group=None, ops: Optional[Ops] = None, fused_gather: bool = True):
        self.group = group
        G, r = _world(group)
        self.G, self.rank = G, r
        self.N = full.weight.shape[0]
        self.local = QuantizedLinear(_split_rows(full.weight, G, r), _split_rows(full.scales, G, r),
                                     _split_rows(full.biases, G, r), full.bits, full.group_size)
        self.ops = ops or kernel_ops()
        self.fused_gather = fused_gather and ops is None
        self._peer = {}
        self._flag = None
        self._pg = PeerGather(group) if (self.fused_gather and G > 1 and torch.cuda.is_available()) else None

    def _fused_ok(self, x2: torch.Tensor) -> bool:
        from . import kernels

        M, K = x2.shape
        Nl = self.local.weight.shape[0]
        return (self.fused_gather and 1 < self.G <= FUSED_GATHER_MAX_RANKS and x2.is_cuda and M >= FUSED_GATHER_MIN_M
                and self.local.group_size == 64 and self.local.bits in (4, 8) and K % 64 == 0
                and Nl * K <= kernels.DENSE_MAX and (self.rank * Nl) % 8 == 0 and self.N % 8 == 0)

    def _gather_dense(self, x2: torch.Tensor) -> torch.Tensor:
        """The dense GEMM of this rank's rows written in place into the gathered layout, then pushed to the peers
        (lq_qmm_dense_gather)."""
        import ctypes

        from . import _lib, kernels

        M, K = x2.shape
        Nl = self.local.weight.shape[0]
        key = (M, x2.dtype)
        if key not in self._peer:
            self._peer[key] = PeerOutputs((M, self.N), x2.dtype, x2.device, self.group)
            self._flag = torch.zeros(1, dtype=torch.float32, device=x2.device)
        y, addrs = self._peer[key].next()
        order = [(self.rank + j) % self.G for j in range(self.G)]  # its own buffer first, then the others in turn
        dst = (ctypes.c_void_p * self.G)(*[addrs[p] for p in order])
        nbytes = int(_lib.lib().lq_qmm_dense_workspace(Nl, K))
        ws = torch.empty(nbytes, dtype=torch.uint8, device=x2.device)  # the dequantized weight rows
        _lib.call("lq_qmm_dense_gather", x2.data_ptr(), self.local.weight.data_ptr(), self.local.scales.data_ptr(),
                  self.local.biases.data_ptr(), dst, self.G, self.rank * Nl, self.N, M, Nl, K, self.local.bits,
                  self.local.group_size, kernels.dtype_code(x2.dtype), ws.data_ptr(), nbytes, None,
                  torch.cuda.current_stream().cuda_stream)
        dist.all_reduce(self._flag, group=self.group)  # every rank's stores are complete before any rank reads y
        return y

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, x.shape[-1])
        if not x2.is_contiguous():
            x2 = x2.contiguous()
        if self._fused_ok(x2):
            return self._gather_dense(x2).reshape(*x.shape[:-1], -1)
        y = self.ops.qmm(x2, (self.local.weight, self.local.scales, self.local.biases), self.local.bits)
        if self._pg is not None and self._pg.ok and gather_ok(y):
            return self._pg(y).reshape(*x.shape[:-1], -1)
        return all_gather_cols(y, self.group).reshape(*x.shape[:-1], -1)


class ShardedQKV:
    """q/k/v projection split at head boundaries; returns full q (M, H, D), k, v (M, KVH, D)."""

    def __init__(self, q: QuantizedLinear, k: QuantizedLinear, v: QuantizedLinear, n_heads: int, n_kv_heads: int,
                 head_dim: int, group=None, ops: Optional[Ops] = None, gather: bool = True):
        G, r = _world(group)
        if n_heads % G or n_kv_heads % G:
            raise ValueError("heads do not split evenly over the ranks")
        self.G, self.rank, self.group, self.gather = G, r, group, gather
        self.H, self.KVH, self.D = n_heads, n_kv_heads, head_dim
        parts = [(m, G, r) for m in (q, k, v)]
        self.w = torch.cat([_split_rows(m.weight, g, i) for m, g, i in parts], 0)
        self.s = torch.cat([_split_rows(m.scales, g, i) for m, g, i in parts], 0)
        self.b = torch.cat([_split_rows(m.biases, g, i) for m, g, i in parts], 0)
        self.bits = q.bits
        self.widths = (n_heads // G * head_dim, n_kv_heads // G * head_dim, n_kv_heads // G * head_dim)
        self.ops = ops

    def __call__(self, x: torch.Tensor):
        x2 = x.reshape(-1, x.shape[-1])
        M = x2.shape[0]
        if self.ops is None:
            from . import kernels

            ql, kl, vl = kernels.qmm_split(x2, self.w, self.s, self.b, self.widths, bits=self.bits)
        else:
            y = self.ops.qmm(x2, (self.w, self.s, self.b), self.bits)
            ql, kl, vl = torch.split(y, list(self.widths), dim=1)
        if not self.gather:
            return (ql.reshape(M, self.H // self.G, self.D), kl.reshape(M, self.KVH // self.G, self.D),
                    vl.reshape(M, self.KVH // self.G, self.D))
        q = all_gather_cols(ql.contiguous(), self.group).reshape(M, self.H, self.D)
        k = all_gather_cols(kl.contiguous(), self.group).reshape(M, self.KVH, self.D)
        v = all_gather_cols(vl.contiguous(), self.group).reshape(M, self.KVH, self.D)
        return q, k, v


class ShardedMLP:
    """down(swiglu(gate x, up x)) with gate/up split by intermediate rows and down by output rows."""

    def __init__(self, gate: QuantizedLinear, up: QuantizedLinear, down: QuantizedLinear, group=None,
                 ops: Optional[Ops] = None):
        G, r = _world(group)
        self.G, self.rank, self.group = G, r, group
        self.gate = tuple(_split_rows(t, G, r) for t in (gate.weight, gate.scales, gate.biases))
        self.up = tuple(_split_rows(t, G, r) for t in (up.weight, up.scales, up.biases))
        self.down = tuple(_split_rows(t, G, r) for t in (down.weight, down.scales, down.biases))
        self.bits = gate.bits
        self.ops = ops or kernel_ops()
        # the two exchanges over peer memory when every rank has its own GPU (kernel ops only), else NCCL
        self._pg = PeerGather(group) if (ops is None and G > 1 and torch.cuda.is_available()) else None

    def _gather(self, t: torch.Tensor) -> torch.Tensor:
        if self._pg is not None and self._pg.ok and gather_ok(t):
            return self._pg(t)
        return all_gather_cols(t, self.group)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        x2 = x.reshape(-1, x.shape[-1])
        h = self._gather(self.ops.glu(x2, self.gate, self.up, self.bits))
        y = self._gather(self.ops.qmm(h, self.down, self.bits))
        return y.reshape(*x.shape[:-1], -1)


class ExpertParallelMoE:
    """Routed MoE with E/G experts and M/G tokens per rank, NCCL all-to-all dispatch and combine."""

    def __init__(self, router_w: torch.Tensor, gate, up, down, top_k: int, mode: int = 0, bits: int = 4,
                 group=None, ops: Optional[Ops] = None):
        G, r = _world(group)
        E = gate[0].shape[0]
        if E % G:
            raise ValueError("experts do not split evenly over the ranks")
        self.G, self.rank, self.group = G, r, group
        self.E, self.EL = E, E // G
        self.router_w, self.k, self.mode, self.bits = router_w, top_k, mode, bits
        self.gate = tuple(_split_rows(t, G, r) for t in gate)
        self.up = tuple(_split_rows(t, G, r) for t in up)
        self.down = tuple(_split_rows(t, G, r) for t in down)
        self.ops = ops or kernel_ops()
        # every rank on its own GPU and the library's kernels: the exchanges over peer memory (_call_peer)
        self._pg = PeerGather(group) if (ops is None and G > 1 and torch.cuda.is_available()) else None

    def _call_peer(self, x_local: torch.Tensor) -> torch.Tensor:
        """Tokens gathered from every rank (peer stores), routed on every rank alike, this rank's experts' pairs
        grouped (the rest in the padding bucket) and computed, each pair's output row stored into every rank's
        pair-ordered buffer, and this rank's tokens combined from it -- the same kernels on the same expert segments as
        one GPU running the whole layer, so the same bits."""
        from . import moe

        T_l, D = x_local.shape
        G, k, EL = self.G, self.k, self.EL
        xa = self._pg.rows(x_local)  # (G T_l, D), rank order
        T = G * T_l
        inds, wts = moe.route(xa, self.router_w, k, self.mode)
        grouping = moe.group_range(inds, self.rank * EL, EL)
        I = self.gate[0].shape[1]
        if T <= moe.GATHER_IN_KERNEL_MAX_ROWS:
            h = moe.experts(xa, grouping, [self.gate, self.up], I, max_rows=T, bits=self.bits, gather_k=k)
        else:
            h = moe.experts(moe.gather(xa, grouping[0], k), grouping, [self.gate, self.up], I, max_rows=T,
                            bits=self.bits)
        ys = moe.experts(h, grouping, [self.down], D, max_rows=T, bits=self.bits)  # (T k, D), grouping order
        ys_all = self._pg.scatter_rows(ys, grouping, EL, T * k)                   # (T k, D), pair order
        mine = slice(self.rank * T_l * k, (self.rank + 1) * T_l * k)
        return moe.combine(ys_all[mine], wts[self.rank * T_l:(self.rank + 1) * T_l].contiguous(), None)

    def _a2a(self, t: torch.Tensor) -> torch.Tensor:
        if self.G == 1:
            return t
        out = torch.empty_like(t)
        dist.all_to_all_single(out, t, group=self.group)
        return out

    def __call__(self, x_local: torch.Tensor) -> torch.Tensor:
        """x_local: this rank's tokens (T, D) -> their MoE outputs (T, D)."""
        if (self._pg is not None and self._pg.ok and x_local.is_cuda and self.bits == 4
                and (x_local.shape[0] * x_local.shape[1] * x_local.element_size()) % 16 == 0):
            return self._call_peer(x_local.contiguous())
        T, D = x_local.shape
        k, G, EL = self.k, self.G, self.EL
        inds, wts = self.ops.route(x_local, self.router_w, k, self.mode)
        P = T * k
        C = P  # capacity per destination: every pair could go to one rank
        flat = inds.reshape(-1).long()
        dest = flat // EL
        # position of each pair inside its destination block: pairs before it with the same destination
        onehot = torch.nn.functional.one_hot(dest, G).to(torch.int32)           # (P, G)
        rank_in_dest = (torch.cumsum(onehot, 0) - onehot).gather(1, dest[:, None])[:, 0].long()
        slot = dest * C + rank_in_dest                                          # row in the send buffer
        send_x = torch.zeros((G * C, D), dtype=x_local.dtype, device=x_local.device)
        send_x.index_copy_(0, slot, x_local.index_select(0, torch.arange(P, device=x_local.device) // k))
        send_id = torch.full((G * C,), -1, dtype=torch.int32, device=x_local.device)
        send_id.index_copy_(0, slot, (flat - dest * EL).to(torch.int32))
        recv_x = self._a2a(send_x)
        recv_id = self._a2a(send_id)
        out = self.ops.experts(recv_x, recv_id, self.gate, self.up, self.down, self.bits, max_rows=G * C)
        out = torch.where((recv_id >= 0)[:, None], out, torch.zeros_like(out))
        back = self._a2a(out.contiguous())
        ys = back.index_select(0, slot)                                          # (P, D), pair order
        return self.ops.combine(ys, wts)
