"""Routed mixture-of-experts on MLX affine experts (the counterpart of the reference's locals/moe.py
router/routing and locals/moe_kernel.py grouped experts; config: mlx-lm's SwitchGLU block).

One step: router logits in float32 (locals/moe.py:86-139) -> top-k with softmax (or the reference's
sigmoid, locals/moe.py:36-82) renormalised -> counting sort of the (token, slot) pairs by expert
(locals/moe_kernel.py:28-66) -> the pairs' tokens gathered in expert order -> grouped gate/up +
SwiGLU (each used expert's weights read once for all its pairs, locals/moe_kernel.py:1-12) ->
grouped down projection -> weighted combine over each token's slots in float32 (locals/moe.py:339-348).
Every stage is a liblq.so kernel; buffers are allocated here (torch), never by the library.
"""

from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch

from . import _lib
from ._lib import call
from .kernels import _check_cuda, _check_format, _stream, dtype_code

SOFTMAX, SIGMOID = 0, 1


def router_logits(x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
    """float32 x (..., D) . w (E, D)^T of 16-bit x and w (their dtypes may differ)."""
    D = x.shape[-1]
    x2 = x.reshape(-1, D).contiguous()
    _check_cuda(x2, w)
    T, E = x2.shape[0], w.shape[0]
    out = torch.empty((T, E), dtype=torch.float32, device=x.device)
    call("lq_router_logits", x2.data_ptr(), dtype_code(x.dtype), w.data_ptr(), dtype_code(w.dtype), out.data_ptr(), T,
         E, D, _stream())
    return out.reshape(*x.shape[:-1], E)


def route_topk(logits: torch.Tensor, k: int, mode: int = SOFTMAX) -> Tuple[torch.Tensor, torch.Tensor]:
    """(inds int32 (T, k), weights float32 (T, k)) of float32 logits (T, E)."""
    E = logits.shape[-1]
    l2 = logits.reshape(-1, E).contiguous()
    _check_cuda(l2)
    T = l2.shape[0]
    inds = torch.empty((T, k), dtype=torch.int32, device=logits.device)
    wts = torch.empty((T, k), dtype=torch.float32, device=logits.device)
    call("lq_route_topk", l2.data_ptr(), T, E, k, mode, inds.data_ptr(), wts.data_ptr(), _stream())
    return inds, wts


def group(inds: torch.Tensor, E: int):
    """(order, starts, experts, nseg, pos) of the flat expert ids (the reference's group(),
    locals/moe_kernel.py:191-197, plus the inverse permutation)."""
    flat = inds.reshape(-1).contiguous()
    _check_cuda(flat)
    P = flat.numel()
    S = min(E, P)
    dev = inds.device
    order = torch.empty(P, dtype=torch.int32, device=dev)
    pos = torch.empty(P, dtype=torch.int32, device=dev)
    starts = torch.empty(S + 1, dtype=torch.int32, device=dev)
    experts = torch.empty(S, dtype=torch.int32, device=dev)
    nseg = torch.empty(1, dtype=torch.int32, device=dev)
    call("lq_moe_group", flat.data_ptr(), P, E, order.data_ptr(), starts.data_ptr(), experts.data_ptr(),
         nseg.data_ptr(), pos.data_ptr(), _stream())
    return order, starts, experts, nseg, pos


def group_range(inds: torch.Tensor, lo: int, count: int):
    """The grouping of only the pairs routed to experts [lo, lo + count), under local ids 0 .. count - 1, every other
    pair in the padding bucket ``count`` (sorted last; the grouped expert kernels skip it): one rank's share of an
    expert-parallel layer (lq_moe_group_range)."""
    flat = inds.reshape(-1).contiguous()
    _check_cuda(flat)
    P = flat.numel()
    S = min(count + 1, P)
    dev = inds.device
    order = torch.empty(P, dtype=torch.int32, device=dev)
    pos = torch.empty(P, dtype=torch.int32, device=dev)
    starts = torch.empty(S + 1, dtype=torch.int32, device=dev)
    experts = torch.empty(S, dtype=torch.int32, device=dev)
    nseg = torch.empty(1, dtype=torch.int32, device=dev)
    call("lq_moe_group_range", flat.data_ptr(), P, lo, count, order.data_ptr(), starts.data_ptr(), experts.data_ptr(),
         nseg.data_ptr(), pos.data_ptr(), _stream())
    return order, starts, experts, nseg, pos


# Up to this many tokens a step, each (token, slot) pair is its own segment in pair order and the counting sort is
# skipped (one launch less): a token's top-k experts are distinct, so every expert's weights are still read once. The
# reference's own decode path computes each slot straight from its expert the same way (locals/moe.py:243-349).
DIRECT_MAX_TOKENS = 1
_DIRECT: dict = {}


def direct_grouping(inds: torch.Tensor):
    """(order, starts, experts, nseg, pos) with one segment a pair, pairs in their own order: order and starts are
    the identity, experts the pairs' expert ids, pos None (the combine reads row t * k + r)."""
    flat = inds.reshape(-1).contiguous()
    _check_cuda(flat)
    P = flat.numel()
    key = (P, flat.device)
    c = _DIRECT.get(key)
    if c is None:
        ar = torch.arange(P + 1, dtype=torch.int32, device=flat.device)
        c = (ar[:P], ar, torch.full((1,), P, dtype=torch.int32, device=flat.device))
        _DIRECT[key] = c
    order, starts, nseg = c
    return order, starts, flat.view(torch.int32), nseg, None


def gather(x: torch.Tensor, order: torch.Tensor, k: int) -> torch.Tensor:
    D = x.shape[-1]
    P = order.numel()
    xs = torch.empty((P, D), dtype=x.dtype, device=x.device)
    call("lq_moe_gather", x.data_ptr(), order.data_ptr(), P, k, D, xs.data_ptr(), _stream())
    return xs


def experts(xs: torch.Tensor, grouping, mats: Sequence, N: int, max_rows: int, bits: int = 4,
            group_size: int = 64, gather_k: int = 0) -> torch.Tensor:
    """Grouped projections: mats = [gate, up] (SwiGLU) or [w]; each (weight (E, N, K*bits/32), scales
    (E, N, K/64), biases). With gather_k, xs is the token matrix (T, K) and the kernel fetches each pair's
    token (grouping order // gather_k) itself; otherwise xs holds one row per pair in expert order."""
    order, starts, experts_, nseg, _ = grouping
    K = xs.shape[-1]
    P = order.numel()
    E = mats[0][0].shape[0]
    glu = len(mats) == 2
    w0, s0, b0 = mats[0]
    w1, s1, b1 = mats[1] if glu else (w0, s0, b0)
    for w_, s_, b_ in mats:
        _check_format(w_, s_, b_, K, bits, group_size)
        if w_.dim() != 3 or w_.shape[0] != E or w_.shape[1] != N:
            raise ValueError(f"expert stack {tuple(w_.shape)} is not ({E}, {N}, K*bits/32)")
    out = torch.empty((P, N), dtype=xs.dtype, device=xs.device)
    call("lq_moe_experts", xs.data_ptr(), starts.data_ptr(), experts_.data_ptr(), nseg.data_ptr(), P, max_rows,
         1 if glu else 0, w0.data_ptr(), s0.data_ptr(), b0.data_ptr(), w1.data_ptr(), s1.data_ptr(), b1.data_ptr(),
         out.data_ptr(), E, N, K, bits, group_size, dtype_code(xs.dtype),
         order.data_ptr() if gather_k else None, gather_k, _stream())
    return out


def down_combine(h: torch.Tensor, grouping, weights: torch.Tensor, down, bits: int = 4,
                 group_size: int = 64) -> Optional[torch.Tensor]:
    """One token's down projections and the weighted combine of its k slots in one kernel (lq_moe_down_combine):
    y (1, D), or None when the shape is outside the fused kernel (use experts + combine then)."""
    k = weights.shape[-1]
    if weights.numel() != k or bits != 4:
        return None
    _, _, experts_, _, pos = grouping
    w, s, b = down
    E, N = w.shape[0], w.shape[1]
    K = h.shape[-1]
    _check_format(w, s, b, K, bits, group_size)
    y = torch.empty((1, N), dtype=h.dtype, device=h.device)
    rc = _lib.lib().lq_moe_down_combine(h.data_ptr(), experts_.data_ptr(), None if pos is None else pos.data_ptr(),
                                        weights.data_ptr(), w.data_ptr(), s.data_ptr(), b.data_ptr(), y.data_ptr(), k,
                                        E, N, K, bits, group_size, dtype_code(h.dtype), _stream())
    if rc == _lib.LQ_E_SHAPE:
        return None
    if rc != _lib.LQ_OK:
        raise _lib.LQError("lq_moe_down_combine", rc)
    return y


def combine(ys: torch.Tensor, weights: torch.Tensor, pos: Optional[torch.Tensor]) -> torch.Tensor:
    T, k = weights.shape
    D = ys.shape[-1]
    y = torch.empty((T, D), dtype=ys.dtype, device=ys.device)
    call("lq_moe_combine", ys.data_ptr(), weights.data_ptr(), None if pos is None else pos.data_ptr(), y.data_ptr(),
         T, k, D, dtype_code(ys.dtype), _stream())
    return y


def combine_norm(ys: torch.Tensor, weights: torch.Tensor, pos: Optional[torch.Tensor], res: torch.Tensor,
                 nw: torch.Tensor, eps: float, shared: Optional[torch.Tensor] = None) -> tuple:
    """The combine, the shared expert's output, the layer's residual add and the next layer's input norm in one
    kernel (locals/moe.py:353-389): (y, n) with y = res + combine(...) (+ shared), n = rms_norm(y) * nw."""
    T, k = weights.shape
    D = ys.shape[-1]
    y = torch.empty((T, D), dtype=ys.dtype, device=ys.device)
    n = torch.empty((T, D), dtype=ys.dtype, device=ys.device)
    sh = None if shared is None else shared.reshape(T, D).contiguous()
    rs = res.reshape(T, D).contiguous()
    call("lq_moe_combine_norm", ys.data_ptr(), weights.data_ptr(), None if pos is None else pos.data_ptr(),
         None if sh is None else sh.data_ptr(), rs.data_ptr(), nw.data_ptr(), y.data_ptr(), n.data_ptr(), T, k, D,
         float(eps), dtype_code(ys.dtype), _stream())
    return y, n


GATHER_IN_KERNEL_MAX_ROWS = 16  # up to this many tokens the GLU kernel fetches the pairs' tokens itself


def route(x: torch.Tensor, w: torch.Tensor, k: int, mode: int = SOFTMAX):
    """Router logits and top-k in one kernel: (inds int32 (T, k), weights float32 (T, k))."""
    D = x.shape[-1]
    x2 = x.reshape(-1, D).contiguous()
    _check_cuda(x2, w)
    T, E = x2.shape[0], w.shape[0]
    inds = torch.empty((T, k), dtype=torch.int32, device=x.device)
    wts = torch.empty((T, k), dtype=torch.float32, device=x.device)
    call("lq_moe_route", x2.data_ptr(), dtype_code(x.dtype), w.data_ptr(), dtype_code(w.dtype), T, E, D, k, mode,
         inds.data_ptr(), wts.data_ptr(), None, _stream())
    return inds, wts


def switch_glu(x: torch.Tensor, inds: torch.Tensor, gate, up, down, bits: int = 4, group_size: int = 64,
               grouping=None) -> torch.Tensor:
    """mlx-lm SwitchGLU for rows x (M, D) and experts inds (M, k): (M, k, D), slot r of token t in row (t, r) (the
    reference's switch_glu, locals/moe_kernel.py:230-239, which returns the pairs in their own order)."""
    M, k = inds.shape
    if grouping is None:
        grouping = group(inds, gate[0].shape[0])
    ys = switch_glu_grouped(x, inds, gate, up, down, bits, group_size, grouping)
    pos = grouping[4]
    if pos is not None:  # expert order -> pair order: row j of the result is row pos[j] of ys
        ys = gather(ys, pos, 1)
    return ys.reshape(M, k, -1)


def switch_glu_grouped(x: torch.Tensor, inds: torch.Tensor, gate, up, down, bits: int = 4, group_size: int = 64,
                       grouping=None) -> torch.Tensor:
    """SwitchGLU with its (M*k, D) rows left in the grouping's expert order (row order[j] of the pairs in row j; the
    combine reads them back through the inverse permutation pos)."""
    M, k = inds.shape
    E = gate[0].shape[0]
    I = gate[0].shape[1]
    D = x.shape[-1]
    if grouping is None:
        grouping = group(inds, E)
    if M <= GATHER_IN_KERNEL_MAX_ROWS:
        h = experts(x.contiguous(), grouping, [gate, up], I, max_rows=M, bits=bits, group_size=group_size,
                    gather_k=k)
    else:
        xs = gather(x, grouping[0], k)
        h = experts(xs, grouping, [gate, up], I, max_rows=M, bits=bits, group_size=group_size)
    return experts(h, grouping, [down], D, max_rows=M, bits=bits, group_size=group_size)


_DECODE_WORK: dict = {}


def decode_workspace(E: int, k: int, D: int, I: int, device) -> Optional[torch.Tensor]:
    """The zero-filled workspace of lq_moe_decode for a shape (one per shape and device; launches in stream order may
    share it -- the kernel leaves it zeroed), or None when the shape is outside the fused kernel."""
    key = (E, k, D, I, str(device))
    w = _DECODE_WORK.get(key)
    if w is None:
        n = int(_lib.lib().lq_moe_decode_workspace(E, k, D, I))
        if n == 0:
            return None
        w = torch.zeros(n, dtype=torch.uint8, device=device)
        _DECODE_WORK[key] = w
    return w


def decode(x: torch.Tensor, router_w: torch.Tensor, gate, up, down, k: int, mode: int = SOFTMAX, bits: int = 4,
           group_size: int = 64, inds: Optional[torch.Tensor] = None, weights: Optional[torch.Tensor] = None,
           workspace: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
    """One token's routed MoE layer in one kernel (lq_moe_decode): y (1, D), or None when the shape is outside the
    fused kernel (the caller then runs route + experts + down_combine). inds (1, k) int32 and weights (1, k) float32,
    when given, receive the routing."""
    x2 = x.reshape(-1, x.shape[-1]).contiguous()
    if x2.shape[0] != 1 or bits != 4 or group_size != 64:
        return None
    _check_cuda(x2, router_w)
    D = x2.shape[1]
    E = router_w.shape[0]
    I = gate[0].shape[1]
    for m in (gate, up):
        _check_format(*m, D, bits, group_size)
    _check_format(*down, I, bits, group_size)
    if router_w.shape[-1] != D or any(m[0].shape[0] != E for m in (gate, up, down)) or down[0].shape[1] != D:
        raise ValueError("router / expert stacks do not match the token width or the expert count")
    work = workspace if workspace is not None else decode_workspace(E, k, D, I, x2.device)
    if work is None:
        return None
    y = torch.empty((1, D), dtype=x2.dtype, device=x2.device)
    rc = _lib.lib().lq_moe_decode(x2.data_ptr(), router_w.data_ptr(), dtype_code(router_w.dtype), E, k, mode,
                                  gate[0].data_ptr(), gate[1].data_ptr(), gate[2].data_ptr(), up[0].data_ptr(),
                                  up[1].data_ptr(), up[2].data_ptr(), down[0].data_ptr(), down[1].data_ptr(),
                                  down[2].data_ptr(), D, I, bits, group_size, dtype_code(x2.dtype), y.data_ptr(),
                                  None if inds is None else inds.data_ptr(),
                                  None if weights is None else weights.data_ptr(), work.data_ptr(), work.numel(),
                                  _stream())
    if rc == _lib.LQ_E_SHAPE:
        return None
    if rc != _lib.LQ_OK:
        raise _lib.LQError("lq_moe_decode", rc)
    return y


class MoELayer:
    """Router + top-k experts + combine over stacked MLX-affine experts (softmax routing, top-k renormalised)."""

    def __init__(self, router_w: torch.Tensor, gate, up, down, top_k: int, mode: int = SOFTMAX, bits: int = 4,
                 group_size: int = 64, fused_decode: bool = True):
        self.router_w, self.gate, self.up, self.down = router_w, gate, up, down
        self.top_k, self.mode, self.bits, self.group_size = top_k, mode, bits, group_size
        self.fused_decode = fused_decode  # one token: lq_moe_decode (else route + experts + down_combine)
        self.n_experts = gate[0].shape[0]

    def route(self, x: torch.Tensor):
        return route(x, self.router_w, self.top_k, self.mode)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        D = x.shape[-1]
        x2 = x.reshape(-1, D).contiguous()
        if x2.shape[0] == 1 and self.fused_decode:  # one token: the whole layer in one kernel
            y = decode(x2, self.router_w, self.gate, self.up, self.down, self.top_k, self.mode, self.bits,
                       self.group_size)
            if y is not None:
                return y.reshape(x.shape)
        inds, wts = self.route(x2)
        grouping = direct_grouping(inds) if x2.shape[0] <= DIRECT_MAX_TOKENS else group(inds, self.n_experts)
        if x2.shape[0] == 1:  # one token: the down projections and the combine in one kernel
            M, k = inds.shape
            h = experts(x2, grouping, [self.gate, self.up], self.gate[0].shape[1], max_rows=M, bits=self.bits,
                        group_size=self.group_size, gather_k=k)
            y = down_combine(h, grouping, wts, self.down, self.bits, self.group_size)
            if y is not None:
                return y.reshape(x.shape)
            ys = experts(h, grouping, [self.down], self.down[0].shape[1], max_rows=M, bits=self.bits,
                         group_size=self.group_size)
            return combine(ys, wts, grouping[4]).reshape(x.shape)
        ys = switch_glu_grouped(x2, inds, self.gate, self.up, self.down, self.bits, self.group_size, grouping)
        return combine(ys, wts, grouping[4]).reshape(x.shape)
