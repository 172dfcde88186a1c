"""numpy front end of the CPU oracle (test infrastructure only).

Only tests/, __graft_entry__.smoke() and bench.py's CPU legs import this module, as the checker
or as the timed CPU restatement; the product (locals_b200) never does. Every function cites the
reference arithmetic it restates in lq_oracle.c's header. MLX (the reference's numerics library,
mlx 0.32.3 per uv.lock:376-377) is absent here, so the quantizer's parity is UNPINNED; the
matmul, routing and grouping arithmetic is pinned by the hand-derived vectors in tests/golden/.

Arrays of 16-bit floats travel as numpy float32 holding exactly representable values, or as
uint16 bit patterns (``to_bits`` / ``from_bits``).
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

from . import build as _build

F16, BF16, F32 = 0, 1, 2
_DT = {"float16": F16, "bfloat16": BF16, "float32": F32, F16: F16, BF16: BF16, F32: F32}

_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _build.build()
        L = ctypes.CDLL(path)
        f32p = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
        u32p = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
        i32p = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
        u8p = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")
        i64, ci = ctypes.c_int64, ctypes.c_int
        L.lqo_quantize.argtypes = [f32p, i64, i64, ci, ci, u32p, f32p, f32p]
        L.lqo_unpack.argtypes = [u32p, i64, i64, ci, u8p]
        L.lqo_dequantize.argtypes = [u32p, f32p, f32p, i64, i64, ci, ci, f32p]
        L.lqo_qmm.argtypes = [f32p, i64, i64, u32p, f32p, f32p, i64, ci, ci, f32p, ci]
        L.lqo_router.argtypes = [f32p, f32p, i64, i64, i64, f32p]
        L.lqo_topk_softmax.argtypes = [f32p, i64, ci, ci, u32p, f32p]
        L.lqo_topk_sigmoid.argtypes = [f32p, i64, ci, ci, u32p, f32p]
        L.lqo_group.argtypes = [u32p, i64, ci, i32p, i32p, i32p, i32p]
        L.lqo_swiglu.argtypes = [f32p, f32p, i64, ci, f32p]
        L.lqo_combine.argtypes = [f32p, f32p, i64, ci, i64, f32p]
        L.lqo_add_rms.argtypes = [f32p, f32p, f32p, i64, i64, ctypes.c_float, ci, f32p, f32p]
        L.lqo_combine_norm.argtypes = [f32p, f32p, ctypes.c_void_p, f32p, f32p, i64, ci, i64, ctypes.c_float, ci,
                                       f32p, f32p]
        L.lqo_kv_attend.argtypes = [f32p, u32p, f32p, f32p, u32p, f32p, f32p, ctypes.c_void_p, i64, ctypes.c_void_p,
                                    ctypes.c_float, i64, i64, i64, i64, i64, f32p]
        L.lqo_round.argtypes = [f32p, i64, ci]
        _lib = L
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32)


# ---- 16-bit helpers --------------------------------------------------------------------------

def round_to(a, dtype) -> np.ndarray:
    """float32 copy of ``a`` rounded to ``dtype`` ("float16", "bfloat16", "float32"), ties to even."""
    out = _f32(a).copy()
    lib().lqo_round(out.reshape(-1), out.size, _DT[dtype])
    return out


def to_bits(a, dtype) -> np.ndarray:
    """uint16 bit patterns of ``a`` rounded to a 16-bit dtype."""
    r = round_to(a, dtype)
    if dtype in ("float16", F16):
        return r.astype(np.float16).view(np.uint16)
    return (r.view(np.uint32) >> 16).astype(np.uint16)


def from_bits(u, dtype) -> np.ndarray:
    u = np.ascontiguousarray(u, dtype=np.uint16)
    if dtype in ("float16", F16):
        return u.view(np.float16).astype(np.float32)
    return (u.astype(np.uint32) << 16).view(np.float32)


# ---- format ----------------------------------------------------------------------------------

def quantize(w, group_size: int = 64, bits: int = 4, dtype="float32"):
    """MLX affine quantization of ``w`` (N, K) -> (packed uint32 (N, K*bits/32), scales, biases), the
    scales and biases rounded to ``dtype`` after the codes are chosen (float32 input: the
    weights are generated in fp32)."""
    w = _f32(w)
    N, K = w.shape
    assert K % group_size == 0 and group_size % (32 // bits) == 0
    wq = np.zeros((N, K * bits // 32), np.uint32)
    s = np.zeros((N, K // group_size), np.float32)
    b = np.zeros((N, K // group_size), np.float32)
    lib().lqo_quantize(w, N, K, bits, group_size, wq, s, b)
    return wq, round_to(s, dtype), round_to(b, dtype)


def unpack(wq, K: int, bits: int = 4) -> np.ndarray:
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    N = wq.shape[0]
    codes = np.zeros((N, K), np.uint8)
    lib().lqo_unpack(wq, N, K, bits, codes)
    return codes


def dequantize(wq, scales, biases, group_size: int = 64, bits: int = 4) -> np.ndarray:
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    N = wq.shape[0]
    K = wq.shape[1] * 32 // bits
    out = np.zeros((N, K), np.float32)
    lib().lqo_dequantize(wq, _f32(scales), _f32(biases), N, K, bits, group_size, out)
    return out


def qmm(x, wq, scales, biases, group_size: int = 64, bits: int = 4, threads: int = 0) -> np.ndarray:
    """float32 y = x . dequant(W)^T (MLX qmv factoring, float32 accumulation); not rounded."""
    x = _f32(x)
    wq = np.ascontiguousarray(wq, dtype=np.uint32)
    M, K = x.shape
    N = wq.shape[0]
    assert wq.shape[1] * 32 // bits == K
    y = np.zeros((M, N), np.float32)
    lib().lqo_qmm(x, M, K, wq, _f32(scales), _f32(biases), N, bits, group_size, y, threads)
    return y


# ---- MoE -------------------------------------------------------------------------------------

def router(x, w) -> np.ndarray:
    x, w = _f32(x), _f32(w)
    T, D = x.shape
    E = w.shape[0]
    out = np.zeros((T, E), np.float32)
    lib().lqo_router(x, w, T, E, D, out)
    return out


def topk(logits, k: int, mode: str = "softmax"):
    logits = _f32(logits)
    T, E = logits.shape
    inds = np.zeros((T, k), np.uint32)
    wts = np.zeros((T, k), np.float32)
    fn = lib().lqo_topk_softmax if mode == "softmax" else lib().lqo_topk_sigmoid
    fn(logits, T, E, k, inds, wts)
    return inds, wts


def group(inds, E: int):
    inds = np.ascontiguousarray(inds, dtype=np.uint32).reshape(-1)
    P = inds.size
    S = min(E, P)
    order = np.zeros(P, np.int32)
    starts = np.zeros(S + 1, np.int32)
    experts = np.zeros(S, np.int32)
    nseg = np.zeros(1, np.int32)
    lib().lqo_group(inds, P, E, order, starts, experts, nseg)
    return order, starts, experts, int(nseg[0])


def swiglu(g, u, dtype) -> np.ndarray:
    g, u = _f32(g), _f32(u)
    h = np.zeros_like(g)
    lib().lqo_swiglu(g.reshape(-1), u.reshape(-1), g.size, _DT[dtype], h.reshape(-1))
    return h


def combine(ys, w) -> np.ndarray:
    w = _f32(w)
    T, k = w.shape
    ys = _f32(ys).reshape(T * k, -1)
    D = ys.shape[1]
    y = np.zeros((T, D), np.float32)
    lib().lqo_combine(ys, w, T, k, D, y)
    return y


def add_rms(x, r, w, eps, dtype):
    """(h, n) of the fused residual add + RMS norm (norm_kernel.add_rms)."""
    x, r, w = _f32(x), _f32(r), _f32(w)
    rows, D = x.shape
    h = np.zeros_like(x)
    n = np.zeros_like(x)
    lib().lqo_add_rms(x, r, w, rows, D, eps, _DT[dtype], h, n)
    return h, n


def combine_norm(ys, w, res, nw, eps, dtype, shared=None):
    """(y, n): the MoE combine + shared expert + residual add + RMS norm (moe.py:353-389); ys (T*k, D) in
    slot order."""
    w = _f32(w)
    T, k = w.shape
    ys = _f32(ys).reshape(T * k, -1)
    D = ys.shape[1]
    res, nw = _f32(res), _f32(nw)
    y = np.zeros((T, D), np.float32)
    n = np.zeros((T, D), np.float32)
    sh = None
    if shared is not None:
        shared = _f32(shared)
        sh = shared.ctypes.data_as(ctypes.c_void_p)
    lib().lqo_combine_norm(ys, w, sh, res, nw, T, k, D, eps, _DT[dtype], y, n)
    return y, n


def kv_attend(q, keys, values, n: int, sinks, scale: float, start=None) -> np.ndarray:
    """qkv.attend (locals/qkv.py:213-249) on the CPU: q (B, H, HD); keys / values = (words uint32 (B, KVH, cap,
    HD/4), scales, biases (B, KVH, cap, HD/64)); sinks (H,) or None; start (B,) or None. Float32 (B, H, HD)."""
    q = _f32(q)
    B, H, HD = q.shape
    kq = np.ascontiguousarray(keys[0], dtype=np.uint32)
    vq = np.ascontiguousarray(values[0], dtype=np.uint32)
    ks, kb, vs, vb = (_f32(a) for a in (keys[1], keys[2], values[1], values[2]))
    KVH, cap = kq.shape[1], kq.shape[2]
    st = None if start is None else np.ascontiguousarray(start, dtype=np.int32)
    sk = None if sinks is None else _f32(sinks)
    out = np.zeros((B, H, HD), np.float32)
    lib().lqo_kv_attend(q, kq, ks, kb, vq, vs, vb, None if st is None else st.ctypes.data_as(ctypes.c_void_p), int(n),
                        None if sk is None else sk.ctypes.data_as(ctypes.c_void_p), float(scale), B, H, KVH, cap, HD,
                        out)
    return out


def linear(x, q, dtype) -> np.ndarray:
    """A quantized linear layer's output rounded to ``dtype``: q = (wq, scales, biases, bits)."""
    wq, s, b, bits = q
    return round_to(qmm(x, wq, s, b, 64, bits), dtype)


def moe(x, inds, weights, gate, up, down, dtype) -> np.ndarray:
    """mlx-lm SwitchGLU + weighted combine: per (token, slot) expert e: h = swiglu(T(gate_e x), T(up_e x)),
    y_slot = T(down_e h), y = T(sum_k w_k y_slot) (float32 sum). gate/up/down: lists over experts of
    (wq, scales, biases, bits). Rows are independent, so each expert's rows are computed together."""
    x = _f32(x)
    inds = np.asarray(inds)
    M, k = inds.shape
    D = x.shape[1]
    flat = inds.reshape(-1)
    ys = np.zeros((M * k, D), np.float32)
    for e in np.unique(flat):
        slots = np.where(flat == e)[0]
        xe = x[slots // k]
        h = swiglu(linear(xe, gate[e], dtype), linear(xe, up[e], dtype), dtype)
        ys[slots] = linear(h, down[e], dtype)
    return round_to(combine(ys, weights), dtype)
