"""Quantized-linear dispatch for MLX affine weights on B200 (the counterpart of the reference's
locals/kernels.py).

The reference routes every 4-bit quantized linear through ``_linear_call_inner``
(locals/kernels.py:1031-1054): prefill-size inputs (M >= PREFILL_M = 128) to a dequantize + dense
GEMM or MLX's quantized GEMM (locals/kernels.py:854-866,1020-1025), few-row inputs to the autotuned
fastest small-M kernel (``_small_matmul`` -> ``_choose`` -> ``_launcher``, locals/kernels.py:516-621,
797-807), everything else to ``mx.quantized_matmul``. Here the same contract holds --
``launch(choice, M, K, N, dtype) -> f(x, w, scales, biases) -> y`` with unchanged MLX tensors -- but
every path is a hand-written sm_100a kernel of liblq.so:

* ``("qmv", MT, WK, KS, NS)`` -- decode family (TMA-staged packed weights, register dequant into
  mma.sync fragments, cluster split-K), any M (weights streamed once per 64 rows);
* ``("qmvg", FR, NS)`` -- dense 4-bit decode for M <= 16: each warp takes one 64-wide group of every stage for
  all of its CTA's 16-row fragments (x loaded once per group), fragments spread over every SM;
* ``("qmvq", FR, NS)`` -- the same split with the codes fed raw to the MMA and each group's scale and bias folded in
  fp32 (the reference's fragq formulation): the weights are never rounded to the activation dtype;
* ``("tcv", NTOK, KS, WS[, PERSISTENT])`` -- the tensor-core family with weights dequantized into tensor
  memory as the MMA's A operand and tokens as its N side (16..256 columns); PERSISTENT = 1 runs one CTA
  per SM over all tiles (K % 256 == 0 at 4 bits);
* ``("tc", ...)`` -- prefill family (dequantized tiles in shared memory feeding tcgen05.mma with
  TMEM accumulators), M >= 128.

There is no CPU or library fallback: a shape the kernels reject raises ``LQError``.
"""

from __future__ import annotations

import threading
from typing import Callable, Optional, Sequence, Tuple

import torch

from . import _lib
from ._lib import call

PREFILL_M = 128  # locals/kernels.py:854: from this many rows the prefill family computes the layer
MAX_SMALL_M = 64  # the decode family's register tiles hold up to 64 rows per pass

_DT = {torch.float16: _lib.F16, torch.bfloat16: _lib.BF16, torch.float32: _lib.F32}


def dtype_code(dt: torch.dtype) -> int:
    try:
        return _DT[dt]
    except KeyError:
        raise TypeError(f"unsupported dtype {dt}") from None


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t: Optional[torch.Tensor]) -> Optional[int]:
    return None if t is None else t.data_ptr()


def _check_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if not t.is_cuda:
            raise ValueError("locals_b200 kernels take CUDA tensors")
        if not t.is_contiguous():
            raise ValueError("locals_b200 kernels take contiguous tensors")


def _check_format(w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, K: int, bits: int,
                  group_size: int) -> None:
    """The MLX affine layout for rows of K inputs: w (..., K*bits/32) 32-bit words, scales and biases
    (..., K/group_size) with the same leading dimensions (mx.quantized_matmul rejects mismatched shapes the same way).
    The kernels read whole rows of K through raw pointers, so a mismatch is refused here, before any launch."""
    if bits not in (4, 8) or K % group_size or (K * bits) % 32:
        raise ValueError(f"K={K} does not fit {bits}-bit codes in groups of {group_size}")
    if w.shape[-1] != K * bits // 32 or scales.shape[-1] != K // group_size:
        raise ValueError(f"weights {tuple(w.shape)} / scales {tuple(scales.shape)} do not match K={K} at {bits} bits, "
                         f"group {group_size}")
    if tuple(scales.shape) != tuple(biases.shape) or tuple(w.shape[:-1]) != tuple(scales.shape[:-1]):
        raise ValueError(f"weights {tuple(w.shape)}, scales {tuple(scales.shape)} and biases {tuple(biases.shape)} "
                         "disagree on their rows")


# ---- format ------------------------------------------------------------------------------------

def quantize(w: torch.Tensor, group_size: int = 64, bits: int = 4, dtype: Optional[torch.dtype] = None):
    """MLX affine quantization (mx.quantize) of w (N, K) on the GPU: (wq uint32 (N, K*bits/32),
    scales, biases (N, K/group_size) in ``dtype``, default w's dtype)."""
    _check_cuda(w)
    N, K = w.shape
    dtype = dtype or w.dtype
    wq = torch.empty((N, K * bits // 32), dtype=torch.int32, device=w.device)
    s = torch.empty((N, K // group_size), dtype=dtype, device=w.device)
    b = torch.empty_like(s)
    call("lq_quantize", w.data_ptr(), dtype_code(w.dtype), N, K, bits, group_size, wq.data_ptr(), s.data_ptr(),
         b.data_ptr(), dtype_code(dtype), _stream())
    return wq, s, b  # (uint32 words carried as int32: the same bits)


def dequantize(wq: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, group_size: int = 64,
               bits: int = 4) -> torch.Tensor:
    """mx.dequantize: (N, K) in the scales' dtype."""
    _check_cuda(wq, scales, biases)
    N = wq.shape[0]
    K = wq.shape[1] * 32 // bits
    out = torch.empty((N, K), dtype=scales.dtype, device=wq.device)
    call("lq_dequantize", wq.data_ptr(), scales.data_ptr(), biases.data_ptr(), N, K, bits, group_size,
         dtype_code(scales.dtype), out.data_ptr(), _stream())
    return out


# ---- matmul ------------------------------------------------------------------------------------

_FAMILY = {"auto": _lib.FAM_AUTO, "qmv": _lib.FAM_QMV, "tc": _lib.FAM_TC, "tcv": _lib.FAM_TCV, "qmvg": _lib.FAM_QMVG,
           "qmvq": _lib.FAM_QMVQ}


def _cfg(choice: Optional[Sequence]):
    if choice is None:
        return None
    fam = _FAMILY[choice[0]]
    return _lib.cfg(fam, *choice[1:])


# The reference's dense prefill rule (locals/kernels.py:854-866): dequantize + dense GEMM for weights of at most
# DENSE_MAX values. Here from DENSE_M rows: below that the fused kernels win (the dequantize pass is a fixed
# ~25 us on a 14336 x 4096 matrix; measured on B200).
DENSE_MAX = 1 << 27
DENSE_M = 512


def dense_default(M: int, N: int, K: int, bits: int, group_size: int = 64) -> bool:
    return M >= DENSE_M and N * K <= DENSE_MAX and group_size == 64 and bits in (4, 8) and K % 64 == 0 and N >= 16


def _qmm_dense(x2: torch.Tensor, w, scales, biases, y, M, N, K, bits, group_size, bn: int = 0) -> None:
    nbytes = int(_lib.lib().lq_qmm_dense_workspace(N, K))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=x2.device)  # the dequantized weights (a temporary, as MLX's)
    cfg = _lib.cfg(_lib.FAM_TC, bn) if bn else None
    call("lq_qmm_dense", x2.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(), y.data_ptr(), M, N, K,
         bits, group_size, dtype_code(x2.dtype), ws.data_ptr(), nbytes, cfg, _stream())


def quantized_matmul(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
                     transpose: bool = True, group_size: int = 64, bits: int = 4,
                     choice: Optional[Sequence] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x . dequant(w)^T (mx.quantized_matmul(x, w, scales, biases, transpose=True, group_size, bits))
    for x (..., K) fp16/bf16. ``choice`` = ("qmv", MT, WK, KS, NS) / ("tc", ...) / ("dense"[, BN]) / None (auto:
    from DENSE_M rows, the reference's dequantize + dense GEMM path, locals/kernels.py:999-1025)."""
    if not transpose:
        raise NotImplementedError("only transpose=True (the layout of every reference call site)")
    shape = x.shape
    K = shape[-1]
    x2 = x.reshape(-1, K)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    M = x2.shape[0]
    N = w.shape[0]
    if choice is not None and tuple(choice) == ("auto",):  # the library's own choice, recorded by the tuner
        choice = None
    _check_cuda(x2, w, scales, biases)
    _check_format(w, scales, biases, K, bits, group_size)
    if scales.dtype != x.dtype or biases.dtype != x.dtype:
        raise TypeError("scales and biases must have the activations' dtype")
    y = out if out is not None else torch.empty((M, N), dtype=x.dtype, device=x.device)
    if (choice is not None and choice[0] == "dense") or (choice is None and dense_default(M, N, K, bits, group_size)):
        _qmm_dense(x2, w, scales, biases, y, M, N, K, bits, group_size, int(choice[1]) if choice and len(choice) > 1 else 0)
        return y.reshape(*shape[:-1], N)
    call("lq_qmm", x2.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(), y.data_ptr(), M, N, K, bits,
         group_size, dtype_code(x.dtype), _cfg(choice), _stream())
    return y.reshape(*shape[:-1], N)


def qmm_split(x: torch.Tensor, w: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor,
              widths: Sequence[int], group_size: int = 64, bits: int = 4,
              choice: Optional[Sequence] = None) -> Tuple[torch.Tensor, ...]:
    """One fused projection whose output columns go to len(widths) separate (M, width) tensors."""
    K = x.shape[-1]
    x2 = x.reshape(-1, K).contiguous()
    M, N = x2.shape[0], w.shape[0]
    _check_cuda(x2, w, scales, biases)
    _check_format(w, scales, biases, K, bits, group_size)
    outs = [torch.empty((M, wd), dtype=x.dtype, device=x.device) for wd in widths]
    import ctypes
    ptrs = (ctypes.c_void_p * len(outs))(*[o.data_ptr() for o in outs])
    wds = (ctypes.c_int * len(outs))(*widths)
    call("lq_qmm_split", x2.data_ptr(), w.data_ptr(), scales.data_ptr(), biases.data_ptr(), len(outs), ptrs, wds, M,
         N, K, bits, group_size, dtype_code(x.dtype), _cfg(choice), _stream())
    return tuple(o.reshape(*x.shape[:-1], o.shape[-1]) for o in outs)


def qmm_glu(x: torch.Tensor, gate: Tuple[torch.Tensor, torch.Tensor, torch.Tensor],
            up: Tuple[torch.Tensor, torch.Tensor, torch.Tensor], group_size: int = 64, bits: int = 4,
            choice: Optional[Sequence] = None, rows: Optional[int] = None) -> torch.Tensor:
    """swiglu(x . gate^T, x . up^T) in one kernel (gate/up: (weight, scales, biases), each (I, ...)
    or views into a concatenated gate||up)."""
    K = x.shape[-1]
    x2 = x.reshape(-1, K).contiguous()
    M = x2.shape[0]
    I = rows if rows is not None else gate[0].shape[0]
    _check_cuda(x2)
    for m in (gate, up):
        _check_format(*m, K, bits, group_size)
        if m[0].shape[0] < I:
            raise ValueError(f"{I} rows asked of a {m[0].shape[0]}-row matrix")
    h = torch.empty((M, I), dtype=x.dtype, device=x.device)
    call("lq_qmm_glu", x2.data_ptr(), gate[0].data_ptr(), gate[1].data_ptr(), gate[2].data_ptr(), up[0].data_ptr(),
         up[1].data_ptr(), up[2].data_ptr(), h.data_ptr(), M, I, K, bits, group_size, dtype_code(x.dtype),
         _cfg(choice), _stream())
    return h.reshape(*x.shape[:-1], I)


# ---- the reference's launcher contract -----------------------------------------------------------

_LAUNCH: dict = {}


def launch(choice: Sequence, M: int, K: int, N: int, dtype: torch.dtype, bits: int = 4,
           group_size: int = 64) -> Callable:
    """A cached closure ``f(x2, w, scales, biases) -> y`` for one tuning choice, as the reference's
    ``_launcher(choice, M, K, N, dtype)`` (locals/kernels.py:516-576)."""
    key = (tuple(choice), M, K, N, dtype, bits, group_size)
    f = _LAUNCH.get(key)
    if f is None:
        ch = tuple(choice)

        def f(x2, w, sc, bi, _ch=ch):
            return quantized_matmul(x2, w, sc, bi, group_size=group_size, bits=bits, choice=_ch)

        _LAUNCH[key] = f
    return f


_FAMILY_NAME = {v: k for k, v in _FAMILY.items()}
_NPARAM = {"qmv": 4, "tcv": 4, "tc": 1, "qmvg": 2, "qmvq": 4}


def candidates(M: int, K: int, N: int, bits: int = 4, dtype: torch.dtype = torch.bfloat16) -> list:
    """Tuning candidates for one shape (the analogue of locals/kernels.py:654-674), from the library's own
    list (``lq_list_configs``): decode tilings ("qmv", MT token tiles of 8, WK warps splitting K per
    16-row fragment, KS cluster split-K, NS stages), ("tcv", NTOK token tile, KS split-K, WS weight slots,
    PERSISTENT), from 65 rows ("tc", BN), and from 128 rows for matrices of at most DENSE_MAX weights ("dense"[, BN])
    (dequantize once + dense GEMM); 0 = the library's choice."""
    L = _lib.lib()
    n = L.lq_list_configs(M, N, K, bits, 64, dtype_code(dtype), None, 0)
    arr = (_lib.Cfg * max(n, 1))()
    L.lq_list_configs(M, N, K, bits, 64, dtype_code(dtype), arr, n)
    out = []
    for c in arr[:n]:
        name = _FAMILY_NAME[c.family]
        out.append((name,) + tuple(int(v) for v in c.p[: _NPARAM[name]]))
    # the reference's dense prefill path (dequantize + dense GEMM, timed per shape like its own choice between MLX's
    # quantized GEMM and dequantize + matmul, locals/kernels.py:872-898) from the prefill row count
    if M >= 128 and N * K <= DENSE_MAX and K % 64 == 0 and N >= 16 and bits in (4, 8):
        out += [("dense",)] + [("dense", bn) for bn in (224, 256) if N % bn == 0 or bn == 256]
    return out


def supported(family: str, M: int, K: int, N: int, bits: int = 4, dtype: torch.dtype = torch.bfloat16) -> bool:
    """Whether a kernel family takes this shape (``lq_supported``)."""
    return bool(_lib.lib().lq_supported(_FAMILY[family], M, N, K, bits, 64, dtype_code(dtype)))


# ---- a quantized linear layer ----------------------------------------------------------------------

# ---- row packing of right-padded batches (locals/kernels.py:809-851) --------------------------------

_PACK = threading.local()  # .ctx: (B, L, valid flat row indices int32 (R,), R) while a packed_rows block is active


class packed_rows:
    """While active, a QuantizedLinear applied to right-padded (B, L, K) activations computes only the valid
    rows (lengths[b] of row block b) and scatters them back, zeros elsewhere -- padding costs no matmul work
    (the reference's ``packed_rows``, locals/kernels.py:814-830). The gather and scatter are the library's
    row kernels (``lq_moe_gather`` with k = 1, ``lq_scatter_rows``)."""

    def __init__(self, B: int, L: int, lengths: Sequence[int], device=None):
        idx = [b * L + i for b, n in enumerate(lengths) for i in range(int(n))]
        self.ctx = (B, L, torch.tensor(idx, dtype=torch.int32, device=device or "cuda"), len(idx))

    def __enter__(self):
        self.prev = getattr(_PACK, "ctx", None)
        _PACK.ctx = self.ctx
        return self

    def __exit__(self, *a):
        _PACK.ctx = self.prev


def gather_rows(x2: torch.Tensor, idx: torch.Tensor) -> torch.Tensor:
    """x2[idx] for a (rows, K) matrix (16-byte rows)."""
    R, K = idx.numel(), x2.shape[-1]
    xs = torch.empty((R, K), dtype=x2.dtype, device=x2.device)
    if R:
        call("lq_moe_gather", x2.data_ptr(), idx.data_ptr(), R, 1, K, xs.data_ptr(), _stream())
    return xs


def scatter_rows(ys: torch.Tensor, idx: torch.Tensor, rows: int) -> torch.Tensor:
    """A (rows, N) matrix of zeros with row idx[j] = ys[j]."""
    N = ys.shape[-1]
    y = torch.empty((rows, N), dtype=ys.dtype, device=ys.device)
    call("lq_scatter_rows", ys.data_ptr(), idx.data_ptr(), idx.numel(), N, y.data_ptr(), rows, dtype_code(ys.dtype),
         _stream())
    return y


def _maybe_packed(x: torch.Tensor, fn: Callable) -> torch.Tensor:
    ctx = getattr(_PACK, "ctx", None)
    if ctx is not None and x.dim() == 3 and x.shape[0] == ctx[0] and x.shape[1] == ctx[1] and ctx[3] < ctx[0] * ctx[1]:
        B, L, idx, R = ctx
        xs = gather_rows(x.reshape(B * L, -1).contiguous(), idx)
        ys = fn(xs)
        return scatter_rows(ys, idx, B * L).reshape(B, L, -1)
    return fn(x)


def pad_rows(N: int, K: int, M: int, dtype: torch.dtype, bits: int = 4) -> int:
    """The rows to compute M rows of this shape at (the reference's ``_pad_rows``, locals/kernels.py:764-794):
    up to 2M rows where the tuner's recorded times say the shape runs at least 7% faster there (8 to 16 rows
    unless LOCALS_PAD_ROWS=all; LOCALS_PAD_ROWS=0 never pads)."""
    import os

    from . import tune

    mode = os.environ.get("LOCALS_PAD_ROWS", "1")
    if mode == "0" or not (8 <= M <= 16 or mode == "all"):
        return M
    tm = tune.best_time(N, K, M, dtype, bits)
    best, bt = M, tm
    if tm is None:
        return M
    for m2 in range(M + 1, min(MAX_SMALL_M, 2 * M) + 1):
        t2 = tune.best_time(N, K, m2, dtype, bits)
        if t2 is not None and t2 < 0.93 * tm and t2 < bt:
            best, bt = m2, t2
    return best


class QuantizedLinear:
    """MLX QuantizedLinear's tensors (weight uint32 (N, K*bits/32), scales, biases (N, K/64)) with the
    reference's routing (locals/kernels.py:1031-1054): the tuned choice for (N, K, M, dtype) if one is
    cached (locals_b200.tune), else the kernel library's own pick."""

    def __init__(self, weight: torch.Tensor, scales: torch.Tensor, biases: torch.Tensor, bits: int = 4,
                 group_size: int = 64, bias: Optional[torch.Tensor] = None):
        self.weight, self.scales, self.biases = weight, scales, biases
        self.bits, self.group_size, self.bias = bits, group_size, bias

    @property
    def out_features(self) -> int:
        return self.weight.shape[0]

    @property
    def in_features(self) -> int:
        return self.weight.shape[1] * 32 // self.bits

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return _maybe_packed(x, self._call)

    def _call(self, x: torch.Tensor) -> torch.Tensor:
        from . import tune

        K = x.shape[-1]
        M = x.numel() // K
        P = pad_rows(self.out_features, K, M, x.dtype, self.bits)
        if P > M:  # more rows run faster for this shape: compute them, keep these
            x2 = torch.cat([x.reshape(M, K), x.new_zeros((P - M, K))])
            choice = tune.lookup(self.out_features, K, P, x.dtype, self.bits)
            y = quantized_matmul(x2, self.weight, self.scales, self.biases, group_size=self.group_size,
                                 bits=self.bits, choice=choice)[:M].reshape(*x.shape[:-1], -1)
        else:
            choice = tune.lookup(self.out_features, K, M, x.dtype, self.bits)
            y = quantized_matmul(x, self.weight, self.scales, self.biases, group_size=self.group_size, bits=self.bits,
                                 choice=choice)
        if self.bias is not None:
            y = y + self.bias
        return y


_STATUS_LOCK = threading.Lock()


def device_status(clear: bool = True) -> int:
    """The kernels' device status word (0 = no bounded wait gave up, no index check failed)."""
    with _STATUS_LOCK:
        return _lib.device_status(clear)
