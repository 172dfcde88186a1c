"""Keys and values in 8 bits, attended to without unpacking them (the counterpart of the reference's
locals/qkv.py).

``attend(q, keys, values, n, sinks, scale, start)`` takes the reference's arguments (qkv.py:213-249): one query a
row and head against a cache's whole buffers, MLX affine 8-bit groups of 64 read in place, positions ``start[b]``
to ``n`` of row b, softmax over those keys and the head's sink. It runs ``lq_kv_attend``: a flash-decoding pass on
the tensor cores (sm_100a) and, when the keys are split over several blocks, a join with the sinks.

``QuantizedKVCache8`` keeps the reference's cache layout and growth rule (BatchQuantizedKVCache.update_and_fetch,
qkv.py:300-326): buffers of (words, scales, biases) (B, KVH, capacity, ...) grown in steps of 256 positions, new
keys and values quantized on the GPU (``lq_quantize``, 8 bits, groups of 64).
"""

from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch

from . import kernels
from ._lib import call, lib
from .kernels import _check_cuda, _stream, dtype_code

BITS, GROUP = 8, 64
HEAD_DIM = 128
MAX_GROUP = 16  # query heads a key/value head

Triple = Tuple[torch.Tensor, torch.Tensor, torch.Tensor]


def quantize(x: torch.Tensor) -> Triple:
    """mx.quantize(x, group_size=64, bits=8) of keys or values (..., D): (words uint32 carried as int32
    (..., D/4), scales, biases (..., D/64)) in x's dtype."""
    shape, D = x.shape[:-1], x.shape[-1]
    wq, s, b = kernels.quantize(x.reshape(-1, D).contiguous(), group_size=GROUP, bits=BITS)
    return wq.reshape(*shape, D * BITS // 32), s.reshape(*shape, D // GROUP), b.reshape(*shape, D // GROUP)


def dequantized(t: Triple) -> torch.Tensor:
    """mx.dequantize of a (words, scales, biases) triple (qkv.py:252-253)."""
    wq, s, b = t
    D = wq.shape[-1] * 32 // BITS
    out = kernels.dequantize(wq.reshape(-1, wq.shape[-1]).contiguous(), s.reshape(-1, s.shape[-1]).contiguous(),
                             b.reshape(-1, b.shape[-1]).contiguous(), group_size=GROUP, bits=BITS)
    return out.reshape(*wq.shape[:-1], D)


def supported(H: int, KVH: int, head_dim: int) -> bool:
    return head_dim == HEAD_DIM and KVH >= 1 and H % KVH == 0 and 1 <= H // KVH <= MAX_GROUP


def attend(q: torch.Tensor, keys: Sequence[torch.Tensor], values: Sequence[torch.Tensor], n: int,
           sinks: Optional[torch.Tensor], scale: float, start: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One query a row against 8-bit keys and values: ``q`` (B, H, 1, 128); ``keys`` / ``values`` a cache's whole
    buffers (words (B, KVH, cap, 32), scales, biases (B, KVH, cap, 2)), of which positions ``start[b]`` .. ``n``-1
    are row b's; ``sinks`` (H,) logits (or None). Returns (B, H, 1, 128) in q's dtype."""
    B, H, L, HD = q.shape
    if L != 1:
        raise ValueError("attend takes one query a row (decode)")
    kq, ks, kb = keys
    vq, vs, vb = values
    KVH, cap = kq.shape[1], kq.shape[2]
    if not supported(H, KVH, HD):
        raise ValueError(f"attend: H={H}, KVH={KVH}, head_dim={HD} not supported")
    for t in (ks, kb, vs, vb):
        if t.dtype != q.dtype:
            raise TypeError("scales and biases must have the queries' dtype")
    if kq.shape != (B, KVH, cap, HD // 4) or vq.shape != kq.shape or ks.shape != (B, KVH, cap, HD // GROUP):
        raise ValueError("keys / values are not (B, KVH, cap, ...) 8-bit triples of q's rows")
    q2 = q.contiguous()
    _check_cuda(q2, kq, ks, kb, vq, vs, vb)
    st = None
    if start is not None:
        st = start.to(device=q.device, dtype=torch.int32).contiguous()
    sk = None
    if sinks is not None:
        sk = sinks.to(device=q.device, dtype=torch.float32).contiguous()
    nbytes = int(lib().lq_kv_attend_workspace(B, H, KVH, int(n)))
    ws = torch.empty(nbytes, dtype=torch.uint8, device=q.device) if nbytes else None
    out = torch.empty((B, H, 1, HD), dtype=q.dtype, device=q.device)
    call("lq_kv_attend", q2.data_ptr(), kq.data_ptr(), ks.data_ptr(), kb.data_ptr(), vq.data_ptr(), vs.data_ptr(),
         vb.data_ptr(), None if st is None else st.data_ptr(), int(n), None if sk is None else sk.data_ptr(),
         float(scale), B, H, KVH, cap, HD, dtype_code(q.dtype), None if ws is None else ws.data_ptr(), nbytes,
         out.data_ptr(), _stream())
    return out


def _zeros(B: int, H: int, n: int, D: int, dtype: torch.dtype, device) -> Triple:
    return (torch.zeros((B, H, n, D * BITS // 32), dtype=torch.int32, device=device),
            torch.zeros((B, H, n, D // GROUP), dtype=dtype, device=device),
            torch.zeros((B, H, n, D // GROUP), dtype=dtype, device=device))


class QuantizedKVCache8:
    """The reference's BatchQuantizedKVCache buffers (left-padded rows, one buffer index ``_idx``) with keys and
    values as 8-bit (words, scales, biases) triples (qkv.py:295-326)."""

    step = 256
    bits, group_size = BITS, GROUP

    def __init__(self, left_padding: Optional[Sequence[int]] = None):
        self.keys: Optional[Triple] = None
        self.values: Optional[Triple] = None
        self._pad = list(left_padding) if left_padding is not None else None
        self.left_padding: Optional[torch.Tensor] = None
        self._idx = 0

    def update_and_fetch(self, keys: torch.Tensor, values: torch.Tensor):
        """Store keys / values (B, KVH, S, D) at positions _idx .. _idx+S-1 (growing the buffers by a multiple of
        256 positions when full, as qkv.py:309-319) and return the valid part of the buffers."""
        prev, S = self._idx, keys.shape[2]
        if self.keys is None or prev + S > self.keys[0].shape[2]:
            B, H, _, D = keys.shape
            n = (self.step + S - 1) // self.step * self.step
            nk = _zeros(B, H, n, D, keys.dtype, keys.device)
            nv = _zeros(B, H, n, values.shape[3], values.dtype, values.device)
            if self.keys is None:
                self.keys, self.values = nk, nv
            else:
                self.keys = tuple(torch.cat([a[..., :prev, :], z], dim=2) for a, z in zip(self.keys, nk))
                self.values = tuple(torch.cat([a[..., :prev, :], z], dim=2) for a, z in zip(self.values, nv))
            if self.left_padding is None and self._pad is not None:
                self.left_padding = torch.tensor(self._pad, dtype=torch.int32, device=keys.device)
        self._idx += S
        for buf, new in ((self.keys, quantize(keys)), (self.values, quantize(values))):
            for a, x in zip(buf, new):
                a[..., prev:self._idx, :] = x
        return self.keys_and_values()

    def keys_and_values(self):
        return (tuple(a[..., :self._idx, :] for a in self.keys), tuple(a[..., :self._idx, :] for a in self.values))

    def attend(self, q: torch.Tensor, scale: float, sinks: Optional[torch.Tensor] = None) -> torch.Tensor:
        """One decode step's attention over the whole cache (qkv.attention's one-query branch, qkv.py:262-269)."""
        return attend(q, self.keys, self.values, self._idx, sinks, scale, self.left_padding)
