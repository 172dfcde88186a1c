"""The residual add and RMS norm between a decoder layer's projections (the counterpart of the reference's
locals/norm_kernel.py): ``add_rms(x, r, w, eps) -> (h, n)`` with h = x + r and n = rms_norm(h) * w, one
sm_100a kernel (``lq_add_rms_norm``), h rounded to the activation dtype and the sum of squares in fp32 as
the reference's kernel (norm_kernel.py:16-85)."""

from __future__ import annotations

import torch

from ._lib import call
from .kernels import _check_cuda, _stream, dtype_code

MAX_D = 8192


def supported(D: int) -> bool:
    """Rows of D values with D % 8 == 0 (16-byte vectors), D <= 8192 (norm_kernel.supported: D % 128, <= 4096)."""
    return D % 8 == 0 and 8 <= D <= MAX_D


def add_rms(x: torch.Tensor, r: torch.Tensor, w: torch.Tensor, eps: float) -> tuple:
    """(h, n) for x, r of shape (..., D) and w of shape (D,)."""
    D = x.shape[-1]
    x2 = x.reshape(-1, D).contiguous()
    r2 = r.reshape(-1, D).contiguous()
    _check_cuda(x2, r2, w)
    if not supported(D):
        raise ValueError(f"add_rms: D={D} not supported")
    h = torch.empty_like(x2)
    n = torch.empty_like(x2)
    call("lq_add_rms_norm", x2.data_ptr(), r2.data_ptr(), w.data_ptr(), h.data_ptr(), n.data_ptr(), x2.shape[0], D,
         float(eps), dtype_code(x.dtype), _stream())
    return h.reshape(x.shape), n.reshape(x.shape)
