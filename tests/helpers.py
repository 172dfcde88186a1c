"""Shared helpers for the parity tests: seeded MLX-format weights made by the CPU oracle, moved to
the GPU, and the output tolerance (1e-2 of the largest reference value)."""

from __future__ import annotations

import numpy as np

from oracle import oracle as O

TOL_REL = 1e-2  # max|y - ref| <= 1e-2 * max|ref| (fp32 accumulation)


def qweights(rng, N, K, bits, dtype, std=0.02):
    w = (rng.standard_normal((N, K), dtype=np.float32) * std).astype(np.float32)
    wq, s, b = O.quantize(w, 64, bits, dtype)
    return wq, s, b


def to_torch(wq, s, b, dtype, device):
    import torch

    tdt = torch.bfloat16 if dtype == "bfloat16" else torch.float16
    return (torch.from_numpy(wq.view(np.int32).copy()).to(device), torch.from_numpy(s).to(device=device, dtype=tdt),
            torch.from_numpy(b).to(device=device, dtype=tdt))


def act(rng, M, K, dtype):
    return O.round_to(rng.standard_normal((M, K), dtype=np.float32), dtype)


def x_torch(x, dtype, device):
    import torch

    tdt = torch.bfloat16 if dtype == "bfloat16" else torch.float16
    return torch.from_numpy(x).to(device=device, dtype=tdt)


def rel_err(got, ref):
    got = np.asarray(got, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    return float(np.max(np.abs(got - ref)) / max(float(np.max(np.abs(ref))), 1e-30))
