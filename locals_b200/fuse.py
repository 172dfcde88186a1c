"""Projection fusion for MLX affine weights (the counterpart of the reference's locals/fuse.py:22-199).

Quantization groups run along the input dimension, so stacking quantized matrices along the output
dimension keeps the format exact (locals/fuse.py:3-6). ``concat_quantized`` builds the stacked
tensors (locals/fuse.py:28-46); ``FusedQKV`` is the q/k/v projection with its output written straight
into separate q, k, v tensors in head layout (FusedAttention's reshape + split, locals/fuse.py:49-54);
``FusedMLP`` is down(swiglu(gate_up(x))) (locals/fuse.py:160-164) with the gate/up matmul and the
SwiGLU in one kernel.
"""

from __future__ import annotations

from typing import Sequence, Tuple

import torch

from . import kernels
from .kernels import QuantizedLinear


def fusable(mods: Sequence[QuantizedLinear]) -> bool:
    """Same bits and group size, and a bias on all or none (locals/fuse.py:22-25)."""
    return len({(m.bits, m.group_size) for m in mods}) == 1 and len({m.bias is None for m in mods}) == 1


def concat_quantized(mods: Sequence[QuantizedLinear]) -> QuantizedLinear:
    if not fusable(mods):
        raise ValueError("projections with different quantization or biases do not fuse")
    first = mods[0]
    w = torch.cat([m.weight for m in mods], 0)
    s = torch.cat([m.scales for m in mods], 0)
    b = torch.cat([m.biases for m in mods], 0)
    bias = torch.cat([m.bias for m in mods], 0) if first.bias is not None else None
    return QuantizedLinear(w, s, b, first.bits, first.group_size, bias)


class FusedQKV:
    """q, k, v = one quantized matmul over the stacked [Wq; Wk; Wv], output (M, H, D), (M, KVH, D) x 2."""

    def __init__(self, q: QuantizedLinear, k: QuantizedLinear, v: QuantizedLinear, n_heads: int, n_kv_heads: int,
                 head_dim: int):
        self.qkv = concat_quantized([q, k, v])
        self.n_heads, self.n_kv_heads, self.head_dim = n_heads, n_kv_heads, head_dim
        self.widths = (n_heads * head_dim, n_kv_heads * head_dim, n_kv_heads * head_dim)
        self.choice = None

    def __call__(self, x: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        m = self.qkv
        q, k, v = kernels.qmm_split(x, m.weight, m.scales, m.biases, self.widths, m.group_size, m.bits,
                                    choice=self.choice)
        lead = x.shape[:-1]
        return (q.view(*lead, self.n_heads, self.head_dim), k.view(*lead, self.n_kv_heads, self.head_dim),
                v.view(*lead, self.n_kv_heads, self.head_dim))


class FusedMLP:
    """down(swiglu(gate(x), up(x))) with gate||up stacked (locals/fuse.py:195-199) and the SwiGLU fused
    into the gate/up kernel's epilogue."""

    def __init__(self, gate: QuantizedLinear, up: QuantizedLinear, down: QuantizedLinear):
        self.gate_up = concat_quantized([gate, up])
        self.hidden = gate.out_features
        self.down = down
        self.choice_up = None
        self.choice_down = None

    def gate_up_views(self):
        m, I = self.gate_up, self.hidden
        return (m.weight[:I], m.scales[:I], m.biases[:I]), (m.weight[I:], m.scales[I:], m.biases[I:])

    def hidden_act(self, x: torch.Tensor) -> torch.Tensor:
        g, u = self.gate_up_views()
        return kernels.qmm_glu(x, g, u, self.gate_up.group_size, self.gate_up.bits, choice=self.choice_up)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        h = self.hidden_act(x)
        d = self.down
        return kernels.quantized_matmul(h, d.weight, d.scales, d.biases, group_size=d.group_size, bits=d.bits,
                                        choice=self.choice_down)
