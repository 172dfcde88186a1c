"""locals_b200: the MLX affine group-quantized matmul path of Generated-Computers/Locals, rebuilt for
NVIDIA B200 (sm_100a) as hand-written CUDA kernels behind a C ABI (include/lq.h, liblq.so).

Public surface (names follow the reference):
  kernels.quantize / dequantize / quantized_matmul / launch / QuantizedLinear   (locals/kernels.py)
  fuse.concat_quantized / FusedQKV / FusedMLP                                  (locals/fuse.py)
  moe.router_logits / route_topk / group / switch_glu / MoELayer               (locals/moe.py, moe_kernel.py)
  tune.choose / lookup                                                         (locals/kernels.py tuner)
  shard.ColumnShardedLinear / ExpertParallelMoE                                (multi-GPU, NCCL)
"""

from . import _lib  # noqa: F401
from .kernels import QuantizedLinear, dequantize, launch, quantize, quantized_matmul  # noqa: F401

__all__ = ["QuantizedLinear", "dequantize", "launch", "quantize", "quantized_matmul"]
