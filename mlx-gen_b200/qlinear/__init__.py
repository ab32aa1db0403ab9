"""qlinear -- host API of the B200 group-wise affine Q4/Q8 quantized-linear path.

Mirrors the reference's operator and module surface (mlx-rs ``ops::quantize /
dequantize / quantized_matmul``; ``AdaptableLinear``, ``Adapter``, ``TokenEmbedding``;
``quant::{lin, embedding, quantize_map, DEFAULT_GROUP_SIZE}``) on top of the C ABI in
include/qlinear.h.  All arithmetic runs in libqlinear.so (CUDA, sm_100a).
"""
from ._lib import (ACT_GELU_ERF, ACT_GELU_TANH, ACT_NONE, ACT_SWIGLU, KERNEL_AUTO, KERNEL_GEMM, KERNEL_GEMM_PAIR,
                   KERNEL_GEMV, KERNEL_GEMV_REGS, KERNEL_GEMV_TC, KERNEL_GEMV_TMA, KERNEL_GENERIC, QlError,
                   device_error)
from .nn import (DEFAULT_GROUP_SIZE, AdaptableLinear, Linear, Lokr, Lora, QuantizedLinear,
                 TokenEmbedding)
from .ops import dequantize, dequantize_rows, layernorm_modulate, quantize, quantized_matmul, workspace_size
from .quant import PackedShapeError, embedding, lin, packed_bits, quantize_map
from .adapters import reconstruct_loha_delta, reconstruct_lokr_delta, reconstruct_lokr_delta_scaled

__all__ = [
    "ACT_GELU_ERF", "ACT_GELU_TANH", "ACT_NONE", "ACT_SWIGLU", "KERNEL_AUTO", "KERNEL_GEMM", "KERNEL_GEMM_PAIR",
    "KERNEL_GEMV", "KERNEL_GEMV_REGS", "KERNEL_GEMV_TC", "KERNEL_GEMV_TMA", "KERNEL_GENERIC", "QlError", "device_error", "DEFAULT_GROUP_SIZE",
    "AdaptableLinear", "Linear", "Lokr", "Lora", "QuantizedLinear", "TokenEmbedding", "dequantize",
    "dequantize_rows", "layernorm_modulate", "quantize", "quantized_matmul", "workspace_size", "embedding", "lin",
    "packed_bits", "PackedShapeError", "quantize_map", "reconstruct_lokr_delta", "reconstruct_lokr_delta_scaled",
    "reconstruct_loha_delta",
]
