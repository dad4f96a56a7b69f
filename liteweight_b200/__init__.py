"""liteweight_b200: B200-native (sm_100a) weight-only quantized inference.

A drop-in for liteweight's API (liteweight/__init__.py:1-17): the same
quantization format and functions, QuantLinear, swap_linears /
save_quantized / load_quantized and generate / KVCache, with the matmul hot
path and the decode step running hand-written CUDA kernels for B200.
"""

from liteweight_b200.perf import B200, DeviceSpec
from liteweight_b200.quantize import (dequantize_int4, dequantize_int8, fakequant_matmul, fakequant_matmul_int4,
                                      quantize_int4, quantize_int8)
from liteweight_b200.quantlinear import QuantLinear
from liteweight_b200.serialize import load_quantized, save_quantized, swap_linears
from liteweight_b200.generate import KVCache, generate

__all__ = [
    "DeviceSpec", "B200",
    "quantize_int8", "dequantize_int8", "fakequant_matmul",
    "quantize_int4", "dequantize_int4", "fakequant_matmul_int4",
    "QuantLinear",
    "swap_linears", "save_quantized", "load_quantized",
    "generate", "KVCache",
]
