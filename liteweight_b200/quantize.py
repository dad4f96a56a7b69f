"""liteweight's weight format: RTN symmetric group-wise INT8 / packed INT4.

Same functions and results as liteweight/quantize.py (the format is the
drop-in contract, so the arithmetic is necessarily the same):

* quantize: per group of ``group_size`` consecutive K elements, scale =
  absmax / 127 (INT8) or / 7 (INT4) in fp32, clamped to >= 1e-8; codes =
  round-half-even(w / scale) clipped to [-127, 127] / [-8, 7]; the scale is
  stored as fp16 (quantize.py:7-27, :65-99).
* INT4 packing: even K -> low nibble, odd K -> high nibble, two's
  complement (quantize.py:90-97).
* dequantize: fp16(float(code) * float(scale)) (quantize.py:30-43, :102-128).
  On CUDA tensors it runs the library's bit-exact dequant kernel.

These run wherever the tensors are (quantization happens on CPU when an HF
model is converted there); none of them is on the matmul hot path. CUDA
tensors go through the library's kernels (lw_quantize_*, lw_dequant_*), which
give the same bits.
"""

from __future__ import annotations

import torch
from torch import Tensor

from liteweight_b200 import _native as nat


def _rtn(weight: Tensor, group_size: int, qmax: float, lo: int, hi: int) -> tuple[Tensor, Tensor]:
    assert weight.ndim == 2, "weight must be [N, K]"
    n, k = weight.shape
    assert k % group_size == 0, f"K={k} must be divisible by group_size={group_size}"
    w = weight.float().reshape(n, k // group_size, group_size)
    scale = (w.abs().amax(dim=-1, keepdim=True) / qmax).clamp(min=1e-8)
    q = torch.round(w / scale).clamp(lo, hi).to(torch.int8).reshape(n, k)
    return q, scale.reshape(n, k // group_size).half()


def _quant_cuda(fn: str, weight: Tensor, group_size: int, packed: bool) -> tuple[Tensor, Tensor]:
    assert weight.ndim == 2, "weight must be [N, K]"
    n, k = weight.shape
    assert k % group_size == 0, f"K={k} must be divisible by group_size={group_size}"
    if weight.dtype not in (torch.float16, torch.float32):
        weight = weight.float()
    weight = weight.contiguous()
    q = torch.empty((n, k // 2) if packed else (n, k), dtype=torch.uint8 if packed else torch.int8,
                    device=weight.device)
    s = torch.empty((n, k // group_size), dtype=torch.float16, device=weight.device)
    nat.call(fn, weight.data_ptr(), int(weight.dtype == torch.float32), q.data_ptr(), s.data_ptr(), n, k,
             group_size, nat.stream_of(weight))
    return q, s


def quantize_int8(weight: Tensor, group_size: int = 128) -> tuple[Tensor, Tensor]:
    """fp16/fp32 [N, K] -> (int8 [N, K], fp16 scales [N, K // group_size])."""
    if weight.is_cuda:
        return _quant_cuda("lw_quantize_int8", weight, group_size, False)
    return _rtn(weight, group_size, 127.0, -127, 127)


def pack_int4(q: Tensor) -> Tensor:
    """int8 codes in [-8, 7], [N, K] -> uint8 [N, K // 2] (even K in the low nibble)."""
    lo = q[:, 0::2].to(torch.uint8) & 0x0F
    hi = (q[:, 1::2].to(torch.uint8) & 0x0F) << 4
    return (lo | hi).to(torch.uint8)


def unpack_int4(qweight: Tensor) -> Tensor:
    """uint8 [N, K // 2] -> int8 codes [N, K] (4-bit sign extension)."""
    lo = (qweight & 0x0F).to(torch.int8)
    hi = (qweight >> 4).to(torch.int8)
    lo = torch.where(lo >= 8, lo - 16, lo)
    hi = torch.where(hi >= 8, hi - 16, hi)
    return torch.stack([lo, hi], dim=-1).reshape(qweight.shape[0], qweight.shape[1] * 2)


def quantize_int4(weight: Tensor, group_size: int = 128) -> tuple[Tensor, Tensor]:
    """fp16/fp32 [N, K] -> (uint8 packed [N, K // 2], fp16 scales [N, K // group_size])."""
    assert weight.ndim == 2, "weight must be [N, K]"
    assert weight.shape[1] % 2 == 0
    if weight.is_cuda:
        return _quant_cuda("lw_quantize_int4", weight, group_size, True)
    q, s = _rtn(weight, group_size, 7.0, -8, 7)
    return pack_int4(q), s


def _dequant_cuda(fn: str, qweight: Tensor, scales: Tensor, n: int, k: int, group_size: int) -> Tensor:
    qweight, scales = qweight.contiguous(), scales.contiguous()
    out = torch.empty((n, k), dtype=torch.float16, device=qweight.device)
    nat.call(fn, qweight.data_ptr(), scales.data_ptr(), out.data_ptr(), n, k, group_size, nat.stream_of(out))
    return out


def dequantize_int8(qweight: Tensor, scales: Tensor, group_size: int = 128) -> Tensor:
    """int8 [N, K] + fp16 [N, K // G] -> fp16 [N, K]."""
    n, k = qweight.shape
    if qweight.is_cuda:
        return _dequant_cuda("lw_dequant_w8", qweight, scales, n, k, group_size)
    w = qweight.float().reshape(n, k // group_size, group_size)
    s = scales.float().reshape(n, k // group_size, 1)
    return (w * s).reshape(n, k).half()


def dequantize_int4(qweight: Tensor, scales: Tensor, group_size: int = 128) -> Tensor:
    """uint8 [N, K // 2] + fp16 [N, K // G] -> fp16 [N, K]."""
    n, kh = qweight.shape
    k = kh * 2
    if qweight.is_cuda:
        return _dequant_cuda("lw_dequant_w4", qweight, scales, n, k, group_size)
    w = unpack_int4(qweight).float().reshape(n, k // group_size, group_size)
    s = scales.float().reshape(n, k // group_size, 1)
    return (w * s).reshape(n, k).half()


def fakequant_matmul(act: Tensor, weight: Tensor, group_size: int = 128) -> Tensor:
    """INT8 quantize -> dequantize -> fp32 matmul -> fp16 (quantize.py:46-60)."""
    q, s = quantize_int8(weight, group_size)
    return act.float().mm(dequantize_int8(q, s, group_size).float().T).half()


def fakequant_matmul_int4(act: Tensor, weight: Tensor, group_size: int = 128) -> Tensor:
    """INT4 variant of fakequant_matmul (quantize.py:131-135)."""
    q, s = quantize_int4(weight, group_size)
    return act.float().mm(dequantize_int4(q, s, group_size).float().T).half()
