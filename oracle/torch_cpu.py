"""torch (CPU) restatement of liteweight's dequantize-then-matmul path.

Test infrastructure only (see ``oracle/__init__.py``); used as the timed CPU
baseline (``bench.py --impl reference`` and the ``cpu_baseline`` leg).

liteweight's ``QuantLinear`` cannot run its Triton kernel on a CPU, so the
reference's CPU path for this hot path is its correctness oracle applied to
the stored packed weights: ``dequantize_int8`` / ``dequantize_int4``
(liteweight/quantize.py:30-43, :102-128) followed by
``act.float().mm(w_dq.float().T).half()`` (liteweight/quantize.py:60, :135).
These functions restate that arithmetic with torch tensor ops, so the CPU
work (elementwise unpack passes, an fp32 copy of the weight, one BLAS fp32
GEMM) is the same kind and size as the reference's; the numpy oracle
(``oracle/quant.py``) is the bit-level statement the tests pin, and
``tests/test_oracle_golden.py`` checks these functions against it.
"""

from __future__ import annotations

import torch


def dequantize_int8(qweight: torch.Tensor, scales: torch.Tensor, group_size: int) -> torch.Tensor:
    """liteweight/quantize.py:30-43: fp16 of the fp32 product code * scale, per group."""
    n, k = qweight.shape
    codes = qweight.to(torch.float32).view(n, k // group_size, group_size)
    return (codes * scales.to(torch.float32).unsqueeze(-1)).view(n, k).to(torch.float16)


def dequantize_int4(qweight: torch.Tensor, scales: torch.Tensor, group_size: int) -> torch.Tensor:
    """liteweight/quantize.py:102-128: low nibble = even k, high nibble = odd k,
    4-bit two's complement, then the same fp32 product rounded to fp16."""
    n, kh = qweight.shape
    k = 2 * kh
    b = qweight.view(torch.int8)                     # the same bytes as signed: arithmetic shifts sign-extend
    codes = torch.stack(((b << 4) >> 4, b >> 4), dim=-1).view(n, k)   # [..., 2p] = low, [..., 2p+1] = high
    codes = codes.to(torch.float32).view(n, k // group_size, group_size)
    return (codes * scales.to(torch.float32).unsqueeze(-1)).view(n, k).to(torch.float16)


def quant_linear(act: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor, group_size: int,
                 bits: int) -> torch.Tensor:
    """One QuantLinear call on the CPU: dequantize, fp32 matmul, fp16 result
    (liteweight/quantize.py:60)."""
    w = (dequantize_int4 if bits == 4 else dequantize_int8)(qweight, scales, group_size)
    return act.to(torch.float32).mm(w.to(torch.float32).t()).to(torch.float16)


def fp16_linear(act: torch.Tensor, weight: torch.Tensor) -> torch.Tensor:
    """The fp16 lm_head through the same fp32-accumulating matmul."""
    return act.to(torch.float32).mm(weight.to(torch.float32).t()).to(torch.float16)
