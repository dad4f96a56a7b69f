"""QuantLinear: nn.Linear drop-in whose forward runs the sm_100a dequant GEMV/GEMM.

Same constructor, buffers (names, dtypes, shapes), ``forward`` contract and
``from_linear`` as liteweight/quantlinear.py:16-94, so ``state_dict`` and the
safetensors layout of liteweight/serialize.py are unchanged:

    qweight  int8 [out, in]          (bits=8)   or uint8 [out, in // 2] (bits=4)
    scales   fp16 [out, in // group_size]
    bias     fp16 [out] or None

fp16 in / fp16 out; the bias add (quantlinear.py:63-64) is fused into the
kernel epilogue with the same rounding (fp16 result, then fp16 add).
"""

from __future__ import annotations

import torch
import torch.nn as nn
from torch import Tensor

from liteweight_b200 import _native as nat
from liteweight_b200.quantize import quantize_int4, quantize_int8


class QuantLinear(nn.Module):
    def __init__(self, in_features: int, out_features: int, group_size: int = 128, bias: bool = False,
                 bits: int = 8):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.group_size = group_size
        self.bits = bits
        assert bits in (4, 8), f"bits must be 4 or 8, got {bits}"
        assert in_features % group_size == 0
        if bits == 8:
            self.register_buffer("qweight", torch.zeros(out_features, in_features, dtype=torch.int8))
        else:
            self.register_buffer("qweight", torch.zeros(out_features, in_features // 2, dtype=torch.uint8))
        self.register_buffer("scales",
                             torch.zeros(out_features, in_features // group_size, dtype=torch.float16))
        if bias:
            self.register_buffer("bias", torch.zeros(out_features, dtype=torch.float16))
        else:
            self.register_buffer("bias", None)

    def forward(self, x: Tensor) -> Tensor:
        orig_shape = x.shape
        x = x.reshape(-1, self.in_features).to(torch.float16).contiguous()
        nat.require_cuda(x, self.qweight)
        m = x.shape[0]
        out = torch.empty((m, self.out_features), dtype=torch.float16, device=x.device)
        if m:
            fn = "lw_gemm_w8a16" if self.bits == 8 else "lw_gemm_w4a16"
            stream = nat.stream_of(x)
            ws, ws_bytes = nat.matmul_workspace(self.bits, m, self.out_features, self.in_features, x.device, stream)
            nat.call(fn, x.data_ptr(), self.qweight.data_ptr(), self.scales.data_ptr(), nat.ptr(self.bias),
                     out.data_ptr(), m, self.out_features, self.in_features, self.group_size, ws, ws_bytes, stream)
        return out.reshape(*orig_shape[:-1], self.out_features)

    @classmethod
    def from_linear(cls, linear: nn.Linear, group_size: int = 128, bits: int = 8) -> "QuantLinear":
        ql = cls(linear.in_features, linear.out_features, group_size=group_size,
                 bias=linear.bias is not None, bits=bits)
        w = linear.weight.data.float().half()
        q, s = (quantize_int8 if bits == 8 else quantize_int4)(w, group_size)
        ql = ql.to(w.device)
        ql.qweight.copy_(q)
        ql.scales.copy_(s)
        if linear.bias is not None:
            ql.bias.copy_(linear.bias.data.half())
        return ql

    def extra_repr(self) -> str:
        return f"in={self.in_features}, out={self.out_features}, bits={self.bits}, group_size={self.group_size}"
