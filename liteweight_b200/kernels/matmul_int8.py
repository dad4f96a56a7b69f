"""INT8 weight-dequant matmul (replaces kernels/matmul_int8.py:103-145).

out[m, n] = sum_k act[m, k] * (qweight[n, k] * scales[n, k // G]), fp32
accumulation over fp16-rounded dequantized weights, fp16 output.
"""

import torch

from liteweight_b200 import _native as nat


def matmul_int8(act: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor,
                group_size: int = 128) -> torch.Tensor:
    """Dequanting INT8 matmul.

    Args:
        act:      fp16 [M, K]
        qweight:  int8 [N, K]
        scales:   fp16 [N, K // group_size]
        group_size: must match how qweight was quantized

    Returns:
        fp16 [M, N]   (act @ dequant(qweight).T)
    """
    # kernels/matmul_int8.py:120-131
    assert act.dtype == torch.float16
    assert qweight.dtype == torch.int8
    assert scales.dtype == torch.float16
    act = act.contiguous()
    qweight = qweight.contiguous()
    scales = scales.contiguous()
    M, K = act.shape
    N, Kw = qweight.shape
    assert K == Kw
    assert scales.shape == (N, K // group_size)
    nat.require_cuda(act, qweight, scales)
    out = torch.empty((M, N), device=act.device, dtype=torch.float16)
    if M == 0 or N == 0:
        return out
    stream = nat.stream_of(act)
    ws, ws_bytes = nat.matmul_workspace(8, M, N, K, act.device, stream)
    nat.call("lw_gemm_w8a16", act.data_ptr(), qweight.data_ptr(), scales.data_ptr(), None, out.data_ptr(),
             M, N, K, group_size, ws, ws_bytes, stream)
    return out
