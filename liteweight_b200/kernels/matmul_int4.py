"""INT4 weight-dequant matmul (replaces kernels/matmul_int4.py:122-165).

qweight is packed uint8 [N, K//2]: low nibble = element at even K, high
nibble = odd K, 4-bit two's complement in [-8, 7].
"""

import torch

from liteweight_b200 import _native as nat


def matmul_int4(act: torch.Tensor, qweight: torch.Tensor, scales: torch.Tensor,
                group_size: int = 128) -> torch.Tensor:
    """Dequanting INT4 matmul.

    Args:
        act:      fp16 [M, K]
        qweight:  uint8 [N, K // 2]  (nibble-packed)
        scales:   fp16  [N, K // group_size]

    Returns:
        fp16 [M, N]
    """
    # kernels/matmul_int4.py:138-149
    assert act.dtype == torch.float16
    assert qweight.dtype == torch.uint8
    assert scales.dtype == torch.float16
    act = act.contiguous()
    qweight = qweight.contiguous()
    scales = scales.contiguous()
    M, K = act.shape
    N, K_half = qweight.shape
    assert K == K_half * 2
    assert scales.shape == (N, K // group_size)
    nat.require_cuda(act, qweight, scales)
    out = torch.empty((M, N), device=act.device, dtype=torch.float16)
    if M == 0 or N == 0:
        return out
    stream = nat.stream_of(act)
    ws, ws_bytes = nat.matmul_workspace(4, M, N, K, act.device, stream)
    nat.call("lw_gemm_w4a16", act.data_ptr(), qweight.data_ptr(), scales.data_ptr(), None, out.data_ptr(),
             M, N, K, group_size, ws, ws_bytes, stream)
    return out
