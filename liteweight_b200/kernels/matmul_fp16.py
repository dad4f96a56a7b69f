"""FP16 matmul (replaces kernels/matmul_fp16.py:67-85): a [M,K] @ b [K,N] -> [M,N].

When ``b`` is the transpose of a contiguous [N, K] weight (``W.T``, how the
reference's benchmarks call it, bench/benchmark.py:133) the weight is read in
place through the nn.Linear-layout kernel - no transposed copy is made.
"""

import torch

from liteweight_b200 import _native as nat


def matmul_fp16(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """a [M, K] fp16 @ b [K, N] fp16 -> [M, N] fp16 (fp32 accumulate)."""
    assert a.dtype == torch.float16 and b.dtype == torch.float16
    a = a.contiguous()
    M, K = a.shape
    Kb, N = b.shape
    assert K == Kb
    nat.require_cuda(a, b)
    c = torch.empty((M, N), device=a.device, dtype=torch.float16)
    if M == 0 or N == 0:
        return c
    s = nat.stream_of(a)
    if b.t().is_contiguous():
        # b = w.T with w [N, K] contiguous
        ws, ws_bytes = nat.matmul_workspace(16, M, N, K, a.device, s)
        nat.call("lw_gemm_f16", a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K, ws, ws_bytes, s)
    else:
        b = b.contiguous()
        nat.call("lw_gemm_f16_kn", a.data_ptr(), b.data_ptr(), c.data_ptr(), M, N, K, s)
    return c
