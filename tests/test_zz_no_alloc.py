"""lw_gemm_w4a16_noalloc: the INT4 matmul for callers that cannot allocate (GPU).

Some callers of this library cannot allocate device memory - a serving
runtime that plans all of its device memory at start-up, a plugin host that
forbids cudaMalloc after initialisation - so they cannot hand lw_gemm_w4a16
the scratch it uses to combine weight tiles split between warps. The
no-allocation entry point keeps that scratch in a fixed array inside the
library. This test calls it through the C ABI twice in a row, on a shape whose
tiles are split (so the array is used), and checks each result against the
regular entry point given a torch-allocated workspace: both run the same plan
and kernel, so the outputs must be bit-identical; one comparison against the
oracle (dequantize, fp32 matmul) within the row-scaled tolerance of the other
kernel tests guards both. It also checks that a problem needing more scratch
than the array holds is rejected, and that a bad group size is rejected
before anything is enqueued.

The file is named to be collected last, so a run that stops at the first
failure has run every other test before this one.
"""

import numpy as np
import pytest
import torch

from oracle import quant as oq

pytestmark = pytest.mark.gpu
DEV = "cuda"
SCRATCH_BYTES = 4 << 20


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from liteweight_b200 import _native as nat
    from liteweight_b200 import build
    build.build()
    return nat


def _quantized(N, K, seed):
    g = np.random.default_rng(seed)
    return oq.quantize_int4((g.standard_normal((N, K)) * 0.02).astype(np.float16), 128)


def test_noalloc_matches_regular_entry_point_twice(lib):
    M, N, K = 3, 512, 8192
    need = int(lib.lib().lw_gemm_workspace_size(4, M, N, K))
    assert 0 < need <= SCRATCH_BYTES, need        # the split-tile scratch is really used
    q, s = _quantized(N, K, seed=5)
    qt, st = torch.from_numpy(q).to(DEV), torch.from_numpy(s).to(DEV)
    ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
    stream = torch.cuda.current_stream().cuda_stream
    rng = np.random.default_rng(9)
    for call in range(2):
        act = torch.from_numpy(rng.standard_normal((M, K)).astype(np.float16)).to(DEV)
        got = torch.empty(M, N, dtype=torch.float16, device=DEV)
        ref = torch.empty(M, N, dtype=torch.float16, device=DEV)
        lib.call("lw_gemm_w4a16_noalloc", act.data_ptr(), qt.data_ptr(), st.data_ptr(), None, got.data_ptr(),
                 M, N, K, 128, stream)
        lib.call("lw_gemm_w4a16", act.data_ptr(), qt.data_ptr(), st.data_ptr(), None, ref.data_ptr(),
                 M, N, K, 128, ws.data_ptr(), need, stream)
        torch.cuda.synchronize()
        g = got.float().cpu().numpy()
        assert np.isfinite(g).all(), call
        assert torch.equal(got, ref), (call, float((got.float() - ref.float()).abs().max()))
        o = oq.packed_matmul(act.cpu().numpy(), q, s, 128, 4).astype(np.float32)
        assert np.all(np.abs(g - o) <= oq.row_tolerance(o)), (call, float(np.abs(g - o).max()))


def test_noalloc_rejects_problems_beyond_its_scratch(lib):
    for M, N, K in [(32, 65536, 16384), (32, 131072, 16384), (32, 262144, 8192)]:
        need = int(lib.lib().lw_gemm_workspace_size(4, M, N, K))
        if need > SCRATCH_BYTES:
            # pointers are never touched: the size check fails before any launch
            status = lib.lib().lw_gemm_w4a16_noalloc(0x1000, 0x1000, 0x1000, None, 0x1000, M, N, K, 128,
                                                     torch.cuda.current_stream().cuda_stream)
            assert status == 7, status            # LW_ERR_WORKSPACE
            return
    pytest.skip("no candidate shape needs more scratch than the array on this device")


def test_noalloc_rejects_bad_group_before_enqueueing(lib):
    # K % group_size != 0: rejected with LW_ERR_BAD_GROUP; pointers are never touched
    status = lib.lib().lw_gemm_w4a16_noalloc(0x1000, 0x1000, 0x1000, None, 0x1000, 1, 512, 8192, 96,
                                             torch.cuda.current_stream().cuda_stream)
    assert status == 3, status                    # LW_ERR_BAD_GROUP
