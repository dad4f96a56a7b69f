"""lw_prefill_gemm: the prompt-chunk GEMM on the tensor cores (tcgen05).

Checked against a torch fp32 reference of the same arithmetic (dequantize
exactly to fp16, fp32 sums, the epilogue's fp16 rounding points), within the
row-scaled tolerance, for INT4 and INT8, M from 1 to 256 (ragged, padded to
16 inside), several group sizes, K in one CTA per tile or sliced over a
cluster of 2 / 4 CTAs (summed over distributed shared memory), and each
epilogue (residual add, SwiGLU, RoPE + KV-cache append). lw_rmsnorm_rows against the oracle's RMSNorm.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import llama as ol
from oracle import quant as oq

pytestmark = pytest.mark.gpu
DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from liteweight_b200 import build
    build.build()


def _weights(bits, N, K, G, seed):
    rng = np.random.default_rng(seed)
    w = (rng.standard_normal((N, K)) * 0.05).astype(np.float16)
    q, s = (oq.quantize_int4 if bits == 4 else oq.quantize_int8)(w, G)
    deq = (oq.dequantize_int4 if bits == 4 else oq.dequantize_int8)(q, s, G)
    return torch.from_numpy(q).to(DEV), torch.from_numpy(s).to(DEV), torch.from_numpy(deq).to(DEV)


def _run(**kw):
    from liteweight_b200 import _native as nat
    from liteweight_b200 import engine as E
    a = E.PrefillGemmArgs(pdl=1)
    keep = []
    for k, v in kw.items():
        if isinstance(v, torch.Tensor):
            keep.append(v)
            v = v.data_ptr()
        setattr(a, k, v)
    nat.check("lw_prefill_gemm", nat.lib().lw_prefill_gemm(ctypes.byref(a), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    assert int(nat.lib().lw_take_device_error()) == 0


def _close(got, ref):
    g = got.float().cpu().numpy().astype(np.float64)
    r = ref.float().cpu().numpy().astype(np.float64)
    tol = oq.row_tolerance(r)
    err = np.abs(g - r)
    assert np.all(err <= tol), float((err / tol).max())


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M,N,K,G", [(1, 128, 64, 64), (5, 256, 256, 128), (16, 128, 512, 32), (37, 384, 192, 64),
                                     (128, 256, 1024, 128), (256, 128, 256, 256),
                                     (64, 512, 4096, 128), (200, 128, 2048, 64), (33, 256, 1088, 64),
                                     # long K (>= 128 blocks of 64): sliced over a 2-CTA cluster
                                     (64, 128, 8192, 128)])
@pytest.mark.parametrize("residual", [False, True])
def test_gemm_residual(bits, M, N, K, G, residual):
    q, s, deq = _weights(bits, N, K, G, seed=M + N + K)
    gen = torch.Generator(device=DEV).manual_seed(M)
    act = torch.randn(M, K, generator=gen, device=DEV).half()
    out = torch.randn(M, N, generator=gen, device=DEV).half() if residual else torch.zeros(M, N, device=DEV).half()
    res = out.clone()
    y = (act.float() @ deq.float().T).half()
    ref = (res.float() + y.float()).half() if residual else y
    _run(bits=bits, epilogue=0, M=M, N=N, K=K, group_size=G, lda=K, ldo=N, act=act, weight=q, scales=s, out=out,
         residual=out if residual else None)
    _close(out, ref)


@pytest.mark.parametrize("splits", [2, 4])
@pytest.mark.parametrize("M,N,K,G", [(64, 512, 4096, 128), (200, 128, 2048, 64), (33, 256, 1088, 64)])
def test_gemm_k_slices(M, N, K, G, splits, monkeypatch):
    """K sliced over a cluster of 2 or 4 CTAs per tile (forced: the default
    slices only rows of >= 128 blocks of 64), ragged slices, partial tiles
    summed over distributed shared memory."""
    monkeypatch.setenv("LW_B200_TC_SPLITS", str(splits))
    for bits in (4, 8):
        q, s, deq = _weights(bits, N, K, G, seed=M + N + K + splits)
        gen = torch.Generator(device=DEV).manual_seed(M + splits)
        act = torch.randn(M, K, generator=gen, device=DEV).half()
        out = torch.randn(M, N, generator=gen, device=DEV).half()
        ref = (out.float() + (act.float() @ deq.float().T).half().float()).half()
        _run(bits=bits, epilogue=0, M=M, N=N, K=K, group_size=G, lda=K, ldo=N, act=act, weight=q, scales=s,
             out=out, residual=out)
        _close(out, ref)


@pytest.mark.parametrize("bits", [16, 4])
@pytest.mark.parametrize("M", [1, 40, 64])
def test_gemm_argmax(bits, M):
    """LW_TC_EPI_ARGMAX (the lm_head of a large decode batch): fp16 logits
    within the row tolerance of an fp32 reference, and per row the key of the
    first maximum of those logits - the key lw_fused_gemv's argmax writes
    ((order key of the fp16 value) << 32 | ~(index + offset))."""
    N, K, G, offset = 1024, 512, 128, 3000
    gen = torch.Generator(device=DEV).manual_seed(M + bits)
    act = torch.randn(M, K, generator=gen, device=DEV).half()
    if bits == 16:
        w = (torch.randn(N, K, generator=gen, device=DEV) * 0.05).half()
        q, s, deq = w, None, w
    else:
        q, s, deq = _weights(bits, N, K, G, seed=M)
    out = torch.zeros(M, N, device=DEV).half()
    keys = torch.zeros(M, dtype=torch.int64, device=DEV)
    _run(bits=bits, epilogue=4, M=M, N=N, K=K, group_size=G, lda=K, ldo=N, act=act, weight=q, scales=s, out=out,
         argmax_keys=keys, argmax_offset=offset)
    _close(out, (act.float() @ deq.float().T).half())
    idx = out.float().argmax(dim=1)          # the first maximum of the kernel's own fp16 logits
    got = (0xFFFFFFFF - (keys & 0xFFFFFFFF)) - offset
    assert torch.equal(got.cpu(), idx.cpu())


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M", [3, 64, 200])
@pytest.mark.parametrize("K", [512, 2048])
def test_gemm_swiglu(bits, M, K):
    from liteweight_b200 import engine as E
    I = 256
    q, s, deq = _weights(bits, 2 * I, K, 128, seed=M)
    gen = torch.Generator(device=DEV).manual_seed(M)
    act = torch.randn(M, K, generator=gen, device=DEV).half()
    y = (act.float() @ deq.float().T).half().float()        # rows in stored (interleaved) order
    rows = torch.arange(2 * I, device=DEV).reshape(-1, 2, 8)
    gate, up = y[:, rows[:, 0].reshape(-1)], y[:, rows[:, 1].reshape(-1)]
    silu = (gate / (1 + torch.exp(-gate))).half().float()
    ref = (silu * up).half()
    out = torch.zeros(M, I, device=DEV).half()
    _run(bits=bits, epilogue=1, M=M, N=2 * I, K=K, group_size=128, lda=K, ldo=I, act=act, weight=q, scales=s, out=out)
    _close(out, ref)
    assert E.TC_EPI_SWIGLU == 1


@pytest.mark.parametrize("M,pos0,K", [(7, 0, 256), (128, 40, 256), (50, 3, 2048)])
def test_gemm_rope_kv(M, pos0, K):
    """The q|k|v epilogue: rows stored in rope-pair order; RoPE (fp16 after
    each op, modeling_llama.py:161-162) at positions pos0 + m; q to q_out,
    k and v to the cache of sequence 1 only."""
    from liteweight_b200 import engine as E
    hd, nq, nkv, S = 64, 4, 2, 256
    N = (nq + 2 * nkv) * hd
    q, s, deq = _weights(4, N, K, 128, seed=3)
    gen = torch.Generator(device=DEV).manual_seed(9)
    act = torch.randn(M, K, generator=gen, device=DEV).half()
    cos, sin = E.rope_tables(E.default_inv_freq(hd, 500000.0), S, 1.0, DEV)
    pos = torch.tensor([pos0], dtype=torch.int32, device=DEV)
    seq = torch.tensor([1], dtype=torch.int32, device=DEV)
    qo = torch.zeros(M, nq * hd, device=DEV).half()
    kc = torch.zeros(2, nkv, S, hd, device=DEV).half()
    vc = torch.zeros_like(kc)
    _run(bits=4, epilogue=2, M=M, N=N, K=K, group_size=128, lda=K, ldo=nq * hd, act=act, weight=q, scales=s,
         out=qo, head_dim=hd, n_q_heads=nq, n_kv_heads=nkv, max_seq=S, rope_cos=cos, rope_sin=sin, pos=pos,
         seq=seq, q_out=qo, k_cache=kc, v_cache=vc)
    # reference: natural row order, then RoPE with the same rounding points
    y = (act.float() @ deq.float().T).half().float()
    perm = E.rope_pair_order(nq + 2 * nkv, hd, DEV)
    nat_rows = y[:, torch.argsort(perm)].reshape(M, nq + 2 * nkv, hd)
    c = cos[pos0:pos0 + M].float()[:, None, :]
    sn = sin[pos0:pos0 + M].float()[:, None, :]
    h = hd // 2
    rot = torch.cat([-nat_rows[..., h:], nat_rows[..., :h]], dim=-1)
    roped = ((nat_rows * c).half().float() + (rot * sn).half().float()).half()
    _close(qo.reshape(M, nq, hd).reshape(-1, hd), roped[:, :nq].reshape(-1, hd))
    kref = roped[:, nq:nq + nkv]                      # [M, nkv, hd]
    vref = nat_rows[:, nq + nkv:].half()
    _close(kc[1, :, pos0:pos0 + M].transpose(0, 1).reshape(-1, hd), kref.reshape(-1, hd))
    _close(vc[1, :, pos0:pos0 + M].transpose(0, 1).reshape(-1, hd), vref.reshape(-1, hd))
    assert torch.count_nonzero(kc[0]) == 0 and torch.count_nonzero(vc[0]) == 0
    assert torch.count_nonzero(kc[1, :, pos0 + M:]) == 0


def test_rmsnorm_rows():
    from liteweight_b200 import _native as nat
    M, K = 9, 4096
    rng = np.random.default_rng(0)
    x = rng.standard_normal((M, K)).astype(np.float16)
    gamma = (1 + 0.1 * rng.standard_normal(K)).astype(np.float16)
    h = torch.zeros(M, K, device=DEV).half()
    xt, gt = torch.from_numpy(x).to(DEV), torch.from_numpy(gamma).to(DEV)
    nat.check("norm", nat.lib().lw_rmsnorm_rows(xt.data_ptr(), gt.data_ptr(), h.data_ptr(), M, K, 1e-5, 1,
                                                torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    ref = ol.rmsnorm(x, gamma, 1e-5).astype(np.float32)
    got = h.float().cpu().numpy()
    assert np.abs(got - ref).max() <= 2e-3 * np.abs(ref).max()


def test_resid_rmsnorm_rows():
    """x = fp16(x + fp16(psum)) in place, then RMSNorm of the new x (the
    tensor-parallel prompt chunk's residual add and norm)."""
    from liteweight_b200 import _native as nat
    M, K = 7, 4096
    rng = np.random.default_rng(1)
    x = rng.standard_normal((M, K)).astype(np.float16)
    psum = rng.standard_normal((M, K)).astype(np.float32)
    gamma = (1 + 0.1 * rng.standard_normal(K)).astype(np.float16)
    xt, pt, gt = (torch.from_numpy(a).to(DEV) for a in (x, psum, gamma))
    h = torch.zeros(M, K, device=DEV).half()
    nat.check("norm", nat.lib().lw_resid_rmsnorm_rows(xt.data_ptr(), pt.data_ptr(), gt.data_ptr(), h.data_ptr(),
                                                      M, K, 1e-5, 1, torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    x_new = (x.astype(np.float32) + psum.astype(np.float16).astype(np.float32)).astype(np.float16)
    assert np.array_equal(xt.cpu().numpy(), x_new)
    ref = ol.rmsnorm(x_new, gamma, 1e-5).astype(np.float32)
    got = h.float().cpu().numpy()
    assert np.abs(got - ref).max() <= 2e-3 * np.abs(ref).max()


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M,K", [(5, 256), (128, 2048)])
def test_gemm_f32_partial(bits, M, K):
    """LW_TC_EPI_F32: the fp32 sums of a row-split linear (a tensor-parallel
    rank's partial), before any fp16 rounding."""
    N = 256
    q, s, deq = _weights(bits, N, K, 128, seed=11 + M)
    gen = torch.Generator(device=DEV).manual_seed(M)
    act = torch.randn(M, K, generator=gen, device=DEV).half()
    out = torch.full((M, N), float("nan"), device=DEV)
    _run(bits=bits, epilogue=3, M=M, N=N, K=K, group_size=128, lda=K, ldo=N, act=act, weight=q, scales=s, out=out)
    ref = act.float() @ deq.float().T
    err = (out - ref).abs().max().item()
    assert err <= 1e-3 * ref.abs().max().item(), err
