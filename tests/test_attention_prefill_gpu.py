"""Prompt-chunk attention (lw_attention_decode with prefill_seq set) against an
fp32 torch restatement of causal attention over the KV cache.

Row r of the chunk is position p0 + r of cache sequence `seq` and attends keys
0 .. p0 + r, the same rule the token-by-token decode applies one position at a
time (reference: liteweight/model.py, the attention of a decode step over the
cache). Tolerance: 4e-3 absolute on outputs of magnitude <= 1 (fp16 scores
weights P and the fp16 output each round at 2^-11 relative)."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda", 0)


def ref_attention(q, k, v, p0, seq, hd):
    R, nq = q.shape[0], q.shape[1] // hd
    nkv = k.shape[1]
    gq = nq // nkv
    qf = q.float().view(R, nq, hd)
    out = torch.empty(R, nq, hd, device=q.device)
    for r in range(R):
        L = p0 + r + 1
        kk = k[seq, :, :L].float().repeat_interleave(gq, 0)   # [nq, L, hd]
        vv = v[seq, :, :L].float().repeat_interleave(gq, 0)
        s = torch.einsum("hd,hld->hl", qf[r], kk) / hd ** 0.5
        out[r] = torch.einsum("hl,hld->hd", torch.softmax(s, -1), vv)
    return out.view(R, nq * hd)


@pytest.mark.parametrize("hd", [64, 128])
@pytest.mark.parametrize("gq", [1, 2, 4, 8])
@pytest.mark.parametrize("R,p0", [(1, 0), (7, 13), (16, 0), (45, 70), (128, 200)])
def test_prefill_attention_matches_torch(hd, gq, R, p0):
    from liteweight_b200 import _native as nat
    from liteweight_b200 import engine as E
    nkv, B, S = 2, 3, 384
    nq = nkv * gq
    g = torch.Generator(device=DEV).manual_seed(hd * 1000 + gq * 100 + R + p0)
    q = (torch.randn(R, nq * hd, device=DEV, generator=g) * 2).half()
    k = torch.randn(B, nkv, S, hd, device=DEV, generator=g).half()
    v = torch.randn(B, nkv, S, hd, device=DEV, generator=g).half()
    out = torch.full((R, nq * hd), float("nan"), device=DEV).half()
    seq = 1
    pos = torch.tensor([p0], dtype=torch.int32, device=DEV)
    seqt = torch.tensor([seq], dtype=torch.int32, device=DEV)
    a = E.AttentionArgs(q.data_ptr(), k.data_ptr(), v.data_ptr(), out.data_ptr(), pos.data_ptr(),
                        R, nq, nkv, hd, S, 0, seqt.data_ptr())
    nat.check("lw_attention_decode",
              nat.lib().lw_attention_decode(ctypes.byref(a), torch.cuda.current_stream().cuda_stream))
    torch.cuda.synchronize()
    want = ref_attention(q, k, v, p0, seq, hd)
    err = (out.float() - want).abs().max().item()
    assert err <= 4e-3, err
