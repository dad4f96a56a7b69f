"""The tensor-parallel exchange kernels on one GPU, with two emulated ranks.

Both ranks' receive buffers live on the same device; every producing launch
(LW_EPI_PEER_*) of both ranks is enqueued before any consuming launch, so no
wait ever depends on a kernel launched after it. Checks, bit for bit, that
  * LW_EPI_PEER_F32 stores the same partial the local LW_EPI_F32 writes, into
    every rank's slot;
  * LW_PRO_PEER_RESID_NORM equals LW_PRO_RESID_NORM given psum = p0 + p1
    (the sum an NCCL all-reduce of two ranks produces);
  * LW_EPI_PEER_ARGMAX + the waiting sampler pick the first maximum of the
    concatenated vocabulary shards;
and that a wait nobody answers, or answers only with words of an earlier
step, gives up with LW_ERR_TIMEOUT, leaving the context usable.
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import quant as oq

pytestmark = pytest.mark.gpu
DEV = "cuda"
G = 128


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from liteweight_b200 import build
    build.build()


def _q4(n, k, seed):
    rng = np.random.default_rng(seed)
    q, s = oq.quantize_int4((rng.standard_normal((n, k)) * 0.05).astype(np.float16), G)
    return torch.from_numpy(q).to(DEV), torch.from_numpy(s).to(DEV)


class Rank:
    """One emulated rank's receive side (flagged 8-byte words): keys slots
    [world][M], two slot sets [world][M][H]; plus its step counter, error flag,
    local argmax keys and the lm_head's arrival count."""

    def __init__(self, world, M, H):
        self.keys_in = torch.zeros(world, M, dtype=torch.int64, device=DEV)
        self.slots = torch.zeros(2, world, M, H, dtype=torch.int64, device=DEV)
        self.keys = torch.zeros(M, dtype=torch.int64, device=DEV)
        self.step = torch.zeros(1, dtype=torch.int32, device=DEV)
        self.error = torch.zeros(1, dtype=torch.int32, device=DEV)
        self.arrivals = torch.zeros(1, dtype=torch.int32, device=DEV)


TAGS = 3   # partial exchanges 0, 1 and the keys exchange 2


def _exchanges(ranks, timeout_s=5.0):
    """(outs[r][e], ins[r][e]) for partial exchanges e = 0, 1 and the keys exchange e = 2."""
    from liteweight_b200 import engine as E
    world = len(ranks)
    outs, ins = [], []
    for r, R in enumerate(ranks):
        o_r, i_r = [], []
        for e in range(TAGS):
            o = E.ExchangeOut(world=world, rank=r, step=R.step.data_ptr(), tag=e, tags_per_step=TAGS,
                              arrivals=R.arrivals.data_ptr())
            for d, D in enumerate(ranks):   # receive buffers; the kernel adds rank * M (* ldo)
                o.dst[d] = D.keys_in.data_ptr() if e == 2 else D.slots[e % 2].data_ptr()
            o_r.append(o)
            src = R.keys_in.data_ptr() if e == 2 else R.slots[e % 2].data_ptr()
            i_r.append(E.ExchangeIn(world=world, tag=e, tags_per_step=TAGS, src=src, step=R.step.data_ptr(),
                                    error=R.error.data_ptr(), timeout_ns=int(timeout_s * 1e9)))
        outs.append(o_r)
        ins.append(i_r)
    return outs, ins


def _words(values_f32: torch.Tensor, flag: int) -> torch.Tensor:
    bits = values_f32.contiguous().view(torch.int32).to(torch.int64) & 0xFFFFFFFF
    return bits | (flag << 32) if flag < 2 ** 31 else bits | ((flag - 2 ** 32) << 32)


def _gemv(**kw):
    from liteweight_b200 import engine as E
    a = E.FusedGemvArgs()
    a.pdl, a.eps = 1, 1e-5
    for k, v in kw.items():
        if isinstance(v, torch.Tensor):
            v = v.data_ptr()
        elif isinstance(v, ctypes.Structure):
            v = ctypes.addressof(v)
        setattr(a, k, v)
    return a


def _run(a, keep):
    from liteweight_b200 import _native as nat
    keep.append(a)
    nat.check("lw_fused_gemv", nat.lib().lw_fused_gemv(ctypes.byref(a), torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("M", [1, 3, 20])
def test_partial_exchange_matches_local_sum(M):
    from liteweight_b200 import engine as E
    H, Kr, I = 512, 256, 512
    ranks = [Rank(2, M, H) for _ in range(2)]
    outs, ins = _exchanges(ranks)
    keep = []
    gen = torch.Generator(device=DEV).manual_seed(M)
    acts = [torch.randn(M, Kr, generator=gen, device=DEV).half() for _ in range(2)]
    W = [_q4(H, Kr, 10 + r) for r in range(2)]
    local = [torch.zeros(M, H, dtype=torch.float32, device=DEV) for _ in range(2)]
    for r in range(2):
        common = dict(bits=4, prologue=E.PRO_PLAIN, M=M, N=H, K=Kr, group_size=G, weight=W[r][0], scales=W[r][1],
                      act=acts[r], lda=Kr, ldo=H)
        _run(_gemv(epilogue=E.EPI_F32, out_f32=local[r], **common), keep)
        _run(_gemv(epilogue=E.EPI_PEER_F32, xout=outs[r][0], **common), keep)
    torch.cuda.synchronize()
    flag = E.exchange_flag(0, 0, TAGS)
    for R in ranks:
        for r in range(2):
            assert torch.equal(R.slots[0, r], _words(local[r], flag))

    # consumers: gate|up + SwiGLU over x + (p0 + p1)
    x = torch.randn(M, H, generator=gen, device=DEV).half()
    gamma = (1 + 0.1 * torch.randn(H, generator=gen, device=DEV)).half()
    gu = _q4(2 * I, H, 20)
    psum = local[0] + local[1]
    ref_out = torch.zeros(M, I, dtype=torch.float16, device=DEV)
    ref_x = torch.zeros(M, H, dtype=torch.float16, device=DEV)
    common = dict(bits=4, epilogue=E.EPI_SWIGLU, M=M, N=2 * I, K=H, group_size=G, weight=gu[0], scales=gu[1],
                  gamma=gamma, act=x, lda=H, ldo=I)
    _run(_gemv(prologue=E.PRO_RESID_NORM, psum=psum, x_out=ref_x, out=ref_out, **common), keep)
    got = []
    for r in range(2):
        o = torch.zeros(M, I, dtype=torch.float16, device=DEV)
        xo = torch.zeros(M, H, dtype=torch.float16, device=DEV)
        _run(_gemv(prologue=E.PRO_PEER_RESID_NORM, xin=ins[r][0], x_out=xo, out=o, **common), keep)
        got.append((o, xo))
    torch.cuda.synchronize()
    for o, xo in got:
        assert torch.equal(xo, ref_x)
        assert torch.equal(o, ref_out)
    assert all(int(R.error) == 0 for R in ranks)


def test_stale_flags_are_not_read():
    """Words of the previous step (or of the other exchange sharing the slot
    set) are not taken: a consumer whose words carry the wrong flag waits
    until its limit, then reports LW_ERR_TIMEOUT."""
    from liteweight_b200 import engine as E
    M, H, I = 1, 256, 256
    ranks = [Rank(2, M, H) for _ in range(2)]
    _outs, ins = _exchanges(ranks, timeout_s=0.02)
    R = ranks[0]
    R.slots[0] = _words(torch.ones(2, M, H, device=DEV), E.exchange_flag(0, 0, TAGS))   # step 0's words
    R.step.fill_(1)                                                                      # consumer is at step 1
    keep = []
    gu = _q4(2 * I, H, 3)
    out = torch.zeros(M, I, dtype=torch.float16, device=DEV)
    xo = torch.zeros(M, H, dtype=torch.float16, device=DEV)
    _run(_gemv(bits=4, prologue=E.PRO_PEER_RESID_NORM, epilogue=E.EPI_SWIGLU, M=M, N=2 * I, K=H, group_size=G,
               weight=gu[0], scales=gu[1], gamma=torch.ones(H, dtype=torch.float16, device=DEV),
               act=torch.zeros(M, H, dtype=torch.float16, device=DEV), lda=H, x_out=xo, out=out, ldo=I,
               xin=ins[0][0]), keep)
    torch.cuda.synchronize()
    assert int(R.error) == 8


def test_argmax_exchange_and_sampler():
    from liteweight_b200 import _native as nat
    from liteweight_b200 import engine as E
    M, H, V = 3, 256, 2 * 384
    Vr = V // 2
    ranks = [Rank(2, M, H) for _ in range(2)]
    outs, ins = _exchanges(ranks)
    keep = []
    gen = torch.Generator(device=DEV).manual_seed(1)
    lm = (torch.randn(V, H, generator=gen, device=DEV) * 0.05).half()
    lm[Vr + 5] = lm[7]                      # a tie across the shards: index 7 must win
    x = torch.randn(M, H, generator=gen, device=DEV).half()
    x[1] = lm[7].float().mul(40).half()     # row 1 aligned with the tied rows
    gamma = torch.ones(H, dtype=torch.float16, device=DEV)
    logits = []
    for r, R in enumerate(ranks):
        lg = torch.zeros(M, Vr, dtype=torch.float16, device=DEV)
        _run(_gemv(bits=16, prologue=E.PRO_NORM, epilogue=E.EPI_PEER_ARGMAX, M=M, N=Vr, K=H, group_size=H,
                   weight=lm[r * Vr:(r + 1) * Vr], gamma=gamma, act=x, lda=H, out=lg, ldo=Vr,
                   argmax_offset=r * Vr, argmax_keys=R.keys, xout=outs[r][2]), keep)
        logits.append(lg)
    embed = torch.randn(V, H, generator=gen, device=DEV).half()
    toks = []
    for r, R in enumerate(ranks):
        tokens = torch.full((4, M), -1, dtype=torch.int32, device=DEV)
        pos = torch.zeros(1, dtype=torch.int32, device=DEV)
        done = torch.zeros(1, dtype=torch.int32, device=DEV)
        xr = torch.zeros(M, H, dtype=torch.float16, device=DEV)
        nat.check("lw_sample_tokens", nat.lib().lw_sample_tokens(
            tokens.data_ptr(), R.keys.data_ptr(), embed.data_ptr(), xr.data_ptr(), pos.data_ptr(), done.data_ptr(),
            R.step.data_ptr(), ctypes.addressof(ins[r][2]), M, H, 1, torch.cuda.current_stream().cuda_stream))
        toks.append((tokens, pos, xr))
    torch.cuda.synchronize()
    full = torch.cat(logits, 1).float()
    want = full.argmax(1)                    # first index of the maximum
    assert int(want[1]) == 7
    for (tokens, pos, xr), R in zip(toks, ranks):
        assert torch.equal(tokens[1].long(), want)
        assert int(pos) == 1 and int(R.step) == 1 and int(R.error) == 0
        assert int(R.keys.abs().sum()) == 0 and int(R.arrivals) == 0
        assert torch.equal(xr, embed[want])


def test_unanswered_wait_times_out():
    """A consumer whose words nobody writes gives up after its limit, reports
    LW_ERR_TIMEOUT in the error flag and the context stays usable."""
    from liteweight_b200 import engine as E
    M, H, I = 1, 256, 256
    ranks = [Rank(2, M, H) for _ in range(2)]
    _outs, ins = _exchanges(ranks, timeout_s=0.02)
    keep = []
    gu = _q4(2 * I, H, 3)
    x = torch.randn(M, H, device=DEV).half()
    out = torch.zeros(M, I, dtype=torch.float16, device=DEV)
    xo = torch.zeros(M, H, dtype=torch.float16, device=DEV)
    _run(_gemv(bits=4, prologue=E.PRO_PEER_RESID_NORM, epilogue=E.EPI_SWIGLU, M=M, N=2 * I, K=H, group_size=G,
               weight=gu[0], scales=gu[1], gamma=torch.ones(H, dtype=torch.float16, device=DEV), act=x, lda=H,
               x_out=xo, out=out, ldo=I, xin=ins[0][0]), keep)
    torch.cuda.synchronize()
    assert int(ranks[0].error) == 8          # LW_ERR_TIMEOUT
    y = torch.ones(4, device=DEV) * 2
    assert float(y.sum()) == 8.0


def test_exchange_argument_validation():
    from liteweight_b200 import _native as nat
    from liteweight_b200 import engine as E
    M, H = 1, 256
    ranks = [Rank(2, M, H) for _ in range(2)]
    outs, ins = _exchanges(ranks)
    w = _q4(H, H, 1)
    x = torch.zeros(M, H, dtype=torch.float16, device=DEV)
    a = _gemv(bits=4, prologue=E.PRO_PLAIN, epilogue=E.EPI_PEER_F32, M=M, N=H, K=H, group_size=G, weight=w[0],
              scales=w[1], act=x, lda=H, ldo=H)
    s = torch.cuda.current_stream().cuda_stream
    assert nat.lib().lw_fused_gemv(ctypes.byref(a), s) == 1           # no xout
    bad = E.ExchangeOut.from_buffer_copy(outs[0][0])
    bad.rank = 2
    a.xout = ctypes.addressof(bad)
    assert nat.lib().lw_fused_gemv(ctypes.byref(a), s) == 2           # rank >= world
    bad.rank, bad.tag = 0, TAGS
    assert nat.lib().lw_fused_gemv(ctypes.byref(a), s) == 2           # tag out of range
    bad.tag, bad.dst[1] = 0, None
    assert nat.lib().lw_fused_gemv(ctypes.byref(a), s) == 1           # missing destination
