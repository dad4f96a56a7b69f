"""Parity of the sm_100a dequant-matmul kernels against the oracle (GPU).

Every case computes the same packed weights two ways: the CUDA kernel through
the drop-in ops / C ABI, and the numpy oracle (dequantize, fp32 matmul, fp16).
Tolerances:
  * bit-exact for dequantized weights (lw_dequant_*) and one-hot probes;
  * outputs: max-abs error <= 1e-2 * ||ref[m, :]||_2 / sqrt(N) per row (the
    row-scaled bound), and also the reference's own allclose (atol 1e-2 /
    rtol 1e-3 for fp16 and INT8, 0.05 / 1e-2 for INT4; tests/test_kernels.py).
"""

import ctypes

import numpy as np
import pytest
import torch

from oracle import quant as oq

pytestmark = pytest.mark.gpu

DEV = "cuda"


@pytest.fixture(scope="module", autouse=True)
def _lib():
    if not torch.cuda.is_available():
        pytest.skip("CUDA device required")
    from liteweight_b200 import build
    build.build()


def kern():
    from liteweight_b200 import kernels
    return kernels


def check_rows(got: torch.Tensor, ref: np.ndarray, what: str):
    g = got.float().cpu().numpy()
    r = ref.astype(np.float32)
    assert g.shape == r.shape, (g.shape, r.shape)
    assert np.isfinite(g).all(), what
    tol = oq.row_tolerance(r)
    err = np.abs(g - r)
    ratio = (err / np.maximum(tol, 1e-12)).max()
    assert np.all(err <= tol), f"{what}: max err {err.max():.4g}, worst err/tol {ratio:.3f}"
    return ratio


def quantized(N, K, G, bits, seed, scale=0.02):
    g = torch.Generator().manual_seed(seed)
    W = (torch.randn(N, K, generator=g) * scale).half()
    if bits == 8:
        return oq.quantize_int8(W.numpy(), G)
    return oq.quantize_int4(W.numpy(), G)


def run_quant(act_np, q, s, G, bits):
    k = kern()
    act = torch.from_numpy(act_np).to(DEV)
    qt, st = torch.from_numpy(q).to(DEV), torch.from_numpy(s).to(DEV)
    return (k.matmul_int8 if bits == 8 else k.matmul_int4)(act, qt, st, group_size=G)


# ------------------------------------------------ the reference's kernel tests

@pytest.mark.parametrize("M,K,N", [(1, 2048, 8192), (4, 2048, 8192), (16, 2048, 2048), (128, 512, 512)])
def test_fp16_close_to_torch(M, K, N):
    torch.manual_seed(0)
    a = torch.randn(M, K, dtype=torch.float16, device=DEV)
    b = torch.randn(K, N, dtype=torch.float16, device=DEV)
    got = kern().matmul_fp16(a, b)
    ref = (a.float().cpu().numpy() @ b.float().cpu().numpy()).astype(np.float16)
    assert got.shape == (M, N) and got.dtype == torch.float16
    assert torch.allclose(got.cpu(), torch.from_numpy(ref), atol=1e-2, rtol=1e-3)
    check_rows(got, ref, "fp16 kn")


@pytest.mark.parametrize("M,K,N", [(1, 2048, 8192), (4, 2048, 8192), (16, 2048, 2048), (3, 70, 130)])
def test_fp16_transposed_weight(M, K, N):
    torch.manual_seed(0)
    a = torch.randn(M, K, dtype=torch.float16, device=DEV)
    w = torch.randn(N, K, dtype=torch.float16, device=DEV)
    got = kern().matmul_fp16(a, w.T)
    ref = (a.float().cpu().numpy() @ w.float().cpu().numpy().T).astype(np.float16)
    assert torch.allclose(got.cpu(), torch.from_numpy(ref), atol=1e-2, rtol=1e-3)


def test_fp16_non_tile_multiple_shape():
    a = torch.randn(3, 70, dtype=torch.float16, device=DEV)
    b = torch.randn(70, 130, dtype=torch.float16, device=DEV)
    got = kern().matmul_fp16(a, b)
    ref = torch.from_numpy((a.float().cpu().numpy() @ b.float().cpu().numpy()).astype(np.float16))
    assert torch.allclose(got.cpu(), ref, atol=1e-2)


@pytest.mark.parametrize("M,K,N,G", [(1, 2048, 8192, 128), (4, 2048, 8192, 128), (16, 2048, 2048, 128),
                                     (1, 2048, 8192, 2048)])
def test_int8_matches_oracle(M, K, N, G):
    torch.manual_seed(1)
    act = torch.randn(M, K, dtype=torch.float16)
    W = torch.randn(N, K, dtype=torch.float16)
    q, s = oq.quantize_int8(W.numpy(), G)
    got = run_quant(act.numpy(), q, s, G, 8)
    oracle = oq.fakequant_matmul(act.numpy(), W.numpy(), G)
    assert got.shape == (M, N) and got.dtype == torch.float16
    assert torch.allclose(got.cpu(), torch.from_numpy(oracle), atol=1e-2, rtol=1e-3)
    check_rows(got, oracle, f"int8 {M}x{K}x{N} G{G}")


def test_int8_no_nan():
    act = torch.randn(1, 256, dtype=torch.float16)
    W = torch.randn(64, 256, dtype=torch.float16)
    q, s = oq.quantize_int8(W.numpy(), 128)
    out = run_quant(act.numpy(), q, s, 128, 8)
    assert not out.isnan().any() and not out.isinf().any()


@pytest.mark.parametrize("M,K,N", [(1, 2048, 8192), (4, 2048, 8192), (16, 2048, 2048)])
def test_int4_matches_oracle(M, K, N):
    torch.manual_seed(2)
    act = torch.randn(M, K, dtype=torch.float16)
    W = torch.randn(N, K, dtype=torch.float16)
    q, s = oq.quantize_int4(W.numpy(), 128)
    got = run_quant(act.numpy(), q, s, 128, 4)
    oracle = oq.fakequant_matmul_int4(act.numpy(), W.numpy(), 128)
    assert torch.allclose(got.cpu(), torch.from_numpy(oracle), atol=0.05, rtol=1e-2)
    check_rows(got, oracle, f"int4 {M}x{K}x{N}")


# ------------------------------------------------ golden vectors from the reference

def test_golden_fakequant_outputs(golden_dir):
    qg = dict(np.load(golden_dir / "quant_golden.npz"))
    names = sorted({k.split("/")[0] for k in qg if k.endswith("/act")})
    assert names
    for name in names:
        act, G = qg[f"{name}/act"], int(qg[f"{name}/G"])
        for bits in (8, 4):
            got = run_quant(act, qg[f"{name}/q{bits}"], qg[f"{name}/s{bits}"], G, bits)
            ref = qg[f"{name}/out{bits}"]
            atol, rtol = (1e-2, 1e-3) if bits == 8 else (0.05, 1e-2)
            assert torch.allclose(got.cpu(), torch.from_numpy(ref), atol=atol, rtol=rtol), name
            check_rows(got, ref, f"{name} int{bits}")


def test_dequant_kernels_bit_exact(golden_dir):
    from liteweight_b200.quantize import dequantize_int4, dequantize_int8
    qg = dict(np.load(golden_dir / "quant_golden.npz"))
    d4 = dequantize_int4(torch.from_numpy(qg["codes4/q"]).to(DEV), torch.from_numpy(qg["codes4/s"]).to(DEV), 128)
    assert np.array_equal(d4.cpu().numpy().view(np.uint16), qg["codes4/dq"].view(np.uint16))
    d8 = dequantize_int8(torch.from_numpy(qg["codes8/q"]).to(DEV), torch.from_numpy(qg["codes8/s"]).to(DEV), 128)
    assert np.array_equal(d8.cpu().numpy().view(np.uint16), qg["codes8/dq"].view(np.uint16))
    for name in ("tq_64x256", "tq_32x512", "ties_i8", "group_axis"):
        G = int(qg[f"{name}/G"])
        d8 = dequantize_int8(torch.from_numpy(qg[f"{name}/q8"]).to(DEV), torch.from_numpy(qg[f"{name}/s8"]).to(DEV), G)
        assert np.array_equal(d8.cpu().numpy().view(np.uint16), qg[f"{name}/dq8"].view(np.uint16)), name
        d4 = dequantize_int4(torch.from_numpy(qg[f"{name}/q4"]).to(DEV), torch.from_numpy(qg[f"{name}/s4"]).to(DEV), G)
        assert np.array_equal(d4.cpu().numpy().view(np.uint16), qg[f"{name}/dq4"].view(np.uint16)), name


def test_every_code_through_the_gemv():
    """All 16 nibble codes (incl. -8) and all 256 int8 codes (incl. -128) through the
    fast path: one-hot activation rows select single weight columns, so the output
    must equal the dequantized weight bit for bit."""
    g = np.random.default_rng(5)
    N, K = 32, 256
    q4 = g.integers(0, 256, (N, K // 2), dtype=np.uint8)
    q8 = g.integers(-128, 128, (N, K), dtype=np.int8)
    s = (g.random((N, K // 128)) * 0.05 + 1e-3).astype(np.float16)
    for bits, q in ((4, q4), (8, q8)):
        w = oq.dequantize_int4(q, s, 128) if bits == 4 else oq.dequantize_int8(q, s, 128)
        for k0 in range(0, K, 32):
            act = np.eye(K, dtype=np.float16)[k0:k0 + 32]
            got = run_quant(act, q, s, 128, bits).cpu().numpy()
            assert np.array_equal(got.view(np.uint16), w[:, k0:k0 + 32].T.copy().view(np.uint16)), (bits, k0)


# ------------------------------------------------ config-2 sweep (Llama-3.2-1B shapes)

SWEEP_KN = [(2048, 2048), (2048, 512), (2048, 8192), (8192, 2048)]
SWEEP_M = [1, 2, 4, 8, 16, 32, 64, 128, 256]
_cache = {}


def sweep_weights(K, N, bits):
    key = (K, N, bits)
    if key not in _cache:
        q, s = quantized(N, K, 128, bits, seed=K * 7 + N + bits)
        w = (oq.dequantize_int4 if bits == 4 else oq.dequantize_int8)(q, s, 128).astype(np.float32)
        _cache[key] = (w, torch.from_numpy(q).to(DEV), torch.from_numpy(s).to(DEV))
    return _cache[key]


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("K,N", SWEEP_KN)
def test_sweep_parity(bits, K, N):
    w, qt, st = sweep_weights(K, N, bits)
    k = kern()
    fn = k.matmul_int4 if bits == 4 else k.matmul_int8
    rng = np.random.default_rng(K + N)
    for M in SWEEP_M:
        act = rng.standard_normal((M, K)).astype(np.float16)
        ref = (act.astype(np.float32) @ w.T).astype(np.float16)
        got = fn(torch.from_numpy(act).to(DEV), qt, st, group_size=128)
        check_rows(got, ref, f"int{bits} M={M} K={K} N={N}")


# ------------------------------------------------ edge cases

@pytest.mark.parametrize("bits,M,K,N,G", [
    (4, 1, 192, 40, 64),      # K tail inside a chunk, N not a multiple of 16
    (4, 3, 2048, 17, 128),    # ragged N
    (8, 5, 48, 24, 16),       # tiny K, G = 16
    (8, 2, 320, 33, 8),       # G below the 16-element piece -> generic path
    (4, 2, 70, 10, 35),       # odd group -> generic path
    (8, 40, 1024, 96, 128),   # M above one launch block (M blocking)
    (4, 33, 4096, 64, 4096),  # per-output-channel INT4, M = 33
    (8, 9, 8192, 48, 128),    # two n8 batch tiles
])
def test_edge_shapes(bits, M, K, N, G):
    q, s = quantized(N, K, G, bits, seed=M * 1000 + N)
    act = np.random.default_rng(M + K).standard_normal((M, K)).astype(np.float16)
    got = run_quant(act, q, s, G, bits)
    ref = oq.packed_matmul(act, q, s, G, bits)
    check_rows(got, ref, f"int{bits} {M}x{K}x{N} G{G}")


def test_empty_m():
    q, s = quantized(16, 256, 128, 8, seed=1)
    out = run_quant(np.zeros((0, 256), np.float16), q, s, 128, 8)
    assert out.shape == (0, 16)


def test_non_contiguous_activation():
    q, s = quantized(64, 512, 128, 4, seed=3)
    big = torch.randn(4, 1024, dtype=torch.float16, device=DEV)
    act = big[:, ::2]
    got = kern().matmul_int4(act, torch.from_numpy(q).to(DEV), torch.from_numpy(s).to(DEV), group_size=128)
    ref = oq.packed_matmul(act.cpu().numpy(), q, s, 128, 4)
    check_rows(got, ref, "strided act")


def test_assertions_like_reference():
    k = kern()
    q, s = quantized(16, 256, 128, 8, seed=1)
    act = torch.zeros(1, 256, dtype=torch.float32, device=DEV)
    with pytest.raises(AssertionError):
        k.matmul_int8(act, torch.from_numpy(q).to(DEV), torch.from_numpy(s).to(DEV))
    with pytest.raises(AssertionError):
        k.matmul_int4(act.half(), torch.from_numpy(q).to(DEV), torch.from_numpy(s).to(DEV))


def test_quantlinear_bias_and_shape():
    from liteweight_b200.quantlinear import QuantLinear
    torch.manual_seed(4)
    lin = torch.nn.Linear(256, 96, bias=True).half()
    for bits in (8, 4):
        ql = QuantLinear.from_linear(lin, group_size=128, bits=bits).to(DEV)
        x = torch.randn(2, 3, 256, dtype=torch.float16, device=DEV)
        y = ql(x)
        assert y.shape == (2, 3, 96)
        q, s = ql.qweight.cpu().numpy(), ql.scales.cpu().numpy()
        ref = oq.packed_matmul(x.reshape(-1, 256).cpu().numpy(), q, s, 128, bits)
        ref = (ref.astype(np.float32) + ql.bias.cpu().numpy().astype(np.float32)).astype(np.float16)
        check_rows(y.reshape(-1, 96), ref, f"QuantLinear bits={bits}")


def test_deterministic_and_graph_capturable():
    q, s = quantized(2048, 2048, 128, 4, seed=9)
    qt, st = torch.from_numpy(q).to(DEV), torch.from_numpy(s).to(DEV)
    act = torch.randn(4, 2048, dtype=torch.float16, device=DEV)
    k = kern()
    a = k.matmul_int4(act, qt, st)
    b = k.matmul_int4(act, qt, st)
    assert torch.equal(a, b)
    out = [None]
    g = torch.cuda.CUDAGraph()
    s_ = torch.cuda.Stream()
    with torch.cuda.stream(s_):
        k.matmul_int4(act, qt, st)
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s_):
            out[0] = k.matmul_int4(act, qt, st)
    g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out[0], a)


@pytest.mark.parametrize("bits,M,K,N", [(4, 1, 8192, 512), (8, 3, 14336, 256), (16, 2, 4096, 1024),
                                        (4, 9, 4096, 64), (8, 1, 2048, 2048)])
def test_split_tiles_with_workspace(bits, M, K, N):
    """Tiles shared between warps (workspace given) and whole tiles (no
    workspace) both match the oracle; the workspace is left zeroed and repeated
    calls are bit-identical."""
    from liteweight_b200 import _native as nat
    rng = np.random.default_rng(bits * 100 + M)
    act = rng.standard_normal((M, K)).astype(np.float16)
    if bits == 16:
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
        ref = oq.matmul_dequant(act, w)
        q, s = w, None
    else:
        q, s = quantized(N, K, 128, bits, seed=N + K)
        ref = oq.packed_matmul(act, q, s, 128, bits)
    a = torch.from_numpy(act).to(DEV)
    qt = torch.from_numpy(q).to(DEV)
    st = torch.from_numpy(s).to(DEV) if s is not None else None
    need = int(nat.lib().lw_gemm_workspace_size(bits, M, N, K))
    assert need > 0, "shape chosen to split tiles"
    ws = torch.zeros(need, dtype=torch.uint8, device=DEV)
    outs = []
    stream = torch.cuda.current_stream().cuda_stream
    for wsp, wsb in ((ws.data_ptr(), need), (ws.data_ptr(), need), (None, 0)):
        o = torch.empty(M, N, dtype=torch.float16, device=DEV)
        if bits == 16:
            nat.call("lw_gemm_f16", a.data_ptr(), qt.data_ptr(), o.data_ptr(), M, N, K, wsp, wsb, stream)
        else:
            fn = "lw_gemm_w4a16" if bits == 4 else "lw_gemm_w8a16"
            nat.call(fn, a.data_ptr(), qt.data_ptr(), st.data_ptr(), None, o.data_ptr(), M, N, K, 128, wsp, wsb,
                     stream)
        torch.cuda.synchronize()
        outs.append(o)
        check_rows(o, ref, f"bits={bits} ws={wsb}")
    assert torch.equal(outs[0], outs[1])
    # the per-tile counters at the head of the workspace are back to zero
    assert int(ws[: 64 * 1024].count_nonzero()) == 0


def test_workspace_reuse_across_shapes():
    """One workspace serves calls of different shapes in any order (the counter
    region never overlaps the slots of a previous call)."""
    k = kern()
    rng = np.random.default_rng(17)
    for bits, M, K, N in [(8, 16, 2048, 2048), (8, 1, 2048, 8192), (4, 3, 8192, 256), (4, 1, 4096, 28672),
                          (8, 2, 2048, 512)]:
        q, s = quantized(N, K, 128, bits, seed=N)
        act = rng.standard_normal((M, K)).astype(np.float16)
        got = run_quant(act, q, s, 128, bits)
        check_rows(got, oq.packed_matmul(act, q, s, 128, bits), f"reuse int{bits} {M}x{K}x{N}")


def test_graph_survives_workspace_growth():
    """A graph captured with a small shape keeps its workspace after a larger
    shape grows the stream's workspace: replaying it afterwards still matches
    the oracle, and the larger call's output is right too. (M = 12 runs the
    split-tile kernel, whose workspace grows with N.)"""
    from liteweight_b200 import _native as nat
    k = kern()
    rng = np.random.default_rng(23)
    M = 12
    s_ = torch.cuda.Stream()
    with torch.cuda.stream(s_):
        key = (torch.device(DEV).index or 0, s_.cuda_stream)
        old = nat._workspaces.pop(key, None)   # start this stream from a small workspace
        if old is not None:
            nat._retired.append(old)
        q1, sc1 = quantized(512, 4096, 128, 4, seed=31)
        act1 = rng.standard_normal((M, 4096)).astype(np.float16)
        a1 = torch.from_numpy(act1).to(DEV)
        qt1, st1 = torch.from_numpy(q1).to(DEV), torch.from_numpy(sc1).to(DEV)
        need1 = int(nat.lib().lw_gemm_workspace_size(4, M, 512, 4096))
        need2 = int(nat.lib().lw_gemm_workspace_size(4, M, 28672, 4096))
        assert 0 < need1 and need2 > max(need1, 1 << 20), (need1, need2)
        k.matmul_int4(a1, qt1, st1)
        torch.cuda.synchronize()
        small_ws = nat._workspaces[key].data_ptr()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s_):
            out1 = k.matmul_int4(a1, qt1, st1)
        # a much larger split-tile problem grows (replaces) the stream's workspace
        q2, sc2 = quantized(28672, 4096, 128, 4, seed=32)
        act2 = rng.standard_normal((M, 4096)).astype(np.float16)
        big = k.matmul_int4(torch.from_numpy(act2).to(DEV), torch.from_numpy(q2).to(DEV),
                            torch.from_numpy(sc2).to(DEV))
        torch.cuda.synchronize()
        assert nat._workspaces[key].data_ptr() != small_ws, "the larger call did not grow the workspace"
        # fill freshly allocated memory with garbage: if the retired block had
        # been handed back, these tensors could own it
        junk = [torch.full((1 << 20,), 255, dtype=torch.uint8, device=DEV) for _ in range(8)]
        for _ in range(3):
            out1.fill_(0)
            g.replay()
        torch.cuda.synchronize()
        del junk
    check_rows(out1, oq.packed_matmul(act1, q1, sc1, 128, 4), "graph replay after workspace growth")
    check_rows(big, oq.packed_matmul(act2, q2, sc2, 128, 4), "the call that grew the workspace")


@pytest.mark.parametrize("bits,M,K,N,G", [
    (4, 1, 2080, 1000, 32),      # row bytes 1040: the last 128-byte stage half past K; N not whole row blocks
    (8, 3, 2064, 200, 16),       # INT8 row bytes 2064; 200 rows = 2 row blocks, the second ragged
    (4, 8, 4096, 4096, 4096),    # per-output-channel scales (G = K), eight rows
    (8, 1, 2048, 8192, 2048),    # the single W8A16 QuantLinear: per-output-channel, M = 1
    (4, 2, 14336, 4096, 128),    # a long row (112 stages): many units per row block
    (16, 5, 4096, 3000, 4096),   # fp16 weights
])
def test_ring_edges(bits, M, K, N, G):
    """M <= 8 shapes on the TMA-ring GEMV: ragged row blocks, partial last
    stages, per-channel scales, long rows; bit-identical on a repeat call and
    the workspace's counters are zero again afterwards."""
    from liteweight_b200 import _native as nat
    rng = np.random.default_rng(bits * 31 + M)
    act = rng.standard_normal((M, K)).astype(np.float16)
    if bits == 16:
        w = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
        q, s, ref = w, None, oq.matmul_dequant(act, w)
    else:
        q, s = quantized(N, K, G, bits, seed=N + K)
        ref = oq.packed_matmul(act, q, s, G, bits)
    a = torch.from_numpy(act).to(DEV)
    qt = torch.from_numpy(q).to(DEV)
    st = torch.from_numpy(s).to(DEV) if s is not None else None
    need = int(nat.lib().lw_gemm_workspace_size(bits, M, N, K))
    ws = torch.zeros(max(need, 64 * 1024), dtype=torch.uint8, device=DEV)
    nat.lib().lw_take_device_error()   # start from clear device error flags
    stream = torch.cuda.current_stream().cuda_stream
    outs = []
    for _ in range(2):
        o = torch.empty(M, N, dtype=torch.float16, device=DEV)
        if bits == 16:
            nat.call("lw_gemm_f16", a.data_ptr(), qt.data_ptr(), o.data_ptr(), M, N, K, ws.data_ptr(), need, stream)
        else:
            fn = "lw_gemm_w4a16" if bits == 4 else "lw_gemm_w8a16"
            nat.call(fn, a.data_ptr(), qt.data_ptr(), st.data_ptr(), None, o.data_ptr(), M, N, K, G,
                     ws.data_ptr(), need, stream)
        outs.append(o)
    torch.cuda.synchronize()
    assert nat.lib().lw_take_device_error() == 0
    check_rows(outs[0], ref, f"ring bits={bits} {M}x{K}x{N} G{G}")
    assert torch.equal(outs[0], outs[1])
    assert int(ws[: 64 * 1024].count_nonzero()) == 0


@pytest.mark.parametrize("bits,M,K,N,G", [
    (4, 1, 4096, 4096, 128),     # a decode projection
    (4, 5, 3072, 3000, 128),     # partial last stage (3-D copy fills zeros), ragged last tile
    (4, 8, 4096, 2048, 4096),    # per-output-channel scales
    (4, 2, 14336, 4096, 128),    # a long row
    (8, 1, 2048, 8192, 2048),    # per-output-channel INT8
    (8, 3, 4096, 4096, 128),
])
def test_ring_codes_variant(bits, M, K, N, G):
    """The ring GEMV's codes variant (fold_scales: codes as fp16 subnormals,
    per-chunk fp32 scale): within one fp16 rounding of the exact fp64
    sum_k code * scale * a, inside the drop-in row tolerance of the oracle's
    exact-dequant matmul, and bit-identical on a repeat call."""
    from liteweight_b200 import _native as nat
    from liteweight_b200 import engine as E
    rng = np.random.default_rng(bits * 7 + M + K)
    act = rng.standard_normal((M, K)).astype(np.float16)
    q, s = quantized(N, K, G, bits, seed=N + K + 1)
    codes = oq.unpack_int4(q) if bits == 4 else q
    w64 = codes.astype(np.float64) * np.repeat(s.astype(np.float64), G, axis=1)
    exact = act.astype(np.float64) @ w64.T
    a, qt, st = (torch.from_numpy(x).to(DEV) for x in (act, q, s))
    args = E.FusedGemvArgs()
    args.bits, args.prologue, args.epilogue = bits, E.PRO_PLAIN, E.EPI_PLAIN
    args.M, args.N, args.K, args.group_size, args.lda, args.ldo = M, N, K, G, K, N
    args.act, args.weight, args.scales = a.data_ptr(), qt.data_ptr(), st.data_ptr()
    args.fold_scales, args.kernel, args.pdl = 1, 0, 0
    need = int(nat.lib().lw_fused_gemv_workspace_size(ctypes.byref(args)))
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=DEV)
    args.workspace, args.workspace_bytes = ws.data_ptr(), ws.numel()
    nat.lib().lw_take_device_error()
    outs = []
    for _ in range(2):
        o = torch.empty(M, N, dtype=torch.float16, device=DEV)
        args.out = o.data_ptr()
        nat.check("lw_fused_gemv", nat.lib().lw_fused_gemv(ctypes.byref(args), torch.cuda.current_stream().cuda_stream))
        outs.append(o)
    torch.cuda.synchronize()
    assert nat.lib().lw_take_device_error() == 0
    got = outs[0].float().cpu().numpy().astype(np.float64)
    # one fp16 rounding of the exact value (half an ulp), plus the fp32 sums'
    # rounding, bounded by a small multiple of sum_k |code * scale * a|
    ulp = np.spacing(np.abs(exact).astype(np.float16)).astype(np.float64)
    absmag = np.abs(act.astype(np.float64)) @ np.abs(w64).T
    err = np.abs(got - exact)
    bound = 0.5 * ulp + 1e-5 * absmag + 1e-7
    assert np.all(err <= bound), f"codes bits={bits}: worst err/bound {(err / bound).max():.3f}"
    check_rows(outs[0], oq.packed_matmul(act, q, s, G, bits), f"codes bits={bits} vs exact dequant")
    assert torch.equal(outs[0], outs[1])
    assert int(ws[: 64 * 1024].count_nonzero()) == 0


def test_quantize_kernels_bit_exact(golden_dir):
    """lw_quantize_int8/int4 reproduce the reference's quantize_int8/int4
    bit for bit on its golden vectors (every group size there, round-half-even
    ties, the per-output-channel case), from fp16 and from fp32 weights."""
    from liteweight_b200 import quantize as lq
    qg = dict(np.load(golden_dir / "quant_golden.npz"))
    names = sorted({k.split("/")[0] for k in qg if k.endswith("/W")})
    assert names
    for name in names:
        W, G = qg[f"{name}/W"], int(qg[f"{name}/G"])
        for dt in (torch.float16, torch.float32):
            if W.dtype == np.float32 and dt == torch.float16:
                continue   # an fp32 golden input is only exact as fp32
            w = torch.from_numpy(W).to(device=DEV, dtype=dt)
            q8, s8 = lq.quantize_int8(w, G)
            q4, s4 = lq.quantize_int4(w, G)
            torch.cuda.synchronize()
            np.testing.assert_array_equal(q8.cpu().numpy(), qg[f"{name}/q8"], err_msg=f"{name} {dt}")
            np.testing.assert_array_equal(s8.cpu().numpy().view(np.uint16), qg[f"{name}/s8"].view(np.uint16))
            np.testing.assert_array_equal(q4.cpu().numpy(), qg[f"{name}/q4"], err_msg=f"{name} {dt}")
            np.testing.assert_array_equal(s4.cpu().numpy().view(np.uint16), qg[f"{name}/s4"].view(np.uint16))


@pytest.mark.parametrize("N,K,G", [(4096, 4096, 128), (1000, 2048, 2048), (64, 6, 3), (33, 60, 15), (128, 256, 32)])
def test_quantize_kernels_match_oracle(N, K, G):
    """Large, per-channel and odd group sizes (INT4 bytes straddling two groups)
    against the numpy oracle, bit for bit."""
    from liteweight_b200 import quantize as lq
    rng = np.random.default_rng(N + K + G)
    W = (rng.standard_normal((N, K)) * 0.02).astype(np.float16)
    W[0, :G] = 0.0                                   # an all-zero group: scale clamped to 1e-8
    w = torch.from_numpy(W).to(DEV)
    for bits, fn, ofn in ((8, lq.quantize_int8, oq.quantize_int8), (4, lq.quantize_int4, oq.quantize_int4)):
        q, s = fn(w, G)
        rq, rs = ofn(W, G)
        torch.cuda.synchronize()
        np.testing.assert_array_equal(q.cpu().numpy(), rq, err_msg=f"int{bits} codes {N}x{K} G{G}")
        np.testing.assert_array_equal(s.cpu().numpy().view(np.uint16), rs.view(np.uint16),
                                      err_msg=f"int{bits} scales {N}x{K} G{G}")


@pytest.mark.parametrize("bits", [4, 8])
@pytest.mark.parametrize("M", [33, 64, 300])
def test_tensor_core_route_with_bias(bits, M):
    """Past the GEMV crossover the drop-in matmul runs the tcgen05 GEMM (here
    with QuantLinear's bias in its epilogue, and M = 300 in two row blocks)."""
    from liteweight_b200.quantlinear import QuantLinear
    torch.manual_seed(bits + M)
    lin = torch.nn.Linear(512, 384, bias=True).half()
    ql = QuantLinear.from_linear(lin, group_size=128, bits=bits).to(DEV)
    x = torch.randn(M, 512, dtype=torch.float16, device=DEV)
    y = ql(x)
    q, s = ql.qweight.cpu().numpy(), ql.scales.cpu().numpy()
    ref = oq.packed_matmul(x.cpu().numpy(), q, s, 128, bits)
    ref = (ref.astype(np.float32) + ql.bias.cpu().numpy().astype(np.float32)).astype(np.float16)
    check_rows(y, ref, f"tcgen05 route bits={bits} M={M}")
