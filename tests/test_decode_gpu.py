"""Parity of the fused decode step against the HF golden decode and the oracle (GPU).

Tolerance (the one the dequant GEMV uses): every logit row within
1e-2 * ||ref row||_2 / sqrt(V) max-abs of the reference; greedy token match
rate reported and required >= 0.9 on the golden fixtures.
"""

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


def _t(a):
    return torch.from_numpy(np.ascontiguousarray(a)).to(DEV)


def engine_from_oracle(w: ol.LlamaWeights, bits: int, group: int, batch: int, max_seq: int, graph_pdl=True,
                       fold=False):
    from liteweight_b200 import engine as E
    s = w.shape
    spec = E.LlamaSpec(hidden=s.hidden, inter=s.inter, n_layers=s.n_layers, n_heads=s.n_heads,
                       n_kv_heads=s.n_kv_heads, head_dim=s.head_dim, vocab=s.vocab, bits=bits, group_size=group,
                       eps=s.eps)
    layers = []
    for L in w.layers:
        lin = {n: (_t(getattr(L, n).qweight), _t(getattr(L, n).scales)) for n in
               ("q", "k", "v", "o", "gate", "up", "down")}
        layers.append(E.LayerWeights(in_norm=_t(L.in_norm), post_norm=_t(L.post_norm), **lin))
    lm = None if w.lm_head is w.embed else _t(w.lm_head)
    return E.build_engine(spec, layers, _t(w.embed), _t(w.norm), lm, torch.from_numpy(w.inv_freq), batch, max_seq,
                          DEV, attention_scaling=w.attention_scaling, pdl=graph_pdl, fold_scales=fold)


def run_engine(eng, prompt, steps, forced=None, graph=True):
    eng.start(torch.from_numpy(prompt), None if forced is None else torch.from_numpy(forced))
    if graph:
        eng.capture()
    P = prompt.shape[1]
    logits = []
    for p in range(steps):
        eng.step(1, graph=graph)
        if p >= P - 1:
            logits.append(eng.logits.float().cpu().numpy().copy())
    torch.cuda.synchronize()
    return np.stack(logits, 0)


def assert_rows(got, ref, what):
    g = got.reshape(-1, got.shape[-1]).astype(np.float64)
    r = ref.reshape(-1, ref.shape[-1]).astype(np.float64)
    tol = oq.row_tolerance(r)
    err = np.abs(g - r)
    assert np.all(err <= tol), f"{what}: worst err/tol {(err / tol).max():.3f}"
    return float((err / tol).max())


@pytest.mark.parametrize("graph", [False, True])
@pytest.mark.parametrize("fixture", ["llama_tiny_int8.npz", "llama_tiny_int4.npz"])
def test_golden_teacher_forced(golden_dir, fixture, graph):
    d = dict(np.load(golden_dir / fixture))
    w = ol.from_fixture(d)
    prompt, tokens = d["prompt"], d["tokens"]
    P, T = prompt.shape[1], tokens.shape[1]
    eng = engine_from_oracle(w, int(d["bits"]), int(d["group_size"]), batch=2, max_seq=64)
    got = run_engine(eng, prompt, P + T - 1, forced=tokens, graph=graph)
    assert_rows(got, d["logits"].astype(np.float32), f"{fixture} vs HF golden")
    oracle = ol.teacher_forced_logits(w, prompt, tokens)
    assert_rows(got, oracle, f"{fixture} vs oracle")
    match = (got.argmax(-1) == tokens.T).mean()
    assert match >= 0.9, match


@pytest.mark.parametrize("fixture", ["llama_tiny_int8.npz", "llama_tiny_int4.npz"])
def test_golden_free_running_greedy(golden_dir, fixture):
    d = dict(np.load(golden_dir / fixture))
    w = ol.from_fixture(d)
    prompt, tokens = d["prompt"], d["tokens"]
    P, T = prompt.shape[1], tokens.shape[1]
    eng = engine_from_oracle(w, int(d["bits"]), int(d["group_size"]), batch=2, max_seq=64)
    run_engine(eng, prompt, P + T - 1)
    gen = eng.generated(T).cpu().numpy()
    assert (gen == tokens).mean() >= 0.9, (gen, tokens)


def random_model(hidden, inter, layers, heads, kv, hd, vocab, bits, seed):
    rng = np.random.default_rng(seed)
    shape = ol.LlamaShape(hidden=hidden, inter=inter, n_layers=layers, n_heads=heads, n_kv_heads=kv, head_dim=hd,
                          vocab=vocab)
    quant = oq.quantize_int4 if bits == 4 else oq.quantize_int8

    def lin(n, k):
        q, s = quant((rng.standard_normal((n, k)) * 0.02).astype(np.float16), 128)
        return ol.QLinear(q, s, bits, 128)

    Ls = []
    for _ in range(layers):
        Ls.append(ol.LlamaLayer(
            in_norm=(1 + 0.1 * rng.standard_normal(hidden)).astype(np.float16),
            post_norm=(1 + 0.1 * rng.standard_normal(hidden)).astype(np.float16),
            q=lin(heads * hd, hidden), k=lin(kv * hd, hidden), v=lin(kv * hd, hidden), o=lin(hidden, heads * hd),
            gate=lin(inter, hidden), up=lin(inter, hidden), down=lin(hidden, inter)))
    embed = (rng.standard_normal((vocab, hidden)) * 0.02).astype(np.float16)
    inv = (1.0 / (500000.0 ** (np.arange(0, hd, 2) / hd))).astype(np.float32)
    return ol.LlamaWeights(shape=shape, embed=embed, layers=Ls,
                           norm=(1 + 0.1 * rng.standard_normal(hidden)).astype(np.float16), lm_head=embed,
                           inv_freq=inv)


@pytest.mark.parametrize("fold", [False, True])
@pytest.mark.parametrize("bits,batch,hd,heads,kv", [(4, 1, 64, 8, 2), (8, 3, 64, 8, 2), (4, 4, 128, 8, 1),
                                                    (8, 1, 128, 4, 4)])
def test_random_model_vs_oracle(bits, batch, hd, heads, kv, fold):
    """Free-running greedy decode; the oracle replays the engine's own tokens
    (teacher forcing), so every step's logits are compared on equal inputs.
    Vocab 1000 (not a multiple of 16) exercises the ragged lm_head tile."""
    w = random_model(512, 1536, 3, heads, kv, hd, 1000, bits, seed=bits * 10 + batch)
    P, T = 5, 7
    prompt = np.random.default_rng(batch).integers(0, 1000, (batch, P))
    eng = engine_from_oracle(w, bits, 128, batch=batch, max_seq=48, fold=fold)
    got = run_engine(eng, prompt, P + T - 1)
    gen = eng.generated(T).cpu().numpy()
    oracle = ol.teacher_forced_logits(w, prompt, gen)
    assert_rows(got, oracle, f"bits={bits} B={batch} hd={hd} fold={fold}")


@pytest.mark.parametrize("tc", [True, False])
@pytest.mark.parametrize("bits,kv,vocab", [(4, 2, 1000), (8, 2, 1000), (4, 8, 1000), (4, 2, 1024)])
def test_large_batch_vs_oracle(bits, kv, vocab, tc, monkeypatch):
    """Batch 40: the step's linears on the tensor-core GEMM with decode rows
    (row m = sequence m at *pos), or - with the tensor-core decode switched off
    - every GEMV as row blocks (32 + 8 sequences). The lm_head runs on the
    tensor cores (argmax epilogue) when the vocabulary is whole 128-row tiles
    (1024), else as GEMV row blocks (1000). 40 x 2 kv heads run the attention
    in 2-CTA clusters, 40 x 8 in single CTAs. Teacher-forced logits against
    the oracle."""
    from liteweight_b200 import engine as E
    monkeypatch.setenv("LW_B200_TC_DECODE_MIN", "24" if tc else "0")
    w = random_model(512, 1536, 3, 8, kv, 64, vocab, bits, seed=bits * 10 + 40 + kv)
    P, T, B = 5, 7, 40
    prompt = np.random.default_rng(40).integers(0, vocab, (B, P))
    eng = engine_from_oracle(w, bits, 128, batch=B, max_seq=48)
    assert eng.tc_decode == tc and E.tc_supported(eng.spec)
    got = run_engine(eng, prompt, P + T - 1)
    gen = eng.generated(T).cpu().numpy()
    oracle = ol.teacher_forced_logits(w, prompt, gen)
    assert_rows(got, oracle, f"bits={bits} B={B} tc={tc}")


def test_graph_equals_eager_and_long_context():
    """Bit-identical logits graph vs eager over a context longer than one
    attention round of the cluster (8 CTAs x 8 warps x 8 positions = 512)."""
    w = random_model(256, 512, 2, 4, 2, 64, 512, 4, seed=3)
    P, T = 1100, 4
    prompt = np.random.default_rng(0).integers(0, 512, (2, P))
    a = run_engine(engine_from_oracle(w, 4, 128, 2, 1200), prompt, P + T - 1, graph=False)
    b = run_engine(engine_from_oracle(w, 4, 128, 2, 1200), prompt, P + T - 1, graph=True)
    assert np.array_equal(a, b)
    eng = engine_from_oracle(w, 4, 128, 2, 1200)
    got = run_engine(eng, prompt, P + T - 1)
    oracle = ol.teacher_forced_logits(w, prompt, eng.generated(T).cpu().numpy())
    assert_rows(got, oracle, "long context")


class _Tok:
    """Minimal tokenizer: ids are space-separated integers."""
    eos_token_id = None

    def __call__(self, text, return_tensors="pt"):
        class R:
            pass
        r = R()
        r.input_ids = torch.tensor([[int(t) for t in text.split()]])
        return r

    def decode(self, ids, skip_special_tokens=True):
        return " ".join(str(i) for i in ids)


def _hf_model(bits):
    from transformers import LlamaConfig, LlamaForCausalLM
    from liteweight_b200.serialize import swap_linears
    cfg = LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=64, vocab_size=640, rms_norm_eps=1e-5, tie_word_embeddings=True,
                      max_position_embeddings=512, rope_parameters={"rope_type": "default", "rope_theta": 500000.0})
    torch.manual_seed(5)
    model = LlamaForCausalLM(cfg).half().eval()
    swap_linears(model, group_size=128, bits=bits)
    return model.to(DEV)


@pytest.mark.parametrize("bits", [8, 4])
def test_generate_api_matches_hf_loop(bits):
    from liteweight_b200 import engine as E
    from liteweight_b200.generate import _generate_hf, generate
    model = _hf_model(bits)
    assert E.supports(model)
    tok = _Tok()
    prompt = " ".join(str(i) for i in np.random.default_rng(1).integers(0, 640, 12))
    text = generate(model, tok, prompt, max_new_tokens=10)
    ids = tok(prompt).input_ids.to(DEV)
    ref = tok.decode(_generate_hf(model, ids, 10, 0.0, None, set()))
    a, b = text.split(), ref.split()
    assert len(a) == 10
    assert sum(x == y for x, y in zip(a, b)) >= 8, (a, b)
    sampled = generate(model, tok, prompt, max_new_tokens=6, temperature=0.8, top_k=20)
    assert len(sampled.split()) == 6


@pytest.mark.parametrize("path", ["gemv", "tc"])
@pytest.mark.parametrize("bits,batch,P,down_block", [(4, 1, 20, 3), (8, 2, 9, 0), (4, 3, 1, 0)])
def test_chunked_prefill(bits, batch, P, down_block, path, monkeypatch):
    """generate() runs the prompt in chunks (here 4 positions, so a prompt
    spans several chunks and a ragged last one). On the fused-GEMV path (with
    down_block, the down_proj in row blocks) the first layer's KV cache equals
    that of the token-by-token path bit for bit (same GEMV sums per row); the
    chunk attention (tensor-core tiles over key blocks) and, on the tensor-core
    path, lw_prefill_gemm sum in another order, so later layers match within
    the row tolerance and the picks match the oracle."""
    from liteweight_b200 import engine as E
    if down_block:
        monkeypatch.setattr(E, "down_rows", lambda spec, tp_size=1: down_block)
    w = random_model(512, 1024, 2, 8, 2, 64, 1000, bits, seed=7 + bits + batch)
    T = 6
    prompt = np.random.default_rng(P).integers(0, 1000, (batch, P))
    a = engine_from_oracle(w, bits, 128, batch=batch, max_seq=48)
    run_engine(a, prompt, P + T - 1)
    ref_tokens = a.generated(T).cpu().numpy()
    b = engine_from_oracle(w, bits, 128, batch=batch, max_seq=48)
    assert b.use_tc   # every linear of this model tiles for the tensor-core GEMM
    b.use_tc = path == "tc"
    b.prefill_rows = 4
    b.pf = b._buffers(4)
    got = b.generate(torch.from_numpy(prompt), T).numpy()
    if path == "gemv":
        assert torch.equal(a.k_cache[0][:, :, :P], b.k_cache[0][:, :, :P])
        assert torch.equal(a.v_cache[0][:, :, :P], b.v_cache[0][:, :, :P])
    for ka, kb in zip(a.k_cache + a.v_cache, b.k_cache + b.v_cache):
        r = ka[:, :, :P].float().reshape(-1, ka.shape[-1]).cpu().numpy()
        g = kb[:, :, :P].float().reshape(-1, kb.shape[-1]).cpu().numpy()
        assert np.all(np.abs(g - r) <= oq.row_tolerance(r) + 1e-3)
    assert (got == ref_tokens).mean() >= 0.8
    oracle = ol.teacher_forced_logits(w, prompt, got)
    assert (oracle.argmax(-1) == got.T).mean() >= 0.9


@pytest.mark.parametrize("path,R,chunks,bits", [("gemv", 4, 5, 4), ("tc", 4, 5, 8), ("tc", 64, 2, 4),
                                                ("tc", 128, 2, 8)])
def test_prefill_final_logits_vs_oracle(path, R, chunks, bits):
    """The logits the prompt pass computes at the prompt's last position (the
    ones that pick the first new token) against the oracle's, within the row
    tolerance, for chunks of 4 rows and for 64- and 128-row chunks on the
    tcgen05 GEMM (the prompt pass of generate() and of the bench)."""
    w = random_model(512, 1024, 2, 8, 2, 64, 1000, bits, seed=31 + R + bits)
    P = R * chunks   # whole chunks: the last one is the engine's own chunk buffers
    prompt = np.random.default_rng(R).integers(0, 1000, (1, P))
    eng = engine_from_oracle(w, bits, 128, batch=1, max_seq=P + 8)
    eng.use_tc = path == "tc"
    eng.prefill_rows = R
    eng.pf = eng._buffers(R)
    eng.start(torch.from_numpy(prompt))
    eng.prefill()
    torch.cuda.synchronize()
    eng.check()
    got = eng.pf.logits[R - 1].float().cpu().numpy()[None]
    first = eng.tokens[P].item()
    ref = ol.teacher_forced_logits(w, prompt, np.array([[first]]))[0]
    assert_rows(got, ref, f"prefill {path} rows {R} int{bits}")
    assert first == int(ref[0].argmax()) or ref[0][first] >= ref[0].max() - oq.row_tolerance(ref)[0, 0]


@pytest.mark.parametrize("head_bits,bits", [(4, 4), (8, 4), (8, 8)])
def test_quantized_lm_head_vs_oracle(head_bits, bits):
    """The lm_head quantized like swap_linears does when it is not skipped:
    the engine's logits (the GEMV dequantizes the head exactly) match the
    oracle whose head is the dequantized fp16 weight, and both pick alike."""
    from liteweight_b200 import engine as E
    w = random_model(512, 1024, 2, 8, 2, 64, 1000, bits, seed=21 + head_bits)
    quant, deq = ((oq.quantize_int4, oq.dequantize_int4) if head_bits == 4
                  else (oq.quantize_int8, oq.dequantize_int8))
    hq, hs = quant(w.embed, 128)
    w.lm_head = deq(hq, hs, 128)
    s = w.shape
    spec = E.LlamaSpec(hidden=s.hidden, inter=s.inter, n_layers=s.n_layers, n_heads=s.n_heads,
                       n_kv_heads=s.n_kv_heads, head_dim=s.head_dim, vocab=s.vocab, bits=bits, group_size=128,
                       eps=s.eps)
    layers = []
    for L in w.layers:
        lin = {n: (_t(getattr(L, n).qweight), _t(getattr(L, n).scales)) for n in
               ("q", "k", "v", "o", "gate", "up", "down")}
        layers.append(E.LayerWeights(in_norm=_t(L.in_norm), post_norm=_t(L.post_norm), **lin))
    eng = E.build_engine(spec, layers, _t(w.embed), _t(w.norm), None, torch.from_numpy(w.inv_freq), 2, 48, DEV,
                         lm_head_quant=(_t(hq), _t(hs), head_bits, 128))
    P, T = 6, 6
    prompt = np.random.default_rng(head_bits).integers(0, 1000, (2, P))
    got = run_engine(eng, prompt, P + T - 1)
    gen = eng.generated(T).cpu().numpy()
    oracle = ol.teacher_forced_logits(w, prompt, gen)
    assert_rows(got, oracle, f"lm_head int{head_bits}")
    # the tensor-core prompt path ends with the same quantized head
    out = eng.generate(torch.from_numpy(prompt), T).numpy()
    assert (out == gen).mean() >= 0.8


def test_generate_with_quantized_head_matches_hf_loop():
    """swap_linears(skip=()) quantizes the lm_head as well: generate() runs it
    on the engine (the head's QuantLinear buffers) and agrees with the HF loop."""
    from transformers import LlamaConfig, LlamaForCausalLM
    from liteweight_b200 import engine as E
    from liteweight_b200.generate import _generate_hf, generate
    from liteweight_b200.quantlinear import QuantLinear
    from liteweight_b200.serialize import swap_linears
    cfg = LlamaConfig(hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=4,
                      num_key_value_heads=2, head_dim=64, vocab_size=640, rms_norm_eps=1e-5, tie_word_embeddings=False,
                      max_position_embeddings=512, rope_parameters={"rope_type": "default", "rope_theta": 500000.0})
    torch.manual_seed(6)
    model = LlamaForCausalLM(cfg).half().eval()
    swap_linears(model, group_size=128, bits=4, skip=())
    model = model.to(DEV)
    assert isinstance(model.lm_head, QuantLinear) and E.supports(model)
    tok = _Tok()
    prompt = " ".join(str(i) for i in np.random.default_rng(2).integers(0, 640, 10))
    text = generate(model, tok, prompt, max_new_tokens=8)
    ids = tok(prompt).input_ids.to(DEV)
    ref = tok.decode(_generate_hf(model, ids, 8, 0.0, None, set()))
    a, b = text.split(), ref.split()
    assert len(a) == 8
    assert sum(x == y for x, y in zip(a, b)) >= 6, (a, b)
