"""Generate the golden fixtures in this folder from the reference itself.

Run where the liteweight sources are present, giving their root directory
(the one holding ``liteweight/``):

    python tests/golden/make_golden.py <reference-root>

It imports the reference's ``liteweight.quantize`` and ``liteweight.serialize``
and the installed ``transformers`` (5.5.0) ``LlamaForCausalLM``, and writes:

* ``quant_golden.npz`` - inputs and outputs of ``quantize_int8/int4``,
  ``dequantize_int8/int4`` and ``fakequant_matmul(_int4)`` for the seeds and
  shapes of the reference's tests (tests/test_quantize.py,
  tests/test_kernels.py), a round-half-even tie case, the per-output-channel
  case (G = K), and random packed bytes covering every int8 / nibble code
  (including -128 and -8, which the quantizer never emits but the format holds).
* ``llama_tiny_int{8,4}.npz`` - a tiny random-init Llama (2 layers, GQA,
  head_dim 64) quantized by the reference's ``swap_linears``, its packed
  buffers, and the fp16 logits of an HF greedy decode in which every
  ``QuantLinear.forward`` is the reference's dequantize-then-fp32-matmul
  (liteweight/quantize.py:60) - the same math its Triton kernels implement.

Nothing on the GPU test path reads the reference; the fixtures are committed.
"""

from __future__ import annotations

import sys
from pathlib import Path

import numpy as np
import torch

OUT = Path(__file__).resolve().parent


def _np(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().numpy()


def quant_cases(lq):
    cases = {}

    def add(name, W, G, act=None, store_dq=True):
        q8, s8 = lq.quantize_int8(W, group_size=G)
        q4, s4 = lq.quantize_int4(W, group_size=G)
        d = {"W": _np(W), "G": np.int64(G), "q8": _np(q8), "s8": _np(s8), "q4": _np(q4), "s4": _np(s4)}
        if store_dq:
            d["dq8"] = _np(lq.dequantize_int8(q8, s8, G))
            d["dq4"] = _np(lq.dequantize_int4(q4, s4, G))
        if act is not None:
            d["act"] = _np(act)
            d["out8"] = _np(lq.fakequant_matmul(act, W, group_size=G))
            d["out4"] = _np(lq.fakequant_matmul_int4(act, W, group_size=G))
        for k, v in d.items():
            cases[f"{name}/{k}"] = v

    # tests/test_quantize.py:11-13 make_weight shapes and seeds
    torch.manual_seed(0)
    add("tq_64x256", torch.randn(64, 256, dtype=torch.float16), 128)
    torch.manual_seed(0)
    add("tq_32x512", torch.randn(32, 512, dtype=torch.float16), 128)
    add("zeros_4x128", torch.zeros(4, 128, dtype=torch.float16), 128)
    W = torch.zeros(4, 256, dtype=torch.float16)
    W[0, :128] = 1.0
    add("group_axis", W, 128)                      # tests/test_quantize.py:48-56
    # round-half-even ties: absmax 127c (resp. 7c) with c a power of two makes
    # w / scale land exactly on .5
    c = 2.0 ** -6
    row8 = [127 * c] + [(i + 0.5) * c * (1 if i % 2 else -1) for i in range(127)]
    row4 = [7 * c] + [((i % 7) + 0.5) * c * (1 if i % 3 else -1) for i in range(127)]
    add("ties_i8", torch.tensor([row8], dtype=torch.float32), 128)
    add("ties_i4", torch.tensor([row4], dtype=torch.float32), 128)
    # tests/test_kernels.py:60-120 seeds, smaller N so the fixture stays small
    for M, K, N, G, seed in [(1, 2048, 24, 128, 1), (4, 2048, 24, 128, 1), (16, 512, 48, 128, 2),
                             (1, 2048, 24, 2048, 1), (3, 256, 40, 128, 2)]:
        torch.manual_seed(seed)
        act = torch.randn(M, K, dtype=torch.float16)
        Wk = torch.randn(N, K, dtype=torch.float16)
        add(f"tk_M{M}_K{K}_N{N}_G{G}", Wk, G, act, store_dq=K <= 512)
    # benchmark distribution (W ~ N(0, 0.02), act ~ N(0, 1)), per-output-channel
    torch.manual_seed(0)
    act = torch.randn(2, 2048, dtype=torch.float16)
    Wb = (torch.randn(16, 2048) * 0.02).half()
    add("bench_perchan", Wb, 2048, act, store_dq=False)
    # every code: random packed bytes / int8 codes with random positive fp16 scales
    g = torch.Generator().manual_seed(7)
    qb = torch.randint(0, 256, (16, 256), dtype=torch.uint8, generator=g)
    sb = (torch.rand(16, 4, generator=g) * 0.05 + 1e-3).half()
    cases["codes4/q"] = _np(qb)
    cases["codes4/s"] = _np(sb)
    cases["codes4/dq"] = _np(lq.dequantize_int4(qb, sb, 128))
    qi = torch.randint(-128, 128, (16, 512), dtype=torch.int8, generator=g)
    cases["codes8/q"] = _np(qi)
    cases["codes8/s"] = _np(sb)
    cases["codes8/dq"] = _np(lq.dequantize_int8(qi, sb, 128))
    return cases


TINY = dict(hidden_size=128, intermediate_size=256, num_hidden_layers=2, num_attention_heads=4,
            num_key_value_heads=2, head_dim=64, vocab_size=512, rms_norm_eps=1e-5,
            tie_word_embeddings=True, max_position_embeddings=256)


def llama_case(ref_root: str, bits: int, rope_scaling: dict | None, seed: int):
    from transformers import LlamaConfig, LlamaForCausalLM
    from liteweight.quantize import dequantize_int4, dequantize_int8
    from liteweight.quantlinear import QuantLinear
    from liteweight.serialize import swap_linears

    params = {"rope_type": "default", "rope_theta": 500000.0}
    if rope_scaling:
        params = dict(rope_scaling, rope_theta=500000.0)
    cfg = LlamaConfig(**TINY, rope_parameters=params)
    cfg._attn_implementation = "sdpa"
    torch.manual_seed(seed)
    model = LlamaForCausalLM(cfg)
    with torch.no_grad():   # non-trivial norm weights so the gamma multiply is exercised
        for name, p in model.named_parameters():
            if name.endswith("norm.weight"):
                p.copy_(1.0 + 0.1 * torch.randn_like(p))
    model = model.half().eval()
    swap_linears(model, group_size=128, bits=bits)

    def shim(self, x):   # liteweight/quantlinear.py:54-66 with the kernel replaced by its oracle
        shp = x.shape
        x = x.reshape(-1, self.in_features).to(torch.float16)
        deq = dequantize_int8 if self.bits == 8 else dequantize_int4
        w = deq(self.qweight, self.scales, self.group_size)
        out = x.float().mm(w.float().T).half()
        if self.bias is not None:
            out = out + self.bias
        return out.reshape(*shp[:-1], self.out_features)

    QuantLinear.forward = shim
    B, P, NEW = 2, 8, 6
    g = torch.Generator().manual_seed(seed + 100)
    prompt = torch.randint(0, cfg.vocab_size, (B, P), generator=g)
    logits_steps, tokens = [], []
    with torch.no_grad():
        out = model(prompt, use_cache=True)
        past = out.past_key_values
        logits = out.logits[:, -1, :]
        for _ in range(NEW):                       # liteweight/generate.py:106-124, batched
            logits_steps.append(_np(logits))
            nxt = logits.argmax(dim=-1)
            tokens.append(_np(nxt))
            out = model(nxt[:, None], past_key_values=past, use_cache=True)
            past = out.past_key_values
            logits = out.logits[:, -1, :]
    d = {
        "prompt": _np(prompt), "tokens": np.stack(tokens, 1), "logits": np.stack(logits_steps, 0),
        "bits": np.int64(bits), "group_size": np.int64(128),
        "inv_freq": _np(model.model.rotary_emb.inv_freq.float()),
        "attention_scaling": np.float64(model.model.rotary_emb.attention_scaling),
        "embed": _np(model.model.embed_tokens.weight), "norm": _np(model.model.norm.weight),
    }
    assert model.lm_head.weight.data_ptr() == model.model.embed_tokens.weight.data_ptr()  # tied
    for k, v in TINY.items():
        d[f"cfg/{k}"] = np.int64(v) if isinstance(v, (int, bool)) else np.float64(v)
    for i, layer in enumerate(model.model.layers):
        d[f"L{i}/in_norm"] = _np(layer.input_layernorm.weight)
        d[f"L{i}/post_norm"] = _np(layer.post_attention_layernorm.weight)
        mods = {"q": layer.self_attn.q_proj, "k": layer.self_attn.k_proj, "v": layer.self_attn.v_proj,
                "o": layer.self_attn.o_proj, "gate": layer.mlp.gate_proj, "up": layer.mlp.up_proj,
                "down": layer.mlp.down_proj}
        for n, m in mods.items():
            d[f"L{i}/{n}/qweight"] = _np(m.qweight)
            d[f"L{i}/{n}/scales"] = _np(m.scales)
    return d


def main(ref_root: str):
    sys.path.insert(0, ref_root)
    import liteweight.quantize as lq
    np.savez_compressed(OUT / "quant_golden.npz", **quant_cases(lq))
    np.savez_compressed(OUT / "llama_tiny_int8.npz", **llama_case(ref_root, 8, None, 11))
    llama3 = {"rope_type": "llama3", "factor": 32.0, "high_freq_factor": 4.0, "low_freq_factor": 1.0,
              "original_max_position_embeddings": 8192}
    np.savez_compressed(OUT / "llama_tiny_int4.npz", **llama_case(ref_root, 4, llama3, 12))
    for f in sorted(OUT.glob("*.npz")):
        print(f.name, f.stat().st_size)


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit("usage: python tests/golden/make_golden.py <reference-root>")
    main(sys.argv[1])
