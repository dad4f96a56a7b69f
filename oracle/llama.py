"""numpy restatement of one Llama decode step over liteweight-quantized linears.

Test infrastructure only (see ``oracle/__init__.py``).

The reference's ``generate`` (liteweight/generate.py:62-126) drives the
third-party ``transformers`` ``LlamaForCausalLM`` (version 5.5.0 installed;
``transformers/models/llama/modeling_llama.py``) whose every ``nn.Linear``
except ``lm_head`` is a ``QuantLinear`` (liteweight/serialize.py:13-64). This
module restates that forward for one new token per sequence, rounding to
fp16 exactly where the fp16 HF model holds an fp16 tensor:

  * RMSNorm (modeling_llama.py:53-70): fp32 mean of squares, ``x * rsqrt(var +
    eps)`` in fp32, cast to fp16, then ``weight * x`` in fp16.
  * QuantLinear (liteweight/quantlinear.py:54-66): dequantize the packed
    weight (liteweight/quantize.py:30-43, :102-128), fp32 matmul, fp16 out,
    then ``+ bias`` in fp16.
  * RoPE (modeling_llama.py:124-167): ``freqs = inv_freq * pos`` in fp32,
    ``cos/sin`` of ``cat(freqs, freqs)`` cast to fp16, then
    ``q*cos + rotate_half(q)*sin`` with an fp16 rounding after each op.
  * Attention (modeling_llama.py:197-222, 255-289): GQA, scale hd**-0.5,
    fp32 softmax; output rounded to fp16.
  * Residual adds in fp16 (modeling_llama.py:320-335); SwiGLU
    ``down(silu(gate) * up)`` (modeling_llama.py:171-184) with silu and the
    product each rounded to fp16.
  * ``lm_head`` fp16 linear (fp32 accumulation) over the final norm
    (modeling_llama.py:429-500); greedy pick = first index of the max
    (liteweight/generate.py:49-52).
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

from oracle.quant import dequantize_int4, dequantize_int8

F32 = np.float32
F16 = np.float16


@dataclass
class LlamaShape:
    hidden: int
    inter: int
    n_layers: int
    n_heads: int
    n_kv_heads: int
    head_dim: int
    vocab: int
    eps: float = 1e-5
    rope_theta: float = 500000.0


@dataclass
class QLinear:
    """Packed weight of one QuantLinear (liteweight/quantlinear.py:34-52)."""
    qweight: np.ndarray
    scales: np.ndarray
    bits: int
    group_size: int
    bias: np.ndarray | None = None
    _w: np.ndarray | None = field(default=None, repr=False)

    def dequantized(self, cache: bool = True) -> np.ndarray:
        if self._w is not None:
            return self._w
        if self.bits == 8:
            w = dequantize_int8(self.qweight, self.scales, self.group_size)
        else:
            w = dequantize_int4(self.qweight, self.scales, self.group_size)
        w = w.astype(F32)
        if cache:
            self._w = w
        return w

    def __call__(self, x: np.ndarray, cache: bool = True) -> np.ndarray:
        out = (x.astype(F32) @ self.dequantized(cache).T).astype(F16)
        if self.bias is not None:
            out = (out.astype(F32) + self.bias.astype(F32)).astype(F16)
        return out


@dataclass
class LlamaLayer:
    in_norm: np.ndarray
    post_norm: np.ndarray
    q: QLinear
    k: QLinear
    v: QLinear
    o: QLinear
    gate: QLinear
    up: QLinear
    down: QLinear


@dataclass
class LlamaWeights:
    shape: LlamaShape
    embed: np.ndarray            # fp16 [V, H]
    layers: list
    norm: np.ndarray             # fp16 [H]
    lm_head: np.ndarray          # fp16 [V, H] (the tied embedding for Llama-3.2-1B)
    inv_freq: np.ndarray         # fp32 [hd/2] (the model's rotary buffer)
    attention_scaling: float = 1.0


def f16(x) -> np.ndarray:
    return np.asarray(x).astype(F16)


def rmsnorm(x: np.ndarray, weight: np.ndarray, eps: float) -> np.ndarray:
    """modeling_llama.py:63-68."""
    xf = x.astype(F32)
    var = (xf * xf).mean(axis=-1, keepdims=True, dtype=F32)
    xn = (xf * (F32(1.0) / np.sqrt(var + F32(eps)))).astype(F16)
    return (weight.astype(F32) * xn.astype(F32)).astype(F16)


def rope_tables(inv_freq: np.ndarray, positions: np.ndarray, scaling: float = 1.0):
    """modeling_llama.py:124-136: fp32 cos/sin of cat(freqs, freqs), cast to fp16."""
    freqs = positions.astype(F32)[:, None] * inv_freq.astype(F32)[None, :]
    emb = np.concatenate([freqs, freqs], axis=-1)
    cos = (np.cos(emb) * F32(scaling)).astype(F16)
    sin = (np.sin(emb) * F32(scaling)).astype(F16)
    return cos, sin


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """modeling_llama.py:138-167 with fp16 rounding after each elementwise op.

    x fp16 [..., hd]; cos/sin fp16 broadcastable to x.
    """
    h = x.shape[-1] // 2
    rot = np.concatenate([-x[..., h:], x[..., :h]], axis=-1)
    a = (x.astype(F32) * cos.astype(F32)).astype(F16)
    b = (rot.astype(F32) * sin.astype(F32)).astype(F16)
    return (a.astype(F32) + b.astype(F32)).astype(F16)


def silu_f16(x: np.ndarray) -> np.ndarray:
    xf = x.astype(F32)
    return (xf / (F32(1.0) + np.exp(-xf))).astype(F16)


def attention(q: np.ndarray, kc: np.ndarray, vc: np.ndarray, length: int) -> np.ndarray:
    """GQA attention of one query per sequence over ``length`` cached positions.

    q [B, nh, hd] fp16; kc/vc [B, nkv, S, hd] fp16 -> [B, nh*hd] fp16.
    """
    b, nh, hd = q.shape
    nkv = kc.shape[1]
    rep = nh // nkv
    k = kc[:, :, :length].astype(F32)
    v = vc[:, :, :length].astype(F32)
    k = np.repeat(k, rep, axis=1)           # repeat_kv, modeling_llama.py:187-195
    v = np.repeat(v, rep, axis=1)
    s = np.einsum("bhd,bhsd->bhs", q.astype(F32), k) * F32(hd ** -0.5)
    s = s - s.max(axis=-1, keepdims=True)
    p = np.exp(s)
    p = p / p.sum(axis=-1, keepdims=True)
    o = np.einsum("bhs,bhsd->bhd", p, v)
    return o.astype(F16).reshape(b, nh * hd)


class KVState:
    """Preallocated per-layer K/V, laid out like liteweight/generate.py:22-25
    (``[B, n_kv, max_seq, hd]`` fp16)."""

    def __init__(self, shape: LlamaShape, batch: int, max_seq: int):
        dims = (batch, shape.n_kv_heads, max_seq, shape.head_dim)
        self.k = [np.zeros(dims, F16) for _ in range(shape.n_layers)]
        self.v = [np.zeros(dims, F16) for _ in range(shape.n_layers)]
        self.pos = 0


def decode_step(w: LlamaWeights, kv: KVState, tokens: np.ndarray, cache: bool = True) -> np.ndarray:
    """One token per sequence at position ``kv.pos``; returns fp16 logits [B, V]
    and advances ``kv.pos``."""
    s = w.shape
    b = tokens.shape[0]
    pos = kv.pos
    x = w.embed[tokens].astype(F16)                                  # [B, H]
    cos, sin = rope_tables(w.inv_freq, np.array([pos]), w.attention_scaling)
    for li, L in enumerate(w.layers):
        h = rmsnorm(x, L.in_norm, s.eps)
        q = L.q(h, cache).reshape(b, s.n_heads, s.head_dim)
        k = L.k(h, cache).reshape(b, s.n_kv_heads, s.head_dim)
        v = L.v(h, cache).reshape(b, s.n_kv_heads, s.head_dim)
        q = apply_rope(q, cos[0], sin[0])
        k = apply_rope(k, cos[0], sin[0])
        kv.k[li][:, :, pos] = k
        kv.v[li][:, :, pos] = v
        a = attention(q, kv.k[li], kv.v[li], pos + 1)
        o = L.o(a, cache)
        x = (x.astype(F32) + o.astype(F32)).astype(F16)
        h = rmsnorm(x, L.post_norm, s.eps)
        g = L.gate(h, cache)
        u = L.up(h, cache)
        act = (silu_f16(g).astype(F32) * u.astype(F32)).astype(F16)
        d = L.down(act, cache)
        x = (x.astype(F32) + d.astype(F32)).astype(F16)
    h = rmsnorm(x, w.norm, s.eps)
    logits = (h.astype(F32) @ w.lm_head.astype(F32).T).astype(F16)
    kv.pos = pos + 1
    return logits


def greedy(logits: np.ndarray) -> np.ndarray:
    """First index of the maximum per row (torch.argmax semantics)."""
    return np.argmax(logits.astype(F32), axis=-1)


def greedy_decode(w: LlamaWeights, prompt: np.ndarray, new_tokens: int, max_seq: int | None = None,
                  cache: bool = True):
    """Prefill token by token, then ``new_tokens`` greedy steps.

    prompt int [B, P]. Returns (generated int [B, new_tokens], list of fp16
    logits [B, V] for every step whose argmax was taken).
    """
    b, p = prompt.shape
    kv = KVState(w.shape, b, max_seq or (p + new_tokens))
    logits = None
    for i in range(p):
        logits = decode_step(w, kv, prompt[:, i], cache)
    out, all_logits = [], []
    for _ in range(new_tokens):
        all_logits.append(logits)
        nxt = greedy(logits)
        out.append(nxt)
        logits = decode_step(w, kv, nxt, cache)
    return np.stack(out, axis=1), all_logits


def from_fixture(d) -> LlamaWeights:
    """Build oracle weights from a ``tests/golden/llama_tiny_*.npz`` mapping."""
    cfg = {k[4:]: d[k] for k in d.keys() if k.startswith("cfg/")}
    shape = LlamaShape(hidden=int(cfg["hidden_size"]), inter=int(cfg["intermediate_size"]),
                       n_layers=int(cfg["num_hidden_layers"]), n_heads=int(cfg["num_attention_heads"]),
                       n_kv_heads=int(cfg["num_key_value_heads"]), head_dim=int(cfg["head_dim"]),
                       vocab=int(cfg["vocab_size"]), eps=float(cfg["rms_norm_eps"]))
    bits, g = int(d["bits"]), int(d["group_size"])
    layers = []
    for i in range(shape.n_layers):
        lin = {n: QLinear(d[f"L{i}/{n}/qweight"], d[f"L{i}/{n}/scales"], bits, g)
               for n in ("q", "k", "v", "o", "gate", "up", "down")}
        layers.append(LlamaLayer(in_norm=d[f"L{i}/in_norm"], post_norm=d[f"L{i}/post_norm"], **lin))
    lm_head = d["lm_head"] if "lm_head" in d else d["embed"]
    return LlamaWeights(shape=shape, embed=d["embed"], layers=layers, norm=d["norm"], lm_head=lm_head,
                        inv_freq=d["inv_freq"], attention_scaling=float(d["attention_scaling"]))


def teacher_forced_logits(w: LlamaWeights, prompt: np.ndarray, tokens: np.ndarray, cache: bool = True):
    """Logits [T, B, V] after the prompt and after each of the given tokens but
    the last: the logits a greedy decode that produced ``tokens`` saw."""
    b, p = prompt.shape
    t = tokens.shape[1]
    kv = KVState(w.shape, b, p + t)
    logits = None
    for i in range(p):
        logits = decode_step(w, kv, prompt[:, i], cache)
    out = [logits]
    for j in range(t - 1):
        logits = decode_step(w, kv, tokens[:, j], cache)
        out.append(logits)
    return np.stack(out, 0)
