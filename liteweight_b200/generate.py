"""Prefill + decode loop (liteweight/generate.py:1-126).

``generate`` keeps the reference's signature and result. For Llama-family
models it runs the native decode engine (liteweight_b200.engine): fused
sm_100a kernels over a preallocated KV cache, one CUDA graph per step, greedy
argmax on the device. Other models run the HF forward with the QuantLinear
kernels, as the reference does.
"""

from __future__ import annotations

import torch
from torch import Tensor


class KVCache:
    """Pre-allocated key/value cache for all transformer layers (generate.py:7-46).

    k[layer], v[layer]: fp16 [batch, n_kv_heads, max_seq, head_dim].
    """

    def __init__(self, n_layers: int, n_kv_heads: int, head_dim: int, max_seq: int, device: torch.device,
                 batch: int = 1):
        self.pos = 0
        shape = (batch, n_kv_heads, max_seq, head_dim)
        self.k = [torch.zeros(shape, dtype=torch.float16, device=device) for _ in range(n_layers)]
        self.v = [torch.zeros(shape, dtype=torch.float16, device=device) for _ in range(n_layers)]

    def append(self, layer: int, k: Tensor, v: Tensor) -> tuple[Tensor, Tensor]:
        """Write k, v [B, n_kv, new_len, hd] at ``pos``; return the valid [.., :pos+new_len, ..] slices."""
        new_len = k.shape[2]
        self.k[layer][:, :, self.pos:self.pos + new_len, :] = k
        self.v[layer][:, :, self.pos:self.pos + new_len, :] = v
        end = self.pos + new_len
        return self.k[layer][:, :, :end, :], self.v[layer][:, :, :end, :]

    def advance(self, n: int = 1) -> None:
        self.pos += n


def _sample(logits: Tensor, temperature: float, top_k: int | None) -> Tensor:
    """Next token id per row of logits [B, vocab] (generate.py:49-59)."""
    if temperature == 0.0:
        return logits.argmax(dim=-1)
    logits = logits / temperature
    if top_k is not None:
        v, _ = torch.topk(logits, min(top_k, logits.size(-1)))
        logits[logits < v[:, [-1]]] = float("-inf")
    probs = torch.softmax(logits.float(), dim=-1)
    return torch.multinomial(probs, num_samples=1).squeeze(-1)


def _eos_set(tokenizer) -> set[int]:
    eos_id = getattr(tokenizer, "eos_token_id", None)
    if eos_id is None:
        return set()
    return {eos_id} if isinstance(eos_id, int) else set(eos_id)


def generate(model: torch.nn.Module, tokenizer, prompt: str, max_new_tokens: int, temperature: float = 0.0,
             top_k: int | None = None) -> str:
    """Prefill + decode; returns the generated text (without the prompt)."""
    device = next(model.parameters()).device
    input_ids = tokenizer(prompt, return_tensors="pt").input_ids.to(device)
    eos_ids = _eos_set(tokenizer)
    from liteweight_b200 import engine as _engine
    if _engine.supports(model):
        ids = _engine.generate_ids(model, input_ids, max_new_tokens, temperature=temperature, top_k=top_k,
                                   eos_ids=eos_ids)
        return tokenizer.decode(ids[0], skip_special_tokens=True)
    return tokenizer.decode(_generate_hf(model, input_ids, max_new_tokens, temperature, top_k, eos_ids),
                            skip_special_tokens=True)


def _generate_hf(model, input_ids: Tensor, max_new_tokens: int, temperature: float, top_k: int | None,
                 eos_ids: set[int]) -> list[int]:
    """The reference loop (generate.py:97-124) over the HF forward."""
    with torch.no_grad():
        out = model(input_ids, use_cache=True)
    past_kv = out.past_key_values
    logits = out.logits[:, -1, :]
    generated: list[int] = []
    for _ in range(max_new_tokens):
        next_id = _sample(logits, temperature, top_k)
        token = next_id.item()
        if token in eos_ids:
            break
        generated.append(token)
        with torch.no_grad():
            out = model(next_id.unsqueeze(0), past_key_values=past_kv, use_cache=True)
        past_kv = out.past_key_values
        logits = out.logits[:, -1, :]
    return generated
