"""The decode line's parity checker (bench.py TorchDecodeReference) restates
the same arithmetic as the pinned numpy oracle: on a tiny random model its
teacher-forced logits agree with oracle.llama within the row-scaled tolerance
and pick the same greedy tokens. Runs on the CPU."""

import numpy as np
import torch

import bench
from liteweight_b200 import engine as E
from oracle import llama as ol
from oracle import quant as oq


class _TinyWorkload:
    def __init__(self, bits):
        self.spec = E.LlamaSpec(hidden=128, inter=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=32,
                                vocab=512, bits=bits, group_size=32)
        self.dev = torch.device("cpu")
        self.torch = torch
        g = torch.Generator().manual_seed(5)
        self.embed = (torch.randn(self.spec.vocab, self.spec.hidden, generator=g) * 0.5).half()
        self.norm = (1.0 + 0.1 * torch.randn(self.spec.hidden, generator=g)).half()
        self.inv_freq = E.default_inv_freq(self.spec.head_dim, self.spec.rope_theta)
        self.cos, self.sin = E.rope_tables(self.inv_freq, 64, 1.0, "cpu")
        self.lm_quant = None

    def layer_weights(self, li):
        return E.synthetic_layers(E.LlamaSpec(**{**self.spec.__dict__, "n_layers": 1}), self.dev, seed=1000 + li,
                                  std=0.1)[0]


def _oracle_weights(wl):
    sp = wl.spec
    layers = []
    for li in range(sp.n_layers):
        L = wl.layer_weights(li)
        lin = {n: ol.QLinear(getattr(L, n)[0].numpy(), getattr(L, n)[1].numpy(), sp.bits, sp.group_size)
               for n in ("q", "k", "v", "o", "gate", "up", "down")}
        layers.append(ol.LlamaLayer(in_norm=L.in_norm.numpy(), post_norm=L.post_norm.numpy(), **lin))
    shape = ol.LlamaShape(hidden=sp.hidden, inter=sp.inter, n_layers=sp.n_layers, n_heads=sp.n_heads,
                          n_kv_heads=sp.n_kv_heads, head_dim=sp.head_dim, vocab=sp.vocab, eps=sp.eps)
    return ol.LlamaWeights(shape=shape, embed=wl.embed.numpy(), layers=layers, norm=wl.norm.numpy(),
                           lm_head=wl.embed.numpy(), inv_freq=wl.inv_freq.numpy())


def test_torch_reference_matches_oracle():
    for bits in (4, 8):
        wl = _TinyWorkload(bits)
        rng = np.random.default_rng(bits)
        prompt = rng.integers(0, wl.spec.vocab, (2, 7))
        toks = rng.integers(0, wl.spec.vocab, (2, 5))
        ref = ol.teacher_forced_logits(_oracle_weights(wl), prompt, toks).astype(np.float32)   # [T, B, V]
        allt = torch.from_numpy(np.concatenate([prompt, toks], axis=1)).long()
        got = bench.TorchDecodeReference(wl).logits(allt[:, :-1], prompt.shape[1] - 1, toks.shape[1])
        got = got.transpose(0, 1).numpy()                                                         # [T, B, V]
        tol = oq.row_tolerance(ref.reshape(-1, ref.shape[-1])).reshape(ref.shape[0], ref.shape[1], 1)
        assert np.all(np.abs(got - ref) <= tol), (bits, float((np.abs(got - ref) / tol).max()))
        assert (got.argmax(-1) == ref.argmax(-1)).mean() >= 0.9
