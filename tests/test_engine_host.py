"""Host-side logic of the decode engine (CPU): weight packing orders,
tensor-parallel sharding, byte accounting and the C-ABI struct layout."""

import ctypes

import pytest
import torch

from liteweight_b200 import engine as E
from liteweight_b200 import build as lwbuild


def test_struct_layout_matches_library():
    lwbuild.build()
    E.check_abi()
    assert ctypes.sizeof(E.FusedGemvArgs) == 256 and ctypes.sizeof(E.AttentionArgs) == 72
    assert ctypes.sizeof(E.ExchangeOut) == 96 and ctypes.sizeof(E.ExchangeIn) == 56


@pytest.mark.parametrize("hd", [64, 128])
def test_rope_pair_order(hd):
    perm = E.rope_pair_order(3, hd, "cpu")
    assert sorted(perm.tolist()) == list(range(3 * hd))
    for tile in range(3 * hd // 16):
        rows = perm[tile * 16:(tile + 1) * 16]
        head = rows[0].item() // hd
        assert all(r.item() // hd == head for r in rows)          # a tile never straddles heads
        for g in range(8):
            assert rows[g + 8].item() - rows[g].item() == hd // 2  # rotate_half partners


def test_interleave8():
    a = torch.arange(32).reshape(16, 2)
    b = torch.arange(100, 132).reshape(16, 2)
    out = E.interleave8(a, b)
    assert torch.equal(out[0:8], a[0:8]) and torch.equal(out[8:16], b[0:8])
    assert torch.equal(out[16:24], a[8:16]) and torch.equal(out[24:32], b[8:16])


def _layer(spec, seed=0):
    g = torch.Generator().manual_seed(seed)
    lin = {}
    for name, n, k in spec.linear_shapes():
        kb = k // 2 if spec.bits == 4 else k
        q = torch.randint(0, 255, (n, kb), generator=g, dtype=torch.uint8)
        lin[name] = (q, torch.rand(n, k // spec.group_size, generator=g).half())
    return E.LayerWeights(in_norm=torch.ones(spec.hidden).half(), post_norm=torch.ones(spec.hidden).half(), **lin)


@pytest.mark.parametrize("tp", [1, 2, 4])
def test_tensor_parallel_shards_reassemble(tp):
    spec = E.LlamaSpec(hidden=256, inter=512, n_layers=1, n_heads=8, n_kv_heads=4, head_dim=64, vocab=1024, bits=4)
    lw = _layer(spec)
    packs = [E.PackedLayer(lw, spec, r, tp, "cpu") for r in range(tp)]
    # o / down: the column shards concatenate back to the full weight (packed bytes and scales)
    assert torch.equal(torch.cat([p.o_w for p in packs], 1), lw.o[0])
    assert torch.equal(torch.cat([p.d_s for p in packs], 1), lw.down[1])
    # q|k|v: inverting the rope-pair order of each shard gives back its q, k, v rows
    nq, nkv, hd = 8 // tp, 4 // tp, 64
    for r, p in enumerate(packs):
        inv_q = torch.argsort(E.rope_pair_order(nq, hd, "cpu"))
        q_rows = p.qkv_w[:nq * hd][inv_q]
        assert torch.equal(q_rows, lw.q[0][r * nq * hd:(r + 1) * nq * hd])
        inv_kv = torch.argsort(E.rope_pair_order(nkv, hd, "cpu"))
        v_rows = p.qkv_w[(nq + nkv) * hd:][inv_kv]
        assert torch.equal(v_rows, lw.v[0][r * nkv * hd:(r + 1) * nkv * hd])
        # gate|up interleave of this rank's intermediate slice
        i = 512 // tp
        assert torch.equal(p.gu_w[:8], lw.gate[0][r * i:r * i + 8])
        assert torch.equal(p.gu_w[8:16], lw.up[0][r * i:r * i + 8])


def test_bytes_per_token_match_the_plan():
    """Per-token bytes of the three decode configs (weights + fp16 scales + fp16 lm_head)."""
    b8 = E.LlamaSpec(**E.LLAMA_3_8B, bits=4).weight_bytes_per_token()
    b1 = E.LlamaSpec(**E.LLAMA_3_2_1B, bits=8).weight_bytes_per_token()
    b70 = E.LlamaSpec(**E.LLAMA_3_70B, bits=4).weight_bytes_per_token()
    assert abs(b8 / 1e9 - 4.650) < 0.01, b8
    assert abs(b1 / 1e9 - 1.514) < 0.01, b1
    assert abs(b70 / 1e9 - 37.40) < 0.05, b70


def test_exchange_flags():
    """Flags are never 0 (receive buffers start zeroed) and differ between the
    exchanges of a step and between consecutive steps."""
    tags = 65
    seen = {E.exchange_flag(s, t, tags) for s in range(3) for t in range(tags)}
    assert len(seen) == 3 * tags and 0 not in seen
    assert E.exchange_flag(0xFFFFFFFF // tags, tags - 1, tags) != 0


def test_prefill_rows_fit_shared_memory():
    """Prompt-chunk rows: the most the norm GEMVs (K=4096 -> 26) stage; the
    down_proj (8B INT4 K=14336 -> 7 rows) runs in row blocks at TP1 and bounds
    the chunk under tensor parallelism (K=7168 at TP2 -> 15)."""
    s8 = E.LlamaSpec(**E.LLAMA_3_8B, bits=4)
    assert [E.prefill_rows(s8, tp) for tp in (1, 2, 4, 8)] == [26, 15, 26, 26]
    assert [E.down_rows(s8, tp) for tp in (1, 2, 4)] == [7, 15, 31]
    s1 = E.LlamaSpec(**E.LLAMA_3_2_1B, bits=8)
    assert E.prefill_rows(s1) == 32 and E.down_rows(s1) == 13


def test_tc_supported_per_rank_shards():
    """The tensor-core prompt path takes a rank's shard when every shard's
    linear tiles (128-row weight tiles, K in 64-element blocks)."""
    from liteweight_b200 import engine as E
    spec = E.LlamaSpec(**E.LLAMA_3_8B, bits=4, group_size=128)
    assert all(E.tc_supported(spec, tp) for tp in (1, 2, 4, 8))
    odd = E.LlamaSpec(**{**E.LLAMA_3_8B, "inter": 14336 + 32}, bits=4, group_size=128)
    assert not E.tc_supported(odd, 1)
