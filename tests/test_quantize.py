"""Quantization format of liteweight_b200 (mirrors liteweight tests/test_quantize.py)
plus bit-exactness against the reference's golden vectors and the oracle."""

import numpy as np
import pytest
import torch

from liteweight_b200.quantize import (dequantize_int4, dequantize_int8, fakequant_matmul, pack_int4,
                                      quantize_int4, quantize_int8, unpack_int4)
from oracle import quant as oq


def make_weight(N=64, K=256, seed=0):
    torch.manual_seed(seed)
    return torch.randn(N, K, dtype=torch.float16)


class TestInt8:
    def test_shapes(self):
        q, s = quantize_int8(make_weight(32, 128), group_size=128)
        assert q.shape == (32, 128) and q.dtype == torch.int8
        assert s.shape == (32, 1) and s.dtype == torch.float16

    def test_shapes_multigroup(self):
        q, s = quantize_int8(make_weight(32, 512), group_size=128)
        assert q.shape == (32, 512) and s.shape == (32, 4)

    def test_roundtrip_close(self):
        W = make_weight(64, 256)
        q, s = quantize_int8(W, group_size=128)
        assert (W - dequantize_int8(q, s, 128)).abs().max().item() < 0.05

    def test_zero_group_no_nan(self):
        q, s = quantize_int8(torch.zeros(4, 128, dtype=torch.float16), group_size=128)
        w = dequantize_int8(q, s, 128)
        assert not w.isnan().any() and not w.isinf().any()

    def test_group_axis_is_k(self):
        W = torch.zeros(4, 256, dtype=torch.float16)
        W[0, :128] = 1.0
        q, s = quantize_int8(W, group_size=128)
        assert s.shape == (4, 2) and s[0, 0].item() != pytest.approx(s[0, 1].item())

    def test_oracle_dtype(self):
        torch.manual_seed(1)
        out = fakequant_matmul(torch.randn(4, 256, dtype=torch.float16), torch.randn(32, 256, dtype=torch.float16))
        assert out.shape == (4, 32) and out.dtype == torch.float16 and not out.isnan().any()

    def test_k_not_multiple_of_group_raises(self):
        with pytest.raises(AssertionError):
            quantize_int8(make_weight(4, 200), group_size=128)


class TestInt4:
    def test_shapes(self):
        q, s = quantize_int4(make_weight(32, 256), group_size=128)
        assert q.shape == (32, 128) and q.dtype == torch.uint8 and s.shape == (32, 2)

    def test_roundtrip_bounded(self):
        W = make_weight(64, 256)
        q, s = quantize_int4(W, group_size=128)
        w = dequantize_int4(q, s, 128)
        assert w.shape == W.shape and not w.isnan().any()
        assert w.abs().max().item() < W.abs().max().item() * 2

    def test_pack_unpack_roundtrip(self):
        g = torch.Generator().manual_seed(3)
        codes = torch.randint(-8, 8, (8, 64), dtype=torch.int8, generator=g)
        assert torch.equal(unpack_int4(pack_int4(codes)), codes)

    def test_nibble_order(self):
        codes = torch.tensor([[1, -2, 7, -8]], dtype=torch.int8)
        assert pack_int4(codes).tolist() == [[0xE1, 0x87]]   # even k low nibble, two's complement


def test_bit_exact_vs_reference_golden(golden_dir):
    qg = dict(np.load(golden_dir / "quant_golden.npz"))
    names = sorted({k.split("/")[0] for k in qg if k.endswith("/W")})
    for name in names:
        W, G = torch.from_numpy(qg[f"{name}/W"]), int(qg[f"{name}/G"])
        q8, s8 = quantize_int8(W, G)
        q4, s4 = quantize_int4(W, G)
        assert np.array_equal(q8.numpy(), qg[f"{name}/q8"]), name
        assert np.array_equal(s8.numpy().view(np.uint16), qg[f"{name}/s8"].view(np.uint16)), name
        assert np.array_equal(q4.numpy(), qg[f"{name}/q4"]), name
        assert np.array_equal(s4.numpy().view(np.uint16), qg[f"{name}/s4"].view(np.uint16)), name
        if f"{name}/dq8" in qg:
            assert np.array_equal(dequantize_int8(q8, s8, G).numpy().view(np.uint16),
                                  qg[f"{name}/dq8"].view(np.uint16)), name
            assert np.array_equal(dequantize_int4(q4, s4, G).numpy().view(np.uint16),
                                  qg[f"{name}/dq4"].view(np.uint16)), name
    d4 = dequantize_int4(torch.from_numpy(qg["codes4/q"]), torch.from_numpy(qg["codes4/s"]), 128)
    assert np.array_equal(d4.numpy().view(np.uint16), qg["codes4/dq"].view(np.uint16))
    d8 = dequantize_int8(torch.from_numpy(qg["codes8/q"]), torch.from_numpy(qg["codes8/s"]), 128)
    assert np.array_equal(d8.numpy().view(np.uint16), qg["codes8/dq"].view(np.uint16))


@pytest.mark.parametrize("N,K,G", [(16, 2048, 2048), (24, 512, 128), (8, 256, 64)])
def test_matches_numpy_oracle(N, K, G):
    g = torch.Generator().manual_seed(N + K)
    W = (torch.randn(N, K, generator=g) * 0.02).half()
    q8, s8 = quantize_int8(W, G)
    r8, t8 = oq.quantize_int8(W.numpy(), G)
    assert np.array_equal(q8.numpy(), r8) and np.array_equal(s8.numpy(), t8)
    q4, s4 = quantize_int4(W, G)
    r4, t4 = oq.quantize_int4(W.numpy(), G)
    assert np.array_equal(q4.numpy(), r4) and np.array_equal(s4.numpy(), t4)
