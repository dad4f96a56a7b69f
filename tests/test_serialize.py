"""Save -> load round trip of the safetensors format (mirrors liteweight
tests/test_serialize.py), plus byte-level compatibility of the tensor names,
dtypes and meta JSON with the reference's format v1 (serialize.py:67-140)."""

import json
import tempfile
from pathlib import Path

import pytest
import torch
import torch.nn as nn
from safetensors.torch import load_file

from liteweight_b200.quantize import dequantize_int8, quantize_int8
from liteweight_b200.quantlinear import QuantLinear
from liteweight_b200.serialize import load_quantized, save_quantized, swap_linears


class TinyModel(nn.Module):
    def __init__(self):
        super().__init__()
        self.fc1 = nn.Linear(256, 512, bias=False)
        self.fc2 = nn.Linear(512, 256, bias=True)
        self.lm_head = nn.Linear(256, 128, bias=False)


class Nested(nn.Module):
    def __init__(self):
        super().__init__()
        self.block = nn.Sequential(nn.Linear(128, 256), nn.ReLU(), nn.Linear(256, 128))
        self.lm_head = nn.Linear(128, 64, bias=False)


def make_model():
    torch.manual_seed(42)
    return TinyModel().eval()


def test_basic_roundtrip():
    model = make_model()
    W_orig = model.fc1.weight.data.half().clone()
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "model.safetensors"
        save_quantized(model, path, group_size=128, bits=8)
        fresh = load_quantized(make_model(), path)
        assert isinstance(fresh.fc1, QuantLinear) and isinstance(fresh.fc2, QuantLinear)
        assert isinstance(fresh.lm_head, nn.Linear)
        q, s = quantize_int8(W_orig, 128)
        assert torch.equal(dequantize_int8(fresh.fc1.qweight, fresh.fc1.scales), dequantize_int8(q, s))


def test_meta_json_content():
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "model.safetensors"
        save_quantized(make_model(), path, group_size=128, bits=8)
        meta = json.loads(Path(str(path) + ".meta.json").read_text())
        assert meta == {"format_version": 1, "bits": 8, "group_size": 128, "skip": ["lm_head"],
                        "layers": {"fc1": {"in": 256, "out": 512, "has_bias": False},
                                   "fc2": {"in": 512, "out": 256, "has_bias": True}}}


def test_tensor_names_and_dtypes():
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "model.safetensors"
        save_quantized(make_model(), path, group_size=128, bits=4)
        t = load_file(path)
        assert sorted(t) == ["fc1.qweight", "fc1.scales", "fc2.bias", "fc2.qweight", "fc2.scales"]
        assert t["fc1.qweight"].dtype == torch.uint8 and t["fc1.qweight"].shape == (512, 128)
        assert t["fc1.scales"].dtype == torch.float16 and t["fc1.scales"].shape == (512, 2)
        assert t["fc2.bias"].dtype == torch.float16


def test_bias_preserved():
    model = make_model()
    bias = model.fc2.bias.data.clone()
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "model.safetensors"
        save_quantized(model, path, group_size=128, bits=8)
        fresh = load_quantized(make_model(), path)
        assert torch.allclose(fresh.fc2.bias, bias.half(), atol=1e-4)


def test_unknown_format_version_raises():
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "model.safetensors"
        save_quantized(make_model(), path)
        mp = Path(str(path) + ".meta.json")
        meta = json.loads(mp.read_text())
        meta["format_version"] = 99
        mp.write_text(json.dumps(meta))
        with pytest.raises(ValueError, match="Unknown format version"):
            load_quantized(make_model(), path)


@pytest.mark.parametrize("bits", [8, 4])
def test_bits_roundtrip(bits):
    with tempfile.TemporaryDirectory() as d:
        path = Path(d) / "model.safetensors"
        save_quantized(make_model(), path, group_size=128, bits=bits)
        fresh = load_quantized(make_model(), path)
        assert isinstance(fresh.fc1, QuantLinear) and fresh.fc1.bits == bits


def test_nested_skip_by_name():
    m = swap_linears(Nested(), group_size=128, bits=8)
    assert isinstance(m.block[0], QuantLinear) and isinstance(m.block[2], QuantLinear)
    assert isinstance(m.lm_head, nn.Linear)


def test_forward_refuses_cpu():
    ql = QuantLinear(128, 64, bits=8)
    with pytest.raises(RuntimeError, match="no CPU fallback"):
        ql(torch.zeros(1, 128, dtype=torch.float16))
