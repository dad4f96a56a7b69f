"""Model surgery and the safetensors packed-weight format (liteweight/serialize.py:1-140).

Format v1, unchanged: ``<path>`` holds ``{module}.qweight``, ``{module}.scales``
and (when present) ``{module}.bias`` for every QuantLinear, and
``<path>.meta.json`` holds ``{"format_version": 1, "bits", "group_size",
"skip", "layers": {name: {"in", "out", "has_bias"}}}``.
"""

from __future__ import annotations

import json
from pathlib import Path

import torch
import torch.nn as nn
from safetensors.torch import load_file, save_file

from liteweight_b200.quantlinear import QuantLinear

FORMAT_VERSION = 1


def swap_linears(model: nn.Module, group_size: int = 128, bits: int = 8,
                 skip: tuple[str, ...] = ("lm_head",)) -> nn.Module:
    """Recursively replace nn.Linear -> QuantLinear, quantizing the live weights."""
    _swap_children(model, group_size, bits, skip, quantize=True)
    return model


def swap_linears_empty(model: nn.Module, group_size: int = 128, bits: int = 8,
                       skip: tuple[str, ...] = ("lm_head",)) -> nn.Module:
    """Recursively replace nn.Linear -> zero-filled QuantLinear (before load_quantized)."""
    _swap_children(model, group_size, bits, skip, quantize=False)
    return model


def _swap_children(module: nn.Module, group_size: int, bits: int, skip: tuple[str, ...], quantize: bool) -> None:
    # Children are replaced through their parent (setattr), matching the name-based
    # skip of serialize.py:47-64: a Linear named in `skip` at any depth is kept.
    for name, child in list(module.named_children()):
        if isinstance(child, nn.Linear) and name not in skip:
            if quantize:
                new = QuantLinear.from_linear(child, group_size, bits)
            else:
                new = QuantLinear(child.in_features, child.out_features, group_size=group_size, bits=bits,
                                  bias=child.bias is not None)
            setattr(module, name, new)
        else:
            _swap_children(child, group_size, bits, skip, quantize)


def save_quantized(model: nn.Module, out_path: str | Path, group_size: int = 128, bits: int = 8,
                   skip: tuple[str, ...] = ("lm_head",)) -> None:
    """Quantize (if no QuantLinear yet) and write <out_path> + <out_path>.meta.json."""
    out_path = Path(out_path)
    if not any(isinstance(m, QuantLinear) for m in model.modules()):
        model = swap_linears(model, group_size=group_size, bits=bits, skip=skip)
    tensors: dict[str, torch.Tensor] = {}
    layers: dict[str, dict] = {}
    for name, module in model.named_modules():
        if isinstance(module, QuantLinear):
            tensors[f"{name}.qweight"] = module.qweight.cpu()
            tensors[f"{name}.scales"] = module.scales.cpu()
            if module.bias is not None:
                tensors[f"{name}.bias"] = module.bias.cpu()
            layers[name] = {"in": module.in_features, "out": module.out_features,
                            "has_bias": module.bias is not None}
    save_file(tensors, out_path)
    meta = {"format_version": FORMAT_VERSION, "bits": bits, "group_size": group_size, "skip": list(skip),
            "layers": layers}
    Path(str(out_path) + ".meta.json").write_text(json.dumps(meta, indent=2))


def load_quantized(model: nn.Module, path: str | Path) -> nn.Module:
    """Rebuild the QuantLinear tree from <path>.meta.json and copy the tensors by name."""
    path = Path(path)
    meta = json.loads(Path(str(path) + ".meta.json").read_text())
    if meta["format_version"] != FORMAT_VERSION:
        raise ValueError(f"Unknown format version: {meta['format_version']}")
    model = swap_linears_empty(model, group_size=meta["group_size"], bits=meta["bits"], skip=tuple(meta["skip"]))
    tensors = load_file(path)
    for name, module in model.named_modules():
        if isinstance(module, QuantLinear):
            module.qweight.copy_(tensors[f"{name}.qweight"])
            module.scales.copy_(tensors[f"{name}.scales"])
            if module.bias is not None:
                module.bias.copy_(tensors[f"{name}.bias"])
    return model
