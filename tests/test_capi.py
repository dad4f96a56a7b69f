"""The C-ABI library loads and exports every symbol include/liteweight_b200.h declares.

Runs without a GPU: only argument validation paths are exercised (they
return before any CUDA call).
"""

import ctypes
import re
from pathlib import Path

import pytest

from liteweight_b200 import _native as nat
from liteweight_b200 import build as lwbuild

INCLUDE = Path(__file__).resolve().parent.parent / "include"


def header_functions() -> list[str]:
    names = set()
    for h in INCLUDE.glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(lw_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


@pytest.fixture(scope="module")
def lib():
    lwbuild.build()
    import liteweight_b200.engine  # noqa: F401  (registers the engine entry points)
    return nat.lib()


def test_header_declares_functions():
    names = header_functions()
    assert "lw_gemm_w8a16" in names and "lw_gemm_w4a16" in names and "lw_gemm_f16" in names


def test_every_declared_symbol_is_exported(lib):
    handle = ctypes.CDLL(str(nat.library_path()))
    for name in header_functions():
        assert hasattr(handle, name), f"{name} declared in the header but not exported"


def test_binding_covers_header(lib):
    assert set(header_functions()) <= set(nat.declared_symbols())


def test_version_and_status_strings(lib):
    assert lib.lw_abi_version() >= 100
    assert lib.lw_status_string(0) == b"ok"
    assert lib.lw_status_string(3) == b"bad group size"
    assert lib.lw_status_string(999) == b"unknown status"


@pytest.mark.parametrize("fn", ["lw_gemm_w8a16", "lw_gemm_w4a16"])
def test_quant_gemm_argument_validation(lib, fn):
    f = getattr(lib, fn)
    fake = 0x1000   # never dereferenced: validation fails first
    assert f(None, fake, fake, None, fake, 1, 64, 256, 128, None, 0, None) == 1          # null act
    assert f(fake, fake, fake, None, fake, 0, 64, 256, 128, None, 0, None) == 2          # M = 0
    assert f(fake, fake, fake, None, fake, 1, 64, 256, 100, None, 0, None) == 3          # K % G
    assert f(fake, fake, fake, None, fake, 1, 64, 256, 0, None, 0, None) == 3            # G = 0
    assert f(fake, fake, None, None, fake, 1, 64, 256, 128, None, 0, None) == 1          # null scales
    assert f(fake + 1, fake, fake, None, fake, 1, 64, 256, 128, None, 0, None) == 4      # odd fp16 pointer
    assert f(fake, fake, fake, None, fake, 1, 64, 256, 128, None, 4096, None) == 7       # bytes without pointer
    assert f(fake, fake, fake, None, fake, 1, 64, 256, 128, fake + 16, 4096, None) == 4  # unaligned workspace


def test_int4_odd_k_rejected(lib):
    fake = 0x1000
    assert lib.lw_gemm_w4a16(fake, fake, fake, None, fake, 1, 8, 255, 255, None, 0, None) == 2


def test_error_becomes_exception(lib):
    with pytest.raises(nat.LiteweightError, match="bad group size"):
        nat.call("lw_gemm_w8a16", 0x1000, 0x1000, 0x1000, None, 0x1000, 1, 64, 256, 100, None, 0, None)
