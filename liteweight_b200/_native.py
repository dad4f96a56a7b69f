"""ctypes binding of the liteweight_b200 C ABI (include/liteweight_b200.h).

The library is ``liteweight_b200/_lib/liblw_b200.so``, built in-tree by
``liteweight_b200.build``. There is no fallback: if the library is missing
or fails to load, every op raises.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

_LIB_PATH = Path(__file__).resolve().parent / "_lib" / "liblw_b200.so"
_lock = threading.Lock()
_lib = None

c_int, c_void_p = ctypes.c_int, ctypes.c_void_p

# name -> argument types (all return int status unless listed in _RESTYPE)
_SIGNATURES: dict[str, list] = {
    "lw_status_string": [c_int],
    "lw_abi_version": [],
    "lw_launch_count": [],
    "lw_take_device_error": [],
    "lw_gemm_workspace_size": [c_int] * 4,
    "lw_gemm_w8a16": [c_void_p] * 5 + [c_int] * 4 + [c_void_p, ctypes.c_size_t, c_void_p],
    "lw_gemm_w4a16": [c_void_p] * 5 + [c_int] * 4 + [c_void_p, ctypes.c_size_t, c_void_p],
    "lw_gemm_f16": [c_void_p] * 3 + [c_int] * 3 + [c_void_p, ctypes.c_size_t, c_void_p],
    "lw_gemm_w4a16_noalloc": [c_void_p] * 5 + [c_int] * 4 + [c_void_p],
    "lw_gemm_f16_kn": [c_void_p] * 3 + [c_int] * 3 + [c_void_p],
    "lw_dequant_w8": [c_void_p] * 3 + [c_int] * 3 + [c_void_p],
    "lw_dequant_w4": [c_void_p] * 3 + [c_int] * 3 + [c_void_p],
    "lw_quantize_int8": [c_void_p, c_int, c_void_p, c_void_p] + [c_int] * 3 + [c_void_p],
    "lw_quantize_int4": [c_void_p, c_int, c_void_p, c_void_p] + [c_int] * 3 + [c_void_p],
}
_RESTYPE = {"lw_status_string": ctypes.c_char_p, "lw_launch_count": ctypes.c_ulonglong,
            "lw_gemm_workspace_size": ctypes.c_size_t}


class LiteweightError(RuntimeError):
    """A liteweight_b200 C-ABI call returned a non-zero status."""

    def __init__(self, fn: str, status: int, msg: str):
        super().__init__(f"{fn} failed: status {status} ({msg})")
        self.status = status


def library_path() -> Path:
    return Path(os.environ.get("LW_B200_LIB", _LIB_PATH))


def declared_symbols() -> list[str]:
    return list(_SIGNATURES)


def register(name: str, args: list, restype=c_int) -> None:
    """Declare another C-ABI function (used by modules that add entry points)."""
    _SIGNATURES[name] = args
    if restype is not c_int:
        _RESTYPE[name] = restype
    if _lib is not None:
        fn = getattr(_lib, name)
        fn.argtypes = args
        fn.restype = restype


def lib() -> ctypes.CDLL:
    """Load (once) and return the C library. Raises if it is not built."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = library_path()
            if not path.exists():
                raise RuntimeError(
                    f"liteweight_b200 CUDA library not found at {path}; build it with "
                    "`python -m liteweight_b200.build` (there is no CPU fallback)")
            handle = ctypes.CDLL(str(path), mode=ctypes.RTLD_LOCAL)
            for name, args in _SIGNATURES.items():
                fn = getattr(handle, name)
                fn.argtypes = args
                fn.restype = _RESTYPE.get(name, c_int)
            _lib = handle
    return _lib


def check(fn: str, status: int) -> None:
    if status != 0:
        msg = lib().lw_status_string(status).decode()
        raise LiteweightError(fn, status, msg)


def call(fn: str, *args) -> None:
    check(fn, getattr(lib(), fn)(*args))


def launch_count() -> int:
    """Kernels the library has enqueued so far (its own counter)."""
    return int(lib().lw_launch_count())


_workspaces: dict = {}
_retired: list = []
_unzeroed: set = set()   # workspaces allocated under stream capture, not yet zeroed


def workspace(device: torch.device, stream: int, nbytes: int) -> torch.Tensor:
    """Zero-initialised scratch for the matmul entry points, one per (device,
    stream) so concurrent streams never share it; grown on demand. The kernels
    leave it zeroed after every call.

    A workspace that is replaced by a larger one is never freed: a CUDA graph
    captured earlier holds its address (split-tile counters and partial-sum
    slots) and keeps writing there on every replay, so the memory must not go
    back to torch's allocator for another tensor to own. Growth is geometric,
    so the retired blocks add up to less than the live one."""
    key = (device.index, stream)
    ws = _workspaces.get(key)
    capturing = torch.cuda.is_current_stream_capturing()
    if ws is None or ws.numel() < nbytes:
        size = max(nbytes, 1 << 20, 2 * ws.numel() if ws is not None else 0)
        if ws is not None:
            _retired.append(ws)
        # Under stream capture the zero fill is recorded into the graph, not
        # run: the block is zeroed again by the first eager call after it.
        ws = torch.zeros(size, dtype=torch.uint8, device=device)
        _workspaces[key] = ws
        if capturing:
            _unzeroed.add(key)
        else:
            _unzeroed.discard(key)
    elif key in _unzeroed and not capturing:
        ws.zero_()
        _unzeroed.discard(key)
    return ws


def matmul_workspace(bits: int, M: int, N: int, K: int, device: torch.device, stream: int) -> tuple[int, int]:
    """(pointer, bytes) of a workspace large enough for this matmul."""
    need = int(lib().lw_gemm_workspace_size(bits, M, N, K))
    if need == 0:
        return 0, 0
    ws = workspace(device, stream, need)
    return ws.data_ptr(), ws.numel()


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream_of(t: torch.Tensor) -> int:
    """Handle of torch's current CUDA stream on ``t``'s device."""
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise RuntimeError("liteweight_b200 ops run on CUDA tensors only (no CPU fallback); "
                               f"got a tensor on {t.device}")
