"""numpy restatement of liteweight's quantization format and its matmul oracle.

Test infrastructure only (see ``oracle/__init__.py``). Every function cites
the reference line it restates (paths relative to the liteweight project).

Format recap (``liteweight/quantize.py``):
  * INT8: symmetric RTN per group of G consecutive K elements,
    scale = absmax / 127 computed in fp32, clamped to >= 1e-8, q = round-half-
    even(w / scale_fp32) clipped to [-127, 127]; the scale is *stored* as fp16
    (so q was computed with the unrounded fp32 scale).
  * INT4: same with 7 and [-8, 7]; two nibbles per byte, even K in the low
    nibble, odd K in the high nibble, two's complement.
  * Dequant: ``(q.float() * s.float()).half()`` - one fp16 rounding of an
    exact fp32 product.
  * Oracle matmul: ``act.float() @ w_dq.float().T`` in fp32, then ``.half()``.
"""

from __future__ import annotations

import numpy as np

F32 = np.float32
F16 = np.float16


def quantize_int8(weight: np.ndarray, group_size: int = 128):
    """liteweight/quantize.py:7-27. weight [N,K] fp16/fp32 -> (int8 [N,K], fp16 [N,K/G])."""
    assert weight.ndim == 2, "weight must be [N, K]"
    n, k = weight.shape
    assert k % group_size == 0, f"K={k} must be divisible by group_size={group_size}"
    w = weight.astype(F32).reshape(n, k // group_size, group_size)
    scale = np.abs(w).max(axis=-1, keepdims=True) / F32(127.0)      # :23
    scale = np.maximum(scale, F32(1e-8))                             # :24
    q = np.clip(np.round(w / scale), -127, 127).astype(np.int8)      # :25
    return q.reshape(n, k), scale.reshape(n, k // group_size).astype(F16)  # :27


def dequantize_int8(qweight: np.ndarray, scales: np.ndarray, group_size: int = 128) -> np.ndarray:
    """liteweight/quantize.py:30-43. -> fp16 [N,K]."""
    n, k = qweight.shape
    w = qweight.astype(F32).reshape(n, k // group_size, group_size)
    s = scales.astype(F32).reshape(n, k // group_size, 1)
    return (w * s).reshape(n, k).astype(F16)


def quantize_int4(weight: np.ndarray, group_size: int = 128):
    """liteweight/quantize.py:65-99. -> (uint8 [N,K/2] packed, fp16 [N,K/G])."""
    assert weight.ndim == 2, "weight must be [N, K]"
    n, k = weight.shape
    assert k % group_size == 0
    assert k % 2 == 0
    w = weight.astype(F32).reshape(n, k // group_size, group_size)
    scale = np.abs(w).max(axis=-1, keepdims=True) / F32(7.0)         # :86
    scale = np.maximum(scale, F32(1e-8))                             # :87
    q = np.clip(np.round(w / scale), -8, 7).astype(np.int8).reshape(n, k)  # :88
    return pack_int4(q), scale.reshape(n, k // group_size).astype(F16)


def pack_int4(q: np.ndarray) -> np.ndarray:
    """liteweight/quantize.py:90-97: even K -> low nibble, odd K -> high nibble."""
    lo = q[:, 0::2].astype(np.uint8) & 0x0F
    hi = (q[:, 1::2].astype(np.uint8) & 0x0F) << 4
    return (lo | hi).astype(np.uint8)


def unpack_int4(qweight: np.ndarray) -> np.ndarray:
    """liteweight/quantize.py:115-124: nibble split, 4-bit sign extension, interleave.

    Returns int8 [N, K] codes in [-8, 7].
    """
    n, kh = qweight.shape
    lo = (qweight & 0x0F).astype(np.int16)
    hi = (qweight >> 4).astype(np.int16)
    lo = np.where(lo >= 8, lo - 16, lo)   # same as int8 (x << 4) >> 4
    hi = np.where(hi >= 8, hi - 16, hi)
    out = np.empty((n, kh * 2), dtype=np.int8)
    out[:, 0::2] = lo
    out[:, 1::2] = hi
    return out


def dequantize_int4(qweight: np.ndarray, scales: np.ndarray, group_size: int = 128) -> np.ndarray:
    """liteweight/quantize.py:102-128. -> fp16 [N,K]."""
    n, kh = qweight.shape
    k = kh * 2
    w = unpack_int4(qweight).astype(F32).reshape(n, k // group_size, group_size)
    s = scales.astype(F32).reshape(n, k // group_size, 1)
    return (w * s).reshape(n, k).astype(F16)


def matmul_dequant(act: np.ndarray, w_dq: np.ndarray) -> np.ndarray:
    """liteweight/quantize.py:60 and :135: ``act.float().mm(w_dq.float().T).half()``."""
    return (act.astype(F32) @ w_dq.astype(F32).T).astype(F16)


def fakequant_matmul(act: np.ndarray, weight: np.ndarray, group_size: int = 128) -> np.ndarray:
    """liteweight/quantize.py:46-60 (INT8 oracle)."""
    q, s = quantize_int8(weight, group_size)
    return matmul_dequant(act, dequantize_int8(q, s, group_size))


def fakequant_matmul_int4(act: np.ndarray, weight: np.ndarray, group_size: int = 128) -> np.ndarray:
    """liteweight/quantize.py:131-135 (INT4 oracle)."""
    q, s = quantize_int4(weight, group_size)
    return matmul_dequant(act, dequantize_int4(q, s, group_size))


def packed_matmul(act: np.ndarray, qweight: np.ndarray, scales: np.ndarray,
                  group_size: int, bits: int) -> np.ndarray:
    """What ``kernels.matmul_int{8,4}`` must equal: dequantize the stored packed
    weights (liteweight/quantize.py:30-43 / :102-128), then the fp32 matmul of
    liteweight/quantize.py:60. act fp16 [M,K] -> fp16 [M,N]."""
    if bits == 8:
        w = dequantize_int8(qweight, scales, group_size)
    elif bits == 4:
        w = dequantize_int4(qweight, scales, group_size)
    else:
        raise ValueError(f"bits must be 4 or 8, got {bits}")
    return matmul_dequant(act, w)


def row_tolerance(ref: np.ndarray, rel: float = 1e-2) -> np.ndarray:
    """Per-row max-abs tolerance ``rel * ||ref[m,:]||_2 / sqrt(N)`` for an
    fp16 output ``ref`` [M,N] of an fp32-accumulated reference."""
    r = ref.astype(np.float64)
    n = r.shape[-1]
    return rel * np.sqrt((r * r).sum(axis=-1, keepdims=True)) / np.sqrt(n)
