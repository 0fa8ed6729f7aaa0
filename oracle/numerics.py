"""Exact scalar conversions used by the oracle (test infrastructure only; see oracle/__init__.py)."""
from __future__ import annotations

import numpy as np


def f32_to_bf16_bits(x) -> np.ndarray:
    """fp32 -> bf16 bit pattern, round to nearest even; NaN -> 0x7FC0 (torch's .to(bfloat16))."""
    x = np.asarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    nan = np.isnan(x)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    r = np.where(nan, 0x7FC0, r)
    return r.astype(np.uint16)


def bf16_bits_to_f32(b) -> np.ndarray:
    b = np.asarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def bf16_round(x) -> np.ndarray:
    """Round fp32 values to bf16 and back (one RNE rounding)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))


def f64_to_bf16_bits(v) -> np.ndarray:
    """fp64 -> bf16 with one RNE rounding (subnormals included): quantum 2^(max(e, -126) - 7)."""
    v = np.asarray(v, dtype=np.float64)
    a = np.abs(v)
    _, ex = np.frexp(a)  # a = m * 2^ex with 0.5 <= m < 1, so the binade exponent is ex - 1
    e = np.where(a > 0, ex - 1, -100000)
    qe = np.maximum(e, -126) - 7
    r = np.rint(np.ldexp(v, -qe)) * np.ldexp(1.0, qe)
    f = r.astype(np.float32)
    bits = (f.view(np.uint32) >> 16).astype(np.uint16)
    return np.where(np.isnan(v), np.uint16(0x7FC0), bits).astype(np.uint16)


def fp8e4m3_to_f32(b) -> np.ndarray:
    """FP8 e4m3fn byte -> fp32 (0x7F / 0xFF are NaN, no infinities)."""
    b = np.asarray(b, dtype=np.uint8).astype(np.int64)
    s = np.where(b & 0x80, -1.0, 1.0)
    e = (b >> 3) & 0xF
    m = b & 7
    val = np.where(e == 0, m * 2.0 ** -9, (1.0 + m / 8.0) * np.ldexp(1.0, (e - 7).astype(np.int64)))
    val = np.where((e == 0xF) & (m == 7), np.nan, val)
    return (s * val).astype(np.float32)


def f32(x) -> np.ndarray:
    return np.asarray(x, dtype=np.float32)
