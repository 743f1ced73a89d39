"""bf16 / fp16 helpers for the oracle (numpy has no bf16 dtype).

bf16 values are carried as uint16 bit patterns; arithmetic happens in float32
and results are rounded to nearest-even, which is what torch does after every
16-bit elementwise op (compute in fp32, round the output).
"""
from __future__ import annotations

import numpy as np


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Round float32 -> bf16 bits, nearest-even (NaN kept quiet)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32)
    nan = np.isnan(x)
    r = ((u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) >> np.uint32(16)).astype(np.uint16)
    if nan.any():
        r = np.where(nan, ((u >> np.uint32(16)) | np.uint32(0x40)).astype(np.uint16), r)
    return r


def round_bf16(x: np.ndarray) -> np.ndarray:
    return bf16_to_f32(f32_to_bf16(x))


def f16_to_f32(bits: np.ndarray) -> np.ndarray:
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def f32_to_f16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).view(np.uint16)


def round_f16(x: np.ndarray) -> np.ndarray:
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


DECODE = {"bf16": bf16_to_f32, "f16": f16_to_f32}
ENCODE = {"bf16": f32_to_bf16, "f16": f32_to_f16}
ROUND = {"bf16": round_bf16, "f16": round_f16, "f32": lambda x: np.asarray(x, np.float32)}
