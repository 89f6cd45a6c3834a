"""bfloat16 <-> float32 on uint16 bit patterns (numpy has no bfloat16).

float32 -> bfloat16 rounds to nearest, ties to even (the rounding torch uses
for ``.to(torch.bfloat16)``), by the usual integer method: add 0x7FFF plus the
lowest kept bit, then truncate.  NaNs map to the quiet NaN 0x7FC0.
"""
from __future__ import annotations

import numpy as np


def bf16_to_f32(u16: np.ndarray) -> np.ndarray:
    return (np.asarray(u16, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    rounded = ((u + np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1))) >> 16).astype(np.uint16)
    nan = np.isnan(np.asarray(x, dtype=np.float32))
    return np.where(nan, np.uint16(0x7FC0), rounded)


def round_to_bf16(x: np.ndarray) -> np.ndarray:
    """float32 values rounded through bfloat16 (returned as float32)."""
    return bf16_to_f32(f32_to_bf16(x))
