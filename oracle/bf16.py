"""bf16 <-> fp32 conversions in numpy (round-to-nearest-even), for the CPU oracle."""

from __future__ import annotations

import numpy as np


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """Round fp32 values to bf16 (nearest, ties to even) and return the raw uint16 bits."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(np.isnan(x), np.uint16(0x7FC0), rounded)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def round_bf16(x: np.ndarray) -> np.ndarray:
    """fp32 values rounded to the nearest bf16 value (returned as fp32)."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))
