"""bf16 / fp16 rounding helpers for the oracle (numpy, round-to-nearest-even).

These emulate the storage precision of the device path so that the oracle can be run either
in pure float32 or with the same storage points rounded to bf16 as the CUDA kernels.
"""
from __future__ import annotations

import numpy as np


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bf16 value (ties to even); returns float32.

    NaN stays NaN; infinities stay infinite.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    lsb = (u >> 16) & 1
    r = (u + 0x7FFF + lsb) & 0xFFFF0000
    out = r.astype(np.uint32).view(np.float32)
    nan = np.isnan(x)
    if nan.any():
        out = out.copy()
        out[nan] = np.nan
    return out


def f32_to_bf16_bits(x: np.ndarray) -> np.ndarray:
    """float32 -> uint16 bf16 bit patterns (round to nearest even)."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def fp16_round(x: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest fp16 value; returns float32."""
    return np.asarray(x, dtype=np.float32).astype(np.float16).astype(np.float32)


def round_to(x: np.ndarray, dtype: str | None) -> np.ndarray:
    """Round to the storage dtype named by ``dtype`` ('bf16', 'fp16' or None for fp32)."""
    if dtype is None or dtype == "fp32":
        return np.asarray(x, dtype=np.float32)
    if dtype == "bf16":
        return bf16_round(x)
    if dtype == "fp16":
        return fp16_round(x)
    raise ValueError(f"unknown dtype {dtype!r}")
