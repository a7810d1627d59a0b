"""bfloat16 bit helpers for the CPU oracle (test infrastructure only).

bf16 tensors are carried as ``uint16`` bit patterns so the oracle never depends
on a framework's bf16 arithmetic.
"""

from __future__ import annotations

import numpy as np


def to_f32(bits: np.ndarray) -> np.ndarray:
    """uint16 bf16 bit patterns -> float32 (exact)."""

    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def from_f32(values: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bits with round-to-nearest-even (NaN stays a quiet NaN)."""

    f = np.ascontiguousarray(values, dtype=np.float32)
    u = f.view(np.uint32).astype(np.uint64)
    rounded = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(f)
    if nan.any():
        rounded = rounded.copy()
        rounded[nan] = ((u[nan] >> 16) | 0x40).astype(np.uint16)
    return rounded


def from_f64(values: np.ndarray) -> np.ndarray:
    """float64 -> bf16 bits, rounding once (via exact float32 when representable)."""

    values = np.asarray(values, dtype=np.float64)
    # Two-step rounding f64->f32->bf16 can double-round; correct it explicitly.
    f32 = values.astype(np.float32)
    bits = from_f32(f32)
    back = to_f32(bits).astype(np.float64)
    # neighbouring candidates
    up = to_f32(bits + np.uint16(1)).astype(np.float64)
    down = to_f32(bits - np.uint16(1)).astype(np.float64)
    best = bits.copy()
    err = np.abs(back - values)
    for cand, cval in ((bits + np.uint16(1), up), (bits - np.uint16(1), down)):
        cerr = np.abs(cval - values)
        better = np.isfinite(cval) & (cerr < err)
        best[better] = cand[better]
        err = np.where(better, cerr, err)
    return best


def ordered(bits: np.ndarray) -> np.ndarray:
    """Map bf16 bits to integers whose difference counts representable steps."""

    b = np.asarray(bits, dtype=np.uint16).astype(np.int64)
    mag = b & 0x7FFF
    return np.where(b & 0x8000, -mag, mag)


def ulp_distance(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    return np.abs(ordered(a) - ordered(b))


def random_bf16(rng: np.random.Generator, shape, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    return from_f32((rng.standard_normal(shape) * std + mean).astype(np.float32))
