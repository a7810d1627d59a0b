"""Dense non-causal softmax attention on the CPU (test infrastructure only).

Restates the SDPA call of src/h3_flash/runtime/parallel/packed_ulysses.py:201-209
(scale 1/sqrt(D), no mask, no dropout) with fp32 (default) or fp64 accumulation,
processed in query blocks so long sequences stay within memory.
"""

from __future__ import annotations

import numpy as np

from .bf16 import to_f32


def attention(q, k, v, scale=None, dtype=np.float32, block=1024):
    """q: [Sq, H, D], k/v: [Sk, H, D] float arrays (or bf16 bits as uint16).
    Returns [Sq, H, D] in ``dtype``."""

    def f(a):
        a = np.asarray(a)
        return (to_f32(a) if a.dtype == np.uint16 else a).astype(dtype)

    q, k, v = f(q), f(k), f(v)
    sq, h, d = q.shape
    if scale is None:
        scale = 1.0 / np.sqrt(d)
    out = np.empty((sq, h, d), dtype=dtype)
    kt = np.ascontiguousarray(k.transpose(1, 2, 0))  # [H, D, Sk]
    vh = np.ascontiguousarray(v.transpose(1, 0, 2))  # [H, Sk, D]
    for start in range(0, sq, block):
        qb = q[start : start + block].transpose(1, 0, 2)  # [H, b, D]
        s = np.matmul(qb, kt) * dtype(scale)  # [H, b, Sk]
        s -= s.max(axis=-1, keepdims=True)
        np.exp(s, out=s)
        denom = s.sum(axis=-1, keepdims=True)
        o = np.matmul(s, vh) / denom  # [H, b, D]
        out[start : start + block] = o.transpose(1, 0, 2)
    return out


def error_metrics(actual: np.ndarray, reference: np.ndarray) -> dict[str, float]:
    """kernels/transformer.py:16-29: max_abs, mean_abs, relative_l2, cosine."""

    a = np.asarray(actual, dtype=np.float64).reshape(-1)
    r = np.asarray(reference, dtype=np.float64).reshape(-1)
    delta = np.abs(a - r)
    denom = max(np.linalg.norm(r), 1e-12)
    cos = float(np.dot(a, r) / max(np.linalg.norm(a) * np.linalg.norm(r), 1e-30))
    return {
        "max_abs": float(delta.max()) if delta.size else 0.0,
        "mean_abs": float(delta.mean()) if delta.size else 0.0,
        "relative_l2": float(np.linalg.norm(delta) / denom),
        "cosine": cos,
    }
