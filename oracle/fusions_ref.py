"""CPU restatement of the fused elementwise ops (test infrastructure only).

Inputs/outputs are bf16 bit patterns (uint16 arrays); cos/sin tables float32.
The reference fusions compute in fp32 and round once when storing; these
functions do the same, in the order the reference kernels write it, so a
correct GPU kernel lands within 1 bf16 ulp (the reduction order of the row sum
is the only freedom). The benchmark-only ops without a reference kernel
(modulate, gated residual, GELU-tanh) are evaluated in float64 and rounded once.
"""

from __future__ import annotations

import numpy as np

from .bf16 import from_f32, from_f64, to_f32


def _store(values: np.ndarray, rounding: str) -> np.ndarray:
    """fp32 -> bf16 bits. "rne" is what a GPU store does (cvt.rn); "trunc" is what the
    Triton CPU interpreter does (it drops the low 16 bits), used to pin this oracle
    bit-exactly against golden vectors recorded from the reference kernels."""

    values = np.ascontiguousarray(values, dtype=np.float32)
    if rounding == "rne":
        return from_f32(values)
    if rounding == "trunc":
        return (values.view(np.uint32) >> 16).astype(np.uint16)
    raise ValueError(f"unknown rounding {rounding!r}")


def _rows(bits: np.ndarray) -> np.ndarray:
    return to_f32(bits).reshape(-1, bits.shape[-1])


def _table_rows(table: np.ndarray, index: np.ndarray, n_rows: int) -> np.ndarray:
    """Row r reads table row index[r % len(index)] (fusions.py:45-46, :88)."""

    t = to_f32(table)
    if t.ndim == 1:
        t = t[None, :]
    idx = np.asarray(index, dtype=np.int64).reshape(-1)
    rows = idx[np.arange(n_rows) % idx.size]
    return t[rows]


def rmsnorm_modulate(x, weight, scale, shift, index, eps, rounding="rne"):
    """src/h3_flash/runtime/kernels/fusions.py:69-96 (_rmsnorm_modulate_kernel)."""

    value = _rows(x)
    n = value.shape[-1]
    variance = np.sum(value * value, axis=-1, dtype=np.float32) / np.float32(n)
    rstd = (np.float32(1.0) / np.sqrt(variance + np.float32(eps))).astype(np.float32)
    normed = value * rstd[:, None]
    w = to_f32(weight)[None, :]
    sc = _table_rows(scale, index, value.shape[0])
    sh = _table_rows(shift, index, value.shape[0])
    out = normed * w * (np.float32(1.0) + sc) + sh
    return _store(out, rounding).reshape(x.shape)


def residual_gate_rmsnorm_modulate(
    residual, branch, gate, weight, scale, shift, index, eps, rounding="rne"
):
    """fusions.py:23-67: hidden stored, norm of the fp32 hidden (not the rounded store)."""

    res = _rows(residual)
    br = _rows(branch)
    g = _table_rows(gate, index, res.shape[0])
    hidden = (res + g * br).astype(np.float32)
    n = hidden.shape[-1]
    variance = np.sum(hidden * hidden, axis=-1, dtype=np.float32) / np.float32(n)
    rstd = (np.float32(1.0) / np.sqrt(variance + np.float32(eps))).astype(np.float32)
    normed = hidden * rstd[:, None] * to_f32(weight)[None, :]
    sc = _table_rows(scale, index, res.shape[0])
    sh = _table_rows(shift, index, res.shape[0])
    out = normed * (np.float32(1.0) + sc) + sh
    return (
        _store(hidden, rounding).reshape(residual.shape),
        _store(out, rounding).reshape(residual.shape),
    )


def swiglu(x, rounding="rne"):
    """fusions.py:98-123: value first, gate second, out = value * (gate * sigmoid(gate)),
    fp32 with sigmoid(g) = 1 / (1 + exp(-g))."""

    v = to_f32(x)
    n = v.shape[-1] // 2
    value, gate = v[..., :n], v[..., n:]
    with np.errstate(over="ignore"):
        sig = np.float32(1.0) / (np.float32(1.0) + np.exp(-gate))
    out = value * (gate * sig)
    return _store(out, rounding)


def qknorm_rope(x, weight, cos, sin, eps, rounding="rne"):
    """fusions.py:125-175: per-head RMSNorm * weight, then rotate-half RoPE on the
    first rotary_dim columns (first half takes -partner), pass-through above.
    x: [B, S, H, D] bf16 bits; cos/sin: float32 [S, rotary_dim]."""

    b, s, h, d = x.shape
    rot = cos.shape[-1]
    if rot > d or rot % 2:
        raise ValueError(
            "fused qknorm+rope requires an even rotary dimension no wider "
            f"than the head, got rotary_dim={rot}, head_dim={d}"
        )
    value = to_f32(x).reshape(b, s, h, d)
    variance = np.sum(value * value, axis=-1, dtype=np.float32) / np.float32(d)
    rstd = (np.float32(1.0) / np.sqrt(variance + np.float32(eps))).astype(np.float32)
    normed = value * rstd[..., None] * to_f32(weight)
    out = normed.copy()
    if rot:
        half = rot // 2
        c = np.asarray(cos, dtype=np.float32)[None, :, None, :]
        sn = np.asarray(sin, dtype=np.float32)[None, :, None, :]
        partner = np.concatenate([-normed[..., half:rot], normed[..., :half]], axis=-1)
        out[..., :rot] = normed[..., :rot] * c + partner * sn
    return _store(out, rounding)


def modulate(x, scale, shift, index):
    """x * (1 + scale[idx]) + shift[idx] (kernels/transformer.py:72-74 without the norm)."""

    value = to_f32(x).reshape(-1, x.shape[-1]).astype(np.float64)
    sc = _table_rows(scale, index, value.shape[0]).astype(np.float64)
    sh = _table_rows(shift, index, value.shape[0]).astype(np.float64)
    return from_f64(value * (1.0 + sc) + sh).reshape(x.shape)


def gated_residual(residual, branch, gate, index):
    """residual + gate[idx] * branch (kernels/transformer.py:123-126)."""

    res = to_f32(residual).reshape(-1, residual.shape[-1]).astype(np.float64)
    br = to_f32(branch).reshape(-1, branch.shape[-1]).astype(np.float64)
    g = _table_rows(gate, index, res.shape[0]).astype(np.float64)
    return from_f64(res + g * br).reshape(residual.shape)


def gelu_tanh(x):
    """torch.nn.functional.gelu(x, approximate="tanh") = 0.5 x (1 + tanh(u)),
    u = sqrt(2/pi)(x + 0.044715 x^3), evaluated in float64 as the identical
    x * sigmoid(2u) = x / (1 + exp(-2u)), which has no cancellation for x << 0."""

    v = to_f32(x).astype(np.float64)
    u = np.sqrt(2.0 / np.pi) * (v + 0.044715 * v**3)
    with np.errstate(over="ignore"):
        out = v / (1.0 + np.exp(-2.0 * u))
    return from_f64(out)
