"""Dense non-causal attention on B200: the tcgen05/TMEM flash-attention kernel of libh3b.so.

``flash_attn_func`` takes FA4's ``[B, S, H, D]`` calling convention
(src/h3_flash/runtime/attention/dense_fa4.py:74-81, :145) and ``packed_attention``
reads Q/K/V in place from the packed-Ulysses receive buffer ``[S, hl, 3D]``
(the SDPA call at src/h3_flash/runtime/parallel/packed_ulysses.py:201-209), writing
the ``[S, hl, D]`` layout the output all-to-all sends.
"""

from __future__ import annotations

import ctypes
import math

import torch

from ..._torch import call, ptr, require_bf16, require_cuda, stream_of

HEAD_DIM = 128


def _check_view(name: str, t: torch.Tensor) -> None:
    if t.stride(-1) != 1:
        raise ValueError(f"{name}: head_dim must be contiguous")
    if t.data_ptr() % 16:
        raise ValueError(f"{name}: base address must be 16-byte aligned")


def attention_bshd(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                   softmax_scale: float | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """softmax(q k^T * scale) v for [B, S, H, D] views (any strides with a contiguous,
    16-byte aligned head_dim=128). Returns a [B, Sq, H, D] tensor."""

    op = "h3b attention"
    require_cuda(op, q, k, v)
    require_bf16(op, q, k, v)
    if q.dim() != 4 or k.dim() != 4 or v.dim() != 4:
        raise ValueError(f"{op}: expected [batch, seq, heads, head_dim] tensors")
    b, sq, h, d = q.shape
    if k.shape[0] != b or k.shape[2] != h or k.shape[3] != d or v.shape != k.shape:
        raise ValueError(f"{op}: q {tuple(q.shape)}, k {tuple(k.shape)}, v {tuple(v.shape)} disagree")
    if d != HEAD_DIM:
        raise RuntimeError(f"{op}: head_dim must be {HEAD_DIM}, got {d}")
    for name, t in (("q", q), ("k", k), ("v", v)):
        _check_view(name, t)
    if out is None:
        out = torch.empty((b, sq, h, d), dtype=q.dtype, device=q.device)
    _check_view("out", out)
    scale = float(softmax_scale) if softmax_scale is not None else 1.0 / math.sqrt(d)
    ws_bytes = workspace_bytes(b, sq, k.shape[1], h, d)
    # Scratch for the split tail (caller-owned: the C ABI never allocates).
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=q.device) if ws_bytes else None
    call("h3b_attention", ptr(out), ptr(q), ptr(k), ptr(v), b, sq, k.shape[1], h, d,
         q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
         v.stride(0), v.stride(1), v.stride(2), out.stride(0), out.stride(1), out.stride(2),
         scale, ptr(ws) if ws is not None else None, ws_bytes, stream_of(q))
    return out


def workspace_bytes(batch: int, seq_q: int, seq_k: int, heads: int, head_dim: int = HEAD_DIM) -> int:
    """Scratch bytes the attention call can use for this shape on the current device."""

    from ... import _lib

    value = ctypes.c_int64(0)
    _lib.check(_lib.load().h3b_attention_workspace_size(batch, seq_q, seq_k, heads, head_dim,
                                                         ctypes.byref(value)),
               "h3b_attention_workspace_size")
    return int(value.value)


def packed_attention(packed: torch.Tensor, head_dim: int = HEAD_DIM,
                     softmax_scale: float | None = None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Attention over the packed receive buffer ``[S, hl, 3*D]`` (q | k | v per head).
    Returns ``[S, hl, D]``."""

    if packed.dim() != 3 or packed.shape[-1] != 3 * head_dim:
        raise ValueError(f"packed attention expects [S, hl, 3*{head_dim}], got {tuple(packed.shape)}")
    if packed.stride(-1) != 1 or packed.stride(-2) != 3 * head_dim:
        packed = packed.contiguous()
    s, hl, _ = packed.shape
    q = packed[..., :head_dim].unsqueeze(0)
    k = packed[..., head_dim : 2 * head_dim].unsqueeze(0)
    v = packed[..., 2 * head_dim :].unsqueeze(0)
    if out is None:
        out = torch.empty((s, hl, head_dim), dtype=packed.dtype, device=packed.device)
    attention_bshd(q, k, v, softmax_scale, out=out.unsqueeze(0))
    return out


def flash_attn_func(q, k, v, softmax_scale=None, causal=False, **kwargs):
    """FA4-compatible entry (``flash_attn.cute.flash_attn_func``): [B, S, H, D] in and out.
    Only the dense non-causal forward used by H3 is provided."""

    if causal:
        raise RuntimeError("h3b attention implements dense (non-causal) attention only")
    unsupported = {key: value for key, value in kwargs.items() if value not in (None, False, 0, 0.0)}
    if unsupported:
        raise RuntimeError(f"h3b attention does not support {sorted(unsupported)}")
    return attention_bshd(q, k, v, softmax_scale)
