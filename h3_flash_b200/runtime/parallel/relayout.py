"""Bit-exact packed-Ulysses relayouts on sm_100a.

Drop-in for ``h3_flash.runtime.parallel.relayout`` (src/h3_flash/runtime/parallel/relayout.py).
``pack_qkv_destination_major`` and ``merge_heads`` run as CUDA copy kernels in
libh3b.so. ``pack_qkv_reference`` is kept with the reference's name and
semantics as the framework-level permute-copy definition of the layout; the
packed all-to-all of this package never selects it (CUDA tensors go through the
kernel, anything else is rejected).

On the block's hot path neither standalone relayout runs: the pack is fused
into the QK-norm+RoPE kernel (``fused_qknorm_rope_pack``) and the merge runs
once on the all-to-all output.
"""

from __future__ import annotations

import torch

from ..._torch import call, ptr, require_cuda, stream_of


def can_pack_qkv(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor) -> bool:
    """Same predicate as relayout.py:70-78: CUDA, 3-D, equal shapes/dtypes, unit last stride."""

    return (
        q.is_cuda
        and q.ndim == 3
        and q.shape == k.shape == v.shape
        and q.dtype == k.dtype == v.dtype
        and q.stride(-1) == k.stride(-1) == v.stride(-1) == 1
    )


def pack_qkv_reference(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, world: int) -> torch.Tensor:
    """Permute-copy definition of the destination-major layout (relayout.py:81-94)."""

    rows, heads, head_dim = q.shape
    if heads % world:
        raise ValueError(f"heads ({heads}) must divide Ulysses degree ({world})")
    heads_local = heads // world
    output = torch.empty((world, rows, heads_local, 3 * head_dim), dtype=q.dtype, device=q.device)
    for index, tensor in enumerate((q, k, v)):
        shards = tensor.reshape(rows, world, heads_local, head_dim).permute(1, 0, 2, 3)
        output[..., index * head_dim : (index + 1) * head_dim].copy_(shards)
    return output


def pack_qkv_destination_major(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, world: int) -> torch.Tensor:
    """out[dst, row, h, 0:D|D:2D|2D:3D] = (q|k|v)[row, dst*hl+h, :] in one CUDA pass
    (relayout.py:97-130). Values are moved, never rounded."""

    rows, heads, head_dim = q.shape
    if heads % world:
        raise ValueError(f"heads ({heads}) must divide Ulysses degree ({world})")
    if not can_pack_qkv(q, k, v):
        require_cuda("pack_qkv_destination_major", q, k, v)
        raise ValueError("pack_qkv_destination_major: q, k, v need equal shapes/dtypes and unit last stride")
    if q.element_size() != 2:
        raise TypeError("pack_qkv_destination_major: 16-bit tensors expected")
    heads_local = heads // world
    output = torch.empty((world, rows, heads_local, 3 * head_dim), dtype=q.dtype, device=q.device)
    call("h3b_pack_qkv", ptr(output), ptr(q), ptr(k), ptr(v), rows, heads, head_dim, world,
         q.stride(0), q.stride(1), k.stride(0), k.stride(1), v.stride(0), v.stride(1),
         stream_of(q))
    return output


def merge_heads(x: torch.Tensor) -> torch.Tensor:
    """[world, rows, hl, D] -> [rows, world*hl, D]: swap the source-rank and row dims
    without changing any value (relayout.py:133-159)."""

    world, rows, heads_local, head_dim = x.shape
    require_cuda("merge_heads", x)
    if x.element_size() != 2:
        raise TypeError("merge_heads: 16-bit tensors expected")
    x = x.contiguous()
    output = torch.empty((rows, world, heads_local, head_dim), dtype=x.dtype, device=x.device)
    call("h3b_merge_heads", ptr(output), ptr(x), world, rows, heads_local * head_dim, stream_of(x))
    return output.reshape(rows, world * heads_local, head_dim)
