"""Fused transformer elementwise ops of the H3 block, backed by sm_100a CUDA kernels.

Drop-in for ``h3_flash.runtime.kernels.fusions`` (src/h3_flash/runtime/kernels/fusions.py):
the same function names, arguments, return shapes and ownership rules (outputs
are fresh tensors, inputs are never mutated, non-contiguous activations are
copied). The reference's Triton kernels become calls into libh3b.so; there is
no CPU path, non-CUDA tensors raise.

Additional ops the benchmark block needs (no reference kernel): ``fused_modulate``,
``fused_gated_residual``, ``fused_gelu_tanh`` and ``fused_qknorm_rope_pack``
(QK-norm + RoPE fused with the packed-Ulysses destination-major pack).
"""

from __future__ import annotations

import torch

from ... import _lib
from ..._torch import (
    call,
    index64,
    ptr,
    require_bf16,
    require_cuda,
    rows_view,
    stream_of,
    table_rows,
)


def _available() -> bool:
    """Whether libh3b.so loads (or builds). A missing toolchain, a missing library
    and an ABI mismatch read as unavailable; the installers then raise."""

    try:
        _lib.load()
        return True
    except (OSError, RuntimeError):
        return False


# The reference exposes HAVE_TRITON; this build's kernels live in libh3b.so.
HAVE_CUDA_KERNELS = _available()


def fused_rmsnorm_modulate(x, weight, scale, shift, index, eps):
    """RMSNorm(x)*weight*(1+scale[idx])+shift[idx], idx = index[row % len(index)].
    Reference: fusions.py:194-215."""

    op = "fused_rmsnorm_modulate"
    require_cuda(op, x, weight, scale, shift)
    require_bf16(op, x, weight, scale, shift)
    columns = x.shape[-1]
    flat = rows_view(x)
    scale, scale_stride = table_rows(scale)
    shift, shift_stride = table_rows(shift)
    idx = index64(index, x.device)
    output = torch.empty(flat.shape, dtype=x.dtype, device=x.device)
    call(
        "h3b_rmsnorm_modulate", ptr(output), ptr(flat), ptr(weight.contiguous()), ptr(scale),
        ptr(shift), ptr(idx), flat.shape[0], columns, idx.numel(), flat.stride(0),
        output.stride(0), scale_stride, shift_stride, float(eps), stream_of(x),
    )
    return output.view(x.shape)


def fused_residual_gate_rmsnorm_modulate(residual, branch, gate, weight, scale, shift, index, eps):
    """hidden = residual + gate[idx]*branch; normed = RMSNorm(hidden)*weight*(1+scale)+shift.
    Returns (hidden, normed). Reference: fusions.py:218-248."""

    op = "fused_residual_gate_rmsnorm_modulate"
    require_cuda(op, residual, branch, gate, weight, scale, shift)
    require_bf16(op, residual, branch, gate, weight, scale, shift)
    columns = residual.shape[-1]
    residual_flat = residual.reshape(-1, columns).contiguous()
    branch_flat = branch.reshape(-1, columns).contiguous()
    if residual_flat.shape != branch_flat.shape:
        raise ValueError("residual and branch must have the same shape")
    gate, gate_stride = table_rows(gate)
    scale, scale_stride = table_rows(scale)
    shift, shift_stride = table_rows(shift)
    idx = index64(index, residual.device)
    hidden = torch.empty_like(residual_flat)
    normed = torch.empty_like(residual_flat)
    call(
        "h3b_residual_gate_rmsnorm_modulate", ptr(hidden), ptr(normed), ptr(residual_flat),
        ptr(branch_flat), ptr(weight.contiguous()), ptr(gate), ptr(scale), ptr(shift), ptr(idx),
        residual_flat.shape[0], columns, idx.numel(), residual_flat.stride(0), gate_stride,
        scale_stride, shift_stride, float(eps), stream_of(residual),
    )
    return hidden.view(residual.shape), normed.view(residual.shape)


def fused_swiglu(x):
    """out = x[..., :n] * silu(x[..., n:]), n = last/2 (value first, gate second).
    Reference: fusions.py:251-265."""

    op = "fused_swiglu"
    require_cuda(op, x)
    require_bf16(op, x)
    if x.shape[-1] % 2:
        raise ValueError("fused_swiglu needs an even last dimension")
    columns = x.shape[-1] // 2
    flat = rows_view(x)
    output = torch.empty(flat.shape[0], columns, dtype=x.dtype, device=x.device)
    call("h3b_swiglu", ptr(output), ptr(flat), flat.shape[0], columns, flat.stride(0),
         output.stride(0), stream_of(x))
    return output.view(*x.shape[:-1], columns)


def fused_qknorm_rope(x, weight, cos, sin, eps):
    """Per-head RMSNorm(x)*weight then rotate-half RoPE on the first rotary_dim columns.
    x: [B, S, H, D]; cos/sin: [S, rotary_dim]. Reference: fusions.py:268-293."""

    op = "fused_qknorm_rope"
    batch, sequence, heads, head_dim = x.shape
    rotary_dim = cos.shape[-1]
    if rotary_dim > head_dim or rotary_dim % 2:
        raise ValueError(
            "fused qknorm+rope requires an even rotary dimension no wider "
            f"than the head, got rotary_dim={rotary_dim}, head_dim={head_dim}"
        )
    require_cuda(op, x, weight, cos, sin)
    require_bf16(op, x, weight)
    flat = x.contiguous()
    cos32 = cos.to(torch.float32).contiguous()
    sin32 = sin.to(torch.float32).contiguous()
    output = torch.empty_like(flat)
    call("h3b_qknorm_rope", ptr(output), ptr(flat), ptr(weight.contiguous()), ptr(cos32),
         ptr(sin32), batch, sequence, heads, head_dim, rotary_dim, float(eps), stream_of(x))
    return output.view(batch, sequence, heads, head_dim)


def fused_modulate(x, scale, shift, index=None):
    """AdaLN modulate without the norm: x*(1+scale[idx])+shift[idx] (benchmark op).
    scale/shift are [d] vectors or [n_table, d] tables addressed through ``index``."""

    op = "fused_modulate"
    require_cuda(op, x, scale, shift)
    require_bf16(op, x, scale, shift)
    flat = rows_view(x)
    scale, scale_stride = table_rows(scale)
    shift, shift_stride = table_rows(shift)
    idx = index64(index, x.device)
    output = torch.empty(flat.shape, dtype=x.dtype, device=x.device)
    call("h3b_modulate", ptr(output), ptr(flat), ptr(scale), ptr(shift), ptr(idx), flat.shape[0],
         flat.shape[1], idx.numel(), flat.stride(0), output.stride(0), scale_stride,
         shift_stride, stream_of(x))
    return output.view(x.shape)


def fused_gated_residual(residual, branch, gate, index=None):
    """residual + gate[idx]*branch in one pass (the block's closing residual,
    kernels/transformer.py:123-126)."""

    op = "fused_gated_residual"
    require_cuda(op, residual, branch, gate)
    require_bf16(op, residual, branch, gate)
    columns = residual.shape[-1]
    residual_flat = residual.reshape(-1, columns).contiguous()
    branch_flat = branch.reshape(-1, columns).contiguous()
    if residual_flat.shape != branch_flat.shape:
        raise ValueError("residual and branch must have the same shape")
    gate, gate_stride = table_rows(gate)
    idx = index64(index, residual.device)
    output = torch.empty_like(residual_flat)
    call("h3b_gated_residual", ptr(output), ptr(residual_flat), ptr(branch_flat), ptr(gate),
         ptr(idx), residual_flat.shape[0], columns, idx.numel(), residual_flat.stride(0),
         gate_stride, stream_of(residual))
    return output.view(residual.shape)


def fused_gelu_tanh(x):
    """torch.nn.functional.gelu(x, approximate="tanh") in one bf16 pass."""

    op = "fused_gelu_tanh"
    require_cuda(op, x)
    require_bf16(op, x)
    flat = rows_view(x)
    output = torch.empty(flat.shape, dtype=x.dtype, device=x.device)
    call("h3b_gelu_tanh", ptr(output), ptr(flat), flat.shape[0], flat.shape[1], flat.stride(0),
         output.stride(0), stream_of(x))
    return output.view(x.shape)


def qknorm_rope_pack_args(op, q, k, v, q_weight, k_weight, cos, sin, world):
    """Checks shared by the packing ops; returns (rotary_dim, cos fp32, sin fp32)."""

    rows, heads, head_dim = q.shape
    if heads % world:
        raise ValueError(f"heads ({heads}) must divide Ulysses degree ({world})")
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError("q, k and v must have the same shape")
    require_cuda(op, q, k, v, q_weight, k_weight)
    require_bf16(op, q, k, v, q_weight, k_weight)
    for t in (q, k, v):
        if t.stride(-1) != 1 or t.stride(-2) != head_dim:
            raise ValueError(f"{op}: heads must be contiguous within a row")
    if cos is None:
        empty = torch.empty(0, dtype=torch.float32, device=q.device)
        return 0, empty, empty
    rotary_dim = cos.shape[-1]
    if rotary_dim > head_dim or rotary_dim % 2:
        raise ValueError(
            "fused qknorm+rope requires an even rotary dimension no wider "
            f"than the head, got rotary_dim={rotary_dim}, head_dim={head_dim}"
        )
    return rotary_dim, cos.to(torch.float32).contiguous(), sin.to(torch.float32).contiguous()


def fused_qknorm_rope_pack(q, k, v, q_weight, k_weight, cos, sin, world, q_eps, k_eps,
                           out=None):
    """QK-norm+RoPE of q and k fused with the packed-Ulysses destination-major pack.

    q, k, v: [rows, heads, head_dim] with contiguous heads inside a row (row stride
    free, e.g. views into one fused QKV projection). cos/sin: [rows, rotary_dim] or
    None (norm only). Returns [world, rows, heads/world, 3*head_dim] equal to
    ``pack_qkv_destination_major(fused_qknorm_rope(q), fused_qknorm_rope(k), v, world)``
    (src/h3_flash/runtime/parallel/packed_ulysses.py:178-200)."""

    op = "fused_qknorm_rope_pack"
    rotary_dim, cos32, sin32 = qknorm_rope_pack_args(op, q, k, v, q_weight, k_weight, cos, sin,
                                                     world)
    rows, heads, head_dim = q.shape
    hl = heads // world
    if out is None:
        out = torch.empty((world, rows, hl, 3 * head_dim), dtype=q.dtype, device=q.device)
    call("h3b_qknorm_rope_pack", ptr(out), ptr(q), ptr(k), ptr(v), q.stride(0), k.stride(0),
         v.stride(0), ptr(q_weight.contiguous()), ptr(k_weight.contiguous()), ptr(cos32),
         ptr(sin32), rows, heads, head_dim, rotary_dim, world, float(q_eps), float(k_eps),
         stream_of(q))
    return out


def qkv_gemm_pack_supported(x: torch.Tensor, weight: torch.Tensor, heads: int, head_dim: int,
                            cos: torch.Tensor | None) -> bool:
    """Whether ``fused_qkv_gemm_pack`` serves this projection: bf16 CUDA tensors,
    head_dim 128, an even head count, dim % 64 == 0, rotary_dim 0/64/96/128."""

    rot = 0 if cos is None else cos.shape[-1]
    return (x.is_cuda and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16
            and head_dim == 128 and heads % 2 == 0 and x.shape[-1] % 64 == 0
            and weight.shape == (3 * heads * head_dim, x.shape[-1]) and rot in (0, 64, 96, 128))


def qkv_gemm_pack_args(op, x, weight, bias, q_weight, k_weight, cos, sin, heads):
    """Checks shared by the GEMM packing ops; returns (x2d, weight, bias, rotary_dim, cos32,
    sin32, workspace): the workspace is the scratch the kernel relays the RoPE tables into
    (rows * rotary_dim * 8 bytes, None without RoPE)."""

    require_cuda(op, x, weight, q_weight, k_weight)
    require_bf16(op, x, weight, q_weight, k_weight)
    x2d = x.reshape(-1, x.shape[-1])
    if x2d.stride(-1) != 1 or x2d.stride(0) % 8 or x2d.data_ptr() % 16:
        x2d = x2d.contiguous()
    weight = weight.contiguous()
    if bias is not None:
        require_bf16(op, bias)
        bias = bias.contiguous()
    if cos is None:
        return x2d, weight, bias, 0, None, None, None
    rotary_dim = cos.shape[-1]
    cos32 = cos.to(torch.float32).contiguous()
    sin32 = sin.to(torch.float32).contiguous()
    if cos32.shape[0] != x2d.shape[0]:
        raise ValueError(f"{op}: rotary tables have {cos32.shape[0]} rows, x has {x2d.shape[0]}")
    workspace = torch.empty(2 * cos32.numel(), dtype=torch.float32, device=cos32.device)
    return x2d, weight, bias, rotary_dim, cos32, sin32, workspace


def fused_qkv_gemm_pack(x, weight, bias, q_weight, k_weight, cos, sin, heads, world, q_eps, k_eps,
                        out=None):
    """The QKV projection with QK-norm + RoPE + the destination-major pack in its
    epilogue (one tcgen05 GEMM). x [..., dim] (rows flattened), weight [3*heads*128, dim]
    (to_q | to_k | to_v stacked), bias [3*heads*128] or None. Returns
    [world, rows, heads/world, 3*128], the layout of ``fused_qknorm_rope_pack``, with the
    projection kept in fp32 up to the norm (src/h3_flash/runtime/parallel/packed_ulysses.py:166-200)."""

    op = "fused_qkv_gemm_pack"
    if heads % world:
        raise ValueError(f"heads ({heads}) must divide Ulysses degree ({world})")
    x2d, weight, bias, rotary_dim, cos32, sin32, workspace = qkv_gemm_pack_args(
        op, x, weight, bias, q_weight, k_weight, cos, sin, heads)
    rows, dim = x2d.shape
    if out is None:
        out = torch.empty((world, rows, heads // world, 3 * 128), dtype=x.dtype, device=x.device)
    if rows == 0:
        return out
    call("h3b_qkv_gemm_pack", ptr(out), world, ptr(x2d), rows, dim, x2d.stride(0), ptr(weight),
         ptr(bias) if bias is not None else None, ptr(q_weight.contiguous()),
         ptr(k_weight.contiguous()), ptr(cos32) if cos32 is not None else None,
         ptr(sin32) if sin32 is not None else None, heads, 128, rotary_dim, float(q_eps),
         float(k_eps), ptr(workspace) if workspace is not None else None,
         workspace.numel() * 4 if workspace is not None else 0, stream_of(x))
    return out


# ---------------------------------------------------------------------------
# GEMMs with the activation in the epilogue (h3b tcgen05 GEMM)
# ---------------------------------------------------------------------------

_ACTIVATIONS = {"none": 0, "gelu-tanh": 1}


def gemm_supported(x: torch.Tensor, weight: torch.Tensor, n_multiple: int = 256) -> bool:
    """Whether the h3b GEMM serves ``x @ weight.T``: bf16 CUDA tensors, a contiguous
    [n, dim] weight, dim % 64 == 0 and n % ``n_multiple`` == 0."""

    return (x.is_cuda and x.dtype == torch.bfloat16 and weight.dtype == torch.bfloat16
            and weight.dim() == 2 and weight.is_contiguous() and x.shape[-1] == weight.shape[1]
            and weight.shape[1] % 64 == 0 and weight.shape[0] % n_multiple == 0)


def _gemm_input(op: str, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None):
    require_cuda(op, x, weight)
    require_bf16(op, x, weight)
    x2d = x.reshape(-1, x.shape[-1])
    if x2d.stride(-1) != 1 or x2d.stride(0) % 8 or x2d.data_ptr() % 16:
        x2d = x2d.contiguous()
    if bias is not None:
        require_bf16(op, bias)
        bias = bias.contiguous()
    return x2d, weight.contiguous(), bias


def fused_linear(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None = None,
                 activation: str = "none", out: torch.Tensor | None = None) -> torch.Tensor:
    """``act(x @ weight.T + bias)`` as one h3b tcgen05 GEMM with the bias and the
    activation in its epilogue: the [rows, n] pre-activation is never stored, and it is
    not rounded to bf16 before the activation. ``activation``: "none" or "gelu-tanh"
    (the GELU-tanh FFN projection of src/h3_flash/runtime/kernels/transformer.py:121-122).
    x [..., dim], weight [n, dim] (nn.Linear layout), bias [n] or None."""

    op = "fused_linear"
    if activation not in _ACTIVATIONS:
        raise ValueError(f"{op}: activation must be one of {sorted(_ACTIVATIONS)}")
    x2d, weight, bias = _gemm_input(op, x, weight, bias)
    rows, n = x2d.shape[0], weight.shape[0]
    if out is None:
        out = torch.empty((rows, n), dtype=x.dtype, device=x.device)
    if rows:
        call("h3b_gemm", ptr(out), out.stride(0), ptr(x2d), rows, x2d.shape[1], x2d.stride(0), ptr(weight), n,
             ptr(bias) if bias is not None else None, _ACTIVATIONS[activation], stream_of(x))
    return out.view(*x.shape[:-1], n)


def interleave_swiglu(weight: torch.Tensor, bias: torch.Tensor | None = None):
    """The SwiGLU projection's weight [2n, dim] (value rows, then gate rows) and bias
    [2n] reordered for ``fused_linear_swiglu``: blocks of 128 value rows alternate with
    the matching 128 gate rows. Needs n % 128 == 0."""

    two_n, dim = weight.shape
    n = two_n // 2
    if two_n % 2 or n % 128:
        raise ValueError(f"interleave_swiglu: projection width {two_n} is not 2 x a multiple of 128")
    value, gate = weight.view(2, n // 128, 128, dim).unbind(0)
    w = torch.stack([value, gate], dim=1).reshape(two_n, dim).contiguous()
    b = None
    if bias is not None:
        bv, bg = bias.view(2, n // 128, 128).unbind(0)
        b = torch.stack([bv, bg], dim=1).reshape(two_n).contiguous()
    return w, b


def fused_linear_swiglu(x: torch.Tensor, weight_interleaved: torch.Tensor,
                        bias_interleaved: torch.Tensor | None = None,
                        out: torch.Tensor | None = None) -> torch.Tensor:
    """``fused_swiglu(x @ W.T + b)`` as one h3b GEMM (value * silu(gate) in its
    epilogue; src/h3_flash/runtime/kernels/transformer.py:112-115, fusions.py:251-265),
    with W and b given by ``interleave_swiglu``. Returns [..., n]."""

    op = "fused_linear_swiglu"
    x2d, w, b = _gemm_input(op, x, weight_interleaved, bias_interleaved)
    rows, n = x2d.shape[0], w.shape[0] // 2
    if out is None:
        out = torch.empty((rows, n), dtype=x.dtype, device=x.device)
    if rows:
        call("h3b_gemm_swiglu", ptr(out), out.stride(0), ptr(x2d), rows, x2d.shape[1], x2d.stride(0), ptr(w), n,
             ptr(b) if b is not None else None, stream_of(x))
    return out.view(*x.shape[:-1], n)


def fused_linear_gated_residual(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
                                residual: torch.Tensor, gate: torch.Tensor, index=None,
                                out: torch.Tensor | None = None) -> torch.Tensor:
    """``residual + gate[index] * (x @ weight.T + bias)`` as one h3b GEMM: the block's
    closing gated residual (src/h3_flash/runtime/kernels/transformer.py:123-126) in the
    epilogue of the FFN output projection (:120), the projection kept in fp32 up to the
    product. residual [..., n] like the output; gate [n_table, n] (rows picked by
    ``index[row % len(index)]``, all rows the first table row when ``index`` is None)."""

    op = "fused_linear_gated_residual"
    x2d, weight, bias = _gemm_input(op, x, weight, bias)
    require_cuda(op, residual, gate)
    require_bf16(op, residual, gate)
    rows, n = x2d.shape[0], weight.shape[0]
    res = residual.reshape(-1, n)
    if res.shape[0] != rows:
        raise ValueError(f"{op}: residual has {res.shape[0]} rows, x has {rows}")
    if res.stride(-1) != 1 or res.stride(0) % 8 or res.data_ptr() % 16:
        res = res.contiguous()
    table, table_stride = table_rows(gate)
    idx = index64(index, x.device)
    if out is None:
        out = torch.empty((rows, n), dtype=x.dtype, device=x.device)
    if rows:
        call("h3b_gemm_gated_residual", ptr(out), out.stride(0), ptr(x2d), rows, x2d.shape[1], x2d.stride(0),
             ptr(weight), n, ptr(bias) if bias is not None else None, ptr(res), res.stride(0), ptr(table),
             table_stride, ptr(idx), idx.numel(), stream_of(x))
    return out.view(*residual.shape[:-1], n)
