"""Install switchable, dense-preserving fused block forwards on an H3-style transformer.

Mirror of src/h3_flash/runtime/kernels/transformer.py. ``install_transformer_fusions``
patches ``block.forward`` (AdaLN/norm/FFN-activation fusions) and ``attn.forward``
(QK-norm+RoPE fused with the packed layout, h3b attention) of every block in
``transformer.transformer_blocks``. The first block records fused-vs-eager error
metrics in ``runtime["gate"]`` exactly as the reference does.

Block math (kernels/transformer.py:50-126):
  shift/scale/gate_msa, shift/scale/gate_mlp = adaln_proj(temb)      # tables [n_table, d]
  normed  = RMSNorm(h)*(1+scale_msa[idx]) + shift_msa[idx]            (fused_rmsnorm_modulate)
  a       = attn(normed, rotary_emb)
  h, normed = h + gate_msa[idx]*a, RMSNorm(h)*(1+scale_mlp)+shift_mlp  (fused_residual_gate_rmsnorm_modulate)
  f       = ff(normed)          # SwiGLU (H3) or GELU-tanh (benchmark) activation fused
  return h + gate_mlp[idx]*f                                           (fused_gated_residual)
"""

from __future__ import annotations

from typing import Any

import torch

from ..timing import TIMER
from .fusions import (
    HAVE_CUDA_KERNELS,
    fused_gated_residual,
    fused_gelu_tanh,
    fused_linear,
    fused_linear_gated_residual,
    fused_linear_swiglu,
    fused_residual_gate_rmsnorm_modulate,
    fused_rmsnorm_modulate,
    fused_swiglu,
    gemm_supported,
    interleave_swiglu,
)


def _error_metrics(actual: Any, reference: Any) -> dict[str, float]:
    """kernels/transformer.py:16-29."""

    from torch.nn import functional

    delta = (actual.float() - reference.float()).abs()
    return {
        "max_abs": float(delta.max()),
        "mean_abs": float(delta.mean()),
        "relative_l2": float(delta.norm() / reference.float().norm().clamp_min(1e-12)),
        "cosine": float(
            functional.cosine_similarity(actual.float().flatten(), reference.float().flatten(), dim=0)
        ),
    }


def _activation_kind(layer: Any, out_proj: Any) -> str | None:
    """'swiglu' for a value|gate projection followed by silu, 'gelu_tanh' for a tanh-GELU
    projection, None when the layer is something this package does not fuse."""

    proj = getattr(layer, "proj", None)
    if proj is None or not hasattr(proj, "out_features"):
        return None
    if getattr(layer, "approximate", None) == "tanh":
        return "gelu_tanh"
    activation = getattr(layer, "activation", None)
    in_features = getattr(out_proj, "in_features", None)
    if isinstance(activation, torch.nn.SiLU) and in_features is not None and proj.out_features == 2 * in_features:
        return "swiglu"
    return None


def _eager_activation(kind: str, projected: torch.Tensor) -> torch.Tensor:
    if kind == "swiglu":
        value, gate = projected.chunk(2, -1)
        return value * torch.nn.functional.silu(gate)
    return torch.nn.functional.gelu(projected, approximate="tanh")


def _swiglu_weights(act_layer: Any) -> tuple[torch.Tensor, torch.Tensor | None]:
    """The SwiGLU projection's weight and bias interleaved for ``fused_linear_swiglu``,
    cached on the layer and rebuilt when the weight or bias changes (in place or by
    reassignment)."""

    proj = act_layer.proj
    key = tuple((t.data_ptr(), t._version) if t is not None else None for t in (proj.weight, proj.bias))
    cached = getattr(act_layer, "_h3b_swiglu_interleaved", None)
    if cached is None or cached[0] != key:
        with torch.no_grad():
            cached = (key, *interleave_swiglu(proj.weight, proj.bias))
        act_layer._h3b_swiglu_interleaved = cached
    return cached[1], cached[2]


def _activated(ff: Any, normed: torch.Tensor, fuse_activation: bool, gate: dict | None,
               gemm_epilogue: bool) -> torch.Tensor | None:
    """The FFN's activated hidden [..., inner] through this package's kernels, or None
    for an FFN this package does not fuse. With ``gemm_epilogue`` the GELU-tanh or
    SwiGLU runs inside the projection GEMM (the h3b tcgen05 GEMM with the bias and the
    activation in its epilogue: the [rows, inner] pre-activation is never stored nor
    rounded to bf16 before the activation); shapes that GEMM does not serve, and
    ``gemm_epilogue=False``, take cuBLAS and then the h3b activation kernel."""

    act_layer, _, output_projection = ff.net
    kind = _activation_kind(act_layer, output_projection) if fuse_activation else None
    if kind is None:
        return None
    proj = act_layer.proj
    if gemm_epilogue and gemm_supported(normed, proj.weight):
        with TIMER.section("gemm"):
            if kind == "gelu_tanh":
                activated = fused_linear(normed, proj.weight, proj.bias, "gelu-tanh")
            else:
                activated = fused_linear_swiglu(normed, *_swiglu_weights(act_layer))
        name = f"{kind}_epilogue"
        if gate is not None and name not in gate:
            gate[name] = _error_metrics(activated, _eager_activation(kind, proj(normed)))
        return activated
    with TIMER.section("gemm"):
        projected = proj(normed)
    with TIMER.section("elementwise"):
        activated = fused_swiglu(projected) if kind == "swiglu" else fused_gelu_tanh(projected)
    if gate is not None and kind not in gate:
        gate[kind] = _error_metrics(activated, _eager_activation(kind, projected))
    return activated


def linear(layer: Any, x: torch.Tensor) -> torch.Tensor:
    """``layer(x)`` for an nn.Linear: the h3b tcgen05 GEMM (bias in its epilogue) where it
    serves the shape, else the layer itself (cuBLAS)."""

    if isinstance(layer, torch.nn.Linear) and gemm_supported(x, layer.weight):
        return fused_linear(x, layer.weight, layer.bias)
    return layer(x)


def feed_forward(ff: Any, normed: torch.Tensor, fuse_activation: bool, gate: dict | None = None,
                 gemm_epilogue: bool = False) -> torch.Tensor:
    """The FFN of one block (``block.ff``) with its activation fused as ``_activated``
    describes; the output projection on the h3b GEMM with ``gemm_epilogue``."""

    activated = _activated(ff, normed, fuse_activation, gate, gemm_epilogue)
    with TIMER.section("gemm"):
        if activated is None:
            return ff(normed)
        output_projection = ff.net[2]
        return linear(output_projection, activated) if gemm_epilogue else output_projection(activated)


def fused_block_forward(block: Any, hidden_states: torch.Tensor, temb: Any, adaln_indices: torch.Tensor,
                        rotary_emb: Any, attention_mask: Any = None, *, modulate: bool = True,
                        swiglu: bool = True, gate: dict | None = None,
                        gemm_epilogue: bool = False) -> torch.Tensor:
    """The patched ``block.forward`` body (kernels/transformer.py:40-126)."""

    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = block.adaln_proj(temb)
    if modulate:
        with TIMER.section("elementwise"):
            normed = fused_rmsnorm_modulate(hidden_states, block.norm1.weight, scale_msa, shift_msa,
                                            adaln_indices, block.norm1.eps)
        if gate is not None and "rmsnorm_modulate" not in gate:
            reference = block.norm1(hidden_states)
            reference = reference * (1.0 + scale_msa.index_select(0, adaln_indices)) + shift_msa.index_select(
                0, adaln_indices)
            gate["rmsnorm_modulate"] = _error_metrics(normed, reference)
    else:
        normed = block.norm1(hidden_states)
        normed = normed * (1.0 + scale_msa.index_select(0, adaln_indices)) + shift_msa.index_select(0, adaln_indices)
    attention_output = block.attn(normed, rotary_emb, attention_mask)
    residual_input = hidden_states
    if modulate:
        with TIMER.section("elementwise"):
            hidden_states, normed = fused_residual_gate_rmsnorm_modulate(
                residual_input, attention_output, gate_msa, block.norm2.weight, scale_mlp, shift_mlp,
                adaln_indices, block.norm2.eps)
        if gate is not None and "residual_chain" not in gate:
            reference_hidden = residual_input + gate_msa.index_select(0, adaln_indices) * attention_output
            reference_normed = block.norm2(reference_hidden)
            reference_normed = reference_normed * (1.0 + scale_mlp.index_select(0, adaln_indices)) + \
                shift_mlp.index_select(0, adaln_indices)
            gate["residual_output"] = _error_metrics(hidden_states, reference_hidden)
            gate["residual_chain"] = _error_metrics(normed, reference_normed)
    else:
        hidden_states = hidden_states + gate_msa.index_select(0, adaln_indices) * attention_output
        normed = block.norm2(hidden_states)
        normed = normed * (1.0 + scale_mlp.index_select(0, adaln_indices)) + shift_mlp.index_select(0, adaln_indices)
    if modulate and gemm_epilogue:
        # The closing gated residual in the epilogue of the FFN output projection.
        activated = _activated(block.ff, normed, swiglu, gate, gemm_epilogue)
        output_projection = block.ff.net[2] if activated is not None else None
        if output_projection is not None and isinstance(output_projection, torch.nn.Linear) and \
                gemm_supported(activated, output_projection.weight):
            with TIMER.section("gemm"):
                return fused_linear_gated_residual(activated, output_projection.weight, output_projection.bias,
                                                   hidden_states, gate_mlp, adaln_indices)
        with TIMER.section("gemm"):
            feed_forward_output = block.ff(normed) if activated is None else linear(output_projection, activated)
    else:
        feed_forward_output = feed_forward(block.ff, normed, swiglu, gate, gemm_epilogue)
    if modulate:
        with TIMER.section("elementwise"):
            return fused_gated_residual(hidden_states, feed_forward_output, gate_mlp, adaln_indices)
    return hidden_states + gate_mlp.index_select(0, adaln_indices) * feed_forward_output


def _patch_blocks(transformer: Any, modulate: bool, swiglu: bool, runtime: dict[str, Any]) -> None:
    gemm_epilogue = bool(runtime.get("gemm_epilogue", False))
    for block_index, block in enumerate(transformer.transformer_blocks):

        def forward(hidden_states, temb, adaln_indices, rotary_emb, attention_mask=None, *, block=block,
                    gate_this_block=block_index == 0):
            return fused_block_forward(
                block, hidden_states, temb, adaln_indices, rotary_emb, attention_mask,
                modulate=modulate, swiglu=swiglu, gate=runtime["gate"] if gate_this_block else None,
                gemm_epilogue=gemm_epilogue,
            )

        block.forward = forward


def _patch_attention(transformer: Any, runtime: dict[str, Any], gemm_pack: bool = True) -> None:
    """Single-device attention: fused QK-norm+RoPE (+ pack with W=1) and h3b attention.
    A later ``install_packed_ulysses`` replaces this with the W-rank exchange path."""

    from ..parallel.packed_ulysses import ulysses_attention_forward

    for block in transformer.transformer_blocks:
        attention = block.attn

        def forward(hidden_states, rotary_emb=None, attention_mask=None, *, attention=attention):
            return ulysses_attention_forward(attention, hidden_states, rotary_emb, attention_mask,
                                             gemm_pack=gemm_pack)

        attention.forward = forward


def install_transformer_fusions(transformer: Any, *, modulate: bool = True, swiglu: bool = True,
                                qknorm_rope: bool = True, gemm_epilogue: bool = True,
                                gemm_pack: bool = True) -> dict[str, Any]:
    """kernels/transformer.py:207-228. ``swiglu`` toggles the fused FFN activation
    (SwiGLU for H3, GELU-tanh for the benchmark block). ``gemm_epilogue`` runs the
    activation inside the FFN projection GEMM (the h3b tcgen05 GEMM's epilogue; SwiGLU
    on a weight whose value and gate rows are interleaved once and cached) instead of
    the h3b elementwise kernel after a cuBLAS GEMM.
    ``gemm_pack`` runs the QKV projection, QK-norm + RoPE and the pack as one
    h3b tcgen05 GEMM where the shapes allow it."""

    if not HAVE_CUDA_KERNELS:
        raise RuntimeError("H3 transformer fusions require the h3b CUDA extension (libh3b.so)")
    runtime = {
        "enabled": True,
        "modulate": modulate,
        "swiglu": swiglu,
        "qknorm_rope": qknorm_rope,
        "gemm_epilogue": gemm_epilogue,
        "gemm_pack": gemm_pack,
        "origin": "B200-native sm_100a kernels (h3b)",
        "gate": {},
    }
    if modulate or swiglu:
        _patch_blocks(transformer, modulate, swiglu, runtime)
    if qknorm_rope:
        _patch_attention(transformer, runtime, gemm_pack)
    return runtime
