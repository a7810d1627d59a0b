"""An H3-style DiT block stack with the attribute layout the installers patch.

The real MiniMax H3 transformer comes from a Diffusers checkout
(``transformer_minimax_h3``) that is not part of this package. This module
provides the same per-block structure, so the installers of this package can be
exercised and benchmarked without Diffusers:

  block.adaln_proj(temb) -> 6 tables [n_table, d]   (shift/scale/gate msa, shift/scale/gate mlp)
  block.norm1, block.norm2                          RMSNorm(d) (weight, eps)
  block.attn.{to_q,to_k,to_v,norm_q,norm_k,to_out,heads,head_dim,processor}
  block.ff.net = [activation-with-.proj, Dropout, Linear]   (GELU-tanh or SwiGLU)

Its own ``forward`` methods are the eager upstream-style math (what a model
looks like before ``install_transformer_fusions`` / ``install_packed_ulysses``
replace them); after installation every forward runs the h3b kernels.
``adaln_proj`` returns a stored table: the request-invariant AdaLN values that
the reference's invariant cache holds (src/h3_flash/runtime/cache/invariants.py:125-157).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F
from torch import nn


class RMSNorm(nn.Module):
    """Upstream-style RMSNorm: fp32 variance, bf16 rescale by the weight."""

    def __init__(self, dim: int, eps: float = 1e-6, **factory) -> None:
        super().__init__()
        self.eps = eps
        self.weight = nn.Parameter(torch.ones(dim, **factory))

    def forward(self, hidden_states: torch.Tensor) -> torch.Tensor:
        variance = hidden_states.to(torch.float32).pow(2).mean(-1, keepdim=True)
        hidden_states = hidden_states * torch.rsqrt(variance + self.eps)
        if self.weight.dtype in (torch.float16, torch.bfloat16):
            hidden_states = hidden_states.to(self.weight.dtype)
        return hidden_states * self.weight


def apply_rotary_emb(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """Rotate-half RoPE on the first rotary_dim columns (first half takes -partner),
    pass-through above; x [..., S, H, D], cos/sin [S, rotary_dim]. This is the
    arithmetic of the reference's fused kernel (fusions.py:149-170)."""

    rot = cos.shape[-1]
    half = rot // 2
    xr = x[..., :rot].float()
    rotated = torch.cat([-xr[..., half:], xr[..., :half]], dim=-1)
    c = cos.float()[:, None, :]
    s = sin.float()[:, None, :]
    out = xr * c + rotated * s
    return torch.cat([out.to(x.dtype), x[..., rot:]], dim=-1)


class AdaLNTable(nn.Module):
    """Request-invariant AdaLN projection: returns six [n_table, d] views of one table."""

    def __init__(self, n_table: int, dim: int, **factory) -> None:
        super().__init__()
        self.table = nn.Parameter(torch.zeros(n_table, 6 * dim, **factory))

    def forward(self, temb=None):
        return self.table.chunk(6, dim=-1)


class AttnProcessor:
    """Diffusers-style processor handle of an attention module: the attention backend
    and context-parallel config a dispatcher reads. Neither is set here (native SDPA,
    no context-parallel hooks)."""

    _attention_backend = None
    _parallel_config = None


class Attention(nn.Module):
    def __init__(self, dim: int, heads: int, head_dim: int, qk_eps: float = 1e-6, bias: bool = True,
                 **factory) -> None:
        super().__init__()
        self.heads = heads
        self.head_dim = head_dim
        self.fused_projections = False
        self.processor = AttnProcessor()
        inner = heads * head_dim
        self.to_q = nn.Linear(dim, inner, bias=bias, **factory)
        self.to_k = nn.Linear(dim, inner, bias=bias, **factory)
        self.to_v = nn.Linear(dim, inner, bias=bias, **factory)
        self.norm_q = RMSNorm(head_dim, qk_eps, **factory)
        self.norm_k = RMSNorm(head_dim, qk_eps, **factory)
        self.to_out = nn.ModuleList([nn.Linear(inner, dim, bias=bias, **factory), nn.Dropout(0.0)])

    def forward(self, hidden_states, rotary_emb=None, attention_mask=None):
        query = self.to_q(hidden_states).unflatten(-1, (self.heads, -1))
        key = self.to_k(hidden_states).unflatten(-1, (self.heads, -1))
        value = self.to_v(hidden_states).unflatten(-1, (self.heads, -1))
        query, key = self.norm_q(query), self.norm_k(key)
        if rotary_emb is not None:
            query = apply_rotary_emb(query, *rotary_emb)
            key = apply_rotary_emb(key, *rotary_emb)
        output = F.scaled_dot_product_attention(
            query.transpose(1, 2), key.transpose(1, 2), value.transpose(1, 2),
            attn_mask=attention_mask, dropout_p=0.0, is_causal=False,
        ).transpose(1, 2)
        output = output.flatten(2, 3).type_as(query)
        return self.to_out[1](self.to_out[0](output))


class GELUProj(nn.Module):
    def __init__(self, dim: int, inner: int, bias: bool = True, **factory) -> None:
        super().__init__()
        self.approximate = "tanh"
        self.proj = nn.Linear(dim, inner, bias=bias, **factory)

    def forward(self, x):
        return F.gelu(self.proj(x), approximate="tanh")


class SwiGLUProj(nn.Module):
    def __init__(self, dim: int, inner: int, bias: bool = True, **factory) -> None:
        super().__init__()
        self.proj = nn.Linear(dim, 2 * inner, bias=bias, **factory)
        self.activation = nn.SiLU()

    def forward(self, x):
        value, gate = self.proj(x).chunk(2, -1)
        return value * self.activation(gate)


class FeedForward(nn.Module):
    def __init__(self, dim: int, inner: int, activation: str = "gelu-tanh", bias: bool = True, **factory) -> None:
        super().__init__()
        act = GELUProj(dim, inner, bias, **factory) if activation == "gelu-tanh" else SwiGLUProj(
            dim, inner, bias, **factory)
        self.net = nn.ModuleList([act, nn.Dropout(0.0), nn.Linear(inner, dim, bias=bias, **factory)])

    def forward(self, x):
        for layer in self.net:
            x = layer(x)
        return x


class H3TransformerBlock(nn.Module):
    def __init__(self, dim: int = 3072, heads: int = 24, head_dim: int = 128, ffn_inner: int = 12288,
                 activation: str = "gelu-tanh", n_table: int = 3, eps: float = 1e-6, qk_eps: float = 1e-6,
                 bias: bool = True, **factory) -> None:
        super().__init__()
        self.adaln_proj = AdaLNTable(n_table, dim, **factory)
        self.norm1 = RMSNorm(dim, eps, **factory)
        self.attn = Attention(dim, heads, head_dim, qk_eps, bias, **factory)
        self.norm2 = RMSNorm(dim, eps, **factory)
        self.ff = FeedForward(dim, ffn_inner, activation, bias, **factory)

    def forward(self, hidden_states, temb, adaln_indices, rotary_emb, attention_mask=None):
        """Upstream eager math (kernels/transformer.py:70-74, :103-111, :121-126)."""

        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = self.adaln_proj(temb)
        pick = lambda t: t.index_select(0, adaln_indices)  # noqa: E731
        normed = self.norm1(hidden_states) * (1.0 + pick(scale_msa)) + pick(shift_msa)
        attention_output = self.attn(normed, rotary_emb, attention_mask)
        hidden_states = hidden_states + pick(gate_msa) * attention_output
        normed = self.norm2(hidden_states) * (1.0 + pick(scale_mlp)) + pick(shift_mlp)
        return hidden_states + pick(gate_mlp) * self.ff(normed)


class H3BlockStack(nn.Module):
    """Holds ``transformer_blocks`` like the H3 transformer, for the installers."""

    def __init__(self, blocks: list[H3TransformerBlock]) -> None:
        super().__init__()
        self.transformer_blocks = nn.ModuleList(blocks)

    def forward(self, hidden_states, temb, adaln_indices, rotary_emb, attention_mask=None):
        for block in self.transformer_blocks:
            hidden_states = block(hidden_states, temb, adaln_indices, rotary_emb, attention_mask)
        return hidden_states
