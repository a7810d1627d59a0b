"""An H3-style transformer around the block stack: the modules on either side of
the blocks that the rank-local I/O and invariant-cache installers act on.

The real MiniMax H3 transformer lives in a Diffusers checkout that is not part
of this package. This module reproduces the attribute surface those installers
use (src/h3_flash/runtime/parallel/rank_local_io.py:139-286,
src/h3_flash/runtime/cache/invariants.py:125-157):

  context_embedder, token_refiner        text tokens -> [B, n_text, d]
  time_proj, time_embedder.linear_1      timestep [T] -> temb [T, d]
  proj_in, audio_proj_in                 video / audio tokens -> [B, n, d]
  rope(position_ids [S, 3]) -> (cos, sin) fp32 [S, rot]
  transformer_blocks[i].adaln_proj(temb) six [T*3, d] tables (index = timestep*3 + tag)
  norm_out(x, temb, timestep_indices), norm_out.linear
  proj_out, audio_proj_out               [B, n, d] -> video / audio outputs

``forward`` is the full-sequence computation (every rank projects every token,
the reference's non-rank-local branch, rank_local_io.py:191-200 and :259-267):
the value the rank-local path must reproduce.
"""

from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F
from torch import nn

from .h3_block import H3TransformerBlock, RMSNorm

N_TAGS = 3  # token tags: 0 text, 1 video, 2 audio


@dataclass
class H3Output:
    sample: torch.Tensor
    audio_sample: torch.Tensor


class TimestepProjection(nn.Module):
    """Sinusoidal timestep features, fp32 [T, freq_dim]."""

    def __init__(self, freq_dim: int = 256) -> None:
        super().__init__()
        self.freq_dim = freq_dim

    def forward(self, timestep: torch.Tensor) -> torch.Tensor:
        half = self.freq_dim // 2
        exponent = -math.log(10000.0) * torch.arange(half, dtype=torch.float32, device=timestep.device) / half
        angles = timestep.float().reshape(-1, 1) * torch.exp(exponent)[None, :]
        return torch.cat([angles.cos(), angles.sin()], dim=-1)


class TimestepEmbedder(nn.Module):
    def __init__(self, freq_dim: int, dim: int, **factory) -> None:
        super().__init__()
        self.linear_1 = nn.Linear(freq_dim, dim, **factory)
        self.linear_2 = nn.Linear(dim, dim, **factory)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self.linear_2(F.silu(self.linear_1(x)))


class TokenRefiner(nn.Module):
    def __init__(self, dim: int, **factory) -> None:
        super().__init__()
        self.linear = nn.Linear(dim, dim, **factory)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return x + F.silu(self.linear(x))


class H3Rope(nn.Module):
    """3-axis rotate-half RoPE tables: per axis ``len(inv_freq)`` frequencies,
    angles of (time, height, width) concatenated, then duplicated
    (rank_local_io.py:74-80); rotary_dim = 6 * len(inv_freq)."""

    def __init__(self, freqs_per_axis: int = 16, theta: float = 10000.0) -> None:
        super().__init__()
        inv_freq = theta ** (-torch.arange(0, 2 * freqs_per_axis, 2, dtype=torch.float32) / (2 * freqs_per_axis))
        self.register_buffer("inv_freq", inv_freq, persistent=False)

    def forward(self, position_ids: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
        angles = position_ids.to(torch.float32).unsqueeze(-1) * self.inv_freq.view(1, 1, -1)
        angles = torch.cat(angles.unbind(dim=1), dim=-1)
        angles = torch.cat((angles, angles), dim=-1)
        return angles.cos(), angles.sin()


class AdaLNProjection(nn.Module):
    """temb [T, d] -> six AdaLN tables [T*3, d] (one row per (timestep, tag)),
    as views of one [T*3, 6d] tensor: the layout the fused kernels index."""

    def __init__(self, dim: int, **factory) -> None:
        super().__init__()
        self.dim = dim
        self.linear = nn.Linear(dim, N_TAGS * 6 * dim, **factory)

    def forward(self, temb: torch.Tensor):
        table = self.linear(F.silu(temb)).reshape(-1, 6 * self.dim)
        return table.chunk(6, dim=-1)


class AdaLNOutputNorm(nn.Module):
    """Final norm: RMSNorm(x) * (1 + scale[ti]) + shift[ti], tables from temb."""

    def __init__(self, dim: int, eps: float = 1e-6, **factory) -> None:
        super().__init__()
        self.norm = RMSNorm(dim, eps, **factory)
        self.linear = nn.Linear(dim, 2 * dim, **factory)

    def forward(self, x: torch.Tensor, temb: torch.Tensor, timestep_indices: torch.Tensor) -> torch.Tensor:
        shift, scale = self.linear(F.silu(temb)).chunk(2, dim=-1)
        return self.norm(x) * (1.0 + scale.index_select(0, timestep_indices)) + shift.index_select(
            0, timestep_indices
        )


class H3Transformer(nn.Module):
    def __init__(self, dim: int, heads: int, head_dim: int, ffn_inner: int, layers: int, *,
                 text_dim: int, video_channels: int, audio_channels: int, freq_dim: int = 256,
                 freqs_per_axis: int = 16, eps: float = 1e-6, activation: str = "gelu-tanh",
                 **factory) -> None:
        super().__init__()
        self.context_embedder = nn.Linear(text_dim, dim, **factory)
        self.token_refiner = TokenRefiner(dim, **factory)
        self.time_proj = TimestepProjection(freq_dim)
        self.time_embedder = TimestepEmbedder(freq_dim, dim, **factory)
        self.proj_in = nn.Linear(video_channels, dim, **factory)
        self.audio_proj_in = nn.Linear(audio_channels, dim, **factory)
        self.rope = H3Rope(freqs_per_axis)
        blocks = []
        for _ in range(layers):
            block = H3TransformerBlock(dim, heads, head_dim, ffn_inner, activation=activation,
                                       eps=eps, qk_eps=eps, **factory)
            block.adaln_proj = AdaLNProjection(dim, **factory)
            blocks.append(block)
        self.transformer_blocks = nn.ModuleList(blocks)
        self.norm_out = AdaLNOutputNorm(dim, eps, **factory)
        self.proj_out = nn.Linear(dim, video_channels, **factory)
        self.audio_proj_out = nn.Linear(dim, audio_channels, **factory)

    def embed(self, hidden_states, audio_hidden_states, encoder_hidden_states, timestep,
              video_indices, audio_indices, text_indices, sequence_length: int):
        """All tokens projected and placed at their sequence positions."""

        text_embeds = self.context_embedder(encoder_hidden_states.to(self.context_embedder.weight.dtype))
        text_embeds = self.token_refiner(text_embeds)
        temb = self.time_embedder(self.time_proj(timestep).to(self.time_embedder.linear_1.weight.dtype))
        video_embeds = self.proj_in(hidden_states.to(self.proj_in.weight.dtype))
        audio_embeds = self.audio_proj_in(audio_hidden_states.to(self.audio_proj_in.weight.dtype))
        full = text_embeds.new_zeros((text_embeds.shape[0], sequence_length, text_embeds.shape[-1]))
        full = full.index_copy(1, text_indices, text_embeds)
        full = full.index_copy(1, video_indices, video_embeds.to(full.dtype))
        full = full.index_copy(1, audio_indices, audio_embeds.to(full.dtype))
        return full, text_embeds, temb

    def forward(self, hidden_states, audio_hidden_states, encoder_hidden_states, timestep,
                timestep_indices, token_tags, position_ids, video_indices, audio_indices,
                text_indices, attention_kwargs=None, return_dict=True):
        sequence_length = position_ids.shape[0]
        full, _, temb = self.embed(hidden_states, audio_hidden_states, encoder_hidden_states, timestep,
                                   video_indices, audio_indices, text_indices, sequence_length)
        rotary_emb = self.rope(position_ids)
        adaln_indices = timestep_indices * N_TAGS + token_tags.clamp(min=0)
        for block in self.transformer_blocks:
            full = block(full, temb, adaln_indices, rotary_emb, None)
        full = self.norm_out(full, temb, timestep_indices).to(self.proj_out.weight.dtype)
        video_output = self.proj_out(full).index_select(1, video_indices)
        audio_output = self.audio_proj_out(full).index_select(1, audio_indices)
        if not return_dict:
            return video_output, audio_output
        return H3Output(sample=video_output, audio_sample=audio_output)


def make_inputs(model: H3Transformer, *, n_text: int, n_video: int, n_audio: int, text_dim: int,
                grid: tuple[int, int, int], n_timesteps: int = 1, seed: int = 0,
                device: str | torch.device = "cpu", dtype: torch.dtype = torch.float32) -> dict:
    """Seeded synthetic request: text first, then video tokens on a (t, h, w)
    grid, then audio tokens; one timestep per modality group."""

    g = torch.Generator().manual_seed(seed)
    video_channels = model.proj_in.in_features
    audio_channels = model.audio_proj_in.in_features
    total = n_text + n_video + n_audio
    text_indices = torch.arange(0, n_text)
    video_indices = torch.arange(n_text, n_text + n_video)
    audio_indices = torch.arange(n_text + n_video, total)
    tags = torch.cat([torch.zeros(n_text), torch.ones(n_video), torch.full((n_audio,), 2.0)]).long()
    t, h, w = grid
    lin = torch.arange(n_video)
    video_pos = torch.stack([lin // (h * w), (lin // w) % h, lin % w], dim=-1)
    text_pos = torch.zeros(n_text, 3, dtype=torch.long)
    audio_pos = torch.stack([torch.arange(n_audio)] * 3, dim=-1)
    position_ids = torch.cat([text_pos, video_pos, audio_pos])
    timestep = torch.rand(n_timesteps, generator=g) * 1000.0
    timestep_indices = (tags % n_timesteps).long() if n_timesteps > 1 else torch.zeros(total, dtype=torch.long)
    to = dict(device=device)
    return {
        "hidden_states": torch.randn(1, n_video, video_channels, generator=g).to(dtype=dtype, **to),
        "audio_hidden_states": torch.randn(1, n_audio, audio_channels, generator=g).to(dtype=dtype, **to),
        "encoder_hidden_states": torch.randn(1, n_text, text_dim, generator=g).to(dtype=dtype, **to),
        "timestep": timestep.to(**to),
        "timestep_indices": timestep_indices.to(**to),
        "token_tags": tags.to(**to),
        "position_ids": position_ids.to(**to),
        "video_indices": video_indices.to(**to),
        "audio_indices": audio_indices.to(**to),
        "text_indices": text_indices.to(**to),
    }
