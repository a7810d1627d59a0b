"""Benchmark workload shapes and seeded synthetic inputs for the LOSSLESS DiT block.

Shapes (d=3072, 24 heads x 128, FFN 4x GELU-tanh) and token counts are the
benchmark configurations; weights are random-init N(0, 0.02), activations
N(0, 1), AdaLN shift/scale/gate tables N(0, 0.1), RMSNorm/QK-norm weights
N(1, 0.02). RoPE tables follow the H3 structure (rank_local_io.py:74-80): per-axis
angles pos_axis * inv_freq_axis for (t, h, w), concatenated, then duplicated
(cos/sin of cat(f, f)); inv_freq_axis = theta^(-2i/32), i < 16, so rotary_dim = 96.
The H3 inv_freq formula lives in an unpinned upstream module, so the tables are
a documented choice; every kernel takes cos/sin as inputs.
Audio tokens follow the video tokens in the joint sequence, at positions
(a, 0, 0); token tags give the AdaLN table row: video 1, audio 2.
"""

from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class BlockConfig:
    name: str
    video_grid: tuple[int, int, int]  # (t, h, w) latent patches
    audio_tokens: int
    dim: int = 3072
    heads: int = 24
    head_dim: int = 128
    ffn_inner: int = 12288
    rotary_dim: int = 96
    theta: float = 10000.0
    eps: float = 1e-6

    @property
    def video_tokens(self) -> int:
        t, h, w = self.video_grid
        return t * h * w

    @property
    def seq(self) -> int:
        return self.video_tokens + self.audio_tokens


CONFIGS = {
    "cpu-gloo": BlockConfig("cpu-gloo", (4, 32, 32), 256),
    "480p-5s": BlockConfig("480p-5s", (32, 30, 52), 1280),
    "768p-5s": BlockConfig("768p-5s", (32, 48, 84), 1280),
    "768p-15s": BlockConfig("768p-15s", (87, 48, 84), 3456),
}


def split_sizes(total: int, parts: int) -> list[int]:
    """Contiguous near-equal row split (rank_local_io.py:13-15)."""

    quotient, remainder = divmod(total, parts)
    return [quotient + (index < remainder) for index in range(parts)]


def split_bounds(total: int, parts: int, rank: int) -> tuple[int, int]:
    sizes = split_sizes(total, parts)
    start = sum(sizes[:rank])
    return start, start + sizes[rank]


def positions(cfg: BlockConfig) -> torch.Tensor:
    t, h, w = cfg.video_grid
    tt, hh, ww = torch.meshgrid(torch.arange(t), torch.arange(h), torch.arange(w), indexing="ij")
    video = torch.stack([tt.reshape(-1), hh.reshape(-1), ww.reshape(-1)], dim=-1)
    audio = torch.stack(
        [torch.arange(cfg.audio_tokens), torch.zeros(cfg.audio_tokens, dtype=torch.long),
         torch.zeros(cfg.audio_tokens, dtype=torch.long)], dim=-1)
    return torch.cat([video, audio], dim=0)  # [S, 3]


def rope_tables(pos: torch.Tensor, rotary_dim: int = 96, theta: float = 10000.0) -> tuple[torch.Tensor, torch.Tensor]:
    """cos, sin fp32 [S, rotary_dim] from integer (t, h, w) positions [S, 3]."""

    if rotary_dim % 6:
        raise ValueError("3-axis RoPE needs rotary_dim divisible by 6")
    per_axis = rotary_dim // 6  # frequencies per axis
    axis_dim = 2 * per_axis
    inv_freq = theta ** (-torch.arange(0, axis_dim, 2, dtype=torch.float64) / axis_dim)  # [per_axis]
    freqs = pos.to(torch.float64)[:, :, None] * inv_freq[None, None, :]  # [S, 3, per_axis]
    freqs = torch.cat([freqs[:, 0], freqs[:, 1], freqs[:, 2]], dim=-1)
    freqs = torch.cat([freqs, freqs], dim=-1)
    return freqs.cos().float(), freqs.sin().float()


def adaln_indices(cfg: BlockConfig) -> torch.Tensor:
    tags = torch.cat([torch.ones(cfg.video_tokens, dtype=torch.long),
                      torch.full((cfg.audio_tokens,), 2, dtype=torch.long)])
    return tags  # timestep index 0: row = 0*3 + tag


def init_block_(block: torch.nn.Module, seed: int = 0) -> torch.nn.Module:
    """Random-init an H3TransformerBlock in place: Linear weights/biases N(0, 0.02),
    norm weights N(1, 0.02), AdaLN table N(0, 0.1)."""

    g = torch.Generator(device="cpu").manual_seed(seed)
    with torch.no_grad():
        for name, p in block.named_parameters():
            if name.endswith("adaln_proj.table"):
                values = torch.randn(p.shape, generator=g) * 0.1
            elif "norm" in name.split(".")[-2]:
                values = 1.0 + torch.randn(p.shape, generator=g) * 0.02
            else:
                values = torch.randn(p.shape, generator=g) * 0.02
            p.copy_(values.to(p.dtype))
    return block


def hidden_states(cfg: BlockConfig, rows: int, dim: int | None = None, seed: int = 1,
                  dtype=torch.bfloat16, device="cpu") -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(seed)
    return torch.randn(1, rows, dim or cfg.dim, generator=g).to(dtype).to(device)
