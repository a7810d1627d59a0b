"""Helpers for the GPU parity tests: bf16 bit patterns <-> CUDA tensors."""

from __future__ import annotations

import numpy as np
import torch


def dev(bits: np.ndarray, device: str = "cuda") -> torch.Tensor:
    """uint16 bf16 bits -> bf16 CUDA tensor."""

    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16).copy()).view(torch.bfloat16).to(device)


def bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


def f32(t: torch.Tensor) -> np.ndarray:
    return t.detach().float().cpu().numpy()


def seeded_bits(seed: int, shape, mean: float = 0.0, std: float = 1.0) -> np.ndarray:
    from oracle.bf16 import random_bf16

    return random_bf16(np.random.default_rng(seed), shape, mean, std)
