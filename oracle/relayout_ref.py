"""CPU restatement of the packed-Ulysses relayouts (test infrastructure only).

Pure data movement: results must match the CUDA kernels bit for bit.
"""

from __future__ import annotations

import numpy as np


def pack_qkv(q: np.ndarray, k: np.ndarray, v: np.ndarray, world: int) -> np.ndarray:
    """src/h3_flash/runtime/parallel/relayout.py:81-94 (pack_qkv_reference):
    out[dst, row, h, p*D:(p+1)*D] = (q, k, v)[p][row, dst*hl + h, :]."""

    rows, heads, head_dim = q.shape
    if heads % world:
        raise ValueError(f"heads ({heads}) must divide Ulysses degree ({world})")
    hl = heads // world
    out = np.empty((world, rows, hl, 3 * head_dim), dtype=q.dtype)
    for p, t in enumerate((q, k, v)):
        out[..., p * head_dim : (p + 1) * head_dim] = t.reshape(rows, world, hl, head_dim).transpose(
            1, 0, 2, 3
        )
    return out


def merge_heads(x: np.ndarray) -> np.ndarray:
    """relayout.py:133-159: [world, rows, hl, D] -> [rows, world*hl, D]."""

    world, rows, hl, d = x.shape
    return np.ascontiguousarray(x.transpose(1, 0, 2, 3)).reshape(rows, world * hl, d)


def exchange(sends: list[np.ndarray], counts: list[int]) -> list[np.ndarray]:
    """The packed QKV all-to-all among W simulated ranks (packed_ulysses.py:85-108).

    sends[r] is rank r's [W, rows_r, hl, 3D] buffer; rank w receives the
    concatenation over sources r of sends[r][w] -> [sum(rows), hl, 3D]."""

    world = len(sends)
    return [np.concatenate([sends[r][w] for r in range(world)], axis=0) for w in range(world)]


def exchange_back(outputs: list[np.ndarray], counts: list[int]) -> list[np.ndarray]:
    """The output all-to-all (packed_ulysses.py:111-128): rank w holds [S, hl, D] for its
    heads; rank r gets [W, rows_r, hl, D] (source-major) then merge_heads."""

    world = len(outputs)
    offsets = np.concatenate([[0], np.cumsum(counts)])
    result = []
    for r in range(world):
        parts = np.stack([outputs[w][offsets[r] : offsets[r + 1]] for w in range(world)])
        result.append(merge_heads(parts))
    return result
