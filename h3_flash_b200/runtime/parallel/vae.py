"""Clip-parallel tile decode for a tiled video VAE (src/h3_flash/runtime/parallel/vae.py:8-128).

A tiled decode of one clip splits the latent into overlapping spatial tiles, decodes each
tile with the decoder and blends the decoded tiles back together. The tiles are
independent, so W ranks can each decode a contiguous share of them:

  tiles (row-major over the tile grid) -> rank r decodes tiles [r*n, (r+1)*n)
  (the list padded to W*n by repeating its last tile) -> one all-gather of the decoded
  tiles into a [W*n, ...] buffer -> the first len(tiles) entries, in the original order,
  go to the VAE's own stitcher.

Every tile is decoded exactly once by the unchanged decoder (the padding repeats are
discarded), so with an eager decoder the result is the single-process decode bit for bit.
Equal-size tiles can be decoded as one batch: the decoder has no operation that reduces
across its batch dimension.

The VAE object provides the tiling interface of the official decoder: ``use_tiling``,
``spatial_compression_ratio``, ``tile_sample_min_height``/``_width``,
``tile_sample_min_overlap_height``/``_width``, ``_split_tiles(size, tile, overlap)`` ->
(starts, lengths, overlaps), ``_stitch_tiles(rows, y_overlaps, x_overlaps)``,
``post_quant_conv``, ``decoder`` and ``_decode_clip``, which the installer replaces.
"""

from __future__ import annotations

from typing import Any

import torch
import torch.distributed as dist


def _tile_grid(vae: Any, z: torch.Tensor):
    """Row-major tile list [(y, height, x, width)] in sample pixels, plus the overlaps."""

    ratio = vae.spatial_compression_ratio
    ys, hs, y_overlaps = vae._split_tiles(z.shape[-2] * ratio, vae.tile_sample_min_height,
                                         vae.tile_sample_min_overlap_height)
    xs, ws, x_overlaps = vae._split_tiles(z.shape[-1] * ratio, vae.tile_sample_min_width,
                                         vae.tile_sample_min_overlap_width)
    tiles = [(y, h, x, w) for y, h in zip(ys, hs) for x, w in zip(xs, ws)]
    return tiles, len(ys), len(xs), y_overlaps, x_overlaps


def _rank_share(tiles: list, world: int, rank: int) -> tuple[list, int]:
    """This rank's contiguous share of the tile list, padded to an equal count per rank
    by repeating the last tile (the repeats are decoded and then discarded)."""

    per_rank = -(-len(tiles) // world)
    padded = tiles + [tiles[-1]] * (per_rank * world - len(tiles))
    return padded[rank * per_rank:(rank + 1) * per_rank], per_rank


def _latent_tile(z: torch.Tensor, tile: tuple[int, int, int, int], ratio: int) -> torch.Tensor:
    """The latent window of a tile given in sample pixels: it starts at the floored
    latent coordinate of the tile's start and spans the floored latent length, so every
    tile of one length has the same latent size whatever its start (vae.py:75-83)."""

    y, h, x, w = tile
    y0, x0 = y // ratio, x // ratio
    return z[..., y0:y0 + h // ratio, x0:x0 + w // ratio]


def _error_gate(got: torch.Tensor, expect: torch.Tensor, group: Any) -> dict[str, float]:
    """max_abs, the ranks' largest mean_abs and relative L2 of compiled vs eager tiles."""

    delta = (got.float() - expect.float()).abs()
    values = torch.stack([delta.max(), delta.mean(),
                          delta.norm() / expect.float().norm().clamp_min(1e-12)])
    dist.all_reduce(values, op=dist.ReduceOp.MAX, group=group)
    return {"max_abs": float(values[0]), "max_rank_mean_abs": float(values[1]),
            "max_rank_relative_l2": float(values[2])}


def install_clip_parallel_video_vae(vae: Any, *, group: Any = None, batched: bool = True,
                                    compile_mode: str | None = None) -> dict[str, Any]:
    """Replace ``vae._decode_clip`` with the clip-parallel tiled decode (vae.py:8-128).

    Collective: every rank of ``group`` decodes every clip. ``batched`` decodes this
    rank's tiles as one batch (they have equal sizes), else one at a time.
    ``compile_mode`` wraps the decoder in ``torch.compile`` with that mode and records
    its first batch against the eager decoder in the returned ``compile_gate``.
    Installing twice returns the first installation's metadata."""

    if not (dist.is_available() and dist.is_initialized()):
        raise RuntimeError("clip-parallel VAE requires an initialized process group")
    group = group or dist.group.WORLD
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if world < 2:
        raise RuntimeError("clip-parallel VAE requires at least two ranks")
    installed = getattr(vae, "_h3_flash_clip_parallel", None)
    if installed is not None:
        return installed

    whole_clip = vae._decode_clip
    eager = vae.decoder
    if compile_mode is not None:
        vae.decoder = torch.compile(eager, mode=compile_mode, dynamic=False)
    gate: dict[str, float] = {}

    def decode_share(latents: list[torch.Tensor]) -> torch.Tensor:
        if not batched:
            return torch.cat([vae.decoder(vae.post_quant_conv(t)) for t in latents], dim=0)
        inputs = vae.post_quant_conv(torch.cat(latents, dim=0))
        decoded = vae.decoder(inputs)
        if compile_mode is not None and not gate:
            gate.update(_error_gate(decoded, eager(inputs), group))
        return decoded

    def clip_parallel_decode(z: torch.Tensor) -> torch.Tensor:
        if not vae.use_tiling:
            return whole_clip(z)
        tiles, n_rows, n_cols, y_overlaps, x_overlaps = _tile_grid(vae, z)
        mine, per_rank = _rank_share(tiles, world, rank)
        ratio = vae.spatial_compression_ratio
        local = decode_share([_latent_tile(z, tile, ratio) for tile in mine]).contiguous()
        # One collective into one buffer: [world * per_rank, ...] in rank order, which is
        # the padded tile order.
        gathered = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]),
                               dtype=local.dtype, device=local.device)
        dist.all_gather_into_tensor(gathered, local, group=group)
        decoded = gathered[:len(tiles)]
        grid = [[decoded[r * n_cols + c].unsqueeze(0) for c in range(n_cols)] for r in range(n_rows)]
        return vae._stitch_tiles(grid, y_overlaps, x_overlaps)

    vae._decode_clip = clip_parallel_decode
    metadata = {
        "backend": "official_tile_clip_parallel",
        "world_size": world,
        "batched_equal_tiles": batched,
        "compile_mode": compile_mode,
        "compile_contract": ("mathematically_equivalent_bounded_numeric_error" if compile_mode is not None
                             else "eager_bit_exact_tile_execution"),
        "compile_gate": gate,
    }
    vae._h3_flash_clip_parallel = metadata
    return metadata
