"""Clip-parallel tiled VAE decode (src/h3_flash/runtime/parallel/vae.py:8-128) on CPU.

The official video VAE lives in an absent Diffusers checkout, so the tests use a small
stand-in with the same tiling interface: equal-size overlapping tiles, a conv decoder
that upsamples 4x, and an averaging stitcher. Over 2 and 3 gloo ranks (3 ranks: the
tile list is padded), the clip-parallel decode must equal the single-process tiled
decode: bit for bit with per-tile decoding, and to fp64 rounding when each rank decodes
its tiles as one batch. Also: the installer's guards, idempotence, the untiled path and
the compile gate's keys.
"""

from __future__ import annotations

import pytest
import torch
from torch import nn

from tests.test_gloo import _run


class TiledVAE(nn.Module):
    spatial_compression_ratio = 4
    tile_sample_min_height = 32
    tile_sample_min_width = 32
    tile_sample_min_overlap_height = 8
    tile_sample_min_overlap_width = 8

    def __init__(self, use_tiling: bool = True) -> None:
        super().__init__()
        torch.manual_seed(0)
        self.use_tiling = use_tiling
        self.post_quant_conv = nn.Conv3d(4, 4, 1)
        self.decoder = nn.Sequential(nn.Conv3d(4, 8, 3, padding=1), nn.SiLU(),
                                     nn.Upsample(scale_factor=(1, 4, 4)), nn.Conv3d(8, 3, 3, padding=1))
        self.double()

    def _split_tiles(self, size, tile, overlap):
        if size <= tile:
            return [0], [size], [0]
        starts = list(range(0, size - tile, tile - overlap)) + [size - tile]
        overlaps = [0] + [starts[i - 1] + tile - starts[i] for i in range(1, len(starts))]
        return starts, [tile] * len(starts), overlaps

    def _stitch_tiles(self, rows, y_overlaps, x_overlaps):
        h, w = rows[0][0].shape[-2:]
        ys = [0]
        for o in y_overlaps[1:]:
            ys.append(ys[-1] + h - o)
        xs = [0]
        for o in x_overlaps[1:]:
            xs.append(xs[-1] + w - o)
        canvas = torch.zeros(rows[0][0].shape[:-2] + (ys[-1] + h, xs[-1] + w), dtype=rows[0][0].dtype)
        weight = torch.zeros_like(canvas)
        for r, row in enumerate(rows):
            for c, tile in enumerate(row):
                canvas[..., ys[r]:ys[r] + h, xs[c]:xs[c] + w] += tile
                weight[..., ys[r]:ys[r] + h, xs[c]:xs[c] + w] += 1
        return canvas / weight

    def _decode_clip(self, z):
        ratio = self.spatial_compression_ratio
        ys, hs, yo = self._split_tiles(z.shape[-2] * ratio, self.tile_sample_min_height,
                                       self.tile_sample_min_overlap_height)
        xs, ws, xo = self._split_tiles(z.shape[-1] * ratio, self.tile_sample_min_width,
                                       self.tile_sample_min_overlap_width)
        if not self.use_tiling:
            return self.decoder(self.post_quant_conv(z))
        rows = [[self.decoder(self.post_quant_conv(
            z[..., y // ratio:y // ratio + h // ratio, x // ratio:x // ratio + w // ratio])) for x, w in zip(xs, ws)]
            for y, h in zip(ys, hs)]
        return self._stitch_tiles(rows, yo, xo)


class OddTiledVAE(TiledVAE):
    """Tiles of 30 sample pixels with an overlap of 10: neither the tile length nor the
    tile stride (20) is a multiple of the compression ratio (4), so tile starts fall
    between latent rows and the latent window must start at the floored coordinate and
    keep the floored length for every tile to come out the same size."""

    tile_sample_min_height = 30
    tile_sample_min_width = 30
    tile_sample_min_overlap_height = 10
    tile_sample_min_overlap_width = 10


def _latent():
    g = torch.Generator().manual_seed(5)
    return torch.randn(1, 4, 2, 22, 30, generator=g, dtype=torch.float64)  # 88 x 120 pixels: 4 x 5 tiles


def _decode_worker(rank, world, batched, odd=False):
    from h3_flash_b200.runtime.parallel.vae import install_clip_parallel_video_vae

    vae = OddTiledVAE() if odd else TiledVAE()
    z = _latent()
    with torch.no_grad():
        expect = vae._decode_clip(z)
        meta = install_clip_parallel_video_vae(vae, batched=batched)
        again = install_clip_parallel_video_vae(vae, batched=not batched)
        got = vae._decode_clip(z)
    return (bool(torch.equal(got, expect)), float((got - expect).abs().max()), tuple(got.shape),
            meta is again, meta["compile_contract"], meta["world_size"])


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("batched", [False, True])
@pytest.mark.parametrize("odd", [False, True])
def test_clip_parallel_decode_equals_single_process(world, batched, odd):
    for equal, max_diff, shape, idempotent, contract, size in _run(world, _decode_worker, batched, odd):
        if not odd:
            assert shape == (1, 3, 2, 88, 120), shape
        if batched:
            assert max_diff <= 1e-12
        else:
            assert equal
        assert idempotent and contract == "eager_bit_exact_tile_execution" and size == world


def _untiled_worker(rank, world):
    from h3_flash_b200.runtime.parallel.vae import install_clip_parallel_video_vae

    vae = TiledVAE(use_tiling=False)
    z = _latent()
    with torch.no_grad():
        expect = vae._decode_clip(z)
        install_clip_parallel_video_vae(vae)
        return bool(torch.equal(vae._decode_clip(z), expect))


def test_untiled_clips_take_the_original_path():
    assert all(_run(2, _untiled_worker))


def test_install_requires_a_process_group():
    from h3_flash_b200.runtime.parallel.vae import install_clip_parallel_video_vae

    with pytest.raises(RuntimeError, match="initialized process group"):
        install_clip_parallel_video_vae(TiledVAE())


def test_rank_shares_cover_every_tile_once_in_order():
    from h3_flash_b200.runtime.parallel.vae import _rank_share

    for n_tiles in range(1, 14):
        tiles = list(range(n_tiles))
        for world in range(2, 6):
            shares = [_rank_share(tiles, world, r) for r in range(world)]
            per_rank = shares[0][1]
            assert all(len(s) == per_rank and p == per_rank for s, p in shares)
            flat = [t for s, _ in shares for t in s]
            assert flat[:n_tiles] == tiles  # rank order is tile order
            assert all(t == tiles[-1] for t in flat[n_tiles:])  # padding repeats the last tile
            assert per_rank * world - n_tiles < world
