"""Sequence-parallel installers of this package, under the import names of
``h3_flash.runtime.parallel``: packed Ulysses (the block's exchanges over NCCL or NVLink
peer stores), the Diffusers context-parallel setup, rank-local input/output and the
clip-parallel VAE tile decode."""

from .context import enable_h3_ulysses, h3_context_parallel_plan
from .packed_ulysses import PackedUlyssesRuntime, install_packed_ulysses
from .rank_local_io import RankLocalIORuntime, install_rank_local_io
from .vae import install_clip_parallel_video_vae

__all__ = sorted([
    "PackedUlyssesRuntime", "RankLocalIORuntime", "enable_h3_ulysses", "h3_context_parallel_plan",
    "install_clip_parallel_video_vae", "install_packed_ulysses", "install_rank_local_io",
])
