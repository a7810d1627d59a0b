"""Distributed execution primitives for the lossless H3 runtime."""

from .context import enable_h3_ulysses, h3_context_parallel_plan
from .packed_ulysses import PackedUlyssesRuntime, install_packed_ulysses

__all__ = [
    "PackedUlyssesRuntime",
    "enable_h3_ulysses",
    "h3_context_parallel_plan",
    "install_packed_ulysses",
]
