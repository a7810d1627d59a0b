"""Explicit-lifetime caches (per request, per denoising timestep) for the H3
transformer's invariant producers, under the import names of ``h3_flash.runtime.cache``."""

from .invariants import H3InvariantCacheRuntime, install_h3_invariant_caches

__all__ = ["H3InvariantCacheRuntime", "install_h3_invariant_caches"]
