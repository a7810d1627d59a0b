"""Request- and schedule-invariant caches of the H3 transformer."""

from .invariants import H3InvariantCacheRuntime, install_h3_invariant_caches

__all__ = ["H3InvariantCacheRuntime", "install_h3_invariant_caches"]
