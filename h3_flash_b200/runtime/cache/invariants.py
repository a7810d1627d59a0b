"""Explicit-lifetime caches for the H3 transformer's invariant producers.

Interface of ``h3_flash.runtime.cache.invariants`` (src/h3_flash/runtime/cache/
invariants.py:10-157): ``H3InvariantCacheRuntime`` with the same attributes, counters,
``audit()`` keys, ``begin_request()`` and ``freeze_fixed_schedule()``, the installer
``install_h3_invariant_caches`` and the same error messages.

Design. Every cached producer is one *site*: a module whose ``forward`` is replaced by
a memoising call that looks its value up in a table chosen by the site's *scope*:

- request scope (text embedder, token refiner, RoPE tables): one table entry per site,
  valid until ``begin_request()`` empties the table;
- schedule scope (each block's AdaLN projection and the output norm's projection): a
  table per site keyed by the current timestep, kept across requests. The key is the
  timestep's shape, dtype and exact value bytes, recorded by the transformer's wrapped
  ``forward`` for the duration of one call. The cached AdaLN value is the
  ``[n_table, 6*d]`` modulation table (six views) that the fused AdaLN kernels index, so
  a hit hands the kernels a resident table without the projection GEMM.

``freeze_fixed_schedule`` releases the AdaLN projection weights once every schedule
site holds the expected number of timesteps; after that an unseen timestep is an error.
A CUDA timestep costs one device-to-host copy per transformer forward (the key needs
its values on the host).
"""

from __future__ import annotations

from dataclasses import dataclass, field
from types import MethodType
from typing import Any, Callable

REQUEST = "request"
SCHEDULE = "schedule"


@dataclass
class H3InvariantCacheRuntime:
    """Cache state owned by one resident H3 transformer."""

    request_values: dict[str, Any] = field(default_factory=dict)
    schedule_values: dict[str, dict[tuple[Any, ...], Any]] = field(default_factory=dict)
    current_timestep_key: tuple[Any, ...] | None = None
    request_hits: int = 0
    request_misses: int = 0
    schedule_hits: int = 0
    schedule_misses: int = 0
    adaln_modules: list[Any] = field(default_factory=list, repr=False)
    schedule_frozen: bool = False
    freed_parameter_bytes: int = 0

    # -- lifetime -------------------------------------------------------------------

    def begin_request(self) -> None:
        """Start a request: request-scope values are dropped and the per-request
        counters restart; schedule-scope values stay (they are keyed by timestep)."""

        self.request_values.clear()
        self.current_timestep_key = None
        for name in ("request_hits", "request_misses", "schedule_hits", "schedule_misses"):
            setattr(self, name, 0)

    def audit(self) -> dict[str, int]:
        entries = 0
        for table in self.schedule_values.values():
            entries += len(table)
        return {
            "request_hits": self.request_hits,
            "request_misses": self.request_misses,
            "schedule_hits": self.schedule_hits,
            "schedule_misses": self.schedule_misses,
            "schedule_entries": entries,
            "schedule_frozen": self.schedule_frozen,
            "freed_parameter_bytes": self.freed_parameter_bytes,
        }

    def freeze_fixed_schedule(self, expected_values_per_site: int = 49) -> int:
        """Release every AdaLN projection's weights once each schedule site holds
        ``expected_values_per_site`` timesteps; returns the bytes released (the same
        figure on repeated calls)."""

        if expected_values_per_site < 1:
            raise ValueError("expected_values_per_site must be positive")
        if self.schedule_frozen:
            return self.freed_parameter_bytes
        complete = bool(self.schedule_values) and min(
            len(table) for table in self.schedule_values.values()) >= expected_values_per_site
        if not complete:
            raise RuntimeError(
                "cannot freeze AdaLN projections before all expected schedule "
                f"values are cached ({expected_values_per_site} per site)"
            )
        self.freed_parameter_bytes = sum(_release_linear(module) for module in self.adaln_modules)
        self.schedule_frozen = True
        return self.freed_parameter_bytes

    # -- lookups used by the cached sites ----------------------------------------------

    def _table(self, scope: str, site: str) -> tuple[dict[Any, Any], Any]:
        """(table, key) of ``site``'s current value."""

        if scope == REQUEST:
            return self.request_values, site
        if self.current_timestep_key is None:
            raise RuntimeError(f"schedule cache {site} called outside H3 transformer forward")
        return self.schedule_values.setdefault(site, {}), self.current_timestep_key

    def _count(self, scope: str, hit: bool) -> None:
        name = f"{scope}_{'hits' if hit else 'misses'}"
        setattr(self, name, getattr(self, name) + 1)


def _release_linear(holder: Any) -> int:
    """Drops ``holder.linear`` and returns the bytes its parameters held."""

    size = sum(p.numel() * p.element_size() for p in holder.linear.parameters())
    holder.linear = None
    return size


def _timestep_key(timestep: Any) -> tuple[Any, ...]:
    """Schedule key of a timestep tensor: shape, dtype and the exact bytes of its
    values, so two timesteps share cached values only if they are the same tensor
    value in the same type."""

    host = timestep.detach().to("cpu").contiguous()
    return (tuple(host.shape), str(host.dtype), host.numpy().tobytes())


def _cache_site(module: Any, site: str, scope: str, runtime: H3InvariantCacheRuntime) -> None:
    """Replace ``module.forward`` by a memoising call of the original."""

    produce: Callable[..., Any] = module.forward
    if scope == SCHEDULE:
        runtime.schedule_values.setdefault(site, {})

    def cached(_self: Any, *args: Any, **kwargs: Any) -> Any:
        table, key = runtime._table(scope, site)
        if key in table:
            runtime._count(scope, hit=True)
            return table[key]
        if scope == SCHEDULE and runtime.schedule_frozen:
            raise RuntimeError(
                f"fixed-schedule cache {site} received an unseen timestep after weights were released"
            )
        value = table[key] = produce(*args, **kwargs)
        runtime._count(scope, hit=False)
        return value

    module.forward = MethodType(cached, module)


def _wrap_request_value(module: Any, name: str, runtime: H3InvariantCacheRuntime) -> None:
    """Request-scope site (src/h3_flash/runtime/cache/invariants.py:80-95)."""

    _cache_site(module, name, REQUEST, runtime)


def _wrap_schedule_value(module: Any, name: str, runtime: H3InvariantCacheRuntime) -> None:
    """Schedule-scope site keyed by the current timestep (invariants.py:98-122)."""

    _cache_site(module, name, SCHEDULE, runtime)


def _timestep_argument(args: tuple[Any, ...], kwargs: dict[str, Any]) -> Any:
    """The transformer forward's ``timestep``: keyword, else the fourth positional."""

    if "timestep" in kwargs and kwargs["timestep"] is not None:
        return kwargs["timestep"]
    if len(args) >= 4:
        return args[3]
    raise RuntimeError("cannot resolve H3 timestep for schedule cache")


def install_h3_invariant_caches(transformer: Any) -> H3InvariantCacheRuntime:
    """Cache the invariant producers of ``transformer`` (invariants.py:125-157):
    request scope for ``context_embedder``, ``token_refiner`` and ``rope``; schedule
    scope for every block's ``adaln_proj`` and for ``norm_out.linear``. Installing
    twice returns the first runtime."""

    existing = getattr(transformer, "_h3_flash_invariant_cache", None)
    if existing is not None:
        return existing
    runtime = H3InvariantCacheRuntime()
    for site in ("context_embedder", "token_refiner", "rope"):
        _cache_site(getattr(transformer, site), site, REQUEST, runtime)
    for index, block in enumerate(transformer.transformer_blocks):
        _cache_site(block.adaln_proj, f"adaln.{index}", SCHEDULE, runtime)
        runtime.adaln_modules.append(block.adaln_proj)
    _cache_site(transformer.norm_out.linear, "norm_out.linear", SCHEDULE, runtime)

    body = transformer.forward

    def forward_with_schedule_key(_self: Any, *args: Any, **kwargs: Any) -> Any:
        runtime.current_timestep_key = _timestep_key(_timestep_argument(args, kwargs))
        try:
            return body(*args, **kwargs)
        finally:
            runtime.current_timestep_key = None

    transformer.forward = MethodType(forward_with_schedule_key, transformer)
    transformer._h3_flash_invariant_cache = runtime
    return runtime
