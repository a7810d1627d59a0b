"""Explicit-lifetime caches for values that do not change within a request or
across a fixed denoising schedule.

Drop-in for ``h3_flash.runtime.cache.invariants``
(src/h3_flash/runtime/cache/invariants.py): same runtime object, key function,
wrappers, installer, counters and error messages.

- Request values (text embedder, token refiner, RoPE tables) are computed once
  per request and returned as the same tensors afterwards
  (invariants.py:72-86).
- Schedule values (every block's AdaLN projection and the output norm's
  projection) depend only on the timestep, so they are keyed by the timestep's
  shape, dtype and values and kept across requests (invariants.py:89-113). The
  cached AdaLN value is the ``[n_table, 6*d]`` modulation table (as six views)
  that the fused AdaLN kernels index with ``adaln_indices``; a hit hands the
  kernels the resident table without recomputing the projection GEMM.
- ``freeze_fixed_schedule`` drops the AdaLN projection weights once every
  schedule value is cached and refuses unseen timesteps afterwards
  (invariants.py:48-68).

The timestep key needs the timestep's values on the host. A CPU timestep is
read directly; a CUDA timestep costs one device-to-host copy per transformer
forward, as in the reference.
"""

from __future__ import annotations

from dataclasses import dataclass, field
from types import MethodType
from typing import Any


@dataclass
class H3InvariantCacheRuntime:
    """State owned by one resident H3 transformer (invariants.py:10-68)."""

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

    def begin_request(self) -> None:
        """Forget request values and reset the per-request counters; schedule
        values survive (they are keyed by timestep)."""

        self.request_values.clear()
        self.current_timestep_key = None
        self.request_hits = 0
        self.request_misses = 0
        self.schedule_hits = 0
        self.schedule_misses = 0

    def audit(self) -> dict[str, int]:
        return {
            "request_hits": self.request_hits,
            "request_misses": self.request_misses,
            "schedule_hits": self.schedule_hits,
            "schedule_misses": self.schedule_misses,
            "schedule_entries": sum(len(values) for values in self.schedule_values.values()),
            "schedule_frozen": self.schedule_frozen,
            "freed_parameter_bytes": self.freed_parameter_bytes,
        }

    def freeze_fixed_schedule(self, expected_values_per_site: int = 49) -> int:
        """Drop the AdaLN projection weights after every fixed-schedule value is
        cached; returns the bytes released."""

        if expected_values_per_site < 1:
            raise ValueError("expected_values_per_site must be positive")
        if self.schedule_frozen:
            return self.freed_parameter_bytes
        if not self.schedule_values or any(
            len(values) < expected_values_per_site for values in self.schedule_values.values()
        ):
            raise RuntimeError(
                "cannot freeze AdaLN projections before all expected schedule "
                f"values are cached ({expected_values_per_site} per site)"
            )
        released = 0
        for module in self.adaln_modules:
            for parameter in module.linear.parameters():
                released += parameter.numel() * parameter.element_size()
            module.linear = None
        self.freed_parameter_bytes = released
        self.schedule_frozen = True
        return released


def _timestep_key(timestep: Any) -> tuple[Any, ...]:
    """(shape, dtype, *values) of a timestep tensor (invariants.py:71-77)."""

    values = timestep.detach().float().cpu().reshape(-1).tolist()
    return (tuple(timestep.shape), str(timestep.dtype), *(float(value) for value in values))


def _wrap_request_value(module: Any, name: str, runtime: H3InvariantCacheRuntime) -> None:
    """Cache ``module``'s first result of a request (invariants.py:80-95)."""

    compute = module.forward

    def forward(_module: Any, *args: Any, **kwargs: Any) -> Any:
        cached = runtime.request_values.get(name, _MISSING)
        if cached is not _MISSING:
            runtime.request_hits += 1
            return cached
        value = compute(*args, **kwargs)
        runtime.request_values[name] = value
        runtime.request_misses += 1
        return value

    module.forward = MethodType(forward, module)


def _wrap_schedule_value(module: Any, name: str, runtime: H3InvariantCacheRuntime) -> None:
    """Cache ``module``'s result per timestep key (invariants.py:98-122)."""

    compute = module.forward
    values = runtime.schedule_values.setdefault(name, {})

    def forward(_module: Any, *args: Any, **kwargs: Any) -> Any:
        key = runtime.current_timestep_key
        if key is None:
            raise RuntimeError(f"schedule cache {name} called outside H3 transformer forward")
        cached = values.get(key, _MISSING)
        if cached is not _MISSING:
            runtime.schedule_hits += 1
            return cached
        if runtime.schedule_frozen:
            raise RuntimeError(
                f"fixed-schedule cache {name} received an unseen timestep after weights were released"
            )
        value = compute(*args, **kwargs)
        values[key] = value
        runtime.schedule_misses += 1
        return value

    module.forward = MethodType(forward, module)


class _Missing:
    pass


_MISSING = _Missing()


def install_h3_invariant_caches(transformer: Any) -> H3InvariantCacheRuntime:
    """Wrap the invariant producers of ``transformer`` (invariants.py:125-157).

    Idempotent: a transformer that already has a cache returns it."""

    installed = getattr(transformer, "_h3_flash_invariant_cache", None)
    if installed is not None:
        return installed
    runtime = H3InvariantCacheRuntime()
    _wrap_request_value(transformer.context_embedder, "context_embedder", runtime)
    _wrap_request_value(transformer.token_refiner, "token_refiner", runtime)
    _wrap_request_value(transformer.rope, "rope", runtime)
    for index, block in enumerate(transformer.transformer_blocks):
        _wrap_schedule_value(block.adaln_proj, f"adaln.{index}", runtime)
        runtime.adaln_modules.append(block.adaln_proj)
    _wrap_schedule_value(transformer.norm_out.linear, "norm_out.linear", runtime)

    forward_body = transformer.forward

    def forward(_module: Any, *args: Any, **kwargs: Any) -> Any:
        timestep = kwargs.get("timestep")
        if timestep is None:
            if len(args) < 4:
                raise RuntimeError("cannot resolve H3 timestep for schedule cache")
            timestep = args[3]
        runtime.current_timestep_key = _timestep_key(timestep)
        try:
            return forward_body(*args, **kwargs)
        finally:
            runtime.current_timestep_key = None

    transformer.forward = MethodType(forward, transformer)
    transformer._h3_flash_invariant_cache = runtime
    return runtime
