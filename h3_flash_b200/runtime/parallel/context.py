"""Padless Ulysses context-parallel setup for the Diffusers MiniMax H3 model.

Mirror of src/h3_flash/runtime/parallel/context.py. These helpers configure
Diffusers' own context-parallel hooks (set-up only, nothing on the per-block
path), so they import Diffusers lazily and fail with the reference's messages
when the process group or Diffusers is missing.
"""

from __future__ import annotations

from typing import Any


def h3_context_parallel_plan() -> dict[str, Any]:
    """Diffusers CP hook plan (context.py:14-52): split the stack input and the
    per-block AdaLN indices/RoPE tables by rows, gather before the output heads."""

    from diffusers.models._modeling_parallel import ContextParallelInput, ContextParallelOutput

    return {
        "rope": {
            0: ContextParallelInput(split_dim=0, expected_dims=2, split_output=True),
            1: ContextParallelInput(split_dim=0, expected_dims=2, split_output=True),
        },
        "transformer_blocks.*": {
            "adaln_indices": ContextParallelInput(split_dim=0, expected_dims=1, split_output=False),
        },
        "transformer_blocks.0": {
            "hidden_states": ContextParallelInput(split_dim=1, expected_dims=3, split_output=False),
        },
        "norm_out": {
            "timestep_indices": ContextParallelInput(split_dim=0, expected_dims=1, split_output=False),
        },
        "proj_out": ContextParallelOutput(gather_dim=1, expected_dims=3),
        "audio_proj_out": ContextParallelOutput(gather_dim=1, expected_dims=3),
    }


def _guard_padless(transformer: Any) -> None:
    """Reject padded packed sequences (context.py:55-72)."""

    if getattr(transformer, "_h3_flash_padless_guard", False):
        return
    original = transformer.forward

    def guarded(*args: Any, **kwargs: Any) -> Any:
        token_tags = kwargs.get("token_tags")
        if token_tags is None and len(args) >= 6:
            token_tags = args[5]
        if token_tags is not None and bool((token_tags < 0).any()):
            raise RuntimeError(
                "H3 lossless context parallelism requires a padless packed "
                "sequence; padding rows would require a row-sharded mask"
            )
        return original(*args, **kwargs)

    transformer.forward = guarded
    transformer._h3_flash_padless_guard = True


def enable_h3_ulysses(transformer: Any, *, degree: int, ulysses_anything: bool = True) -> dict[str, Any]:
    """Enable Diffusers-native dense Ulysses on an initialized process group (context.py:75-119)."""

    import torch.distributed as dist

    if not (dist.is_available() and dist.is_initialized()):
        raise RuntimeError("Ulysses requires an initialized torch process group")
    world_size = dist.get_world_size()
    if degree != world_size:
        raise RuntimeError(f"Ulysses degree {degree} must equal process-group world size {world_size}")
    if degree < 2:
        raise RuntimeError("Ulysses degree must be at least two")
    from diffusers.models._modeling_parallel import ContextParallelConfig

    _guard_padless(transformer)
    transformer.set_attention_backend("native")
    plan = h3_context_parallel_plan()
    transformer.enable_parallelism(
        config=ContextParallelConfig(ulysses_degree=degree, ulysses_anything=ulysses_anything),
        cp_plan=plan,
    )
    transformer._h3_flash_cp_plan = plan
    return {
        "backend": "diffusers_native_ulysses",
        "degree": degree,
        "ulysses_anything": ulysses_anything,
        "semantics": "dense",
    }


def with_context_parallel_reapplied(transformer: Any, action: Any) -> Any:
    """Run ``action`` with Diffusers' CP hooks removed, then re-apply them (context.py:122-145).
    Modules without Diffusers CP configured run ``action`` directly."""

    parallel_config = getattr(transformer, "_parallel_config", None)
    cp_config = getattr(parallel_config, "context_parallel_config", None) if parallel_config is not None else None
    if cp_config is None:
        return action()
    plan = getattr(transformer, "_h3_flash_cp_plan", None)
    if plan is None:
        raise RuntimeError("context parallelism is enabled without its recorded plan")
    from diffusers.hooks.context_parallel import apply_context_parallel, remove_context_parallel

    remove_context_parallel(transformer, plan)
    try:
        return action()
    finally:
        apply_context_parallel(transformer, cp_config, plan)
