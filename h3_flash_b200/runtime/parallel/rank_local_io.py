"""Rank-local H3 input projection and compact output gather.

Drop-in for ``h3_flash.runtime.parallel.rank_local_io``
(src/h3_flash/runtime/parallel/rank_local_io.py). Each rank owns a contiguous
slice of the packed sequence (``_split_sizes``: the first ``total % W`` ranks
get one extra row). Instead of projecting every token on every rank and slicing
(what Diffusers' context-parallel hooks do), a rank:

- projects only the text/video/audio tokens that fall in its slice and places
  them at their local rows (rank_local_io.py:174-191), and builds RoPE tables
  for its rows only;
- runs the block stack on its rows with ``adaln_indices = timestep*3 + tag``;
- applies the output norm and the video/audio heads to its own rows of each
  modality and gathers the (uneven) per-rank results (rank_local_io.py:240-252).

The gather differs from the reference's list ``all_gather`` + concatenate
(rank_local_io.py:44-52) only in how the bytes move: every rank sends a
row-padded block into one contiguous ``[W, B, max_rows, C]`` buffer (one
``all_gather_into_tensor`` on NCCL) and the valid rows are packed with one
concatenation. The result is the same tensor, bit for bit.

The first call (the "gate") also computes the full-sequence reference on every
rank and records error metrics, as the reference does (rank_local_io.py:205-232,
:261-279).
"""

from __future__ import annotations

from types import MethodType
from typing import Any

import torch
import torch.distributed as dist


def _split_sizes(total: int, parts: int) -> list[int]:
    """rank_local_io.py:13-15."""

    quotient, remainder = divmod(total, parts)
    return [quotient + (index < remainder) for index in range(parts)]


def _split_bounds(total: int, parts: int, rank: int) -> tuple[int, int]:
    """rank_local_io.py:18-21."""

    sizes = _split_sizes(total, parts)
    start = sum(sizes[:rank])
    return start, start + sizes[rank]


def _local_modality_indices(indices: torch.Tensor, start: int, stop: int) -> tuple[torch.Tensor, torch.Tensor]:
    """Positions (in ``indices``) of a modality's tokens inside rows [start, stop)
    and their local rows (rank_local_io.py:24-30)."""

    inside = (indices >= start) & (indices < stop)
    source = torch.nonzero(inside, as_tuple=False).flatten()
    return source, indices.index_select(0, source) - start


def _modality_counts(indices: torch.Tensor, row_counts: list[int]) -> list[int]:
    """How many of a (sorted) modality's tokens each rank owns (rank_local_io.py:33-41)."""

    ends = torch.tensor(
        [sum(row_counts[: index + 1]) for index in range(len(row_counts))],
        dtype=indices.dtype, device=indices.device,
    )
    cumulative = torch.searchsorted(indices, ends, right=False)
    cumulative = torch.cat([cumulative.new_zeros(1), cumulative])
    return [int(value) for value in torch.diff(cumulative).tolist()]


def _gather_uneven(value: torch.Tensor, counts: list[int], group: Any) -> torch.Tensor:
    """Concatenate every rank's ``value[:, :counts[rank]]`` along dim 1."""

    world = len(counts)
    batch, rows, channels = value.shape
    longest = max(counts)
    padded = value.new_zeros((batch, longest, channels))
    padded[:, :rows] = value
    if str(dist.get_backend(group)) == "nccl":
        gathered = value.new_empty((world * batch, longest, channels))
        dist.all_gather_into_tensor(gathered, padded, group=group)
        parts = gathered.view(world, batch, longest, channels)
        return torch.cat([parts[w, :, : counts[w]] for w in range(world)], dim=1)
    parts = [torch.empty_like(padded) for _ in range(world)]
    dist.all_gather(parts, padded, group=group)
    return torch.cat([part[:, :rows_w] for part, rows_w in zip(parts, counts, strict=True)], dim=1)


def _metrics(actual: torch.Tensor, reference: torch.Tensor, group: Any) -> dict[str, float]:
    """Max over ranks of max |d|, mean |d| and relative L2 (rank_local_io.py:55-71)."""

    delta = (actual.float() - reference.float()).abs()
    values = torch.stack([delta.max(), delta.mean(),
                          delta.norm() / reference.float().norm().clamp_min(1e-12)])
    dist.all_reduce(values, op=dist.ReduceOp.MAX, group=group)
    return {"max_abs": float(values[0]), "max_rank_mean_abs": float(values[1]),
            "max_rank_relative_l2": float(values[2])}


def _official_rope(module: Any, position_ids: torch.Tensor) -> tuple[torch.Tensor, ...]:
    """The RoPE tables of the upstream model (rank_local_io.py:74-80): angles of
    the (time, height, width) axes concatenated, then duplicated."""

    angles = position_ids.to(torch.float32).unsqueeze(-1) * module.inv_freq.view(1, 1, -1)
    angles = torch.cat(angles.unbind(dim=1), dim=-1)
    angles = torch.cat((angles, angles), dim=-1)
    return angles.cos(), angles.sin()


class RankLocalIORuntime:
    """Settings and first-call gate metrics (rank_local_io.py:83-106)."""

    def __init__(self, *, group: Any, rank_local_inputs: bool, compact_output_gather: bool) -> None:
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.rank_local_inputs = rank_local_inputs
        self.compact_output_gather = compact_output_gather
        self.gate: dict[str, Any] = {}
        self._gate_complete = False

    def provenance(self) -> dict[str, Any]:
        return {
            "enabled": True,
            "rank_local_inputs": self.rank_local_inputs,
            "compact_output_gather": self.compact_output_gather,
            "semantics": "all_rows_projected_exactly_once_then_gathered",
            "gate": self.gate,
            "origin": "B200-native rebuild of the H3-Flash rank-local I/O",
        }


def _full_sequence_inputs(model: Any, hidden_states, audio_hidden_states, text_embeds,
                          video_indices, audio_indices, text_indices, sequence_length: int):
    video = model.proj_in(hidden_states.to(model.proj_in.weight.dtype))
    audio = model.audio_proj_in(audio_hidden_states.to(model.audio_proj_in.weight.dtype))
    full = text_embeds.new_zeros((text_embeds.shape[0], sequence_length, text_embeds.shape[-1]))
    full = full.index_copy(1, text_indices, text_embeds)
    full = full.index_copy(1, video_indices, video.to(full.dtype))
    return full.index_copy(1, audio_indices, audio.to(full.dtype))


def _full_sequence_heads(model: Any, full: torch.Tensor, temb, timestep_indices, video_indices, audio_indices):
    full = model.norm_out(full, temb, timestep_indices).to(model.proj_out.weight.dtype)
    return (model.proj_out(full).index_select(1, video_indices),
            model.audio_proj_out(full).index_select(1, audio_indices))


def _output_class() -> Any:
    """Diffusers' H3 output type when Diffusers is present, else this package's."""

    try:
        from diffusers.models.transformers.transformer_minimax_h3 import MiniMaxH3TransformerOutput

        return MiniMaxH3TransformerOutput
    except ImportError:
        from ..h3_model import H3Output

        return H3Output


def install_rank_local_io(transformer: Any, *, group: Any = None, rank_local_inputs: bool = True,
                          compact_output_gather: bool = True) -> RankLocalIORuntime:
    """Replace the transformer forward with explicit uneven rank-local execution
    (rank_local_io.py:109-309). Install after context parallelism: Diffusers'
    context-parallel hooks are removed because this forward shards by itself."""

    if not (dist.is_available() and dist.is_initialized()):
        raise RuntimeError("rank-local H3 I/O requires an initialized process group")
    group = group or dist.group.WORLD
    runtime = RankLocalIORuntime(group=group, rank_local_inputs=rank_local_inputs,
                                 compact_output_gather=compact_output_gather)
    if runtime.world < 2:
        raise RuntimeError("rank-local H3 I/O requires at least two ranks")
    plan = getattr(transformer, "_h3_flash_cp_plan", None)
    hooked = getattr(getattr(transformer, "_parallel_config", None), "context_parallel_config", None)
    if plan is not None:
        from diffusers.hooks.context_parallel import remove_context_parallel

        remove_context_parallel(transformer, plan)
    elif hooked is not None:
        raise RuntimeError("rank-local H3 I/O must be installed after context parallelism")
    # (A module with no context-parallel hooks at all, like this package's
    # H3Transformer, has nothing to remove.)

    def forward(self, hidden_states, audio_hidden_states, encoder_hidden_states, timestep,
                timestep_indices, token_tags, position_ids, video_indices, audio_indices,
                text_indices, attention_kwargs=None, return_dict=True):
        if attention_kwargs:
            raise RuntimeError("rank-local H3 I/O does not support runtime LoRA scaling")
        if position_ids.ndim != 2 or position_ids.shape[-1] != 3:
            raise ValueError("position_ids must have shape (sequence, 3)")
        sequence_length = position_ids.shape[0]
        if bool((token_tags < 0).any()):
            raise RuntimeError("rank-local H3 I/O requires a padless packed sequence")
        start, stop = _split_bounds(sequence_length, runtime.world, runtime.rank)
        row_counts = _split_sizes(sequence_length, runtime.world)
        local_timesteps = timestep_indices[start:stop].contiguous()
        adaln_indices = local_timesteps * 3 + token_tags[start:stop].clamp(min=0)

        text_embeds = self.context_embedder(encoder_hidden_states.to(self.context_embedder.weight.dtype))
        text_embeds = self.token_refiner(text_embeds)
        temb = self.time_embedder(self.time_proj(timestep).to(self.time_embedder.linear_1.weight.dtype))

        if runtime.rank_local_inputs:
            local = text_embeds.new_zeros((text_embeds.shape[0], stop - start, text_embeds.shape[-1]))
            for indices, values, projection in ((text_indices, text_embeds, None),
                                                (video_indices, hidden_states, self.proj_in),
                                                (audio_indices, audio_hidden_states, self.audio_proj_in)):
                source, destination = _local_modality_indices(indices, start, stop)
                if not source.numel():
                    continue
                selected = values.index_select(1, source)
                if projection is not None:
                    selected = projection(selected.to(projection.weight.dtype))
                local = local.index_copy(1, destination, selected.to(local.dtype))
            rotary_emb = self.rope(position_ids[start:stop])
        else:
            full = _full_sequence_inputs(self, hidden_states, audio_hidden_states, text_embeds,
                                         video_indices, audio_indices, text_indices, sequence_length)
            local = full[:, start:stop].contiguous()
            rotary_emb = tuple(value[start:stop].contiguous() for value in self.rope(position_ids))

        gate_this_call = not runtime._gate_complete
        if gate_this_call and runtime.rank_local_inputs:
            reference = _full_sequence_inputs(self, hidden_states, audio_hidden_states, text_embeds,
                                              video_indices, audio_indices, text_indices, sequence_length)
            rotary_reference = _official_rope(self.rope, position_ids)
            runtime.gate["rank_local_inputs"] = {
                "hidden_states": _metrics(local, reference[:, start:stop], runtime.group),
                "rotary": [_metrics(actual, expected[start:stop], runtime.group)
                           for actual, expected in zip(rotary_emb, rotary_reference, strict=True)],
            }

        for block in self.transformer_blocks:
            local = block(local, temb, adaln_indices, rotary_emb, None)

        if runtime.compact_output_gather:
            def project(indices, head):
                _, destination = _local_modality_indices(indices, start, stop)
                rows = self.norm_out(local.index_select(1, destination), temb,
                                     local_timesteps.index_select(0, destination))
                rows = head(rows.to(head.weight.dtype))
                return _gather_uneven(rows, _modality_counts(indices, row_counts), runtime.group)

            video_output = project(video_indices, self.proj_out)
            audio_output = project(audio_indices, self.audio_proj_out)
        else:
            full = _gather_uneven(local, row_counts, runtime.group)
            video_output, audio_output = _full_sequence_heads(self, full, temb, timestep_indices,
                                                              video_indices, audio_indices)

        if gate_this_call and runtime.compact_output_gather:
            full = _gather_uneven(local, row_counts, runtime.group)
            video_reference, audio_reference = _full_sequence_heads(self, full, temb, timestep_indices,
                                                                    video_indices, audio_indices)
            runtime.gate["compact_output_gather"] = {
                "video": _metrics(video_output, video_reference, runtime.group),
                "audio": _metrics(audio_output, audio_reference, runtime.group),
            }
        runtime._gate_complete = True
        if not return_dict:
            return video_output, audio_output
        return _output_class()(sample=video_output, audio_sample=audio_output)

    # An invariant cache installed earlier keys its schedule values by the
    # timestep of the running forward; keep that scope around the new forward.
    cache_runtime = getattr(transformer, "_h3_flash_invariant_cache", None)
    if cache_runtime is not None:
        from ..cache.invariants import _timestep_key

        body = forward

        def cached_forward(self, *args, **kwargs):
            timestep = kwargs.get("timestep")
            if timestep is None:
                timestep = args[3]
            cache_runtime.current_timestep_key = _timestep_key(timestep)
            try:
                return body(self, *args, **kwargs)
            finally:
                cache_runtime.current_timestep_key = None

        transformer.forward = MethodType(cached_forward, transformer)
    else:
        transformer.forward = MethodType(forward, transformer)
    return runtime
