"""Rank-local H3 input projection and compact output gather.

Interface of ``h3_flash.runtime.parallel.rank_local_io`` (src/h3_flash/runtime/parallel/
rank_local_io.py:83-309): ``install_rank_local_io(transformer, *, group,
rank_local_inputs, compact_output_gather)`` returning a runtime with ``provenance()``
and the first-call ``gate`` metrics, and the same error messages.

Design. The packed sequence (text, video and audio tokens at the positions their index
vectors name) is cut into W contiguous row shards, the first ``S % W`` one row longer.
A ``_Shard`` describes this rank's rows; ``_RankLocalForward`` runs one transformer call
in three stages:

1. inputs: each modality's tokens that fall inside the shard are projected (video and
   audio through their input projections, text already embedded) and scattered to their
   local rows; the RoPE tables are built for the shard's positions only. Without
   ``rank_local_inputs`` the whole sequence is assembled and sliced instead;
2. the block stack on the shard, with ``adaln_indices = timestep_index * 3 + tag``;
3. outputs: with ``compact_output_gather`` each modality's rows of the shard go through
   the output norm and that modality's head here, and only those rows are gathered;
   otherwise the shard's hidden rows are gathered and the heads run on the full sequence.

Uneven gathers move one row-padded ``[B, max_rows, C]`` block per rank into a single
``[W * B, max_rows, C]`` buffer (``all_gather_into_tensor`` on NCCL, ``all_gather`` into
a list on gloo) and keep each rank's valid rows: the same tensor the reference's list
gather and concatenation produce.

On the first call the gate computes the full-sequence inputs, RoPE tables and heads on
every rank and records the differences (max over ranks of max |d|, mean |d|, relative
L2).
"""

from __future__ import annotations

from dataclasses import dataclass
from itertools import accumulate
from types import MethodType
from typing import Any

import torch
import torch.distributed as dist


def _split_sizes(total: int, parts: int) -> list[int]:
    """Contiguous shard lengths: the first ``total % parts`` shards are one longer."""

    base, extra = divmod(total, parts)
    return [base + 1] * extra + [base] * (parts - extra)


def _split_bounds(total: int, parts: int, rank: int) -> tuple[int, int]:
    """[start, stop) of shard ``rank``."""

    ends = [0, *accumulate(_split_sizes(total, parts))]
    return ends[rank], ends[rank + 1]


def _local_modality_indices(indices: torch.Tensor, start: int, stop: int) -> tuple[torch.Tensor, torch.Tensor]:
    """For a modality whose tokens sit at sequence rows ``indices``: which of its tokens
    fall in rows [start, stop) (positions in ``indices``) and their rows in the shard."""

    positions = torch.arange(indices.numel(), device=indices.device)
    keep = (indices >= start) & (indices < stop)
    source = positions[keep]
    return source, indices[keep] - start


def _modality_counts(indices: torch.Tensor, row_counts: list[int]) -> list[int]:
    """How many of a modality's tokens (``indices`` sorted) each shard holds."""

    ends = torch.tensor(list(accumulate(row_counts)), dtype=indices.dtype, device=indices.device)
    shard_of_token = torch.bucketize(indices, ends, right=True)
    return torch.bincount(shard_of_token, minlength=len(row_counts))[: len(row_counts)].tolist()


def _gather_uneven(value: torch.Tensor, counts: list[int], group: Any) -> torch.Tensor:
    """Concatenate every rank's ``value[:, :counts[rank]]`` along dim 1."""

    world = len(counts)
    batch, rows, channels = value.shape
    longest = max(counts)
    block = value.new_zeros((batch, longest, channels))
    block[:, :rows] = value
    if str(dist.get_backend(group)) == "nccl":
        flat = value.new_empty((world * batch, longest, channels))
        dist.all_gather_into_tensor(flat, block, group=group)
        blocks = list(flat.view(world, batch, longest, channels).unbind(0))
    else:
        blocks = [torch.empty_like(block) for _ in range(world)]
        dist.all_gather(blocks, block, group=group)
    return torch.cat([b[:, :n] for b, n in zip(blocks, counts, strict=True)], dim=1)


def _metrics(actual: torch.Tensor, reference: torch.Tensor, group: Any) -> dict[str, float]:
    """Max over ranks of max |d|, mean |d| and relative L2 (the reference's gate keys)."""

    delta = (actual.float() - reference.float()).abs()
    stats = torch.stack([delta.max(), delta.mean(), delta.norm() / reference.float().norm().clamp_min(1e-12)])
    dist.all_reduce(stats, op=dist.ReduceOp.MAX, group=group)
    worst_max, worst_mean, worst_rel = (float(v) for v in stats)
    return {"max_abs": worst_max, "max_rank_mean_abs": worst_mean, "max_rank_relative_l2": worst_rel}


def _official_rope(module: Any, position_ids: torch.Tensor) -> tuple[torch.Tensor, ...]:
    """RoPE tables of the upstream model for ``position_ids`` [S, 3]: per-axis angles
    position * inv_freq, the three axes side by side, the whole repeated twice."""

    angles = torch.cat([position_ids[:, axis:axis + 1].to(torch.float32) * module.inv_freq.view(1, -1)
                        for axis in range(3)], dim=-1)
    angles = angles.repeat(1, 2)
    return angles.cos(), angles.sin()


class RankLocalIORuntime:
    """Settings of an installation and the first call's gate metrics."""

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


@dataclass(frozen=True)
class _Shard:
    start: int
    stop: int
    row_counts: list[int]

    @classmethod
    def of(cls, total: int, runtime: RankLocalIORuntime) -> _Shard:
        start, stop = _split_bounds(total, runtime.world, runtime.rank)
        return cls(start, stop, _split_sizes(total, runtime.world))

    @property
    def rows(self) -> int:
        return self.stop - self.start


class _RankLocalForward:
    """One transformer call, stage by stage (see the module docstring)."""

    def __init__(self, model: Any, runtime: RankLocalIORuntime) -> None:
        self.model = model
        self.rt = runtime

    # -- stage 1 ------------------------------------------------------------------------

    def _assembled_sequence(self, text, video, audio, indices, length: int) -> torch.Tensor:
        """The full input sequence with every modality projected and placed."""

        m = self.model
        text_indices, video_indices, audio_indices = indices
        out = text.new_zeros((text.shape[0], length, text.shape[-1]))
        out[:, text_indices] = text
        out[:, video_indices] = m.proj_in(video.to(m.proj_in.weight.dtype)).to(out.dtype)
        out[:, audio_indices] = m.audio_proj_in(audio.to(m.audio_proj_in.weight.dtype)).to(out.dtype)
        return out

    def _shard_inputs(self, text, video, audio, indices, shard: _Shard) -> torch.Tensor:
        """This shard's rows of the input sequence, projecting only its own tokens."""

        m = self.model
        out = text.new_zeros((text.shape[0], shard.rows, text.shape[-1]))
        sources = ((indices[0], text, None), (indices[1], video, m.proj_in), (indices[2], audio, m.audio_proj_in))
        for token_rows, values, projection in sources:
            picked, local_rows = _local_modality_indices(token_rows, shard.start, shard.stop)
            if picked.numel() == 0:
                continue
            tokens = values[:, picked]
            if projection is not None:
                tokens = projection(tokens.to(projection.weight.dtype))
            out[:, local_rows] = tokens.to(out.dtype)
        return out

    # -- stage 3 ------------------------------------------------------------------------

    def _heads_of_sequence(self, hidden, temb, timestep_indices, video_indices, audio_indices):
        m = self.model
        normed = m.norm_out(hidden, temb, timestep_indices).to(m.proj_out.weight.dtype)
        return m.proj_out(normed)[:, video_indices], m.audio_proj_out(normed)[:, audio_indices]

    def _compact_head(self, local, temb, local_timesteps, token_rows, head, shard: _Shard) -> torch.Tensor:
        _, local_rows = _local_modality_indices(token_rows, shard.start, shard.stop)
        rows = self.model.norm_out(local[:, local_rows], temb, local_timesteps[local_rows])
        rows = head(rows.to(head.weight.dtype))
        return _gather_uneven(rows, _modality_counts(token_rows, shard.row_counts), self.rt.group)

    # -- the call -------------------------------------------------------------------------

    def __call__(self, hidden_states, audio_hidden_states, encoder_hidden_states, timestep, timestep_indices,
                 token_tags, position_ids, video_indices, audio_indices, text_indices, attention_kwargs=None,
                 return_dict=True):
        m, rt = self.model, self.rt
        if attention_kwargs:
            raise RuntimeError("rank-local H3 I/O does not support runtime LoRA scaling")
        if position_ids.ndim != 2 or position_ids.shape[-1] != 3:
            raise ValueError("position_ids must have shape (sequence, 3)")
        if bool((token_tags < 0).any()):
            raise RuntimeError("rank-local H3 I/O requires a padless packed sequence")
        length = position_ids.shape[0]
        shard = _Shard.of(length, rt)
        local_timesteps = timestep_indices[shard.start:shard.stop].contiguous()
        adaln_indices = local_timesteps * 3 + token_tags[shard.start:shard.stop].clamp(min=0)
        text = m.token_refiner(m.context_embedder(encoder_hidden_states.to(m.context_embedder.weight.dtype)))
        temb = m.time_embedder(m.time_proj(timestep).to(m.time_embedder.linear_1.weight.dtype))
        indices = (text_indices, video_indices, audio_indices)
        gating = not rt._gate_complete

        if rt.rank_local_inputs:
            local = self._shard_inputs(text, hidden_states, audio_hidden_states, indices, shard)
            rotary = m.rope(position_ids[shard.start:shard.stop])
            if gating:
                whole = self._assembled_sequence(text, hidden_states, audio_hidden_states, indices, length)
                expected_rotary = _official_rope(m.rope, position_ids)
                rt.gate["rank_local_inputs"] = {
                    "hidden_states": _metrics(local, whole[:, shard.start:shard.stop], rt.group),
                    "rotary": [_metrics(a, b[shard.start:shard.stop], rt.group)
                               for a, b in zip(rotary, expected_rotary, strict=True)],
                }
        else:
            whole = self._assembled_sequence(text, hidden_states, audio_hidden_states, indices, length)
            local = whole[:, shard.start:shard.stop].contiguous()
            rotary = tuple(t[shard.start:shard.stop].contiguous() for t in m.rope(position_ids))

        for block in m.transformer_blocks:
            local = block(local, temb, adaln_indices, rotary, None)

        if rt.compact_output_gather:
            video_out = self._compact_head(local, temb, local_timesteps, video_indices, m.proj_out, shard)
            audio_out = self._compact_head(local, temb, local_timesteps, audio_indices, m.audio_proj_out, shard)
            if gating:
                hidden = _gather_uneven(local, shard.row_counts, rt.group)
                expected = self._heads_of_sequence(hidden, temb, timestep_indices, video_indices, audio_indices)
                rt.gate["compact_output_gather"] = {"video": _metrics(video_out, expected[0], rt.group),
                                                    "audio": _metrics(audio_out, expected[1], rt.group)}
        else:
            hidden = _gather_uneven(local, shard.row_counts, rt.group)
            video_out, audio_out = self._heads_of_sequence(hidden, temb, timestep_indices, video_indices,
                                                           audio_indices)
        rt._gate_complete = True
        if not return_dict:
            return video_out, audio_out
        return _output_class()(sample=video_out, audio_sample=audio_out)


def _output_class() -> Any:
    """Diffusers' H3 output type when Diffusers is present, else this package's."""

    try:
        from diffusers.models.transformers.transformer_minimax_h3 import MiniMaxH3TransformerOutput

        return MiniMaxH3TransformerOutput
    except ImportError:
        from ..h3_model import H3Output

        return H3Output


def _detach_context_parallel_hooks(transformer: Any) -> None:
    """This forward shards by itself, so Diffusers' context-parallel hooks (installed
    with a recorded plan) come off; a model with hooks but no plan was set up in the
    wrong order; a model without hooks (this package's H3Transformer) has none."""

    plan = getattr(transformer, "_h3_flash_cp_plan", None)
    config = getattr(transformer, "_parallel_config", None)
    if plan is not None:
        from diffusers.hooks.context_parallel import remove_context_parallel

        remove_context_parallel(transformer, plan)
    elif getattr(config, "context_parallel_config", None) is not None:
        raise RuntimeError("rank-local H3 I/O must be installed after context parallelism")


def install_rank_local_io(transformer: Any, *, group: Any = None, rank_local_inputs: bool = True,
                          compact_output_gather: bool = True) -> RankLocalIORuntime:
    """Replace ``transformer.forward`` with the rank-local call (rank_local_io.py:109-309).
    Collective: every rank of ``group`` calls the transformer together."""

    if not (dist.is_available() and dist.is_initialized()):
        raise RuntimeError("rank-local H3 I/O requires an initialized process group")
    group = group or dist.group.WORLD
    runtime = RankLocalIORuntime(group=group, rank_local_inputs=rank_local_inputs,
                                 compact_output_gather=compact_output_gather)
    if runtime.world < 2:
        raise RuntimeError("rank-local H3 I/O requires at least two ranks")
    _detach_context_parallel_hooks(transformer)
    call = _RankLocalForward(transformer, runtime)
    cache = getattr(transformer, "_h3_flash_invariant_cache", None)

    def forward(_self: Any, *args: Any, **kwargs: Any) -> Any:
        if cache is None:
            return call(*args, **kwargs)
        # An invariant cache installed earlier keys its schedule values by the running
        # call's timestep; the replaced forward that set it is gone, so set it here.
        from ..cache.invariants import _timestep_argument, _timestep_key

        cache.current_timestep_key = _timestep_key(_timestep_argument(args, kwargs))
        try:
            return call(*args, **kwargs)
        finally:
            cache.current_timestep_key = None

    transformer.forward = MethodType(forward, transformer)
    return runtime
