"""Rank-local input projection and compact output gather
(src/h3_flash/runtime/parallel/rank_local_io.py), on CPU.

The helpers are checked against direct restatements; then two gloo ranks run a
transformer with no blocks (the blocks are covered by the packed-Ulysses
tests): with every combination of rank-local inputs and compact output gather,
each rank's video and audio outputs must equal the full-sequence forward of the
same model, uneven splits included, and the first call's gate metrics must be
recorded.
"""

from __future__ import annotations

import pytest
import torch

from h3_flash_b200.runtime.parallel.rank_local_io import (
    _local_modality_indices,
    _modality_counts,
    _split_bounds,
    _split_sizes,
)


def test_split_sizes_and_bounds():
    assert _split_sizes(10, 3) == [4, 3, 3]
    assert _split_sizes(2, 4) == [1, 1, 0, 0]
    assert [_split_bounds(10, 3, r) for r in range(3)] == [(0, 4), (4, 7), (7, 10)]
    for total in range(0, 40):
        for parts in range(1, 9):
            sizes = _split_sizes(total, parts)
            assert sum(sizes) == total and max(sizes) - min(sizes) <= 1


def test_local_modality_indices_and_counts():
    indices = torch.tensor([1, 2, 5, 6, 7, 11])
    source, destination = _local_modality_indices(indices, 5, 8)
    assert source.tolist() == [2, 3, 4] and destination.tolist() == [0, 1, 2]
    counts = [4, 4, 4]  # rows [0,4) [4,8) [8,12)
    assert _modality_counts(indices, counts) == [2, 3, 1]
    g = torch.Generator().manual_seed(3)
    for _ in range(20):
        total = int(torch.randint(5, 60, (1,), generator=g))
        parts = int(torch.randint(1, 6, (1,), generator=g))
        picked = torch.nonzero(torch.rand(total, generator=g) < 0.4).flatten()
        sizes = _split_sizes(total, parts)
        expect = []
        for r in range(parts):
            lo, hi = _split_bounds(total, parts, r)
            expect.append(int(((picked >= lo) & (picked < hi)).sum()))
        assert _modality_counts(picked, sizes) == expect


def _model():
    from h3_flash_b200.runtime.h3_model import H3Transformer

    torch.manual_seed(0)
    return H3Transformer(32, 2, 16, 64, 0, text_dim=12, video_channels=8, audio_channels=6,
                         freq_dim=16, freqs_per_axis=2, dtype=torch.float64).eval()


def _inputs(model):
    from h3_flash_b200.runtime.h3_model import make_inputs

    return make_inputs(model, n_text=5, n_video=24, n_audio=4, text_dim=12, grid=(2, 3, 4),
                       n_timesteps=2, seed=4, dtype=torch.float64)


def _rank_local_worker(rank, world, rank_local_inputs, compact):
    import torch.distributed as dist

    from h3_flash_b200.runtime.parallel import install_rank_local_io

    model = _model()
    inputs = _inputs(model)
    with torch.no_grad():
        expect = model(**inputs, return_dict=False)
        runtime = install_rank_local_io(model, group=dist.group.WORLD, rank_local_inputs=rank_local_inputs,
                                        compact_output_gather=compact)
        got = model(**inputs, return_dict=False)
        again = model(**inputs, return_dict=False)  # after the gate
    diffs = [float((a - b).abs().max()) for a, b in zip(got, expect)]
    repeat = all(torch.equal(a, b) for a, b in zip(got, again))
    shapes = [tuple(t.shape) for t in got]
    return diffs, repeat, shapes, sorted(runtime.gate), runtime.provenance()["semantics"]


@pytest.mark.parametrize("rank_local_inputs,compact", [(True, True), (True, False), (False, True), (False, False)])
def test_rank_local_io_matches_full_sequence_forward(rank_local_inputs, compact):
    from tests.test_gloo import _run

    results = _run(2, _rank_local_worker, rank_local_inputs, compact)
    for diffs, repeat, shapes, gate, semantics in results:
        assert max(diffs) <= 1e-12, diffs
        assert repeat
        assert shapes == [(1, 24, 8), (1, 4, 6)]
        expect_gate = (["compact_output_gather"] if compact else []) + (["rank_local_inputs"] if rank_local_inputs else [])
        assert gate == sorted(expect_gate)
        assert semantics == "all_rows_projected_exactly_once_then_gathered"


def _errors_worker(rank, world):
    import torch.distributed as dist

    from h3_flash_b200.runtime.parallel import install_rank_local_io

    model = _model()
    inputs = _inputs(model)
    install_rank_local_io(model, group=dist.group.WORLD)
    messages = []
    for bad in (dict(attention_kwargs={"scale": 1.0}),
                dict(position_ids=inputs["position_ids"][:, :2]),
                dict(token_tags=inputs["token_tags"].clone().fill_(-1))):
        try:
            model(**{**inputs, **bad})
        except (RuntimeError, ValueError) as error:
            messages.append(str(error))
    return messages


def test_rank_local_io_errors():
    from tests.test_gloo import _run

    for messages in _run(2, _errors_worker):
        assert "LoRA scaling" in messages[0]
        assert "position_ids must have shape" in messages[1]
        assert "padless packed sequence" in messages[2]


def test_install_requires_process_group():
    from h3_flash_b200.runtime.parallel import install_rank_local_io

    with pytest.raises(RuntimeError, match="initialized process group"):
        install_rank_local_io(object())
