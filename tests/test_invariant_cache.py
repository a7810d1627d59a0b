"""Invariant caches: the behaviour of src/h3_flash/runtime/cache/invariants.py
(request values reused then cleared, schedule values keyed by timestep across
requests, fail-closed outside a forward and after freezing), then the installer
on this package's H3 transformer (CPU, fp32)."""

from __future__ import annotations

import pytest
import torch

from h3_flash_b200.runtime.cache import H3InvariantCacheRuntime, install_h3_invariant_caches
from h3_flash_b200.runtime.cache.invariants import _timestep_key, _wrap_request_value, _wrap_schedule_value


class Counter:
    def __init__(self) -> None:
        self.calls = 0

    def forward(self, value):
        self.calls += 1
        return value + self.calls


def test_request_value_is_reused_within_a_request_and_recomputed_after():
    runtime = H3InvariantCacheRuntime()
    module = Counter()
    _wrap_request_value(module, "value", runtime)
    assert module.forward(10) == 11
    assert module.forward(99) == 11  # cached: the argument is not looked at
    runtime.begin_request()
    assert module.forward(20) == 22
    assert runtime.audit()["request_misses"] == 1


def test_schedule_value_is_keyed_by_timestep_across_requests():
    runtime = H3InvariantCacheRuntime()
    module = Counter()
    _wrap_schedule_value(module, "adaln", runtime)
    runtime.current_timestep_key = (0.5,)
    assert module.forward(10) == 11
    assert module.forward(99) == 11
    runtime.begin_request()
    runtime.current_timestep_key = (0.5,)
    assert module.forward(50) == 11
    runtime.current_timestep_key = (0.25,)
    assert module.forward(50) == 52
    audit = runtime.audit()
    assert audit["schedule_entries"] == 2 and audit["schedule_hits"] == 1


def test_schedule_value_outside_a_forward_fails_closed():
    runtime = H3InvariantCacheRuntime()
    module = Counter()
    _wrap_schedule_value(module, "adaln", runtime)
    with pytest.raises(RuntimeError, match="outside H3 transformer"):
        module.forward(1)


def test_timestep_key_covers_values_shape_and_dtype():
    a = torch.tensor([0.5], dtype=torch.float32)
    assert _timestep_key(a) != _timestep_key(a.double())
    assert _timestep_key(a) != _timestep_key(torch.tensor([0.25]))
    assert _timestep_key(a) != _timestep_key(torch.tensor([[0.5]]))
    assert _timestep_key(a) == _timestep_key(torch.tensor([0.5]))


@pytest.mark.parametrize("expected", [49, 4])
def test_freeze_releases_the_adaln_projection_and_then_refuses_new_timesteps(expected):
    class Holder:
        def __init__(self) -> None:
            self.linear = torch.nn.Linear(2, 3)

    runtime = H3InvariantCacheRuntime()
    holder = Holder()
    size = sum(p.numel() * p.element_size() for p in holder.linear.parameters())
    runtime.adaln_modules.append(holder)
    runtime.schedule_values["adaln"] = {(index,): index for index in range(expected - 1)}
    with pytest.raises(RuntimeError, match="before all expected schedule"):
        runtime.freeze_fixed_schedule(expected_values_per_site=expected)
    runtime.schedule_values["adaln"][(expected - 1,)] = expected - 1
    assert runtime.freeze_fixed_schedule(expected_values_per_site=expected) == size
    assert holder.linear is None
    assert runtime.audit()["schedule_frozen"] is True
    assert runtime.freeze_fixed_schedule(expected_values_per_site=expected) == size  # idempotent
    module = Counter()
    _wrap_schedule_value(module, "new", runtime)
    runtime.current_timestep_key = (100,)
    with pytest.raises(RuntimeError, match="unseen timestep"):
        module.forward(1)
    with pytest.raises(ValueError, match="positive"):
        H3InvariantCacheRuntime().freeze_fixed_schedule(expected_values_per_site=0)


def _small_model():
    from h3_flash_b200.runtime.h3_model import H3Transformer

    torch.manual_seed(0)
    model = H3Transformer(64, 2, 32, 128, 2, text_dim=24, video_channels=16, audio_channels=8,
                          freq_dim=32, freqs_per_axis=4)
    return model.eval()


def test_installer_caches_request_and_schedule_values_of_a_transformer():
    from h3_flash_b200.runtime.h3_model import make_inputs

    model = _small_model()
    inputs = make_inputs(model, n_text=5, n_video=24, n_audio=3, text_dim=24, grid=(2, 3, 4), seed=1)
    with torch.no_grad():
        expect = model(**inputs, return_dict=False)
        runtime = install_h3_invariant_caches(model)
        assert install_h3_invariant_caches(model) is runtime  # idempotent
        first = model(**inputs, return_dict=False)
        second = model(**inputs, return_dict=False)
    for a, b, c in zip(expect, first, second):
        assert torch.equal(a, b) and torch.equal(b, c)
    audit = runtime.audit()
    # rope, context_embedder, token_refiner: one miss each, then hits
    assert audit["request_misses"] == 3 and audit["request_hits"] == 3
    # two blocks' AdaLN + norm_out: computed once for this timestep
    assert audit["schedule_misses"] == 3 and audit["schedule_hits"] == 3
    assert runtime.current_timestep_key is None
    runtime.begin_request()
    other = dict(inputs, timestep=inputs["timestep"] + 1.0)
    with torch.no_grad():
        model(**other, return_dict=False)
    assert runtime.audit()["schedule_misses"] == 3  # new timestep: recomputed
    assert runtime.freeze_fixed_schedule(expected_values_per_site=2) > 0
    assert all(block.adaln_proj.linear is None for block in model.transformer_blocks)
    with torch.no_grad():
        again = model(**inputs, return_dict=False)  # cached timestep still served
    assert torch.equal(again[0], expect[0])
