"""Pins the CPU oracle against golden vectors recorded from the reference's own kernels.

The goldens were produced by the reference Triton kernels executed by the Triton
CPU interpreter (tests/golden/make_golden.py). That interpreter stores bf16 by
truncating fp32; in "trunc" rounding the oracle must reproduce every golden bit.
"""

from __future__ import annotations

import numpy as np
import pytest

from oracle import bf16, fusions_ref, relayout_ref


def _chunks(wide: np.ndarray, cols: int) -> list[np.ndarray]:
    return [wide[:, i * cols : (i + 1) * cols] for i in range(6)]


@pytest.mark.parametrize("case", ["a", "b", "c"])
def test_rmsnorm_modulate_matches_reference_kernel(golden_fusions, case):
    g = golden_fusions
    p = f"mod_{case}_"
    cols = g[p + "x"].shape[-1]
    shift_msa, scale_msa, *_ = _chunks(g[p + "wide"], cols)
    out = fusions_ref.rmsnorm_modulate(
        g[p + "x"], g[p + "weight"], scale_msa, shift_msa, g[p + "index"], float(g[p + "eps"]),
        rounding="trunc",
    )
    np.testing.assert_array_equal(out, g[p + "rmsnorm_modulate"])


@pytest.mark.parametrize("case", ["a", "b", "c"])
def test_residual_gate_rmsnorm_modulate_matches_reference_kernel(golden_fusions, case):
    g = golden_fusions
    p = f"mod_{case}_"
    cols = g[p + "x"].shape[-1]
    _, _, gate_msa, shift_mlp, scale_mlp, _ = _chunks(g[p + "wide"], cols)
    hidden, normed = fusions_ref.residual_gate_rmsnorm_modulate(
        g[p + "x"], g[p + "branch"], gate_msa, g[p + "weight"], scale_mlp, shift_mlp, g[p + "index"],
        float(g[p + "eps"]), rounding="trunc",
    )
    np.testing.assert_array_equal(hidden, g[p + "hidden"])
    np.testing.assert_array_equal(normed, g[p + "normed"])


@pytest.mark.parametrize("case", ["a", "b"])
def test_swiglu_matches_reference_kernel(golden_fusions, case):
    g = golden_fusions
    out = fusions_ref.swiglu(g[f"swiglu_{case}_x"], rounding="trunc")
    np.testing.assert_array_equal(out, g[f"swiglu_{case}_out"])


@pytest.mark.parametrize("case", ["a", "b", "c", "d"])
def test_qknorm_rope_matches_reference_kernel(golden_fusions, case):
    g = golden_fusions
    p = f"rope_{case}_"
    out = fusions_ref.qknorm_rope(g[p + "x"], g[p + "weight"], g[p + "cos"], g[p + "sin"], float(g[p + "eps"]),
                                  rounding="trunc")
    np.testing.assert_array_equal(out, g[p + "out"])


def test_rne_and_trunc_differ_by_at_most_one_ulp(golden_fusions):
    g = golden_fusions
    p = "rope_a_"
    rne = fusions_ref.qknorm_rope(g[p + "x"], g[p + "weight"], g[p + "cos"], g[p + "sin"], float(g[p + "eps"]))
    assert bf16.ulp_distance(rne, g[p + "out"]).max() <= 1


@pytest.mark.parametrize("case", ["a", "b", "c"])
def test_pack_matches_reference_kernel(golden_relayout, case):
    g = golden_relayout
    rows, heads, d, world = (int(v) for v in g[f"pack_{case}_shape"])
    qkv = g[f"pack_{case}_qkv"]
    q, k, v = (qkv[:, i * heads * d : (i + 1) * heads * d].reshape(rows, heads, d) for i in range(3))
    np.testing.assert_array_equal(relayout_ref.pack_qkv(q, k, v, world), g[f"pack_{case}_out"])


@pytest.mark.parametrize("case", ["a", "b"])
def test_merge_matches_reference_kernel(golden_relayout, case):
    g = golden_relayout
    np.testing.assert_array_equal(relayout_ref.merge_heads(g[f"merge_{case}_x"]), g[f"merge_{case}_out"])


def test_exchange_restatement_matches_reference_gloo_run(golden_ulysses):
    g = golden_ulysses
    heads, d = int(g["heads"]), int(g["head_dim"])
    world = 2
    sends = [relayout_ref.pack_qkv(g[f"r{r}_q"], g[f"r{r}_k"], g[f"r{r}_v"], world) for r in range(world)]
    counts = [g[f"r{r}_q"].shape[0] for r in range(world)]
    recv = relayout_ref.exchange(sends, counts)
    for r in range(world):
        np.testing.assert_array_equal(recv[r], g[f"r{r}_packed"])
    back = relayout_ref.exchange_back([g[f"r{r}_attn"] for r in range(world)], counts)
    for r in range(world):
        np.testing.assert_array_equal(back[r], g[f"r{r}_back"])
    assert recv[0].shape == (sum(counts), heads // world, 3 * d)


def test_bf16_rounding_is_nearest_even():
    values = np.array([1.0, 1.0 + 2**-8, 1.0 + 3 * 2**-8, -1.0 - 2**-8, 1.0 + 2**-9], dtype=np.float32)
    out = bf16.to_f32(bf16.from_f32(values))
    np.testing.assert_array_equal(out, np.array([1.0, 1.0, 1.0 + 4 * 2**-8, -1.0, 1.0], dtype=np.float32))
    assert bf16.ulp_distance(np.array([0x3F80], np.uint16), np.array([0x3F81], np.uint16))[0] == 1
    assert bf16.ulp_distance(np.array([0x0000], np.uint16), np.array([0x8000], np.uint16))[0] == 0
