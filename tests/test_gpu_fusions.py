"""GPU parity of the fused elementwise kernels (through the C ABI via the Python surface).

Bar: within 1 bf16 ulp of the oracle (reference arithmetic in fp32, round-to-nearest-even
store); within 2 ulps of the golden vectors, which the Triton CPU interpreter stored by
truncation (one ulp) on top of the fp32 reduction-order freedom (one ulp).
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import bf16, fusions_ref
from tests.gpu_util import bits, dev, seeded_bits

pytestmark = pytest.mark.gpu

ULP = 1  # against the oracle
ULP_GOLDEN = 2  # against interpreter-truncated goldens


def _ulps(a, b):
    return int(bf16.ulp_distance(a, b).max()) if a.size else 0


def _chunks(wide, cols):
    return [wide[:, i * cols : (i + 1) * cols] for i in range(6)]


@pytest.mark.parametrize("case", ["a", "b", "c"])
def test_rmsnorm_modulate_golden(golden_fusions, case):
    from h3_flash_b200.runtime.kernels.fusions import fused_rmsnorm_modulate

    g = golden_fusions
    p = f"mod_{case}_"
    cols = g[p + "x"].shape[-1]
    wide = dev(g[p + "wide"])
    shift_msa, scale_msa, *_ = wide.chunk(6, -1)
    index = torch.from_numpy(g[p + "index"]).cuda()
    out = fused_rmsnorm_modulate(dev(g[p + "x"]), dev(g[p + "weight"]), scale_msa, shift_msa, index,
                                 float(g[p + "eps"]))
    ref = fusions_ref.rmsnorm_modulate(g[p + "x"], g[p + "weight"], _chunks(g[p + "wide"], cols)[1],
                                       _chunks(g[p + "wide"], cols)[0], g[p + "index"], float(g[p + "eps"]))
    assert _ulps(bits(out), ref) <= ULP
    assert _ulps(bits(out), g[p + "rmsnorm_modulate"]) <= ULP_GOLDEN


@pytest.mark.parametrize("case", ["a", "b", "c"])
def test_residual_gate_rmsnorm_modulate_golden(golden_fusions, case):
    from h3_flash_b200.runtime.kernels.fusions import fused_residual_gate_rmsnorm_modulate

    g = golden_fusions
    p = f"mod_{case}_"
    cols = g[p + "x"].shape[-1]
    _, _, gate_msa, shift_mlp, scale_mlp, _ = dev(g[p + "wide"]).chunk(6, -1)
    index = torch.from_numpy(g[p + "index"]).cuda()
    hidden, normed = fused_residual_gate_rmsnorm_modulate(
        dev(g[p + "x"]), dev(g[p + "branch"]), gate_msa, dev(g[p + "weight"]), scale_mlp, shift_mlp, index,
        float(g[p + "eps"]))
    ch = _chunks(g[p + "wide"], cols)
    ref_h, ref_n = fusions_ref.residual_gate_rmsnorm_modulate(
        g[p + "x"], g[p + "branch"], ch[2], g[p + "weight"], ch[4], ch[3], g[p + "index"], float(g[p + "eps"]))
    assert _ulps(bits(hidden), ref_h) <= ULP
    assert _ulps(bits(normed), ref_n) <= ULP
    assert _ulps(bits(hidden), g[p + "hidden"]) <= ULP_GOLDEN
    assert _ulps(bits(normed), g[p + "normed"]) <= ULP_GOLDEN


@pytest.mark.parametrize("case", ["a", "b"])
def test_swiglu_golden(golden_fusions, case):
    from h3_flash_b200.runtime.kernels.fusions import fused_swiglu

    g = golden_fusions
    x = g[f"swiglu_{case}_x"]
    out = bits(fused_swiglu(dev(x)))
    assert _ulps(out, fusions_ref.swiglu(x)) <= ULP
    assert _ulps(out, g[f"swiglu_{case}_out"]) <= ULP_GOLDEN


@pytest.mark.parametrize("case", ["a", "b", "c", "d"])
def test_qknorm_rope_golden(golden_fusions, case):
    from h3_flash_b200.runtime.kernels.fusions import fused_qknorm_rope

    g = golden_fusions
    p = f"rope_{case}_"
    cos = torch.from_numpy(g[p + "cos"]).cuda()
    sin = torch.from_numpy(g[p + "sin"]).cuda()
    out = bits(fused_qknorm_rope(dev(g[p + "x"]), dev(g[p + "weight"]), cos, sin, float(g[p + "eps"])))
    ref = fusions_ref.qknorm_rope(g[p + "x"], g[p + "weight"], g[p + "cos"], g[p + "sin"], float(g[p + "eps"]))
    assert _ulps(out, ref) <= ULP
    assert _ulps(out, g[p + "out"]) <= ULP_GOLDEN


@pytest.mark.parametrize("rows,cols,n_table,n_index", [(333, 3072, 3, 333), (64, 5376, 9, 9), (7, 24, 2, 3),
                                                        (5, 4104, 1, 1), (0, 3072, 3, 1)])
def test_adaln_ops_random(rows, cols, n_table, n_index):
    from h3_flash_b200.runtime.kernels import fusions as F

    x = seeded_bits(1, (1, rows, cols))
    br = seeded_bits(2, (1, rows, cols))
    w = seeded_bits(3, (cols,), 1.0, 0.02)
    wide = seeded_bits(4, (n_table, 6 * cols), 0.0, 0.1)
    idx = np.random.default_rng(5).integers(0, n_table, n_index)
    ch = [wide[:, i * cols : (i + 1) * cols] for i in range(6)]
    wd = dev(wide).chunk(6, -1)
    it = torch.from_numpy(idx).cuda()
    eps = 1e-6
    out = F.fused_rmsnorm_modulate(dev(x), dev(w), wd[1], wd[0], it, eps)
    assert _ulps(bits(out), fusions_ref.rmsnorm_modulate(x, w, ch[1], ch[0], idx, eps)) <= ULP
    h, n = F.fused_residual_gate_rmsnorm_modulate(dev(x), dev(br), wd[2], dev(w), wd[4], wd[3], it, eps)
    rh, rn = fusions_ref.residual_gate_rmsnorm_modulate(x, br, ch[2], w, ch[4], ch[3], idx, eps)
    assert _ulps(bits(h), rh) <= ULP and _ulps(bits(n), rn) <= ULP
    m = F.fused_modulate(dev(x), wd[1], wd[0], it)
    assert _ulps(bits(m), fusions_ref.modulate(x, ch[1], ch[0], idx)) <= ULP
    gr = F.fused_gated_residual(dev(x), dev(br), wd[5], it)
    assert _ulps(bits(gr), fusions_ref.gated_residual(x, br, ch[5], idx)) <= ULP


def test_modulate_with_vectors_and_strided_rows():
    """Benchmark form: [d] shift/scale vectors; activations as a strided row view."""

    from h3_flash_b200.runtime.kernels import fusions as F

    cols = 3072
    big = seeded_bits(11, (40, 2 * cols))
    scale = seeded_bits(12, (cols,), 0.0, 0.1)
    shift = seeded_bits(13, (cols,), 0.0, 0.1)
    x_dev = dev(big)[:, :cols]  # row stride 2*cols
    out = F.fused_modulate(x_dev, dev(scale), dev(shift))
    ref = fusions_ref.modulate(big[:, :cols], scale, shift, np.zeros(1, np.int64))
    assert _ulps(bits(out), ref) <= ULP


@pytest.mark.parametrize("rows,cols", [(97, 12288), (3, 100), (1, 8)])
def test_gelu_tanh(rows, cols):
    from h3_flash_b200.runtime.kernels.fusions import fused_gelu_tanh

    x = seeded_bits(21, (rows, cols), 0.0, 3.0)
    out = bits(fused_gelu_tanh(dev(x)))
    ref = fusions_ref.gelu_tanh(x)
    d = bf16.ulp_distance(out, ref)
    # values below 1e-30 in magnitude are compared in absolute terms
    tiny = np.abs(bf16.to_f32(ref)) < 1e-30
    assert int(d[~tiny].max()) <= ULP
    # and against torch's own GELU (fp32 opmath) within bf16 resolution
    t = torch.nn.functional.gelu(dev(x).float(), approximate="tanh")
    assert torch.allclose(torch.from_numpy(bf16.to_f32(out)).cuda(), t, rtol=2**-7, atol=1e-6)


@pytest.mark.parametrize("rows,n", [(65, 14336), (4, 100)])
def test_swiglu_random(rows, n):
    from h3_flash_b200.runtime.kernels.fusions import fused_swiglu

    x = seeded_bits(31, (rows, 2 * n), 0.0, 2.0)
    assert _ulps(bits(fused_swiglu(dev(x))), fusions_ref.swiglu(x)) <= ULP


@pytest.mark.parametrize("shape,rot", [((1, 33, 24, 128), 96), ((2, 9, 3, 128), 128), ((1, 5, 4, 128), 0),
                                       ((1, 6, 2, 64), 10), ((1, 4, 2, 256), 64)])
def test_qknorm_rope_random(shape, rot):
    from h3_flash_b200.runtime.kernels.fusions import fused_qknorm_rope

    b, s, h, d = shape
    x = seeded_bits(41, shape)
    w = seeded_bits(42, (d,), 1.0, 0.02)
    ang = np.random.default_rng(43).standard_normal((s, rot)).astype(np.float32) * 4
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    out = fused_qknorm_rope(dev(x), dev(w), torch.from_numpy(cos).cuda(), torch.from_numpy(sin).cuda(), 1e-6)
    assert _ulps(bits(out), fusions_ref.qknorm_rope(x, w, cos, sin, 1e-6)) <= ULP


def test_cpu_tensors_are_rejected_loudly():
    from h3_flash_b200.runtime.kernels.fusions import fused_swiglu

    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        fused_swiglu(torch.zeros(2, 8, dtype=torch.bfloat16))
