"""The h3b tcgen05 GEMM with fused epilogues (h3b_gemm, h3b_gemm_swiglu) through the C ABI.

References are fp32 restatements on the same bf16 inputs: y = x W^T + b, then nothing,
GELU-tanh (the FFN activation of src/h3_flash/runtime/kernels/transformer.py:121-122),
or value * silu(gate) (fusions.py:251-265 after the SwiGLU projection). The kernel keeps
y in fp32 up to its one rounding at the store, so the bar is 1 bf16 ulp of the fp32
result, except where a result is far smaller than its row (a sum that cancels): there
the fp32 accumulation order alone moves it by a few fp32 ulps of the row's scale, and
the bar is 2^-16 of the row's largest |y|. Shapes cover row tails (1, 257, 1000 rows),
strided x and output rows, no bias, and the FFN shapes of the benchmark block.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import bf16
from tests.gpu_util import bits

pytestmark = pytest.mark.gpu


def _rand(g, *shape, std=1.0):
    return (torch.randn(*shape, device="cuda", generator=g) * std).to(torch.bfloat16)


def _within(got: torch.Tensor, want: torch.Tensor) -> tuple[float, float]:
    """(fraction within 1 ulp of the fp32 value rounded to bf16, worst excess over the
    conditioning bar among the rest, in units of the bar)."""

    ref16 = want.to(torch.bfloat16)
    ulps = torch.from_numpy(bf16.ulp_distance(bits(got), bits(ref16)).astype(np.int64)).to(got.device)
    scale = want.abs().amax(dim=-1, keepdim=True).clamp_min(2.0 ** -30)
    off = ulps > 1
    worst = float(((got.float() - want).abs() / (2.0 ** -16 * scale))[off].max()) if bool(off.any()) else 0.0
    return float((~off).float().mean()), worst


def _gelu_tanh(y):
    return torch.nn.functional.gelu(y, approximate="tanh")


@pytest.mark.parametrize("rows,dim,n,act,use_bias", [
    (1000, 3072, 512, "gelu-tanh", True), (257, 3072, 12288, "gelu-tanh", True),
    (1, 64, 256, "none", True), (1000, 12288, 3072, "none", True), (300, 512, 768, "none", False),
])
def test_gemm_against_fp32(rows, dim, n, act, use_bias):
    from h3_flash_b200.runtime.kernels.fusions import fused_linear

    g = torch.Generator(device="cuda").manual_seed(rows + n)
    x = _rand(g, rows, dim)
    w = _rand(g, n, dim, std=dim ** -0.5)
    b = _rand(g, n, std=0.5) if use_bias else None
    got = fused_linear(x, w, b, act)
    y = x.float() @ w.float().t() + (b.float() if b is not None else 0.0)
    want = _gelu_tanh(y) if act == "gelu-tanh" else y
    within, worst = _within(got, want)
    assert within >= 0.999 and worst <= 1.0, (within, worst)
    from h3_flash_b200 import _lib

    assert _lib.device_status() == 0


def test_gemm_strided_rows_and_output():
    from h3_flash_b200 import _lib
    from h3_flash_b200._torch import ptr, stream_of

    g = torch.Generator(device="cuda").manual_seed(9)
    base = _rand(g, 333, 1024 + 64)
    x = base[:, 64:]  # row stride 1088
    w = _rand(g, 512, 1024, std=1024 ** -0.5)
    b = _rand(g, 512)
    out = torch.full((333, 640), float("nan"), device="cuda", dtype=torch.bfloat16)
    _lib.call("h3b_gemm", ptr(out), out.stride(0), ptr(x), 333, 1024, x.stride(0), ptr(w), 512, ptr(b), 1,
              stream_of(x))
    want = _gelu_tanh(x.float() @ w.float().t() + b.float())
    within, worst = _within(out[:, :512].contiguous(), want)
    assert within >= 0.999 and worst <= 1.0
    assert torch.isnan(out[:, 512:].float()).all()  # columns past n untouched


@pytest.mark.parametrize("rows,dim,n_out", [(1000, 3072, 1536), (257, 512, 128)])
def test_swiglu_gemm_against_fp32(rows, dim, n_out):
    from h3_flash_b200.runtime.kernels.fusions import fused_linear_swiglu, interleave_swiglu

    g = torch.Generator(device="cuda").manual_seed(rows)
    x = _rand(g, rows, dim)
    w = _rand(g, 2 * n_out, dim, std=dim ** -0.5)
    b = _rand(g, 2 * n_out, std=0.5)
    got = fused_linear_swiglu(x, *interleave_swiglu(w, b))
    y = x.float() @ w.float().t() + b.float()
    value, gate = y.chunk(2, -1)
    want = value * torch.nn.functional.silu(gate)
    within, worst = _within(got, want)
    assert within >= 0.999 and worst <= 1.0, (within, worst)


def test_gemm_rejects_unsupported_widths():
    from h3_flash_b200.runtime.kernels.fusions import fused_linear

    x = torch.zeros(4, 64, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="256"):
        fused_linear(x, torch.zeros(100, 64, device="cuda", dtype=torch.bfloat16))


@pytest.mark.parametrize("rows,n_table", [(1000, 3), (257, 1)])
def test_gated_residual_gemm_against_fp32(rows, n_table):
    """residual + gate[idx] * (x W^T + b) in the GEMM epilogue vs fp32 (the block's
    closing residual, kernels/transformer.py:123-126)."""

    from h3_flash_b200.runtime.kernels.fusions import fused_linear_gated_residual

    g = torch.Generator(device="cuda").manual_seed(rows)
    dim, n = 2048, 768
    x = _rand(g, rows, dim)
    w = _rand(g, n, dim, std=dim ** -0.5)
    b = _rand(g, n, std=0.5)
    res = _rand(g, 1, rows, n)
    table = _rand(g, n_table, 6 * n, std=0.1)
    gate = table.chunk(6, -1)[5]  # a strided view of the AdaLN table, as in the block
    idx = torch.randint(0, n_table, (rows,), device="cuda", generator=g)
    got = fused_linear_gated_residual(x, w, b, res, gate, idx)
    y = x.float() @ w.float().t() + b.float()
    want = res[0].float() + gate.float().index_select(0, idx) * y
    assert got.shape == res.shape
    within, worst = _within(got[0], want)
    assert within >= 0.999 and worst <= 1.0, (within, worst)
