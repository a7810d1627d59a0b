"""Whole-block parity on one GPU: the installed fused block vs the fp32 CPU oracle.

Bar (north star): max-abs <= 2e-2 and cosine >= 0.9999 against the fp32 reference.
The block output is bf16, so an element can differ from the fp32 reference by half
a bf16 spacing of its own magnitude before any arithmetic error (0.016 at |x|=4):
the max-abs bar is applied on top of that rounding. The fused block must also be
at least as accurate as the eager bf16 composition of the same module.
"""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle.attention_ref import error_metrics
from oracle.block_ref import block_forward, fp32_params

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
COSINE = 0.9999


def _setup(rows: int, dim: int, heads: int, ffn: int, activation: str, seed: int = 0):
    from h3_flash_b200.runtime.h3_block import H3BlockStack, H3TransformerBlock
    from h3_flash_b200.workloads import init_block_, rope_tables

    block = init_block_(H3TransformerBlock(dim=dim, heads=heads, head_dim=128, ffn_inner=ffn,
                                           activation=activation), seed=seed)
    block = block.to(device="cuda", dtype=torch.bfloat16)
    stack = H3BlockStack([block])
    g = torch.Generator().manual_seed(seed + 1)
    hidden = torch.randn(1, rows, dim, generator=g).to(torch.bfloat16)
    idx = torch.randint(0, 3, (rows,), generator=g)
    pos = torch.stack([torch.arange(rows) // 64, (torch.arange(rows) // 8) % 8, torch.arange(rows) % 8], -1)
    cos, sin = rope_tables(pos, 96)
    return stack, block, hidden, idx, cos, sin


@pytest.mark.parametrize("rows,dim,heads,ffn,activation", [(300, 384, 3, 1536, "gelu-tanh"),
                                                           (257, 256, 2, 1024, "swiglu"),
                                                           (1024, 3072, 24, 12288, "gelu-tanh")])
def test_fused_block_matches_oracle(rows, dim, heads, ffn, activation):
    from h3_flash_b200.runtime.kernels import install_transformer_fusions

    stack, block, hidden, idx, cos, sin = _setup(rows, dim, heads, ffn, activation)
    params = fp32_params(block)
    ref = block_forward(params, hidden[0].float(), idx, cos, sin, heads=heads, head_dim=128, eps=1e-6,
                        qk_eps=1e-6, activation=activation)
    args = (hidden.cuda(), None, idx.cuda(), (cos.cuda(), sin.cuda()))
    with torch.no_grad():
        eager = stack(*args)  # upstream-style bf16 torch composition (before installation)
    runtime = install_transformer_fusions(stack)
    with torch.no_grad():
        out = stack(*args)
    got = out[0].float().cpu().numpy()
    refn = ref.numpy()
    m = error_metrics(got, refn)
    m_eager = error_metrics(eager[0].float().cpu().numpy(), refn)
    half_ulp = np.ldexp(1.0, np.frexp(np.abs(refn))[1] - 9)  # half a bf16 spacing at |ref|
    excess = np.abs(got - refn) - half_ulp
    assert excess.max() <= MAX_ABS, (m, float(excess.max()))
    assert m["cosine"] >= COSINE, m
    assert m["mean_abs"] <= m_eager["mean_abs"] * 1.05, (m, m_eager)
    assert m["max_abs"] <= max(MAX_ABS, m_eager["max_abs"] * 1.05), (m, m_eager)
    # the reference's first-block gates were recorded
    assert {"rmsnorm_modulate", "residual_chain", "residual_output"} <= set(runtime["gate"])
    for name, gate in runtime["gate"].items():
        assert gate["cosine"] > 0.999, (name, gate)


def test_block_is_deterministic_and_reuses_qkv_cache():
    from h3_flash_b200.runtime.kernels import install_transformer_fusions

    stack, block, hidden, idx, cos, sin = _setup(256, 256, 2, 1024, "gelu-tanh")
    install_transformer_fusions(stack)
    args = (hidden.cuda(), None, idx.cuda(), (cos.cuda(), sin.cuda()))
    with torch.no_grad():
        a = stack(*args)
        b = stack(*args)
    assert torch.equal(a, b)
    # in-place weight update invalidates the fused QKV weight cache
    with torch.no_grad():
        block.attn.to_q.weight.mul_(0.5)
        c = stack(*args)
    assert not torch.equal(a, c)


def test_gelu_in_the_gemm_epilogue_is_tanh_gelu():
    """The FFN projection with GELU in its epilogue (h3b GEMM) vs the fp32 GELU-tanh of the
    fp32 projection: within the bf16 bar, no worse than the unfused GEMM + h3b GELU, and
    tanh-GELU rather than erf-GELU where the two differ by many bf16 spacings (x near -3)."""

    from h3_flash_b200.runtime.h3_block import FeedForward
    from h3_flash_b200.runtime.kernels.transformer import feed_forward

    torch.manual_seed(5)
    ff = FeedForward(512, 2048, "gelu-tanh").to("cuda", torch.bfloat16)
    with torch.no_grad():
        ff.net[0].proj.weight.normal_(0.0, 0.1)
        ff.net[0].proj.bias.normal_(0.0, 0.5)
        x = torch.randn(1, 700, 512, device="cuda").to(torch.bfloat16)
        gate = {}
        # the activation itself: the same h3b GEMM epilogue call feed_forward makes
        from h3_flash_b200.runtime.kernels.fusions import fused_linear

        proj = ff.net[0].proj
        fused = fused_linear(x[0], proj.weight, proj.bias, "gelu-tanh").float()
        unfused = torch.nn.functional.gelu(proj(x[0]).float(), approximate="tanh").to(torch.bfloat16).float()
        pre = x[0].float() @ proj.weight.float().t() + proj.bias.float()
        tanh_ref = torch.nn.functional.gelu(pre, approximate="tanh")
        erf_ref = torch.nn.functional.gelu(pre)
        out = feed_forward(ff, x, True, gate, gemm_epilogue=True)
        out_unfused = feed_forward(ff, x, True, None, gemm_epilogue=False)
    half_ulp = tanh_ref.abs().clamp_min(2.0 ** -126) * 2.0 ** -9
    assert float(((fused - tanh_ref).abs() - half_ulp).max()) <= 2e-2
    assert float((fused - tanh_ref).abs().mean()) <= float((unfused - tanh_ref).abs().mean()) * 1.05
    distinct = (tanh_ref - erf_ref).abs() > 16 * half_ulp
    assert int(distinct.sum()) > 100
    closer = (fused - tanh_ref).abs()[distinct] < (fused - erf_ref).abs()[distinct]
    assert float(closer.float().mean()) > 0.99
    assert gate["gelu_tanh_epilogue"]["cosine"] > 0.9999
    cos = torch.nn.functional.cosine_similarity(out.float().flatten(), out_unfused.float().flatten(), dim=0)
    assert float(cos) > 0.9999
