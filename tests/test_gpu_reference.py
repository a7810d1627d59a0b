"""GPU parity against the reference itself: its own Triton kernels and its LOSSLESS block,
run unmodified from the offline install under baseline/_ref (skipped when it is absent).

- elementwise ops (fused_rmsnorm_modulate, fused_residual_gate_rmsnorm_modulate,
  fused_qknorm_rope, fused_swiglu; src/h3_flash/runtime/kernels/fusions.py:194-293): the
  h3b kernel is within 1 bf16 ulp of the reference's Triton kernel on the same inputs for
  at least 99.99% of the elements, and every other element is a cancellation (a result far
  below the magnitude of its terms) where the two differ by fp32 rounding noise
  (2^-18 of the row's scale): the two kernels sum the row's squares in different orders;
- relayout (pack_qkv_destination_major, merge_heads; src/h3_flash/runtime/parallel/
  relayout.py:97-159): bit-exact;
- the default QKV projection (h3b_qkv_gemm_pack: projection, QK-norm, RoPE and pack in one
  GEMM) against the reference composition it replaces (cuBLAS to_q/to_k/to_v, then the
  reference's fused_qknorm_rope and Triton pack; packed_ulysses.py:166-200). The GEMM keeps
  the projection in fp32 up to the norm where the reference rounds it to bf16 first: v (one
  rounding each) is within 1 ulp everywhere; q/k within 1 ulp for at least 97% of the
  elements, the rest within the reference's own projection rounding carried through the
  rotation plus both output roundings (2^-7 of the row's scale);
- the whole block: the installed h3b block and the reference's LOSSLESS block on the same
  weights and inputs, both against the fp32 oracle (max-abs 2e-2 above the bf16 output's own
  half spacing, cosine >= 0.9999), and the h3b block no less accurate than the reference's.
"""

from __future__ import annotations

import sys
from types import SimpleNamespace

import numpy as np
import pytest
import torch

from oracle import bf16
from tests.gpu_util import bits

pytestmark = pytest.mark.gpu

# Where a result cancels (it is far smaller than the terms it is computed from), two fp32
# evaluations that differ in reduction order or in which product an FMA keeps unrounded
# differ by a few fp32 ulps of the terms: 2^-18 of the row's scale bounds that.
FP32_NOISE = 2.0 ** -18
# The reference rounds the QKV projection to bf16 before the norm (2^-9 relative to each
# element); the rotation x*cos + partner*sin adds two such errors, up to 2^-8 of the row's
# scale, and each side's own output rounding adds half a bf16 ulp, up to 2^-8 together.
PROJECTION_ROUNDING = 2.0 ** -7


@pytest.fixture(scope="module")
def ref():
    import bench

    site = bench._reference_site()
    if site is None:
        pytest.skip("the reference package is not installed under baseline/_ref")
    if str(site) not in sys.path:
        sys.path.insert(0, str(site))
    bench._diffusers_stand_in()
    from h3_flash.runtime.kernels import fusions
    from h3_flash.runtime.parallel import relayout

    return SimpleNamespace(fusions=fusions, relayout=relayout, bench=bench)


def _ulps(a: torch.Tensor, b: torch.Tensor) -> np.ndarray:
    return bf16.ulp_distance(bits(a), bits(b))


def _agree(a: torch.Tensor, b: torch.Tensor, rel: float) -> tuple[float, float]:
    """(fraction of elements within 1 bf16 ulp of b, largest |a - b| / (rel * scale) over
    the elements that are not). An element agrees when it is within 1 bf16 ulp of b, or
    within ``rel`` times its row's scale (the row's largest |b|): a result far smaller
    than the terms it is computed from (x*cos + partner*sin, normed*(1+scale) + shift
    near zero) carries the terms' fp32 rounding, which is many bf16 ulps of itself."""

    ulps = torch.from_numpy(_ulps(a, b).astype(np.int64)).to(a.device)
    a32, b32 = a.float(), b.float()
    diff = (a32 - b32).abs()
    scale = b32.abs().amax(dim=-1, keepdim=True).clamp_min(2.0 ** -30)
    off = ulps > 1
    worst = float((diff / (rel * scale))[off].max()) if bool(off.any()) else 0.0
    return float((~off).float().mean()), worst


def _rand(g, *shape, std=1.0, mean=0.0):
    return (torch.randn(*shape, device="cuda", generator=g) * std + mean).to(torch.bfloat16)


@pytest.mark.parametrize("rows,cols,n_table", [(1000, 3072, 3), (257, 1536, 9), (64, 384, 1)])
def test_adaln_ops_match_reference_kernels(ref, rows, cols, n_table):
    from h3_flash_b200.runtime.kernels import fusions as mine

    g = torch.Generator(device="cuda").manual_seed(rows)
    x, branch = _rand(g, 1, rows, cols), _rand(g, 1, rows, cols)
    weight = _rand(g, cols, std=0.02, mean=1.0)
    table = _rand(g, n_table, 6 * cols, std=0.1)
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, _ = table.chunk(6, -1)
    index = torch.randint(0, n_table, (rows,), device="cuda", generator=g)
    a = mine.fused_rmsnorm_modulate(x, weight, scale_msa, shift_msa, index, 1e-6)
    b = ref.fusions.fused_rmsnorm_modulate(x, weight, scale_msa, shift_msa, index, 1e-6)
    ha, na = mine.fused_residual_gate_rmsnorm_modulate(x, branch, gate_msa, weight, scale_mlp, shift_mlp,
                                                        index, 1e-6)
    hb, nb = ref.fusions.fused_residual_gate_rmsnorm_modulate(x, branch, gate_msa, weight, scale_mlp,
                                                              shift_mlp, index, 1e-6)
    for got, want in ((a, b), (ha, hb), (na, nb)):
        within, worst = _agree(got, want, FP32_NOISE)
        assert within >= 0.9999 and worst <= 1.0, (within, worst)


@pytest.mark.parametrize("rot", [96, 128, 64])
def test_qknorm_rope_matches_reference_kernel(ref, rot):
    from h3_flash_b200.runtime.kernels import fusions as mine

    g = torch.Generator(device="cuda").manual_seed(rot)
    x = _rand(g, 1, 777, 24, 128)
    weight = _rand(g, 128, std=0.02, mean=1.0)
    cos = torch.rand(777, rot, device="cuda", generator=g) * 2 - 1
    sin = torch.rand(777, rot, device="cuda", generator=g) * 2 - 1
    a = mine.fused_qknorm_rope(x, weight, cos, sin, 1e-6)
    b = ref.fusions.fused_qknorm_rope(x, weight, cos, sin, 1e-6)
    within, worst = _agree(a, b, FP32_NOISE)
    assert within >= 0.9999 and worst <= 1.0, (within, worst)


def test_swiglu_matches_reference_kernel(ref):
    from h3_flash_b200.runtime.kernels import fusions as mine

    g = torch.Generator(device="cuda").manual_seed(3)
    x = _rand(g, 513, 2 * 1536, std=2.0)
    within, worst = _agree(mine.fused_swiglu(x), ref.fusions.fused_swiglu(x), FP32_NOISE)
    assert within >= 0.9999 and worst <= 1.0, (within, worst)


@pytest.mark.parametrize("rows,heads,world", [(1000, 24, 8), (333, 24, 2), (64, 6, 3)])
def test_relayout_is_bit_exact_with_reference_kernels(ref, rows, heads, world):
    from h3_flash_b200.runtime.parallel import relayout as mine

    g = torch.Generator(device="cuda").manual_seed(rows)
    qkv = _rand(g, rows, 3 * heads * 128)
    q, k, v = (qkv[:, i * heads * 128:(i + 1) * heads * 128].view(rows, heads, 128) for i in range(3))
    assert torch.equal(mine.pack_qkv_destination_major(q, k, v, world),
                       ref.relayout.pack_qkv_destination_major(q, k, v, world))
    out = _rand(g, world, rows, heads // world, 128)
    assert torch.equal(mine.merge_heads(out), ref.relayout.merge_heads(out))


@pytest.mark.parametrize("rows,world", [(6400, 8), (1111, 2)])
def test_qkv_gemm_pack_ulp_histogram_against_reference_composition(ref, rows, world):
    """The default fused projection against cuBLAS + the reference's QK-norm+RoPE and pack."""

    import torch.nn.functional as F

    from h3_flash_b200.runtime.kernels.fusions import fused_qkv_gemm_pack
    from h3_flash_b200.workloads import CONFIGS, positions, rope_tables

    cfg = CONFIGS["480p-5s"]
    heads, d = cfg.heads, cfg.dim
    g = torch.Generator(device="cuda").manual_seed(rows)
    x = _rand(g, rows, d)
    w = _rand(g, 3 * heads * 128, d, std=0.02)
    bias = _rand(g, 3 * heads * 128, std=0.02)
    wq, wk = _rand(g, 128, std=0.02, mean=1.0), _rand(g, 128, std=0.02, mean=1.0)
    cos, sin = (t[:rows].cuda() for t in rope_tables(positions(cfg), cfg.rotary_dim, cfg.theta))
    got = fused_qkv_gemm_pack(x, w, bias, wq, wk, cos, sin, heads, world, cfg.eps, cfg.eps)
    wq_, wk_, wv_ = w.chunk(3, 0)
    bq, bk, bv = bias.chunk(3, 0)
    q = F.linear(x, wq_, bq).view(rows, heads, 128)
    k = F.linear(x, wk_, bk).view(rows, heads, 128)
    v = F.linear(x, wv_, bv).view(rows, heads, 128)
    q = ref.fusions.fused_qknorm_rope(q.unsqueeze(0), wq, cos, sin, cfg.eps).squeeze(0)
    k = ref.fusions.fused_qknorm_rope(k.unsqueeze(0), wk, cos, sin, cfg.eps).squeeze(0)
    want = ref.relayout.pack_qkv_destination_major(q, k, v, world)
    ulps = _ulps(got, want).reshape(world, rows, heads // world, 3, 128)
    qk, vv = ulps[:, :, :, :2], ulps[:, :, :, 2]
    hist = {u: float((qk == u).mean()) for u in range(4)}
    assert vv.max() <= 1, int(vv.max())
    shape = (world, rows, heads // world, 3, 128)
    within, worst = _agree(got.view(shape)[:, :, :, :2], want.view(shape)[:, :, :, :2], PROJECTION_ROUNDING)
    assert within >= 0.97 and worst <= 1.0, (hist, within, worst)


def _small_cfg():
    from h3_flash_b200.workloads import BlockConfig

    return BlockConfig("ref-block", (4, 16, 16), 128, dim=1024, heads=8, ffn_inner=4096)


def test_block_against_reference_lossless_block(ref):
    """Same weights and inputs: the h3b block and the reference's LOSSLESS block (its
    Triton fusions + SDPA, installed by its own install_transformer_fusions), each against
    the fp32 oracle."""

    from oracle.attention_ref import error_metrics
    from oracle.block_ref import block_forward, fp32_params

    from h3_flash_b200.runtime.h3_block import H3BlockStack, H3TransformerBlock
    from h3_flash_b200.runtime.kernels import install_transformer_fusions
    from h3_flash_b200.workloads import adaln_indices, init_block_, positions, rope_tables

    cfg = _small_cfg()
    ref_stack, _, provenance = ref.bench.reference_stack(cfg, 1)
    assert "baseline" in provenance["package"] or "h3_flash" in provenance["package"]
    block = init_block_(H3TransformerBlock(cfg.dim, cfg.heads, cfg.head_dim, cfg.ffn_inner, eps=cfg.eps,
                                           qk_eps=cfg.eps), seed=0)
    stack = H3BlockStack([block.to("cuda", torch.bfloat16).eval()])
    params = fp32_params(block)  # the bf16 weights the GPU blocks use, in fp32
    install_transformer_fusions(stack)
    g = torch.Generator().manual_seed(1)
    hidden = torch.randn(1, cfg.seq, cfg.dim, generator=g).to(torch.bfloat16)
    idx = adaln_indices(cfg)
    cos, sin = rope_tables(positions(cfg), cfg.rotary_dim, cfg.theta)
    args = (hidden.cuda(), None, idx.cuda(), (cos.cuda(), sin.cuda()))
    with torch.no_grad():
        mine = stack(*args)[0].float().cpu().numpy()
        theirs = ref_stack(*args)[0].float().cpu().numpy()
    want = block_forward(params, hidden[0].float(), idx, cos, sin, heads=cfg.heads, head_dim=cfg.head_dim,
                         eps=cfg.eps, qk_eps=cfg.eps).numpy()
    m_mine, m_ref = error_metrics(mine, want), error_metrics(theirs, want)
    half_ulp = np.ldexp(1.0, np.frexp(np.abs(want))[1] - 9)
    assert (np.abs(mine - want) - half_ulp).max() <= 2e-2 and m_mine["cosine"] >= 0.9999, m_mine
    assert (np.abs(theirs - want) - half_ulp).max() <= 2e-2 and m_ref["cosine"] >= 0.9999, m_ref
    assert m_mine["mean_abs"] <= m_ref["mean_abs"] * 1.05, (m_mine, m_ref)
    assert m_mine["relative_l2"] <= m_ref["relative_l2"] * 1.05, (m_mine, m_ref)
