"""Parity at the benchmark sizes (480p-5s, and 768p-15s, the largest), where the CPU oracle
is too slow.

The checks use properties that hold at any size:
- attention over the full joint sequence (S = 51,200 with 3 heads, the SP8 per-rank shape,
  and 24 heads, one GPU; S = 354,240 with 3 heads) agrees with torch's
  scaled_dot_product_attention. Torch is only the checker here; both are bf16-in,
  fp32-accumulate.
- the fused QK-norm+RoPE+pack at the SP8 per-rank shapes ([6400, 24, 128] and
  [44280, 24, 128], W=8) equals, bit for bit, the standalone fused QK-norm+RoPE followed by
  the destination-major pack, and the pack then the merge of q is the identity.
- the fused block at d=3072 (S = 51,200, and S = 354,240 on one GPU, where the packed buffer
  holds 3.3e9 elements and every offset needs 64 bits) agrees with the same module's eager
  bf16 forward (torch ops and SDPA). Both carry bf16 rounding at every stage (the eager one
  more), so the bar is set for the difference of two approximations: excess over half a
  bf16 spacing <= 6e-2, cosine >= 0.9999, relative L2 <= 1e-2.
"""

from __future__ import annotations

import math

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu

S = 51200
S_MAX = 354240  # 768p-15s


def _metrics(got: torch.Tensor, ref: torch.Tensor):
    got, ref = got.float(), ref.float()
    diff = (got - ref).abs()
    half_ulp = ref.abs().clamp_min(2.0 ** -126) * 2.0 ** -9
    excess = float((diff - half_ulp).clamp_min(0).max())
    cosine = float(F.cosine_similarity(got.flatten(), ref.flatten(), dim=0))
    return float(diff.max()), excess, cosine


@pytest.mark.parametrize("seq,heads", [(S, 3), (S, 24), (S_MAX, 3)])
def test_full_sequence_attention_matches_sdpa(seq, heads):
    from h3_flash_b200 import _lib
    from h3_flash_b200.runtime.attention.dense import packed_attention

    g = torch.Generator(device="cuda").manual_seed(heads)
    packed = torch.randn(seq, heads, 384, device="cuda", generator=g).to(torch.bfloat16)
    out = packed_attention(packed, 128)
    q, k, v = (packed[..., i * 128 : (i + 1) * 128].permute(1, 0, 2).unsqueeze(0) for i in range(3))
    ref = F.scaled_dot_product_attention(q, k, v, scale=1.0 / math.sqrt(128))[0].permute(1, 0, 2)
    torch.cuda.synchronize()
    max_abs, excess, cosine = _metrics(out, ref)
    assert torch.isfinite(out).all()
    # two bf16 computations of the same value: each rounds its output once
    assert max_abs <= 2e-2 and cosine >= 0.9999, (max_abs, cosine)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("config", ["480p-5s", "768p-15s"])
def test_sp8_pack_is_bit_exact_and_inverts(config):
    from h3_flash_b200.runtime.kernels.fusions import fused_qknorm_rope, fused_qknorm_rope_pack
    from h3_flash_b200.runtime.parallel.relayout import merge_heads, pack_qkv_destination_major
    from h3_flash_b200.workloads import CONFIGS, positions, rope_tables

    cfg = CONFIGS[config]
    rows, heads, world = cfg.seq // 8, 24, 8
    g = torch.Generator(device="cuda").manual_seed(7)
    qkv = torch.randn(rows, 3 * heads * 128, device="cuda", generator=g).to(torch.bfloat16)
    q, k, v = (qkv[:, i * heads * 128 : (i + 1) * heads * 128].view(rows, heads, 128) for i in range(3))
    wq = (1 + 0.02 * torch.randn(128, device="cuda", generator=g)).to(torch.bfloat16)
    wk = (1 + 0.02 * torch.randn(128, device="cuda", generator=g)).to(torch.bfloat16)
    cos, sin = (t[:rows].cuda() for t in rope_tables(positions(cfg), cfg.rotary_dim, cfg.theta))
    fused = fused_qknorm_rope_pack(q, k, v, wq, wk, cos, sin, world, 1e-6, 1e-6)
    qn = fused_qknorm_rope(q.unsqueeze(0), wq, cos, sin, 1e-6).squeeze(0)
    kn = fused_qknorm_rope(k.unsqueeze(0), wk, cos, sin, 1e-6).squeeze(0)
    two_step = pack_qkv_destination_major(qn, kn, v.contiguous(), world)
    assert torch.equal(fused, two_step)
    back = merge_heads(fused[..., :128].contiguous())
    assert torch.equal(back, qn)


@pytest.mark.parametrize("config", ["480p-5s", "768p-15s"])
def test_full_size_block_matches_eager(config):
    from h3_flash_b200 import _lib
    from h3_flash_b200.runtime.h3_block import H3BlockStack, H3TransformerBlock
    from h3_flash_b200.runtime.kernels import install_transformer_fusions
    from h3_flash_b200.workloads import CONFIGS, adaln_indices, init_block_, positions, rope_tables

    cfg = CONFIGS[config]
    block = init_block_(H3TransformerBlock(cfg.dim, cfg.heads, cfg.head_dim, cfg.ffn_inner, eps=cfg.eps,
                                           qk_eps=cfg.eps), seed=0)
    block = block.to("cuda", torch.bfloat16).eval()
    stack = H3BlockStack([block])
    g = torch.Generator(device="cuda").manual_seed(1)
    hidden = torch.randn(1, cfg.seq, cfg.dim, device="cuda", generator=g).to(torch.bfloat16)
    idx = adaln_indices(cfg).cuda()
    cos, sin = (t.cuda() for t in rope_tables(positions(cfg), cfg.rotary_dim, cfg.theta))
    with torch.no_grad():
        eager = stack(hidden, None, idx, (cos, sin))
        install_transformer_fusions(stack)
        fused = stack(hidden, None, idx, (cos, sin))
    torch.cuda.synchronize()
    max_abs, excess, cosine = _metrics(fused, eager)
    rel_l2 = float((fused.float() - eager.float()).norm() / eager.float().norm())
    assert torch.isfinite(fused).all()
    assert excess <= 6e-2 and cosine >= 0.9999 and rel_l2 <= 1e-2, (max_abs, excess, cosine, rel_l2)
    assert _lib.device_status() == 0


def _sampled_chunks(seq: int, chunks: int = 8, rows: int = 64) -> list[tuple[int, int]]:
    """``chunks`` runs of ``rows`` query rows spread over the sequence; the last run is
    the sequence's tail (the audio tokens of the joint sequence)."""

    starts = [seq * i // chunks for i in range(chunks - 1)] + [seq - rows]
    return [(a, a + rows) for a in starts]


@pytest.fixture
def fp32_matmul():
    saved = torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = torch.backends.cudnn.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32, torch.backends.cudnn.allow_tf32 = saved


@pytest.mark.parametrize("heads", [24, 3])
def test_headline_attention_against_fp32_on_sampled_rows(fp32_matmul, heads):
    """480p-5s attention (24 heads: one GPU; 3 heads: the SP8 per-rank shape) against an
    fp32 torch reference over all 51,200 keys for 512 query rows spread over the
    sequence. Bar: max-abs <= 2e-2 and cosine >= 0.9999."""

    from oracle.block_ref import attention_heads

    from h3_flash_b200.runtime.attention.dense import packed_attention

    g = torch.Generator(device="cuda").manual_seed(11 + heads)
    packed = torch.randn(S, heads, 384, device="cuda", generator=g).to(torch.bfloat16)
    out = packed_attention(packed, 128)
    q, k, v = (packed[..., i * 128:(i + 1) * 128].float() for i in range(3))
    rows = torch.cat([torch.arange(a, b) for a, b in _sampled_chunks(S)]).cuda()
    want = attention_heads(q.index_select(0, rows).contiguous(), k.contiguous(), v.contiguous(), block=128)
    got = out.index_select(0, rows).float()
    diff = (got - want).abs()
    cosine = float(F.cosine_similarity(got.flatten(), want.flatten(), dim=0))
    assert float(diff.max()) <= 2e-2 and cosine >= 0.9999, (float(diff.max()), cosine)


def test_headline_block_against_fp32_on_sampled_rows(fp32_matmul):
    """The fused 480p-5s block (d=3072, S=51,200, one GPU) against the fp32 block computed
    on the GPU from the same bf16 weights and inputs (the oracle's block math run as fp32
    torch ops: keys and values of every row, then 512 sampled query rows through the whole
    block). Bar: max-abs <= 2e-2 and cosine >= 0.9999 on the sampled rows."""

    from oracle.block_ref import block_forward_rows, project_kv

    from h3_flash_b200 import _lib
    from h3_flash_b200.runtime.h3_block import H3BlockStack, H3TransformerBlock
    from h3_flash_b200.runtime.kernels import install_transformer_fusions
    from h3_flash_b200.workloads import CONFIGS, adaln_indices, init_block_, positions, rope_tables

    cfg = CONFIGS["480p-5s"]
    block = init_block_(H3TransformerBlock(cfg.dim, cfg.heads, cfg.head_dim, cfg.ffn_inner, eps=cfg.eps,
                                           qk_eps=cfg.eps), seed=0)
    block = block.to("cuda", torch.bfloat16).eval()
    params = {name: value.detach().float() for name, value in block.state_dict().items()}
    stack = H3BlockStack([block])
    g = torch.Generator(device="cuda").manual_seed(1)
    hidden = torch.randn(1, cfg.seq, cfg.dim, device="cuda", generator=g).to(torch.bfloat16)
    idx = adaln_indices(cfg).cuda()
    cos, sin = (t.cuda() for t in rope_tables(positions(cfg), cfg.rotary_dim, cfg.theta))
    install_transformer_fusions(stack)
    with torch.no_grad():
        fused = stack(hidden, None, idx, (cos, sin))[0]
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    kw = dict(heads=cfg.heads, head_dim=cfg.head_dim, eps=cfg.eps, qk_eps=cfg.eps)
    x = hidden[0].float()
    k_all = torch.empty(cfg.seq, cfg.heads, cfg.head_dim, device="cuda")
    v_all = torch.empty_like(k_all)
    with torch.no_grad():
        for a in range(0, cfg.seq, 8192):
            b = min(a + 8192, cfg.seq)
            k_all[a:b], v_all[a:b] = project_kv(params, x[a:b], idx[a:b], cos[a:b], sin[a:b], **kw)
        got, want = [], []
        for a, b in _sampled_chunks(cfg.seq):
            want.append(block_forward_rows(params, x[a:b], idx[a:b], cos[a:b], sin[a:b], k_all, v_all, a, **kw))
            got.append(fused[a:b].float())
    got, want = torch.cat(got), torch.cat(want)
    rows = torch.cat([torch.arange(a, b) for a, b in _sampled_chunks(cfg.seq)]).cuda()
    del fused, k_all, v_all, stack
    torch.cuda.empty_cache()
    max_abs, excess, cosine = _metrics(got, want)
    assert torch.isfinite(got).all()
    # the output is bf16: an element may sit half a bf16 spacing of its own magnitude
    # from the fp32 value before any arithmetic error; the 2e-2 bar applies above that
    assert excess <= 2e-2 and cosine >= 0.9999, (max_abs, excess, cosine)
    # and no further from fp32 than the reference's own LOSSLESS block on the same rows
    theirs = _reference_block_rows(cfg, hidden, idx, cos, sin, rows)
    if theirs is not None:
        ref_max, ref_excess, ref_cosine = _metrics(theirs, want)
        assert max_abs <= max(2e-2, 1.05 * ref_max), (max_abs, ref_max)
        assert float((got - want).abs().mean()) <= 1.05 * float((theirs - want).abs().mean())


def _reference_block_rows(cfg, hidden, idx, cos, sin, rows):
    """The reference's LOSSLESS block (its own installers and Triton kernels, from
    baseline/_ref) on the same weights and inputs, at ``rows``; None when absent."""

    import sys
    from pathlib import Path

    sys.path.insert(0, str(Path(__file__).resolve().parents[1]))
    import bench

    if bench._reference_site() is None:
        return None
    stack, _, _ = bench.reference_stack(cfg, 1)
    with torch.no_grad():
        out = stack(hidden, None, idx, (cos, sin))[0].index_select(0, rows).float()
    del stack
    torch.cuda.empty_cache()
    return out
