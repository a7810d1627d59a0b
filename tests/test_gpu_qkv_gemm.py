"""The QKV projection GEMM with the packed-Ulysses epilogue (h3b_qkv_gemm_pack).

Checked against an fp32 restatement of the reference path (to_q/to_k/to_v, QK-norm,
rotate-half RoPE, destination-major pack: packed_ulysses.py:166-200,
relayout.py:97-130): every element within 2^-7 relative + 1e-3 absolute (one bf16
rounding of a value computed in fp32 from bf16 inputs), cosine >= 0.9999. Shapes cover
row tails (rows not a multiple of 256), rotary widths 0/64/96/128, no bias, several
Ulysses degrees, and the p2p form with every 'peer' buffer on this GPU (rows land at
their global offset in every owner's receive buffer).
"""

from __future__ import annotations

import ctypes

import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _reference(x, w, b, wq, wk, cos, sin, heads, world, eps):
    rows = x.shape[0]
    y = x.float() @ w.float().t()
    if b is not None:
        y = y + b.float()
    hd = heads * 128
    q, k, v = (y[:, i * hd:(i + 1) * hd].view(rows, heads, 128) for i in range(3))

    def norm_rope(t, weight):
        n = t * torch.rsqrt(t.pow(2).mean(-1, keepdim=True) + eps) * weight.float()
        if cos is not None:
            rot = cos.shape[-1]
            half = rot // 2
            a, c = n[..., :half].clone(), n[..., half:rot].clone()
            cs, sn = cos[:, None, :].float(), sin[:, None, :].float()
            n[..., :half] = a * cs[..., :half] - c * sn[..., :half]
            n[..., half:rot] = c * cs[..., half:] + a * sn[..., half:]
        return n

    packed = torch.stack([norm_rope(q, wq), norm_rope(k, wk), v], 2)  # [rows, H, 3, D]
    return packed.view(rows, world, heads // world, 384).permute(1, 0, 2, 3).contiguous()


def _close(got, ref):
    got = got.float()
    diff = (got - ref).abs()
    bad = int((diff > ref.abs() * 2.0 ** -7 + 1e-3).sum())
    cos = float(F.cosine_similarity(got.flatten(), ref.flatten(), dim=0))
    return bad, cos


def _inputs(rows, dim, heads, rot, bias, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(rows, dim, device="cuda", generator=g).to(torch.bfloat16)
    w = (torch.randn(3 * heads * 128, dim, device="cuda", generator=g) * dim ** -0.5).to(torch.bfloat16)
    b = (0.1 * torch.randn(3 * heads * 128, device="cuda", generator=g)).to(torch.bfloat16) if bias else None
    wq = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(torch.bfloat16)
    wk = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(torch.bfloat16)
    cos = sin = None
    if rot:
        cos = torch.rand(rows, rot, device="cuda", generator=g) * 2 - 1
        sin = torch.rand(rows, rot, device="cuda", generator=g) * 2 - 1
    return x, w, b, wq, wk, cos, sin


@pytest.mark.parametrize("rows,dim,heads,world,rot,bias", [
    (300, 512, 4, 1, 96, True),
    (1000, 3072, 24, 2, 96, True),
    (777, 1024, 6, 3, 128, True),
    (513, 256, 2, 1, 0, True),
    (256, 768, 8, 4, 64, False),
    (1, 128, 2, 2, 96, True),
])
def test_qkv_gemm_pack_matches_fp32_reference(rows, dim, heads, world, rot, bias):
    from h3_flash_b200 import _lib
    from h3_flash_b200.runtime.kernels.fusions import fused_qkv_gemm_pack

    x, w, b, wq, wk, cos, sin = _inputs(rows, dim, heads, rot, bias, rows + dim)
    out = torch.full((world, rows, heads // world, 384), float("nan"), device="cuda").to(torch.bfloat16)
    fused_qkv_gemm_pack(x, w, b, wq, wk, cos, sin, heads, world, 1e-6, 1e-6, out=out)
    torch.cuda.synchronize()
    bad, cosine = _close(out, _reference(x, w, b, wq, wk, cos, sin, heads, world, 1e-6))
    assert bad == 0 and cosine >= 0.9999, (bad, cosine)
    assert _lib.device_status() == 0


@pytest.mark.parametrize("rows,dim,heads,world,offset", [(1000, 3072, 24, 2, 5), (777, 1024, 6, 3, 0)])
def test_qkv_gemm_pack_p2p_routes_rows_to_owners(rows, dim, heads, world, offset):
    from h3_flash_b200 import _lib

    x, w, b, wq, wk, cos, sin = _inputs(rows, dim, heads, 96, True, 7)
    total = offset + rows + 3
    hl = heads // world
    recv = [torch.full((total, hl, 384), float("nan"), device="cuda").to(torch.bfloat16) for _ in range(world)]
    ptrs = (ctypes.c_void_p * world)(*[t.data_ptr() for t in recv])
    ws = torch.empty(rows * 96 * 2, dtype=torch.float32, device="cuda")
    _lib.call("h3b_qkv_gemm_pack_p2p", ptrs, world, offset, total, x.data_ptr(), rows, dim, dim, w.data_ptr(),
              b.data_ptr(), wq.data_ptr(), wk.data_ptr(), cos.data_ptr(), sin.data_ptr(), heads, 128, 96,
              1e-6, 1e-6, ws.data_ptr(), ws.numel() * 4, torch.cuda.current_stream().cuda_stream)
    local = torch.empty((world, rows, hl, 384), device="cuda").to(torch.bfloat16)
    from h3_flash_b200.runtime.kernels.fusions import fused_qkv_gemm_pack

    fused_qkv_gemm_pack(x, w, b, wq, wk, cos, sin, heads, world, 1e-6, 1e-6, out=local)
    torch.cuda.synchronize()
    for owner in range(world):
        assert torch.equal(recv[owner][offset:offset + rows], local[owner])  # same bits as the local form
        assert torch.isnan(recv[owner][:offset].float()).all() and torch.isnan(recv[owner][offset + rows:].float()).all()
    assert _lib.device_status() == 0


def test_qkv_gemm_pack_close_to_the_unfused_path():
    """The fused kernel and cuBLAS + fused_qknorm_rope_pack differ only by the bf16
    rounding of the projection before the norm (and the GEMM summation order)."""

    from h3_flash_b200.runtime.kernels.fusions import fused_qkv_gemm_pack, fused_qknorm_rope_pack

    rows, dim, heads, world = 640, 3072, 24, 8
    x, w, b, wq, wk, cos, sin = _inputs(rows, dim, heads, 96, True, 3)
    fused = fused_qkv_gemm_pack(x, w, b, wq, wk, cos, sin, heads, world, 1e-6, 1e-6)
    y = F.linear(x, w, b)
    q, k, v = (y[:, i * heads * 128:(i + 1) * heads * 128].view(rows, heads, 128) for i in range(3))
    unfused = fused_qknorm_rope_pack(q, k, v, wq, wk, cos, sin, world, 1e-6, 1e-6)
    ref = _reference(x, w, b, wq, wk, cos, sin, heads, world, 1e-6)
    err_fused = float((fused.float() - ref).abs().mean())
    err_unfused = float((unfused.float() - ref).abs().mean())
    assert err_fused <= err_unfused * 1.05, (err_fused, err_unfused)
    cosine = float(F.cosine_similarity(fused.float().flatten(), unfused.float().flatten(), dim=0))
    assert cosine >= 0.9999


def test_qkv_gemm_pack_empty_rows_is_a_noop():
    from h3_flash_b200.runtime.kernels.fusions import fused_qkv_gemm_pack

    x, w, b, wq, wk, cos, sin = _inputs(0, 256, 2, 96, True, 1)
    out = fused_qkv_gemm_pack(x, w, b, wq, wk, cos, sin, 2, 1, 1e-6, 1e-6)
    assert out.shape == (1, 0, 2, 384)



def test_qkv_gemm_pack_matches_the_oracle_reference_path():
    """Against the oracle of the reference path: the projection rounded to bf16 (what
    to_q/to_k/to_v return), then oracle.fusions_ref.qknorm_rope (pinned to the reference
    kernel's golden vectors) and oracle.relayout_ref.pack_qkv. The fused kernel skips the
    projection's bf16 rounding, so it does not match the oracle to a fixed number of
    spacings where RoPE cancels. The bars, elementwise against the fp32 evaluation T of
    the same math:
    - |fused - T| <= 2^-7 |T| + 1e-3 (one bf16 rounding);
    - |fused - oracle| <= |oracle - T| + 2^-7 |T| + 1e-3 (the oracle's own error plus one
      rounding);
    - on average the fused result is at least as close to T as the oracle path."""

    import numpy as np

    from oracle import fusions_ref, relayout_ref
    from oracle.bf16 import from_f32, to_f32
    from h3_flash_b200.runtime.kernels.fusions import fused_qkv_gemm_pack

    rows, dim, heads, world = 300, 512, 4, 2
    x, w, b, wq, wk, cos, sin = _inputs(rows, dim, heads, 96, True, 21)
    got = fused_qkv_gemm_pack(x, w, b, wq, wk, cos, sin, heads, world, 1e-6, 1e-6)
    truth = _reference(x, w, b, wq, wk, cos, sin, heads, world, 1e-6).cpu().numpy()
    bits = lambda t: t.contiguous().view(torch.int16).cpu().numpy().view(np.uint16)
    y = to_f32(bits(x)) @ to_f32(bits(w)).T + to_f32(bits(b))
    proj = from_f32(y.astype(np.float32))  # the bf16 projection the reference normalises
    hd = heads * 128
    q, k, v = (proj[:, i * hd:(i + 1) * hd].reshape(rows, heads, 128) for i in range(3))
    cos_np, sin_np = cos.cpu().numpy(), sin.cpu().numpy()
    qn = fusions_ref.qknorm_rope(q[None], bits(wq), cos_np, sin_np, 1e-6)[0]
    kn = fusions_ref.qknorm_rope(k[None], bits(wk), cos_np, sin_np, 1e-6)[0]
    oracle = to_f32(relayout_ref.pack_qkv(qn, kn, v, world))
    fused = to_f32(bits(got)).reshape(oracle.shape)
    one_rounding = np.abs(truth) * 2.0 ** -7 + 1e-3
    assert int((np.abs(fused - truth) > one_rounding).sum()) == 0
    assert int((np.abs(fused - oracle) > np.abs(oracle - truth) + one_rounding).sum()) == 0
    assert float(np.abs(fused - truth).mean()) <= float(np.abs(oracle - truth).mean()) * 1.05
