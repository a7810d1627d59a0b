"""GPU parity of the packed-Ulysses relayouts: bit-exact against the reference goldens/oracle."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import bf16, fusions_ref, relayout_ref
from tests.gpu_util import bits, dev, seeded_bits

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", ["a", "b", "c"])
def test_pack_qkv_destination_major_golden(golden_relayout, case):
    from h3_flash_b200.runtime.parallel.relayout import pack_qkv_destination_major

    g = golden_relayout
    rows, heads, d, world = (int(v) for v in g[f"pack_{case}_shape"])
    fused = dev(g[f"pack_{case}_qkv"])
    q, k, v = (t.reshape(rows, heads, d) for t in fused.chunk(3, dim=-1))  # strided views
    out = pack_qkv_destination_major(q, k, v, world)
    np.testing.assert_array_equal(bits(out), g[f"pack_{case}_out"])


@pytest.mark.parametrize("case", ["a", "b"])
def test_merge_heads_golden(golden_relayout, case):
    from h3_flash_b200.runtime.parallel.relayout import merge_heads

    g = golden_relayout
    np.testing.assert_array_equal(bits(merge_heads(dev(g[f"merge_{case}_x"]))), g[f"merge_{case}_out"])


@pytest.mark.parametrize("rows,heads,world,rot", [(37, 24, 8, 96), (5, 24, 1, 96), (13, 8, 4, 128),
                                                  (9, 6, 2, 0), (11, 4, 2, 10)])
def test_fused_qknorm_rope_pack(rows, heads, world, rot):
    """The fused kernel equals pack(rope(norm(q)), rope(norm(k)), v): q/k within 1 ulp of
    the oracle, v and the layout bit-exact."""

    from h3_flash_b200.runtime.kernels.fusions import fused_qknorm_rope_pack

    d = 128
    qkv = seeded_bits(7, (rows, 3 * heads * d))
    wq = seeded_bits(8, (d,), 1.0, 0.02)
    wk = seeded_bits(9, (d,), 1.0, 0.02)
    ang = np.random.default_rng(10).standard_normal((rows, rot)).astype(np.float32)
    cos, sin = np.cos(ang).astype(np.float32), np.sin(ang).astype(np.float32)
    fused = dev(qkv)
    q, k, v = (t.view(rows, heads, d) for t in fused.split(heads * d, dim=-1))
    out = fused_qknorm_rope_pack(q, k, v, dev(wq), dev(wk),
                                 torch.from_numpy(cos).cuda() if rot else None,
                                 torch.from_numpy(sin).cuda() if rot else None, world, 1e-6, 1e-5)
    qn = qkv[:, : heads * d].reshape(1, rows, heads, d)
    kn = qkv[:, heads * d : 2 * heads * d].reshape(1, rows, heads, d)
    vn = qkv[:, 2 * heads * d :].reshape(rows, heads, d)
    rq = fusions_ref.qknorm_rope(qn, wq, cos, sin, 1e-6)[0]
    rk = fusions_ref.qknorm_rope(kn, wk, cos, sin, 1e-5)[0]
    ref = relayout_ref.pack_qkv(rq, rk, vn, world)
    got = bits(out)
    assert got.shape == ref.shape
    assert int(bf16.ulp_distance(got[..., : 2 * d], ref[..., : 2 * d]).max()) <= 1
    np.testing.assert_array_equal(got[..., 2 * d :], ref[..., 2 * d :])


def test_pack_then_merge_roundtrip_is_identity():
    """Size-independent property at a benchmark-like shape: merging the pack's v part
    back returns the original heads bit for bit."""

    from h3_flash_b200.runtime.parallel.relayout import merge_heads, pack_qkv_destination_major

    rows, heads, d, world = 6400, 24, 128, 8
    g = torch.Generator(device="cuda").manual_seed(3)
    q, k, v = (torch.randn(rows, heads, d, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
    packed = pack_qkv_destination_major(q, k, v, world)
    for part, t in enumerate((q, k, v)):
        merged = merge_heads(packed[..., part * d : (part + 1) * d].contiguous())
        assert torch.equal(merged, t)
