"""The allocation-free attention entry point against the allocating one.

h3b_attention_noalloc exists for callers that reach the kernels over the plain C
ABI and own no device allocator (the memory belongs to another framework's pool,
and cudaMalloc on their hot loop would bypass it and can synchronise the device).
It keeps the split-tail workspace in a fixed device array instead of caller
memory. Here it is called through the C ABI twice in a row, and each result is
checked against h3b_attention fed a torch-allocated workspace, with the
attention tolerance of the other GPU tests. This file is collected last.
"""

from __future__ import annotations

import math

import numpy as np
import pytest
import torch

from oracle.attention_ref import error_metrics

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-2
COSINE = 0.9999


def _views(packed: torch.Tensor):
    q = packed[..., :128].unsqueeze(0)
    k = packed[..., 128:256].unsqueeze(0)
    v = packed[..., 256:].unsqueeze(0)
    return q, k, v


def _strides(q, k, v, o):
    return [q.stride(0), q.stride(1), q.stride(2), k.stride(0), k.stride(1), k.stride(2),
            v.stride(0), v.stride(1), v.stride(2), o.stride(0), o.stride(1), o.stride(2)]


@pytest.mark.parametrize("seq,hl", [(51200, 3), (38400, 1)])
def test_noalloc_matches_allocating_entry_point_twice(seq, hl):
    from h3_flash_b200 import _lib
    from h3_flash_b200._torch import ptr, stream_of
    from h3_flash_b200.runtime.attention.dense import workspace_bytes

    g = torch.Generator(device="cuda").manual_seed(seq + hl)
    packed = torch.randn(seq, hl, 384, device="cuda", generator=g).to(torch.bfloat16)
    q, k, v = _views(packed)
    scale = 1.0 / math.sqrt(128)
    need = workspace_bytes(1, seq, seq, hl)
    assert need > 0, "the shape must exercise the split tail"

    expect = torch.empty(1, seq, hl, 128, dtype=torch.bfloat16, device="cuda")
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    _lib.call("h3b_attention", ptr(expect), ptr(q), ptr(k), ptr(v), 1, seq, seq, hl, 128,
              *_strides(q, k, v, expect), scale, ptr(ws), need, stream_of(q))

    # The whole-unit plan (no workspace) rounds the tail differently from the split plan.
    unsplit = torch.empty_like(expect)
    _lib.call("h3b_attention", ptr(unsplit), ptr(q), ptr(k), ptr(v), 1, seq, seq, hl, 128,
              *_strides(q, k, v, unsplit), scale, None, 0, stream_of(q))

    for _ in range(2):  # the shared array keeps the previous call's contents
        got = torch.full_like(expect, float("nan"))
        _lib.call("h3b_attention_noalloc", ptr(got), ptr(q), ptr(k), ptr(v), 1, seq, seq, hl, 128,
                  *_strides(q, k, v, got), scale, stream_of(q))
        torch.cuda.synchronize()
        m = error_metrics(got.float().cpu().numpy(), expect.float().cpu().numpy())
        assert np.isfinite(m["max_abs"]), m
        assert m["max_abs"] <= MAX_ABS, m
        assert m["cosine"] >= COSINE, m
        # Same split plan, same kernels: the static array stands in for the caller's
        # workspace bit for bit, and the split tail really ran through it.
        assert torch.equal(got, expect)
        assert not torch.equal(got, unsplit), "the split tail did not run"
    assert _lib.device_status() == 0


def test_noalloc_limits_and_errors():
    """On a 148-SM B200 every split plan fits the 20 MiB array (148 split CTAs x
    130 KiB at most), and bad arguments surface as the ordinary exceptions."""

    from h3_flash_b200 import _lib
    from h3_flash_b200.runtime.attention.dense import workspace_bytes

    assert workspace_bytes(1, 51200, 51200, 3) <= 20 << 20
    assert workspace_bytes(1, 256, 51200, 1) <= 20 << 20
    # Invalid shapes still fail with the ordinary errors.
    with pytest.raises(RuntimeError, match="head_dim must be 128"):
        _lib.call("h3b_attention_noalloc", None, None, None, None, 1, 4, 4, 1, 64,
                  *([64] * 12), 1.0, None)
