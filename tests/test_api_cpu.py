"""Host-side behaviour of the drop-in surface without a GPU: errors, guards, adapters.

Mirrors the reference's contract tests (tests/test_dense_fa4.py, tests/test_context_parallel.py)
plus the fail-loudly rule: no op of this package computes on CPU tensors.
"""

from __future__ import annotations

from pathlib import Path
from unittest.mock import Mock, patch

import pytest
import torch

from h3_flash_b200.runtime.attention.dense_fa4 import DenseFA4MiniMaxH3Processor, load_fa4
from h3_flash_b200.runtime.kernels import fusions
from h3_flash_b200.runtime.parallel import relayout
from h3_flash_b200.runtime.parallel.context import enable_h3_ulysses
from h3_flash_b200.runtime.parallel.packed_ulysses import install_packed_ulysses


def test_missing_fa4_package_is_rejected(tmp_path: Path) -> None:
    with pytest.raises(RuntimeError, match="CuTe package"):
        load_fa4(tmp_path)


def test_dense_processor_preserves_shape_and_full_sequence() -> None:
    class Attention(torch.nn.Module):
        def __init__(self) -> None:
            super().__init__()
            self.heads = 2
            self.fused_projections = False
            self.to_q = torch.nn.Linear(8, 8, bias=False)
            self.to_k = torch.nn.Linear(8, 8, bias=False)
            self.to_v = torch.nn.Linear(8, 8, bias=False)
            self.norm_q = torch.nn.Identity()
            self.norm_k = torch.nn.Identity()
            self.to_out = torch.nn.ModuleList([torch.nn.Linear(8, 8, bias=False), torch.nn.Identity()])

    seen = {}

    def kernel(q, k, v, **kwargs):
        seen["shapes"] = (q.shape, k.shape, v.shape)
        seen["kwargs"] = kwargs
        return v

    processor = DenseFA4MiniMaxH3Processor(kernel=kernel)
    result = processor(Attention(), torch.randn(1, 7, 8))
    assert result.shape == (1, 7, 8)
    assert seen["shapes"] == ((1, 7, 2, 4),) * 3
    assert seen["kwargs"] == {"causal": False}
    assert processor.calls == 1


def test_dense_processor_rejects_masked_sequence() -> None:
    processor = DenseFA4MiniMaxH3Processor(kernel=lambda *args, **kwargs: None)
    with pytest.raises(RuntimeError, match="padless"):
        processor(None, None, attention_mask=object())


def test_dense_processor_defaults_to_h3b_kernel() -> None:
    from h3_flash_b200.runtime.attention.dense import flash_attn_func

    assert DenseFA4MiniMaxH3Processor().kernel is flash_attn_func


def test_ulysses_requires_initialized_process_group() -> None:
    with patch("torch.distributed.is_initialized", return_value=False), \
            pytest.raises(RuntimeError, match="initialized torch process group"):
        enable_h3_ulysses(Mock(), degree=8)


def test_packed_ulysses_requires_initialized_process_group() -> None:
    with patch("torch.distributed.is_initialized", return_value=False), \
            pytest.raises(RuntimeError, match="initialized process group"):
        install_packed_ulysses(Mock())


@pytest.mark.parametrize(
    "call",
    [
        lambda: fusions.fused_swiglu(torch.zeros(2, 8, dtype=torch.bfloat16)),
        lambda: fusions.fused_gelu_tanh(torch.zeros(2, 8, dtype=torch.bfloat16)),
        lambda: fusions.fused_rmsnorm_modulate(torch.zeros(1, 2, 8, dtype=torch.bfloat16),
                                               torch.ones(8, dtype=torch.bfloat16),
                                               torch.zeros(1, 8, dtype=torch.bfloat16),
                                               torch.zeros(1, 8, dtype=torch.bfloat16),
                                               torch.zeros(1, dtype=torch.long), 1e-6),
        lambda: relayout.merge_heads(torch.zeros(2, 3, 1, 8, dtype=torch.bfloat16)),
    ],
)
def test_cpu_tensors_fail_loudly(call) -> None:
    with pytest.raises(RuntimeError, match="CUDA tensors only"):
        call()


def test_rotary_dimension_checked_before_device() -> None:
    x = torch.zeros(1, 3, 2, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="rotary dimension"):
        fusions.fused_qknorm_rope(x, torch.ones(128), torch.zeros(3, 7), torch.zeros(3, 7), 1e-6)


def test_heads_must_divide_world() -> None:
    q = torch.zeros(4, 6, 128, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="must divide Ulysses degree"):
        relayout.pack_qkv_destination_major(q, q, q, 4)
    with pytest.raises(ValueError, match="must divide Ulysses degree"):
        fusions.fused_qknorm_rope_pack(q, q, q, torch.ones(128), torch.ones(128), None, None, 4, 1e-6, 1e-6)


def test_pack_reference_definition_matches_oracle() -> None:
    import numpy as np

    from oracle import relayout_ref

    g = torch.Generator().manual_seed(0)
    q, k, v = (torch.randn(5, 8, 16, generator=g) for _ in range(3))
    ref = relayout_ref.pack_qkv(q.numpy(), k.numpy(), v.numpy(), 4)
    np.testing.assert_array_equal(relayout.pack_qkv_reference(q, k, v, 4).numpy(), ref)
    assert not relayout.can_pack_qkv(q, k, v)  # CPU tensors never take the kernel path


def test_workload_shapes_match_baseline() -> None:
    from h3_flash_b200.workloads import CONFIGS, rope_tables, positions, split_sizes

    assert CONFIGS["480p-5s"].seq == 49920 + 1280
    assert CONFIGS["768p-5s"].seq == 129024 + 1280
    assert CONFIGS["768p-15s"].seq == 350784 + 3456
    assert CONFIGS["cpu-gloo"].seq == 4096 + 256
    assert split_sizes(10, 4) == [3, 3, 2, 2]
    cos, sin = rope_tables(positions(CONFIGS["cpu-gloo"]), 96)
    assert cos.shape == (4352, 96) and sin.dtype == torch.float32
    assert torch.allclose(cos[:, :48], cos[:, 48:])


def test_qkv_weights_stack_cache_and_rebuild() -> None:
    """The stacked to_q | to_k | to_v weight the QKV GEMM consumes: concatenated once,
    rebuilt after an in-place update, missing biases filled with zeros."""

    from h3_flash_b200.runtime.parallel.packed_ulysses import qkv_weights

    class Attention(torch.nn.Module):
        def __init__(self) -> None:
            super().__init__()
            self.heads, self.head_dim, self.fused_projections = 2, 4, False
            self.to_q = torch.nn.Linear(8, 8)
            self.to_k = torch.nn.Linear(8, 8, bias=False)
            self.to_v = torch.nn.Linear(8, 8)

    attn = Attention()
    weight, bias = qkv_weights(attn)
    assert torch.equal(weight, torch.cat([attn.to_q.weight, attn.to_k.weight, attn.to_v.weight]))
    assert torch.equal(bias, torch.cat([attn.to_q.bias, torch.zeros(8), attn.to_v.bias]))
    assert qkv_weights(attn)[0] is weight  # cached
    with torch.no_grad():
        attn.to_k.weight.mul_(2.0)
    rebuilt, _ = qkv_weights(attn)
    assert rebuilt is not weight and torch.equal(rebuilt[8:16], attn.to_k.weight)
    attn.to_v = torch.nn.Identity()
    assert qkv_weights(attn) is None


def test_qkv_gemm_pack_supported_shapes() -> None:
    from h3_flash_b200.runtime.kernels.fusions import qkv_gemm_pack_supported

    x = torch.empty(4, 256, dtype=torch.bfloat16)
    w = torch.empty(3 * 2 * 128, 256, dtype=torch.bfloat16)
    cos = torch.empty(4, 96)
    assert not qkv_gemm_pack_supported(x, w, 2, 128, cos)  # CPU tensors: never
    if torch.cuda.is_available():  # pragma: no cover - CPU suite
        assert qkv_gemm_pack_supported(x.cuda(), w.cuda(), 2, 128, cos)
