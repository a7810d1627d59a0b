"""The bench's reference LOSSLESS block harness on the CPU.

``bench.reference_stack`` installs the unmodified reference (baseline/_ref) on this
package's H3-style block stack with the reference's own installers. Here its Triton
kernels run under the Triton CPU interpreter (TRITON_INTERPRET=1, which stores bf16 by
truncation) at a tiny shape, and the block output must agree with the fp32 oracle block:
the harness wiring (Diffusers stand-in, processor handle, first-block gates, installer
arguments) is checked without a GPU. Skipped when the reference install is absent.
"""

from __future__ import annotations

import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]

SCRIPT = r"""
import json, sys
sys.path.insert(0, sys.argv[1])
import torch
import bench
from h3_flash_b200.runtime.h3_block import H3TransformerBlock
from h3_flash_b200.workloads import BlockConfig, adaln_indices, init_block_, positions, rope_tables
from oracle.attention_ref import error_metrics
from oracle.block_ref import block_forward, fp32_params

cfg = BlockConfig("tiny", (2, 4, 8), 16, dim=256, heads=2, ffn_inner=1024)
stack, runtime, provenance = bench.reference_stack(cfg, 1, device="cpu")
block = init_block_(H3TransformerBlock(cfg.dim, cfg.heads, cfg.head_dim, cfg.ffn_inner, eps=cfg.eps,
                                       qk_eps=cfg.eps), seed=0)
params = {k: v.to(torch.bfloat16).float() for k, v in fp32_params(block).items()}
g = torch.Generator().manual_seed(1)
hidden = torch.randn(1, cfg.seq, cfg.dim, generator=g).to(torch.bfloat16)
idx = adaln_indices(cfg)
cos, sin = rope_tables(positions(cfg), cfg.rotary_dim, cfg.theta)
with torch.no_grad():
    out = stack(hidden, None, idx, (cos, sin))[0].float()
want = block_forward(params, hidden[0].float(), idx, cos, sin, heads=cfg.heads, head_dim=cfg.head_dim,
                     eps=cfg.eps, qk_eps=cfg.eps)
block0 = stack.transformer_blocks[0]
print(json.dumps({"metrics": error_metrics(out.numpy(), want.numpy()), "provenance": provenance,
                  "patched_block": "forward" in block0.__dict__,
                  "patched_attention": "forward" in block0.attn.__dict__}))
"""


def test_reference_lossless_block_under_the_triton_interpreter():
    sys.path.insert(0, str(ROOT))
    import bench

    if bench._reference_site() is None:
        pytest.skip("the reference package is not installed under baseline/_ref")
    env = dict(os.environ, TRITON_INTERPRET="1")
    result = subprocess.run([sys.executable, "-c", SCRIPT, str(ROOT)], cwd=ROOT, env=env, capture_output=True,
                            text=True, timeout=600)
    assert result.returncode == 0, result.stderr[-3000:]
    line = json.loads(result.stdout.strip().splitlines()[-1])
    assert line["patched_block"] and line["patched_attention"]
    assert "h3_flash" in line["provenance"]["package"]
    m = line["metrics"]
    assert m["cosine"] >= 0.9999 and m["max_abs"] <= 5e-2, m
