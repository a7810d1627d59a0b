"""The bench's reference arm (the CPU port of the reference path) prints one JSON line
with the contract's keys. The h3b arm needs a GPU and runs in the GPU rounds."""

from __future__ import annotations

import json
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_reference_arm_prints_the_contract_line():
    result = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--config", "cpu-gloo",
                             "--steps", "2", "--warmup", "1"],
                            cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert result.returncode == 0, result.stderr[-2000:]
    lines = [line for line in result.stdout.splitlines() if line.startswith("{")]
    assert len(lines) == 1
    line = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line, key
    assert line["impl"] == "reference" and line["unit"] == "ms" and line["higher_is_better"] is False
    assert line["value"] > 0 and line["e2e"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0
    base = line["cpu_baseline"]
    assert base["kind"] == "port" and base["cores"] >= 1 and base["sample"]
    assert "workload" in line["config"]
    # the timed steps cover the sequence once: a measurement, not a scaled sample
    assert base["scaled"] is False and base["rows_measured"] == line["config"]["seq"]
    assert abs(sum(base["chunk_ms"]) - line["value"]) < 0.05 * line["value"]


def _torch_ulysses_worker(rank, world):
    import torch
    import torch.distributed as dist

    sys.path.insert(0, str(ROOT))
    import bench
    from h3_flash_b200.runtime.h3_block import Attention
    from h3_flash_b200.workloads import rope_tables, split_bounds

    torch.manual_seed(0)
    attention = Attention(64, 4, 16, qk_eps=1e-6).double()
    rows_total = 23
    g = torch.Generator().manual_seed(1)
    x = torch.randn(1, rows_total, 64, generator=g, dtype=torch.float64)
    pos = torch.stack([torch.arange(rows_total) // 6, (torch.arange(rows_total) // 2) % 3, torch.arange(rows_total) % 2], -1)
    cos, sin = (t.double() for t in rope_tables(pos, 12))
    with torch.no_grad():
        expect = attention(x, (cos, sin))
        start, stop = split_bounds(rows_total, world, rank)
        counts = [split_bounds(rows_total, world, r)[1] - split_bounds(rows_total, world, r)[0] for r in range(world)]
        got = bench._torch_ulysses_forward(attention, x[:, start:stop], (cos[start:stop], sin[start:stop]),
                                           group=dist.group.WORLD, counts=counts)
    return float((got - expect[:, start:stop]).abs().max())


def test_torch_ulysses_baseline_equals_the_full_sequence_attention():
    """The opt-in N>1 GPU baseline's attention (reference structure, torch ops, all-to-alls)
    computes the module's full-sequence attention: two gloo ranks, fp64, uneven rows."""

    from tests.test_gloo import _run

    for diff in _run(2, _torch_ulysses_worker):
        assert diff <= 1e-12, diff
