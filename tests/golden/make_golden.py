#!/usr/bin/env python3
"""Generate golden vectors from the reference's own kernels (run in the build container).

The reference (fluxmatrix/h3-flash) ships its hot-path kernels as Triton. With
``TRITON_INTERPRET=1`` Triton executes those exact kernel bodies on the CPU, so
this script imports the reference package read-only and records, on small seeded
inputs, what its kernels produce:

* fusions.py: fused_rmsnorm_modulate, fused_residual_gate_rmsnorm_modulate,
  fused_swiglu, fused_qknorm_rope                        -> fusions.npz
* relayout.py: pack_qkv_destination_major, merge_heads    -> relayout.npz
* packed_ulysses.py: _packed_qkv_all_to_all / _packed_output_all_to_all run as
  two gloo ranks (row counts 5 and 6, the reference's CPU routing)  -> ulysses_w2.npz

bf16 tensors are stored as uint16 bit patterns. The fixtures are committed; the
GPU box never needs the reference.

Usage: python tests/golden/make_golden.py [--reference /path/to/h3-flash]
"""

from __future__ import annotations

import argparse
import os
import sys
from pathlib import Path

os.environ["TRITON_INTERPRET"] = "1"

import numpy as np  # noqa: E402
import torch  # noqa: E402

HERE = Path(__file__).resolve().parent


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16).copy()


def fusions_cases(fusions) -> dict[str, np.ndarray]:
    out: dict[str, np.ndarray] = {}
    g = torch.Generator().manual_seed(17)

    def randn(*shape, std=1.0, mean=0.0):
        return (torch.randn(*shape, generator=g) * std + mean).to(torch.bfloat16)

    # (name, rows, cols, n_table, n_index, eps)
    for name, rows, cols, n_table, n_index, eps in (
        ("a", 37, 256, 3, 37, 1e-6),
        ("b", 9, 100, 2, 4, 1e-5),
        ("c", 17, 3072, 9, 17, 1e-6),
    ):
        x = randn(1, rows, cols)
        branch = randn(1, rows, cols)
        weight = randn(cols, mean=1.0, std=0.02)
        wide = randn(n_table, 6 * cols, std=0.1)  # [n_table, 6d] AdaLN table, row stride 6d
        shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, _ = wide.chunk(6, -1)
        index = torch.randint(0, n_table, (n_index,), generator=g, dtype=torch.int64)
        y = fusions.fused_rmsnorm_modulate(x, weight, scale_msa, shift_msa, index, eps)
        hidden, normed = fusions.fused_residual_gate_rmsnorm_modulate(
            x, branch, gate_msa, weight, scale_mlp, shift_mlp, index, eps
        )
        p = f"mod_{name}_"
        out[p + "x"] = bits(x)
        out[p + "branch"] = bits(branch)
        out[p + "weight"] = bits(weight)
        out[p + "wide"] = bits(wide)
        out[p + "index"] = index.numpy()
        out[p + "eps"] = np.array(eps, dtype=np.float64)
        out[p + "rmsnorm_modulate"] = bits(y)
        out[p + "hidden"] = bits(hidden)
        out[p + "normed"] = bits(normed)

    for name, rows, n in (("a", 11, 288), ("b", 3, 100)):
        x = randn(rows, 2 * n, std=2.0)
        out[f"swiglu_{name}_x"] = bits(x)
        out[f"swiglu_{name}_out"] = bits(fusions.fused_swiglu(x))

    # (name, B, S, H, D, rotary, eps)
    for name, b, s, h, d, rot, eps in (
        ("a", 1, 7, 4, 128, 96, 1e-6),
        ("b", 2, 5, 3, 128, 128, 1e-6),
        ("c", 1, 6, 2, 64, 10, 1e-5),
        ("d", 1, 4, 2, 128, 32, 1e-6),
    ):
        x = randn(b, s, h, d)
        weight = randn(d, mean=1.0, std=0.02)
        angles = torch.randn(s, rot, generator=g) * 3.0
        cos, sin = angles.cos(), angles.sin()
        y = fusions.fused_qknorm_rope(x, weight, cos, sin, eps)
        p = f"rope_{name}_"
        out[p + "x"] = bits(x)
        out[p + "weight"] = bits(weight)
        out[p + "cos"] = cos.numpy()
        out[p + "sin"] = sin.numpy()
        out[p + "eps"] = np.array(eps, dtype=np.float64)
        out[p + "out"] = bits(y)
    return out


def relayout_cases(relayout) -> dict[str, np.ndarray]:
    out: dict[str, np.ndarray] = {}
    g = torch.Generator().manual_seed(1000)
    for name, rows, heads, d, world in (("a", 13, 8, 128, 4), ("b", 5, 6, 64, 2), ("c", 3, 4, 16, 4)):
        fused = (torch.randn(rows, 3 * heads * d, generator=g)).to(torch.bfloat16)
        q, k, v = (t.reshape(rows, heads, d) for t in fused.chunk(3, dim=-1))  # strided views
        packed = relayout.pack_qkv_destination_major(q, k, v, world)
        assert torch.equal(packed, relayout.pack_qkv_reference(q, k, v, world))
        p = f"pack_{name}_"
        out[p + "qkv"] = bits(fused)
        out[p + "shape"] = np.array([rows, heads, d, world], dtype=np.int64)
        out[p + "out"] = bits(packed)
    for name, world, rows, hl, d in (("a", 4, 13, 2, 128), ("b", 2, 7, 3, 64)):
        x = torch.randn(world, rows, hl, d, generator=g).to(torch.bfloat16)
        out[f"merge_{name}_x"] = bits(x)
        out[f"merge_{name}_out"] = bits(relayout.merge_heads(x))
    return out


def _ulysses_worker(rank: int, world: int, port: int, reference: str, queue) -> None:
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, reference)
    import torch.distributed as dist

    from h3_flash.runtime.parallel import packed_ulysses as pu

    dist.init_process_group(
        "gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world
    )

    # The reference allocates its row-count buffer on "cuda" (packed_ulysses.py:45);
    # run the identical logic on the CPU for gloo.
    def row_counts(self, rows_local):
        if self._row_counts is not None:
            counts, seen = self._row_counts
            if seen != rows_local:
                raise RuntimeError("row count changed")
            return counts
        buffer = torch.zeros(self.world, dtype=torch.long)
        buffer[dist.get_rank(self.group)] = rows_local
        dist.all_reduce(buffer, group=self.group)
        counts = [int(value) for value in buffer.tolist()]
        self._row_counts = (counts, rows_local)
        return counts

    pu.PackedUlyssesRuntime.row_counts = row_counts
    rows = 5 + rank  # uneven: 5, 6
    heads, d = 8, 32
    g = torch.Generator().manual_seed(1000 + rank)
    q = torch.randn(rows, heads, d, generator=g).to(torch.bfloat16)
    k = torch.randn(rows, heads, d, generator=g).to(torch.bfloat16)
    v = torch.randn(rows, heads, d, generator=g).to(torch.bfloat16)
    runtime = pu.PackedUlyssesRuntime(dist.group.WORLD)
    runtime.begin_request()
    packed = pu._packed_qkv_all_to_all(q, k, v, runtime)
    attn_out = torch.randn(packed.shape[0], heads // world, d, generator=g).to(torch.bfloat16)
    back = pu._packed_output_all_to_all(attn_out, rows, runtime)
    queue.put(
        (
            rank,
            {
                f"r{rank}_q": bits(q),
                f"r{rank}_k": bits(k),
                f"r{rank}_v": bits(v),
                f"r{rank}_packed": bits(packed),
                f"r{rank}_attn": bits(attn_out),
                f"r{rank}_back": bits(back),
            },
        )
    )
    dist.barrier()
    dist.destroy_process_group()


def ulysses_case(reference: str) -> dict[str, np.ndarray]:
    import socket

    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    procs = [
        ctx.Process(target=_ulysses_worker, args=(r, 2, port, reference, queue)) for r in range(2)
    ]
    for p in procs:
        p.start()
    out: dict[str, np.ndarray] = {}
    for _ in procs:
        _, payload = queue.get(timeout=300)
        out.update(payload)
    for p in procs:
        p.join(timeout=60)
        if p.exitcode != 0:
            raise RuntimeError(f"gloo worker failed: exit {p.exitcode}")
    out["heads"] = np.array(8)
    out["head_dim"] = np.array(32)
    return out


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--reference", default=os.environ.get("H3_FLASH_REFERENCE"),
                        help="checkout of fluxmatrix/h3-flash (default: $H3_FLASH_REFERENCE)")
    args = parser.parse_args()
    if not args.reference:
        parser.error("pass --reference or set H3_FLASH_REFERENCE")
    src = str(Path(args.reference) / "src")
    sys.path.insert(0, src)
    from h3_flash.runtime.kernels import fusions
    from h3_flash.runtime.parallel import relayout

    np.savez_compressed(HERE / "fusions.npz", **fusions_cases(fusions))
    np.savez_compressed(HERE / "relayout.npz", **relayout_cases(relayout))
    np.savez_compressed(HERE / "ulysses_w2.npz", **ulysses_case(src))
    for name in ("fusions.npz", "relayout.npz", "ulysses_w2.npz"):
        print(name, (HERE / name).stat().st_size, "bytes")
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
