"""Packed Ulysses on 2+ GPUs against the reference's own multi-GPU path (its package
installed under baseline/_ref; skipped when absent or on a single-GPU box).

On every rank, with uneven row counts:
- ``_packed_qkv_all_to_all`` and ``_packed_output_all_to_all`` of this package (NCCL
  exchange) equal the reference's functions (src/h3_flash/runtime/parallel/
  packed_ulysses.py:85-128: Triton pack, all_to_all_single, Triton merge) bit for bit;
- the whole SP block with this package's defaults (fused QKV GEMM, NVLink peer exchange
  fused into the QKV GEMM and attention epilogues) and the reference's LOSSLESS SP block
  (its install_transformer_fusions + install_packed_ulysses: Triton fusions, NCCL, SDPA)
  are each compared with the fp32 oracle block over the full sequence: max-abs <= 2e-2
  above the bf16 output's half spacing, cosine >= 0.9999, and this package's block no
  less accurate than the reference's (mean-abs within 5%).
"""

from __future__ import annotations

import datetime
import os
import socket
import sys
import traceback
from pathlib import Path

import pytest
import torch

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        sys.path.insert(0, str(ROOT))
        torch.cuda.set_device(rank)
        import numpy as np
        import torch.distributed as dist

        import bench

        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        sys.path.insert(0, str(bench._reference_site()))
        bench._diffusers_stand_in()
        from h3_flash.runtime.parallel import packed_ulysses as ref_pu

        from h3_flash_b200.runtime.h3_block import H3BlockStack, H3TransformerBlock
        from h3_flash_b200.runtime.kernels import install_transformer_fusions
        from h3_flash_b200.runtime.parallel import install_packed_ulysses
        from h3_flash_b200.runtime.parallel import packed_ulysses as pu
        from h3_flash_b200.workloads import BlockConfig, adaln_indices, init_block_, positions, rope_tables
        from h3_flash_b200.workloads import split_bounds
        from oracle.attention_ref import error_metrics
        from oracle.block_ref import block_forward, fp32_params

        # 1) exchanges, uneven rows, against the reference's functions
        rows = 37 + 5 * rank
        heads = 4 * world
        g = torch.Generator(device="cuda").manual_seed(200 + rank)
        q, k, v = (torch.randn(rows, heads, 128, device="cuda", generator=g).to(torch.bfloat16) for _ in range(3))
        mine_rt, ref_rt = pu.PackedUlyssesRuntime(dist.group.WORLD), ref_pu.PackedUlyssesRuntime(dist.group.WORLD)
        mine_rt.begin_request()
        ref_rt.begin_request()
        mine_qkv = pu._packed_qkv_all_to_all(q, k, v, mine_rt)
        ref_qkv = ref_pu._packed_qkv_all_to_all(q, k, v, ref_rt)
        qkv_equal = torch.equal(mine_qkv, ref_qkv)
        out = mine_qkv[..., 256:].contiguous()
        out_equal = torch.equal(pu._packed_output_all_to_all(out, rows, mine_rt),
                                ref_pu._packed_output_all_to_all(out, rows, ref_rt))

        # 2) the SP block, this package's defaults and the reference's LOSSLESS block
        cfg = BlockConfig("sp-ref", (2, 16, 24), 64, dim=128 * 2 * world, heads=2 * world, ffn_inner=1024 * world)
        block = init_block_(H3TransformerBlock(cfg.dim, cfg.heads, cfg.head_dim, cfg.ffn_inner, eps=cfg.eps,
                                               qk_eps=cfg.eps), seed=0)
        stack = H3BlockStack([block.to("cuda", torch.bfloat16).eval()])
        params = fp32_params(block)  # the bf16 weights the GPU blocks use, in fp32
        install_transformer_fusions(stack)
        runtime = install_packed_ulysses(stack)
        runtime.begin_request()
        ref_stack, _, _ = bench.reference_stack(cfg, world)
        gh = torch.Generator().manual_seed(1)
        hidden = torch.randn(1, cfg.seq, cfg.dim, generator=gh).to(torch.bfloat16)
        idx = adaln_indices(cfg)
        cos, sin = rope_tables(positions(cfg), cfg.rotary_dim, cfg.theta)
        start, stop = split_bounds(cfg.seq, world, rank)
        args = (hidden[:, start:stop].contiguous().cuda(), None, idx[start:stop].cuda(),
                (cos[start:stop].cuda(), sin[start:stop].cuda()))
        with torch.no_grad():
            mine = stack(*args)[0].float().cpu().numpy()
            theirs = ref_stack(*args)[0].float().cpu().numpy()
        want = block_forward(params, hidden[0].float(), idx, cos, sin, heads=cfg.heads, head_dim=cfg.head_dim,
                             eps=cfg.eps, qk_eps=cfg.eps)[start:stop].numpy()
        half_ulp = np.ldexp(1.0, np.frexp(np.abs(want))[1] - 9)
        m_mine, m_ref = error_metrics(mine, want), error_metrics(theirs, want)
        stats = (float((np.abs(mine - want) - half_ulp).max()), m_mine["cosine"], m_mine["mean_abs"],
                 float((np.abs(theirs - want) - half_ulp).max()), m_ref["cosine"], m_ref["mean_abs"])
        exchange = runtime.provenance().get("exchange")
        if runtime.peer is not None:
            runtime.peer.close()
        queue.put((rank, True, (qkv_equal, out_equal, stats, exchange)))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException:  # noqa: BLE001
        queue.put((rank, False, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_packed_ulysses_against_the_reference_multi_gpu_path():
    sys.path.insert(0, str(ROOT))
    import bench

    if bench._reference_site() is None:
        pytest.skip("the reference package is not installed under baseline/_ref")
    import torch.multiprocessing as mp

    world = min(torch.cuda.device_count(), 8)
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in procs:
            rank, ok, payload = queue.get(timeout=600)
            assert ok, payload
            results[rank] = payload
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    for rank, (qkv_equal, out_equal, stats, exchange) in results.items():
        assert qkv_equal, f"rank {rank}: packed QKV exchange differs from the reference's"
        assert out_equal, f"rank {rank}: output exchange + merge differs from the reference's"
        excess, cosine, mean_abs, ref_excess, ref_cosine, ref_mean_abs = stats
        assert excess <= 2e-2 and cosine >= 0.9999, (rank, stats)
        assert ref_excess <= 2e-2 and ref_cosine >= 0.9999, (rank, stats)
        assert mean_abs <= 1.05 * ref_mean_abs, (rank, stats)
