"""The whole H3 transformer on the GPU, every installer of this package at once.

* one GPU: ``install_transformer_fusions`` + ``install_h3_invariant_caches`` vs
  the same model's eager forward (upstream-style math, torch SDPA attention),
  within the block tolerance, twice (the second call served from the caches);
* two GPUs (skipped otherwise): fusions + packed Ulysses (peer exchange) +
  rank-local I/O + caches, each rank's video/audio outputs vs the one-GPU fused
  result.
"""

from __future__ import annotations

import datetime
import os
import socket
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_EXCESS = 2e-2  # over half a bf16 spacing at the output's magnitude
COSINE = 0.9999


def _model(device="cuda"):
    from h3_flash_b200.runtime.h3_model import H3Transformer

    torch.manual_seed(0)
    model = H3Transformer(512, 4, 128, 1024, 2, text_dim=64, video_channels=32, audio_channels=16,
                          freq_dim=64, freqs_per_axis=16)
    with torch.no_grad():
        for name, p in model.named_parameters():
            if name.endswith("norm.weight") or name.endswith("norm1.weight") or name.endswith("norm2.weight") \
                    or "norm_q" in name or "norm_k" in name:
                p.copy_(1.0 + 0.02 * torch.randn_like(p))
            elif name.endswith("bias"):
                p.zero_()
            else:
                p.normal_(0.0, 0.02)
    return model.to(device, torch.bfloat16).eval()


def _inputs(model, device="cuda"):
    from h3_flash_b200.runtime.h3_model import make_inputs

    return make_inputs(model, n_text=16, n_video=512, n_audio=33, text_dim=64, grid=(2, 16, 16),
                       n_timesteps=1, seed=2, device=device, dtype=torch.bfloat16)


def _close(got, expect):
    diff = (got.float() - expect.float()).abs()
    half_ulp = expect.float().abs().clamp_min(2.0 ** -126) * 2.0 ** -9
    excess = float((diff - half_ulp).clamp_min(0).max())
    cosine = float(torch.nn.functional.cosine_similarity(got.float().flatten(), expect.float().flatten(), dim=0))
    return excess, cosine


def test_fused_cached_transformer_matches_eager():
    from h3_flash_b200 import _lib
    from h3_flash_b200.runtime.cache import install_h3_invariant_caches
    from h3_flash_b200.runtime.kernels import install_transformer_fusions

    model = _model()
    inputs = _inputs(model)
    with torch.no_grad():
        eager = model(**inputs, return_dict=False)
        install_transformer_fusions(model)
        runtime = install_h3_invariant_caches(model)
        fused = model(**inputs, return_dict=False)
        cached = model(**inputs, return_dict=False)
    torch.cuda.synchronize()
    for e, f, c in zip(eager, fused, cached):
        assert torch.isfinite(f).all()
        excess, cosine = _close(f, e)
        assert excess <= MAX_EXCESS and cosine >= COSINE, (excess, cosine)
        assert torch.equal(f, c)
    assert runtime.audit()["schedule_hits"] == 3
    assert _lib.device_status() == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, queue):
    try:
        os.environ["NCCL_NVLS_ENABLE"] = "0"
        torch.cuda.set_device(rank)
        import torch.distributed as dist

        dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
        from h3_flash_b200 import _lib
        from h3_flash_b200.runtime.cache import install_h3_invariant_caches
        from h3_flash_b200.runtime.kernels import install_transformer_fusions
        from h3_flash_b200.runtime.parallel import install_packed_ulysses, install_rank_local_io

        reference = _model()
        inputs = _inputs(reference)
        install_transformer_fusions(reference)
        with torch.no_grad():
            expect = reference(**inputs, return_dict=False)
        model = _model()
        install_transformer_fusions(model)
        ulysses = install_packed_ulysses(model, exchange="p2p")
        install_h3_invariant_caches(model)
        io = install_rank_local_io(model, group=dist.group.WORLD)
        results = []
        for _ in range(2):
            ulysses.begin_request()
            with torch.no_grad():
                got = model(**inputs, return_dict=False)
            results.append([_close(g, e) for g, e in zip(got, expect)])
        torch.cuda.synchronize()
        ok = all(x <= MAX_EXCESS and c >= COSINE for run in results for x, c in run)
        flags = torch.tensor([int(ok), int(_lib.device_status() == 0)], device="cuda")
        dist.all_reduce(flags, op=dist.ReduceOp.MIN)
        gate = io.gate["compact_output_gather"]["video"]["max_abs"]
        ulysses.peer.close()
        queue.put((rank, True, (flags.tolist(), results, gate, ulysses.attention_calls)))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException:  # noqa: BLE001
        queue.put((rank, False, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sequence_parallel_transformer_matches_single_gpu():
    import torch.multiprocessing as mp

    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = {}
    try:
        for _ in procs:
            rank, ok, payload = queue.get(timeout=300)
            assert ok, payload
            results[rank] = payload
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    flags, metrics, gate, calls = results[0]
    assert flags == [1, 1], metrics
    assert gate < 5e-2  # compact gather vs full gather + heads (GEMMs over fewer rows)
    assert calls == 4  # two blocks, two requests
