#!/usr/bin/env python3
"""Benchmark: one LOSSLESS packed-Ulysses DiT block forward at the 480p-5s shape.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl h3b|reference] [--config 480p-5s]
    torchrun --nproc-per-node N bench.py --gpus N ...          (N > 1: one rank per GPU, NCCL)

A step is one block forward over the whole joint sequence (S = 49,920 video + 1,280
audio tokens, d=3072, 24x128 heads, FFN 12,288 GELU-tanh, bf16), split into W
contiguous row shards (Ulysses SP=W; strong scaling: total work fixed). Inputs are
resident in HBM; each step is timed alone with CUDA events on the compute stream and
L2 is flushed (256 MiB written, then read back) between steps. ms_per_step is the max over ranks.

``e2e`` runs the step through the same public API as a serving loop. Every step copies
its hidden states from pinned host memory and its block output back, inside the timed
region. The copies run on two copy streams, double-buffered, so step i's copies overlap
the compute of steps i-1 and i+1. ``e2e_serial`` is the same without overlap: H2D, block,
D2H back to back for each step. For N>1 each rank first binds to the CPU cores that NVML
reports as local to its GPU, so that its pinned buffers sit on that NUMA node.
``roofline`` covers the dominant kernel (attention) from CUDA events
around its launches inside the timed steps. ``cpu_baseline`` times the CPU oracle
port of the reference path (two gloo ranks) on the benchmark CPU configuration.

``--impl reference`` times that CPU port as the reference arm (rank 0 only).

Other modes print their own line: ``--sweep elementwise`` (benchmark config 2),
``--exchange-bench`` (N>1: the exchange operations alone), ``--transformer-bench``
(the whole H3 transformer per request: invariant caches at N=1, rank-local I/O at N>1),
``--profile-kernel`` (one kernel for ncu captures).
"""

from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
METRIC = "DiT block fwd ms at S=49,920 (480p-5s) on 1/2/4/8 B200; a2a GB/s vs NVLink"
NVLINK_PEER_GBS = 770.0  # measured peer copy, GB/s per direction per GPU
L2_FLUSH_BYTES = 256 << 20


def _peaks() -> dict:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        data = json.loads(path.read_text())
        return {"hbm_gbs": data["hbm_gbs"], "bf16_tflops": data["bf16_tflops"],
                "bf16_tflops_sustained": data.get("bf16_tflops_sustained", data["bf16_tflops"]),
                "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


def _profile_traffic(hl: int, seq: int) -> float | None:
    """DRAM bytes per attention launch from the committed ncu summary, scaled from the
    captured case to this launch by heads (traffic is per (head, sequence) unit)."""

    path = ROOT / "profiles" / "attention_480p5s_sp8.md"
    if not path.exists():
        return None
    m = re.search(r"dram_bytes_per_launch:\s*([0-9.eE+]+)\s+at\s+hl=(\d+)\s+S=(\d+)", path.read_text())
    if not m:
        return None
    bytes_, cap_hl, cap_s = float(m.group(1)), int(m.group(2)), int(m.group(3))
    if cap_s != seq:
        return None
    return bytes_ * hl / cap_hl


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpus: list[int]) -> None:
        self.gpus = set(gpus)
        self.samples: list[tuple[float, float, list[str]]] = []
        self.proc = None
        self.thread = None

    def start(self) -> None:
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200"],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, FileNotFoundError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self) -> None:
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 8:
                continue
            try:
                index = int(parts[0])
                if index not in self.gpus:
                    continue
                sm, sm_max = float(parts[1]), float(parts[2])
            except ValueError:
                continue
            active = [name for name, value in zip(self.REASONS, parts[4:8]) if value.lower() == "active"]
            self.samples.append((sm, sm_max, active))

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        if self.thread is not None:
            self.thread.join(timeout=5)
        if not self.samples:
            return None
        loaded = [s for s in self.samples if s[0] > 0.5 * s[1]] or self.samples
        reasons = sorted({r for s in self.samples for r in s[2]})
        return {"sm_mhz": statistics.median(s[0] for s in loaded), "sm_max_mhz": max(s[1] for s in self.samples),
                "reasons": reasons, "samples": len(self.samples)}


# ---------------------------------------------------------------------------
# CPU reference port (oracle) — the cpu_baseline leg and the --impl reference arm
# ---------------------------------------------------------------------------


def cpu_reference_block(config: str, chunks: int, timed: int, warmup: int) -> dict:
    """The reference path's CPU restatement (the oracle's fp32 block at W=1, every host
    thread) on the bench's own workload.

    The sequence's query rows are cut into ``chunks`` contiguous chunks; one step runs one
    chunk through the whole block (``oracle.block_ref.block_forward_rows``: its own AdaLN,
    projections, QK-norm and RoPE, attention over all S keys, output projection, FFN).
    Keys and values of every row are projected once before the timed steps (untimed) so a
    chunk can attend over the full sequence; each timed chunk projects its own rows' keys
    and values again, so consecutive chunks do exactly the arithmetic of the full block.
    With ``timed == chunks`` the timed steps cover the sequence once and ``value`` is their
    summed time: one block forward, measured. With ``timed < chunks`` the first ``timed``
    chunks are a sample and ``value`` scales their sum by chunks / timed (row-linear)."""

    from h3_flash_b200.runtime.h3_block import H3TransformerBlock
    from h3_flash_b200.workloads import CONFIGS, adaln_indices, init_block_, positions, rope_tables
    from oracle.block_ref import block_forward_rows, fp32_params, project_kv

    cores = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    threads_before = torch.get_num_threads()
    torch.set_num_threads(cores)
    try:
        cfg = CONFIGS[config]
        block = init_block_(H3TransformerBlock(cfg.dim, cfg.heads, cfg.head_dim, cfg.ffn_inner), seed=0)
        params = fp32_params(block)
        del block
        g = torch.Generator().manual_seed(1)
        hidden = torch.randn(cfg.seq, cfg.dim, generator=g)
        idx = adaln_indices(cfg)
        cos, sin = rope_tables(positions(cfg), cfg.rotary_dim, cfg.theta)
        kw = dict(heads=cfg.heads, head_dim=cfg.head_dim, eps=cfg.eps, qk_eps=cfg.eps)
        k_all = torch.empty(cfg.seq, cfg.heads, cfg.head_dim)
        v_all = torch.empty_like(k_all)
        with torch.no_grad():
            for a in range(0, cfg.seq, 4096):
                b = min(a + 4096, cfg.seq)
                k_all[a:b], v_all[a:b] = project_kv(params, hidden[a:b], idx[a:b], cos[a:b], sin[a:b], **kw)
        bounds = [(cfg.seq * i // chunks, cfg.seq * (i + 1) // chunks) for i in range(chunks)]

        def run(a, b):
            block_forward_rows(params, hidden[a:b], idx[a:b], cos[a:b], sin[a:b], k_all, v_all, a, **kw)

        warm_rows = min(bounds[0][1], max(cfg.seq // 4, 1))  # first-touch of the chunk-sized buffers
        with torch.no_grad():
            for _ in range(warmup):
                run(0, warm_rows)
            step_s = []
            for a, b in bounds[:timed]:
                t0 = time.perf_counter()
                run(a, b)
                step_s.append(time.perf_counter() - t0)
    finally:
        torch.set_num_threads(threads_before)
    measured_ms = sum(step_s) * 1e3
    covered = sum(b - a for a, b in bounds[:timed])
    value = measured_ms * cfg.seq / covered
    if timed == chunks:
        sample = (f"the whole {cfg.name} block forward (S={cfg.seq}), measured: {chunks} timed steps each run "
                  f"{cfg.seq // chunks}-{-(-cfg.seq // chunks)} consecutive query rows through the full block "
                  f"(their own projections, attention over all S keys, FFN); value = the sum of the steps")
    else:
        sample = (f"{covered} of the {cfg.seq} query rows of the {cfg.name} block ({timed} of {chunks} row chunks, "
                  f"each through the full block with attention over all S keys), measured "
                  f"{measured_ms:.1f} ms, scaled by rows to the whole block")
    return {"value": value, "unit": "ms", "cores": cores, "kind": "port", "measured_ms": round(measured_ms, 2),
            "rows_measured": covered, "scaled": timed != chunks,
            "chunk_ms": [round(t * 1e3, 2) for t in step_s],
            "sample": "oracle fp32 restatement of the reference block (W=1, torch CPU ops on every host thread): "
                      + sample}


# ---------------------------------------------------------------------------
# The reference's own GPU block (its Triton kernels, NCCL all-to-alls, torch SDPA)
# ---------------------------------------------------------------------------


def _reference_site() -> Path | None:
    """Directory holding the unmodified reference package ``h3_flash``: the offline
    install under baseline/_ref, or $H3_FLASH_REFERENCE_SITE."""

    for candidate in (os.environ.get("H3_FLASH_REFERENCE_SITE"), ROOT / "baseline" / "_ref"):
        if candidate and (Path(candidate) / "h3_flash" / "runtime" / "kernels" / "fusions.py").exists():
            return Path(candidate)
    return None


def _diffusers_stand_in() -> str:
    """Registers the two Diffusers entry points the reference's installers import, when
    Diffusers itself is absent. ``dispatch_attention_fn`` keeps Diffusers' native backend
    semantics ([B, S, H, D] in and out, torch SDPA on the [B, H, S, D] views). The
    context-parallel hook pair is only called for a model that carries a
    context-parallel config, which the block stack here does not."""

    try:
        import diffusers  # noqa: F401

        return "diffusers"
    except ImportError:
        pass
    import types

    import torch.nn.functional as F

    def dispatch_attention_fn(query, key, value, attn_mask=None, dropout_p=0.0, is_causal=False, scale=None,
                              enable_gqa=False, backend=None, parallel_config=None):
        if backend is not None or parallel_config is not None:
            raise RuntimeError("the Diffusers stand-in dispatches the native backend only")
        out = F.scaled_dot_product_attention(query.permute(0, 2, 1, 3), key.permute(0, 2, 1, 3),
                                             value.permute(0, 2, 1, 3), attn_mask=attn_mask, dropout_p=dropout_p,
                                             is_causal=is_causal, scale=scale)
        return out.permute(0, 2, 1, 3)

    def _no_context_parallel(*args, **kwargs):
        raise RuntimeError("the Diffusers stand-in has no context-parallel hooks")

    from h3_flash_b200.runtime.h3_block import apply_rotary_emb

    names = ("diffusers", "diffusers.models", "diffusers.models.attention_dispatch",
             "diffusers.models.transformers", "diffusers.models.transformers.transformer_minimax_h3",
             "diffusers.hooks", "diffusers.hooks.context_parallel")
    modules = {name: types.ModuleType(name) for name in names}
    for name in names:
        if name != "diffusers" and not name.endswith(("attention_dispatch", "minimax_h3", "context_parallel")):
            modules[name].__path__ = []  # a package, so its submodules import
    modules["diffusers"].__path__ = []
    modules["diffusers.models.attention_dispatch"].dispatch_attention_fn = dispatch_attention_fn
    # the rotary the reference's first-block numerical gate compares against
    # (transformer.py:174-190); the rotate-half of the reference's own kernel
    modules["diffusers.models.transformers.transformer_minimax_h3"]._apply_rotary_emb = apply_rotary_emb
    modules["diffusers.hooks.context_parallel"].apply_context_parallel = _no_context_parallel
    modules["diffusers.hooks.context_parallel"].remove_context_parallel = _no_context_parallel
    for name in names[1:]:
        parent, _, child = name.rpartition(".")
        setattr(modules[parent], child, modules[name])
    sys.modules.update(modules)
    return "stand-in (native SDPA dispatch; rotate-half rotary for the first-block gate)"


def reference_stack(cfg, world: int, device: str = "cuda", dtype: torch.dtype = torch.bfloat16):
    """The block stack with the reference's own LOSSLESS installers applied: its Triton
    fusions (transformer.py:207-228; modulate and QK-norm+RoPE on, SwiGLU off for the
    GELU-tanh FFN, which stays eager) and, for world > 1, its packed Ulysses
    (packed_ulysses.py:131-220: Triton pack, NCCL all_to_all_single, torch SDPA, Triton
    merge). Returns (stack, runtime or None, provenance) or raises RuntimeError."""

    site = _reference_site()
    if site is None:
        raise RuntimeError("the reference package is not installed under baseline/_ref")
    if str(site) not in sys.path:
        sys.path.insert(0, str(site))
    dispatch = _diffusers_stand_in()
    import h3_flash
    from h3_flash.runtime.kernels.transformer import install_transformer_fusions as ref_fusions

    from h3_flash_b200.runtime.h3_block import H3BlockStack, H3TransformerBlock
    from h3_flash_b200.workloads import init_block_

    block = init_block_(H3TransformerBlock(cfg.dim, cfg.heads, cfg.head_dim, cfg.ffn_inner, eps=cfg.eps,
                                           qk_eps=cfg.eps), seed=0)
    stack = H3BlockStack([block.to(device=device, dtype=dtype).eval()])
    ref_fusions(stack, modulate=True, swiglu=False, qknorm_rope=True)
    runtime = None
    if world > 1:
        import torch.distributed as dist
        from h3_flash.runtime.parallel.packed_ulysses import install_packed_ulysses as ref_packed

        runtime = ref_packed(stack, group=dist.group.WORLD, fused_qknorm_rope=True)
        runtime.begin_request()
    provenance = {"package": str(Path(h3_flash.__file__).resolve().parent.relative_to(ROOT))
                  if Path(h3_flash.__file__).resolve().is_relative_to(ROOT) else h3_flash.__file__,
                  "diffusers": dispatch}
    return stack, runtime, provenance


def gpu_reference_block(cfg, hidden, idx, rotary, world: int, flush, steps: int) -> tuple[dict, torch.Tensor | None]:
    """Times the reference's LOSSLESS block (``reference_stack``) on this rank's rows,
    every rank taking part. Returns the JSON entry and this rank's output."""

    try:
        stack, runtime, provenance = reference_stack(cfg, world)
        with torch.no_grad():
            ms = _timed(lambda: stack(hidden, None, idx, rotary), steps, 3, flush)
            out = stack(hidden, None, idx, rotary)
        torch.cuda.synchronize()
    except (RuntimeError, ImportError) as error:
        torch.cuda.empty_cache()
        return {"unavailable": f"{type(error).__name__}: {str(error).splitlines()[0][:200]}"}, None
    entry = {"ms_per_step": round(_max_over_ranks(ms, world), 4), "steps": steps, "warmup": 3,
             "what": "the unmodified reference's LOSSLESS block: its Triton fused_rmsnorm_modulate, "
                     "fused_qknorm_rope and fused_residual_gate_rmsnorm_modulate"
                     + (", its packed-Ulysses exchange (Triton pack, NCCL all_to_all_single, Triton merge)"
                        if world > 1 else "")
                     + ", torch SDPA, torch Linears, eager GELU-tanh FFN; installed by its own "
                       "install_transformer_fusions" + (" and install_packed_ulysses" if world > 1 else "")
                     + " on this package's H3-style block stack; L2 flushed between steps",
             **provenance}
    if runtime is not None:
        entry["reference_provenance"] = runtime.provenance()
    del stack
    torch.cuda.empty_cache()
    return entry, out


def attention_ab(cfg, steps: int, flush) -> dict:
    """Attention alone, this package's kernel against torch SDPA, at the N=1 shape (all
    heads) and the SP8 per-rank shape (heads / 8) of the joint sequence, in one process
    under one clock record. SDPA gets the q/k/v views the reference hands it
    (packed_ulysses.py:201-208: [1, h, S, D] transposed views of the packed buffer);
    the h3b kernel reads the same packed buffer. FLOP = 4 S^2 h D."""

    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel

    from h3_flash_b200.runtime.attention.dense import packed_attention

    out = {}
    d = cfg.head_dim
    for label, heads in (("sp1", cfg.heads), ("sp8", cfg.heads // 8)):
        g = torch.Generator(device="cuda").manual_seed(0)
        packed = torch.randn(cfg.seq, heads, 3 * d, device="cuda", generator=g).to(torch.bfloat16)
        q, k, v = (t.transpose(0, 1).unsqueeze(0) for t in packed.split(d, dim=-1))
        flop = 4.0 * cfg.seq * cfg.seq * heads * d
        try:
            choice = SDPBackend(torch._fused_sdp_choice(q, k, v)).name
        except Exception as error:  # noqa: BLE001 - informational
            choice = f"unknown ({type(error).__name__})"
        entry = {"heads": heads, "seq": cfg.seq, "flop": flop, "sdpa_default_backend": choice}
        arms = {"h3b": lambda: packed_attention(packed, d),
                "sdpa_default": lambda: F.scaled_dot_product_attention(q, k, v)}
        for name, backend in (("sdpa_cudnn", SDPBackend.CUDNN_ATTENTION), ("sdpa_flash", SDPBackend.FLASH_ATTENTION)):
            def call(backend=backend):
                with sdpa_kernel(backend):
                    return F.scaled_dot_product_attention(q, k, v)
            arms[name] = call
        for name, fn in arms.items():
            try:
                ms = _timed(fn, steps, 3, flush)
            except RuntimeError as error:
                entry[name] = {"unavailable": str(error).splitlines()[0][:160]}
                continue
            entry[name] = {"ms": round(ms, 4), "tflops": round(flop / (ms * 1e-3) / 1e12, 1)}
        ref = F.scaled_dot_product_attention(q, k, v)[0].transpose(0, 1).float()
        mine = packed_attention(packed, d).float()
        delta = (mine - ref).abs()
        entry["h3b_vs_sdpa"] = {"max_abs": float(delta.max()),
                                "cosine": float(F.cosine_similarity(mine.flatten(), ref.flatten(), dim=0))}
        best_sdpa = min((entry[k]["ms"] for k in entry if k.startswith("sdpa_") and isinstance(entry[k], dict)
                         and "ms" in entry[k]), default=None)
        if best_sdpa and "ms" in entry.get("h3b", {}):
            entry["h3b_speedup_vs_best_sdpa"] = round(best_sdpa / entry["h3b"]["ms"], 4)
        out[label] = entry
        del packed, q, k, v, ref, mine
        torch.cuda.empty_cache()
    return out


# ---------------------------------------------------------------------------
# GPU block benchmark
# ---------------------------------------------------------------------------


def _bind_host_cores(local: int) -> str:
    """Pin this rank's host thread to the CPU cores NVML reports as local to its
    GPU, so pinned host buffers (first touched after this) sit on that NUMA node.
    Reads GPU topology only; changes nothing on the GPU."""

    try:
        import pynvml

        pynvml.nvmlInit()
        props = torch.cuda.get_device_properties(local)
        bus = f"{props.pci_domain_id:08x}:{props.pci_bus_id:02x}:{props.pci_device_id:02x}.0"
        handle = pynvml.nvmlDeviceGetHandleByPciBusId(bus.encode())
        words = (os.cpu_count() + 63) // 64
        masks = pynvml.nvmlDeviceGetCpuAffinity(handle, words)
        cores = {64 * w + b for w, mask in enumerate(masks) for b in range(64) if (mask >> b) & 1}
        cores &= set(range(os.cpu_count()))
        if cores:
            os.sched_setaffinity(0, cores)
            return f"{len(cores)} NUMA-local cores (NVML CPU affinity of {bus})"
    except Exception as error:  # noqa: BLE001 - topology is advisory
        return f"unbound ({type(error).__name__})"
    return "unbound (no affinity reported)"


def _dist_setup(n_gpus: int):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != n_gpus:
        raise SystemExit(f"--gpus {n_gpus} but WORLD_SIZE={world}: launch N>1 under torchrun")
    torch.cuda.set_device(local)
    if world > 1:
        import torch.distributed as dist

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device("cuda", local))
    return rank, world, local


def _barrier(world: int) -> None:
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def pipelined_e2e(step, hidden_host, flush, stream, steps: int, world: int) -> float:
    """ms per step of ``steps`` block forwards fed from and drained to pinned host
    memory the way a serving loop runs them: step i's input goes H2D on one copy
    stream while step i-1 computes, and its output goes D2H on another while
    step i+1 computes. Every step still moves its own input and output."""

    h2d = torch.cuda.Stream()
    d2h = torch.cuda.Stream()
    x_bufs = [torch.empty(hidden_host.shape, dtype=hidden_host.dtype, device="cuda") for _ in range(2)]
    out_bufs = [torch.empty_like(hidden_host).pin_memory() for _ in range(2)]
    loaded = [torch.cuda.Event() for _ in range(2)]
    consumed = [torch.cuda.Event() for _ in range(2)]
    _barrier(world)
    torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    start.record(h2d)
    with torch.cuda.stream(h2d):
        x_bufs[0].copy_(hidden_host, non_blocking=True)
        loaded[0].record(h2d)
    for i in range(steps):
        b = i % 2
        stream.wait_event(loaded[b])
        flush_l2(flush)
        y = step(x_bufs[b])
        consumed[b].record(stream)
        if i + 1 < steps:
            nb = (i + 1) % 2
            if i >= 1:
                h2d.wait_event(consumed[nb])  # step i-1 is done with that buffer
            with torch.cuda.stream(h2d):
                x_bufs[nb].copy_(hidden_host, non_blocking=True)
                loaded[nb].record(h2d)
        d2h.wait_event(consumed[b])
        with torch.cuda.stream(d2h):
            out_bufs[b].copy_(y, non_blocking=True)
        y.record_stream(d2h)
    d2h.wait_stream(h2d)
    end.record(d2h)
    torch.cuda.synchronize()
    _barrier(world)
    return start.elapsed_time(end) / steps


def _max_over_ranks(value: float, world: int) -> float:
    if world == 1:
        return value
    import torch.distributed as dist

    t = torch.tensor([value], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def _torch_ulysses_forward(attention, hidden_states, rotary_emb=None, attention_mask=None, *, group, counts):
    """Packed-Ulysses attention in the reference's structure (packed_ulysses.py:150-215)
    with torch ops in place of its Triton kernels: torch projections, RMSNorm and RoPE,
    the permute-copy pack, NCCL all-to-alls, torch SDPA, the permute merge."""

    import torch.distributed as dist
    import torch.nn.functional as F

    from h3_flash_b200.runtime.h3_block import apply_rotary_emb
    from h3_flash_b200.runtime.parallel.relayout import pack_qkv_reference

    world = dist.get_world_size(group)
    rows = hidden_states.shape[1]
    heads, head_dim = attention.heads, attention.head_dim
    hl = heads // world
    x = hidden_states[0]
    q = attention.norm_q(attention.to_q(x).view(rows, heads, head_dim))
    k = attention.norm_k(attention.to_k(x).view(rows, heads, head_dim))
    v = attention.to_v(x).view(rows, heads, head_dim)
    if rotary_emb is not None:
        q, k = apply_rotary_emb(q, *rotary_emb), apply_rotary_emb(k, *rotary_emb)
    send = pack_qkv_reference(q.contiguous(), k.contiguous(), v.contiguous(), world)
    total = sum(counts)
    block = hl * 3 * head_dim
    recv = torch.empty(total * block, dtype=send.dtype, device=send.device)
    dist.all_to_all_single(recv, send.reshape(-1), [c * block for c in counts], [rows * block] * world,
                           group=group)
    packed = recv.view(total, hl, 3 * head_dim)
    q, k, v = (packed[..., i * head_dim:(i + 1) * head_dim].permute(1, 0, 2).unsqueeze(0) for i in range(3))
    out = F.scaled_dot_product_attention(q, k, v)[0].permute(1, 0, 2).contiguous()  # [S, hl, D]
    block = hl * head_dim
    back = torch.empty(world * rows * block, dtype=out.dtype, device=out.device)
    dist.all_to_all_single(back, out.reshape(-1), [rows * block] * world, [c * block for c in counts],
                           group=group)
    merged = back.view(world, rows, hl, head_dim).permute(1, 0, 2, 3).reshape(1, rows, heads * head_dim)
    return attention.to_out[1](attention.to_out[0](merged))


def eager_sp_baseline(stack, hidden, idx, rotary, rows: int, world: int, flush, steps: int) -> dict:
    """The unfused block over N ranks with ``_torch_ulysses_forward`` as its attention
    (collective: every rank calls it). Restores the blocks' attention forwards after."""

    import torch.distributed as dist

    group = dist.group.WORLD
    counts_t = torch.zeros(world, dtype=torch.long, device="cuda")
    counts_t[dist.get_rank()] = rows
    dist.all_reduce(counts_t)
    counts = [int(c) for c in counts_t.tolist()]
    saved = []
    for block in stack.transformer_blocks:
        attention = block.attn
        saved.append((attention, attention.__dict__.get("forward")))

        def forward(hidden_states, rotary_emb=None, attention_mask=None, *, attention=attention):
            return _torch_ulysses_forward(attention, hidden_states, rotary_emb, attention_mask, group=group,
                                          counts=counts)

        attention.forward = forward
    try:
        with torch.no_grad():
            ms = _timed(lambda: stack(hidden, None, idx, rotary), steps, 3, flush)
    finally:
        for attention, original in saved:
            if original is None:
                del attention.forward
            else:
                attention.forward = original
    return {"ms_per_step": round(_max_over_ranks(ms, world), 4), "steps": steps, "warmup": 3,
            "what": "the block unfused over N ranks in the reference's packed-Ulysses structure, torch ops "
                    "in place of its Triton kernels: torch RMSNorm/RoPE/modulate/GELU, permute-copy pack, "
                    "NCCL all_to_all_single, torch SDPA, permute merge; L2 flushed between steps"}


def run_h3b(args) -> dict | None:
    from h3_flash_b200 import _lib
    from h3_flash_b200.runtime.h3_block import H3BlockStack, H3TransformerBlock
    from h3_flash_b200.runtime.kernels import install_transformer_fusions
    from h3_flash_b200.runtime.timing import TIMER
    from h3_flash_b200.workloads import CONFIGS, adaln_indices, init_block_, positions, rope_tables, split_bounds

    rank, world, local = _dist_setup(args.gpus)
    host_binding = _bind_host_cores(local) if world > 1 else "unbound (one rank)"
    cfg = CONFIGS[args.config]
    if cfg.heads % world:
        raise SystemExit(f"{cfg.heads} heads do not split over {world} ranks")
    torch.manual_seed(0)
    block = init_block_(H3TransformerBlock(cfg.dim, cfg.heads, cfg.head_dim, cfg.ffn_inner, eps=cfg.eps,
                                           qk_eps=cfg.eps), seed=0)
    block = block.to(device="cuda", dtype=torch.bfloat16).eval()
    stack = H3BlockStack([block])
    start, stop = split_bounds(cfg.seq, world, rank)
    rows = stop - start
    g = torch.Generator().manual_seed(1 + start)
    hidden_host = torch.randn(1, rows, cfg.dim, generator=g).to(torch.bfloat16).pin_memory()
    hidden = hidden_host.cuda()
    idx = adaln_indices(cfg)[start:stop].cuda()
    cos, sin = rope_tables(positions(cfg), cfg.rotary_dim, cfg.theta)
    rotary = (cos[start:stop].cuda(), sin[start:stop].cuda())
    out_host = torch.empty_like(hidden_host).pin_memory()
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream()

    # The reference's own LOSSLESS block on the same rows (every rank takes part).
    reference, reference_out = (None, None)
    if not args.no_reference_block:
        reference, reference_out = gpu_reference_block(cfg, hidden, idx, rotary, world, flush,
                                                       min(args.steps, 5))
    # The same block before any of this package's kernels are installed: torch ops,
    # torch SDPA and cuBLAS (N=1), or at N>1 (opt-in) the reference's packed-Ulysses
    # structure with torch ops in place of its Triton kernels.
    eager = None
    if world > 1 and args.eager_sp_baseline:
        eager = eager_sp_baseline(stack, hidden, idx, rotary, rows, world, flush, min(args.steps, 5))
        torch.cuda.empty_cache()
    if world == 1 and not args.no_eager_baseline:
        with torch.no_grad():
            eager_steps = min(args.steps, 5)
            eager_ms = _timed(lambda: stack(hidden, None, idx, rotary), eager_steps, 3, flush)
        eager = {"ms_per_step": round(eager_ms, 4), "steps": eager_steps, "warmup": 3,
                 "what": "the same block unfused: torch RMSNorm/RoPE/modulate/GELU ops, torch SDPA "
                         "attention, cuBLAS GEMMs; L2 flushed between steps"}
        torch.cuda.empty_cache()

    gemm_pack = not args.no_gemm_pack
    install_transformer_fusions(stack, gemm_epilogue=not args.no_gemm_epilogue, gemm_pack=gemm_pack)
    runtime = None
    if world > 1:
        from h3_flash_b200.runtime.parallel import install_packed_ulysses

        runtime = install_packed_ulysses(stack, exchange=args.exchange,
                                         fuse_output_exchange=args.output_exchange == "fused",
                                         gemm_pack=gemm_pack)
        runtime.begin_request()

    def step(x):
        with torch.no_grad():
            return stack(x, None, idx, rotary)

    for _ in range(args.warmup):
        step(hidden)
    torch.cuda.synchronize()

    sampler = ClockSampler(list(range(world))) if rank == 0 else None
    if sampler:
        sampler.start()
        time.sleep(0.3)
    # ---- device-resident timed steps ----
    _lib.reset_launch_count()
    TIMER.reset()
    TIMER.enabled = True
    events = []
    _barrier(world)
    torch.cuda.synchronize()
    for _ in range(args.steps):
        flush_l2(flush)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        step(hidden)
        e.record(stream)
        events.append((s, e))
    torch.cuda.synchronize()
    _barrier(world)
    TIMER.enabled = False
    launches = _lib.launch_count()
    step_ms = [s.elapsed_time(e) for s, e in events]
    sections = TIMER.milliseconds()
    # ---- end-to-end through the public API with host buffers, one step at a time ----
    e2e_events = []
    _barrier(world)
    torch.cuda.synchronize()
    for _ in range(args.steps):
        flush_l2(flush)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record(stream)
        x = hidden_host.to("cuda", non_blocking=True)
        y = step(x)
        out_host.copy_(y, non_blocking=True)
        e.record(stream)
        e2e_events.append((s, e))
    torch.cuda.synchronize()
    _barrier(world)
    e2e_ms = [s.elapsed_time(e) for s, e in e2e_events]
    # ---- end-to-end as a serving loop: the same per-step copies, overlapped ----
    e2e_pipelined_ms = pipelined_e2e(step, hidden_host, flush, stream, args.steps, world)
    clocks = sampler.stop() if sampler else None

    if reference_out is not None:
        import torch.nn.functional as F

        mine = step(hidden).float()
        delta = (mine - reference_out.float()).abs()
        stats = torch.tensor([float(delta.max()), float(F.cosine_similarity(
            mine.flatten(), reference_out.float().flatten(), dim=0))], dtype=torch.float64, device="cuda")
        if world > 1:
            import torch.distributed as dist

            stats[1] = -stats[1]
            dist.all_reduce(stats, op=dist.ReduceOp.MAX)
            stats[1] = -stats[1]
        reference["output_vs_h3b"] = {"max_abs": round(float(stats[0]), 6), "cosine": round(float(stats[1]), 7),
                                      "what": "this rank's block output against the reference block's on the "
                                              "same inputs and weights (worst rank)"}
        del mine, delta, reference_out
    if reference is not None and "ms_per_step" in reference:
        reference["h3b_speedup"] = round(reference["ms_per_step"] / _max_over_ranks(statistics.mean(step_ms), world), 4)
    side = {}
    if world == 8 and not args.no_side_lines and args.config == "480p-5s":
        side["block_768p_15s_sp8"] = sp_side_block(stack, runtime, "768p-15s", rank, world, min(args.steps, 3),
                                                   flush)
    if world == 1 and not args.no_side_lines:
        side["attention_ab"] = attention_ab(cfg, min(args.steps, 10), flush)
        side["gemm_ab"] = gemm_ab(cfg, min(args.steps, 10), flush)
        side["block_768p_5s_sp1"] = side_block(stack, "768p-5s", min(args.steps, 3), flush)
        side["elementwise_sweep"] = elementwise_sweep(argparse.Namespace(steps=min(args.steps, 10), warmup=3))
    status = _lib.device_status()
    if status:
        raise RuntimeError(f"h3b device status {status}: a kernel wait timed out")

    ms_mean = _max_over_ranks(statistics.mean(step_ms), world)
    e2e_mean = _max_over_ranks(statistics.mean(e2e_ms), world)
    e2e_pipelined = _max_over_ranks(e2e_pipelined_ms, world)
    attn_ms = statistics.mean(sections.get("attention", [float("nan")]))
    attn_ms_max = _max_over_ranks(attn_ms, world)
    hl = cfg.heads // world
    attn_flop = 4.0 * cfg.seq * cfg.seq * hl * cfg.head_dim
    peaks = _peaks()
    achieved = attn_flop / (attn_ms_max * 1e-3) / 1e12
    peak = peaks["bf16_tflops_sustained"]
    traffic = _profile_traffic(hl, cfg.seq)

    # secondary rooflines: elementwise HBM bytes, all-to-all bytes over NVLink
    r = rows
    d = cfg.dim
    ew_bytes = (2 * r * d * 2            # rmsnorm_modulate: read x, write
                + 4 * r * d * 2          # residual+rmsnorm+modulate: 2 reads, 2 writes
                + (2 * r * cfg.ffn_inner * 2 if args.no_gemm_epilogue else 0)  # GELU kernel: read, write
                + (3 * r * d * 2 if args.no_gemm_epilogue else 0)  # gated residual (else in the FFN GEMM)
                + (0 if gemm_pack else 2 * 3 * r * d * 2))  # qknorm+rope+pack: read qkv, write packed
    ew_keys = ("elementwise",) if gemm_pack else ("elementwise", "qknorm_rope_pack")
    ew_ms = sum(sum(v) / args.steps for k, v in sections.items() if k in ew_keys)
    ew_ms = _max_over_ranks(ew_ms, world)
    fused_output = world > 1 and args.exchange == "p2p" and args.output_exchange == "fused"
    per_row = r * d * 2 * (world - 1) / world if world > 1 else 0.0  # one [r, d] tensor sent
    a2a_keys = ["all_to_all"]
    covers = "QKV and output rows"
    a2a_bytes = 4 * per_row
    if world > 1 and args.exchange == "p2p":
        if gemm_pack and fused_output:
            a2a_bytes, covers = 0.0, ("barriers only: the QKV rows move inside the QKV GEMM kernel, "
                                      "the output rows inside the attention kernel")
        elif gemm_pack:
            a2a_bytes, covers = per_row, "output rows (scatter + barriers); the QKV rows move inside the QKV GEMM"
        else:
            a2a_keys.append("qknorm_rope_pack")  # the QKV exchange happens inside the pack kernel
            if fused_output:
                a2a_bytes, covers = 3 * per_row, ("QKV rows (pack kernel + barriers); the output rows "
                                                  "move inside the attention kernel")
    a2a_ms = _max_over_ranks(sum(sum(sections.get(k, [0.0])) for k in a2a_keys) / max(args.steps, 1), world)
    sections_total = {k: round(sum(v) / args.steps, 4) for k, v in sections.items()}
    # The exchange's own NVLink rate: with the default path the transfers run inside the
    # QKV GEMM and attention kernels, so time the same rows moved by the standalone peer
    # kernels (and by NCCL) on this rank's shape.
    exchange = None
    if world > 1 and not args.no_exchange_roofline:
        if runtime is not None and runtime.peer is not None:
            runtime.peer.close()
            runtime.peer = None
        torch.cuda.empty_cache()
        exchange = exchange_timings(args.config, rank, world, min(args.steps, 10), 3)

    if rank != 0:
        return None
    result = {
        "metric": METRIC,
        "value": round(ms_mean, 4),
        "unit": "ms",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": round(ms_mean, 4),
        "higher_is_better": False,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: seeded N(0,1) activations, N(0,0.02) weights, N(0,0.1) AdaLN tables, 3D RoPE tables",
        "config": {
            "workload": f"{cfg.name} DiT block forward, packed Ulysses SP{world}",
            "seq": cfg.seq, "video_tokens": cfg.video_tokens, "audio_tokens": cfg.audio_tokens,
            "dim": cfg.dim, "heads": cfg.heads, "head_dim": cfg.head_dim,
            "ffn": f"{cfg.ffn_inner} gelu-tanh" + ("" if args.no_gemm_epilogue else
                                                   " (h3b GEMM epilogues: GELU in the projection, the gated "
                                                   "residual in the output projection)"),
            "rotary_dim": cfg.rotary_dim, "rows_per_rank": rows, "heads_per_rank": hl,
            "parallelism": f"ulysses_sp{world}",
            "qkv_projection": ("h3b tcgen05 GEMM with QK-norm + RoPE + pack (+ QKV exchange at p2p) in its epilogue"
                               if gemm_pack else "cuBLAS GEMM, then the h3b QK-norm + RoPE + pack kernel"),
            "exchange": (args.exchange + (" (output exchange in the attention epilogue)" if fused_output else "")
                         if world > 1 else "none"), "l2": "flushed between timed steps (256 MiB write, then read back)",
        },
        "e2e": {"value": round(e2e_pipelined, 4), "unit": "ms",
                "h2d_bytes_per_step": hidden_host.numel() * hidden_host.element_size(),
                "d2h_bytes_per_step": out_host.numel() * out_host.element_size(),
                "mode": "serving loop: every step copies its input H2D from pinned host memory and "
                        "its output D2H on two copy streams, double-buffered, overlapping the "
                        "neighbouring steps' compute; one L2 flush per step inside the timed region; "
                        "total time of all steps / steps, max over ranks",
                "host_binding": host_binding},
        "e2e_serial": {"value": round(e2e_mean, 4), "unit": "ms",
                       "mode": "each step alone: H2D, block, D2H back to back on one stream"},
        "roofline": {
            "kernel": "h3b attention_fwd (tcgen05)" + (", output rows stored at their owners over NVLink"
                                                     if fused_output else ""),
            "bound": "tensor",
            "achieved": round(achieved, 2),
            "peak": peak,
            "unit": "TFLOP/s",
            "frac": round(achieved / peak, 4),
            "peak_note": "sustained cuBLAS bf16 of measured (kernel timed inside the block step)"
            if peaks["source"] == "measured" else "fallback",
            "frac_of_burst": round(achieved / peaks["bf16_tflops"], 4),
            "traffic": traffic,
            "traffic_source": ("DRAM bytes per launch from the committed ncu capture "
                               "(profiles/attention_480p5s_sp8.md) scaled by heads; not measured in this run")
            if traffic is not None else None,
            "flop_per_launch": attn_flop,
            "ms_per_launch": round(attn_ms_max, 4),
        },
        "rooflines": {
            "elementwise_hbm": {"bytes_per_step": ew_bytes, "ms": round(ew_ms, 4),
                                "achieved_gbs": round(ew_bytes / (ew_ms * 1e-3) / 1e9, 1) if ew_ms else None,
                                "peak_gbs": peaks["hbm_gbs"],
                                "frac": round(ew_bytes / (ew_ms * 1e-3) / 1e9 / peaks["hbm_gbs"], 4)
                                if ew_ms else None},
            "all_to_all_nvlink": {"bytes_sent_per_gpu": a2a_bytes, "ms": round(a2a_ms, 4),
                                  "achieved_gbs": round(a2a_bytes / (a2a_ms * 1e-3) / 1e9, 1)
                                  if a2a_ms and a2a_bytes else None,
                                  "peak_gbs": NVLINK_PEER_GBS, "nominal_gbs": 900.0,
                                  "peak_note": "measured peer copy per direction on this pool",
                                  "covers": covers,
                                  "frac": round(a2a_bytes / (a2a_ms * 1e-3) / 1e9 / NVLINK_PEER_GBS, 4)
                                  if a2a_ms and a2a_bytes else None},
        },
        "exchange_standalone": exchange,
        "sections_ms_per_step": sections_total,
        "gpu_reference_block": reference,
        "gpu_eager_baseline": eager,
        **side,
        "gpu_launches": launches,
        "clocks": clocks,
    }
    if exchange is not None:
        ms = exchange["ms"]
        moving = (ms["pack_p2p_and_barrier"] - ms["barrier"]) + (ms["scatter_p2p_and_barrier"] - ms["barrier"])
        sent = (exchange["remote_mb_per_rank"]["qkv"] + exchange["remote_mb_per_rank"]["output"]) * 1e6
        gbs = sent / (moving * 1e-3) / 1e9 if moving > 0 else None
        result["rooflines"]["all_to_all_nvlink"]["standalone"] = {
            "what": "the QKV rows (pack kernel storing at the owners) and the output rows (scatter kernel) "
                    "of one block moved by the standalone peer kernels, barrier time excluded; the default "
                    "path moves the same rows inside the QKV GEMM and attention kernels",
            "bytes_sent_per_gpu": sent, "ms": round(moving, 4),
            "achieved_gbs": round(gbs, 1) if gbs else None,
            "frac_of_measured_peer_copy": round(gbs / NVLINK_PEER_GBS, 4) if gbs else None,
            "frac_of_900_nominal": round(gbs / 900.0, 4) if gbs else None,
            "nccl_all_to_all_ms": {"qkv": ms["nccl_qkv_all_to_all"],
                                   "output_and_merge": ms["nccl_output_all_to_all_and_merge"]},
        }
    return result


def gemm_ab(cfg, steps: int, flush) -> dict:
    """The block's GEMMs at the N=1 shape (S rows), this package's tcgen05 GEMM with its
    fused epilogue against cuBLAS (and cuBLASLt's bias+GELU epilogue for the FFN
    projection), in one process. TFLOP/s = 2 S K N / time."""

    import torch.nn.functional as F

    from h3_flash_b200.runtime.kernels.fusions import fused_linear, fused_qkv_gemm_pack

    g = torch.Generator(device="cuda").manual_seed(0)
    s, d, f = cfg.seq, cfg.dim, cfg.ffn_inner
    rnd = lambda *shape, std=1.0: (torch.randn(*shape, device="cuda", generator=g) * std).to(torch.bfloat16)  # noqa: E731
    x, h = rnd(s, d), rnd(s, f)
    out = {}

    def entry(name, k, n, arms):
        flop = 2.0 * s * k * n
        row = {"shape": f"[{s}, {k}] x [{k}, {n}]"}
        for arm, fn in arms.items():
            ms = _timed(fn, steps, 3, flush)
            row[arm] = {"ms": round(ms, 4), "tflops": round(flop / (ms * 1e-3) / 1e12, 1)}
        out[name] = row

    w_qkv, b_qkv = rnd(3 * d, d, std=0.02), rnd(3 * d, std=0.02)
    norm_w = torch.ones(cfg.head_dim, device="cuda", dtype=torch.bfloat16)
    from h3_flash_b200.workloads import positions, rope_tables

    cos, sin = (t.cuda() for t in rope_tables(positions(cfg), cfg.rotary_dim, cfg.theta))
    send = torch.empty((1, s, cfg.heads, 3 * cfg.head_dim), device="cuda", dtype=torch.bfloat16)
    entry("qkv_projection", d, 3 * d, {
        "h3b_gemm_qknorm_rope_pack": lambda: fused_qkv_gemm_pack(x, w_qkv, b_qkv, norm_w, norm_w, cos, sin,
                                                                  cfg.heads, 1, cfg.eps, cfg.eps, out=send),
        "cublas_linear": lambda: F.linear(x, w_qkv, b_qkv)})
    w_up, b_up = rnd(f, d, std=0.02), rnd(f, std=0.02)
    up_out = torch.empty((s, f), device="cuda", dtype=torch.bfloat16)
    entry("ffn_up_gelu_tanh", d, f, {
        "h3b_gemm_gelu_epilogue": lambda: fused_linear(x, w_up, b_up, "gelu-tanh", out=up_out),
        "cublaslt_gelu_epilogue": lambda: torch._addmm_activation(b_up, x, w_up.t(), use_gelu=True),
        "cublas_linear_then_torch_gelu": lambda: F.gelu(F.linear(x, w_up, b_up), approximate="tanh")})
    w_down, b_down = rnd(d, f, std=0.02), rnd(d, std=0.02)
    down_out = torch.empty((s, d), device="cuda", dtype=torch.bfloat16)
    entry("ffn_down", f, d, {"h3b_gemm": lambda: fused_linear(h, w_down, b_down, out=down_out),
                             "cublas_linear": lambda: F.linear(h, w_down, b_down)})
    w_o, b_o = rnd(d, d, std=0.02), rnd(d, std=0.02)
    entry("attention_out", d, d, {"h3b_gemm": lambda: fused_linear(x, w_o, b_o, out=down_out),
                                  "cublas_linear": lambda: F.linear(x, w_o, b_o)})
    del x, h, send, up_out
    torch.cuda.empty_cache()
    return out


def side_block(stack, config: str, steps: int, flush) -> dict:
    """The installed (fused) block stack at another benchmark shape on one GPU: ms per
    block forward and the in-step attention rate. Inputs seeded like the main line."""

    from h3_flash_b200.runtime.timing import TIMER
    from h3_flash_b200.workloads import CONFIGS, adaln_indices, positions, rope_tables

    cfg = CONFIGS[config]
    g = torch.Generator().manual_seed(1)
    hidden = torch.randn(1, cfg.seq, cfg.dim, generator=g).to(torch.bfloat16).cuda()
    idx = adaln_indices(cfg).cuda()
    cos, sin = rope_tables(positions(cfg), cfg.rotary_dim, cfg.theta)
    rotary = (cos.cuda(), sin.cuda())
    with torch.no_grad():
        for _ in range(2):
            stack(hidden, None, idx, rotary)
        TIMER.reset()
        TIMER.enabled = True
        ms = _timed(lambda: stack(hidden, None, idx, rotary), steps, 0, flush)
        TIMER.enabled = False
    attn = statistics.mean(TIMER.milliseconds().get("attention", [float("nan")]))
    flop = 4.0 * cfg.seq * cfg.seq * cfg.heads * cfg.head_dim
    del hidden
    torch.cuda.empty_cache()
    return {"config": f"{cfg.name}: S={cfg.seq} ({cfg.video_tokens} video + {cfg.audio_tokens} audio), SP1",
            "ms_per_step": round(ms, 3), "steps": steps, "attention_ms": round(attn, 3),
            "attention_tflops": round(flop / (attn * 1e-3) / 1e12, 1)}


def sp_side_block(stack, runtime, config: str, rank: int, world: int, steps: int, flush) -> dict:
    """The installed packed-Ulysses block stack at another benchmark shape over the same
    ranks (every rank calls it; a new request, so the row counts are exchanged again):
    ms per block forward (max over ranks) and the in-step attention rate."""

    from h3_flash_b200.runtime.timing import TIMER
    from h3_flash_b200.workloads import CONFIGS, adaln_indices, positions, rope_tables, split_bounds

    cfg = CONFIGS[config]
    start, stop = split_bounds(cfg.seq, world, rank)
    g = torch.Generator().manual_seed(1 + start)
    hidden = torch.randn(1, stop - start, cfg.dim, generator=g).to(torch.bfloat16).cuda()
    idx = adaln_indices(cfg)[start:stop].cuda()
    cos, sin = rope_tables(positions(cfg), cfg.rotary_dim, cfg.theta)
    rotary = (cos[start:stop].cuda(), sin[start:stop].cuda())

    def step():
        with torch.no_grad():
            return stack(hidden, None, idx, rotary)

    runtime.begin_request()  # new row counts (and, p2p, buffers sized for them)
    for _ in range(2):
        step()
    TIMER.reset()
    TIMER.enabled = True
    ms = _timed(step, steps, 0, flush)
    TIMER.enabled = False
    attn = statistics.mean(TIMER.milliseconds().get("attention", [float("nan")]))
    flop = 4.0 * cfg.seq * cfg.seq * (cfg.heads // world) * cfg.head_dim
    del hidden
    torch.cuda.empty_cache()
    return {"config": f"{cfg.name}: S={cfg.seq} ({cfg.video_tokens} video + {cfg.audio_tokens} audio), SP{world}",
            "ms_per_step": round(_max_over_ranks(ms, world), 3), "steps": steps,
            "attention_ms": round(_max_over_ranks(attn, world), 3),
            "attention_tflops_per_gpu": round(flop / (_max_over_ranks(attn, world) * 1e-3) / 1e12, 1)}


def flush_l2(buf: torch.Tensor) -> None:
    """Evict L2 between timed steps: write a buffer larger than L2, then read it back so
    the dirty lines are written to DRAM here rather than inside the next timed step."""

    buf.fill_(1)
    buf.view(torch.int64).sum()


def _timed(fn, steps: int, warmup: int, flush: torch.Tensor) -> float:
    """Mean device ms of fn() over ``steps`` launches, L2 flushed before each."""

    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    events = []
    for _ in range(steps):
        flush_l2(flush)
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        events.append((s, e))
    torch.cuda.synchronize()
    return statistics.mean(s.elapsed_time(e) for s, e in events)


def elementwise_sweep(args) -> dict:
    """Benchmark config 2: each fused elementwise kernel at the 1xB200 sweep shapes;
    achieved GB/s = algorithmic bytes (each input read once, each output written once)
    / CUDA-event time, L2 flushed between launches."""

    from h3_flash_b200.runtime.kernels import fusions as F
    from h3_flash_b200.workloads import CONFIGS, positions, rope_tables

    torch.cuda.set_device(0)
    cfg = CONFIGS["480p-5s"]
    s, d = cfg.video_tokens, cfg.dim  # [1, 49920, 3072]
    g = torch.Generator(device="cuda").manual_seed(0)
    rnd = lambda *shape, std=1.0, mean=0.0: (torch.randn(*shape, device="cuda", generator=g) * std + mean).to(  # noqa: E731
        torch.bfloat16)
    x, br = rnd(1, s, d), rnd(1, s, d)
    scale_v, shift_v, gate_v = rnd(d, std=0.1), rnd(d, std=0.1), rnd(d, std=0.1)  # benchmark [d] vectors
    table = rnd(3, 6 * d, std=0.1)
    t = table.chunk(6, -1)
    idx = torch.ones(s, dtype=torch.long, device="cuda")
    w = rnd(d, std=0.02, mean=1.0)
    qk = rnd(1, s, cfg.heads, cfg.head_dim)
    qkw = rnd(cfg.head_dim, std=0.02, mean=1.0)
    cos, sin = (z[:s].cuda() for z in rope_tables(positions(cfg), 96))
    hidden = rnd(s, cfg.ffn_inner)
    qkv = rnd(s, 3 * d)
    q3, k3, v3 = (z.view(s, cfg.heads, cfg.head_dim) for z in qkv.split(d, -1))
    flush = torch.empty(L2_FLUSH_BYTES, dtype=torch.uint8, device="cuda")
    e = s * d * 2  # bytes of one [1, S, d] bf16 tensor
    peaks = _peaks()
    cases = {
        "modulate": (lambda: F.fused_modulate(x, scale_v, shift_v), 2 * e),
        "gated_residual": (lambda: F.fused_gated_residual(x, br, gate_v), 3 * e),
        "rmsnorm_modulate": (lambda: F.fused_rmsnorm_modulate(x, w, t[1], t[0], idx, 1e-6), 2 * e),
        "residual_gate_rmsnorm_modulate": (
            lambda: F.fused_residual_gate_rmsnorm_modulate(x, br, t[2], w, t[4], t[3], idx, 1e-6), 4 * e),
        "qknorm_rope_rot96": (lambda: F.fused_qknorm_rope(qk, qkw, cos, sin, 1e-6), 2 * e + 2 * s * 96 * 4),
        "qknorm_rope_pack_w8": (lambda: F.fused_qknorm_rope_pack(q3, k3, v3, qkw, qkw, cos, sin, 8, 1e-6, 1e-6),
                                6 * e + 2 * s * 96 * 4),
        "gelu_tanh_ffn": (lambda: F.fused_gelu_tanh(hidden), 2 * s * cfg.ffn_inner * 2),
    }
    out = {}
    for name, (fn, nbytes) in cases.items():
        ms = _timed(fn, args.steps, args.warmup, flush)
        gbs = nbytes / (ms * 1e-3) / 1e9
        out[name] = {"ms": round(ms, 4), "bytes": nbytes, "gbs": round(gbs, 1),
                     "frac_of_measured_hbm": round(gbs / peaks["hbm_gbs"], 4),
                     "frac_of_8tbs_nominal": round(gbs / 8000.0, 4)}
    return {"sweep": "elementwise", "shape": f"[1,{s},{d}] / [1,{s},24,128] / FFN [{s},{cfg.ffn_inner}]",
            "hbm_peak_gbs": peaks["hbm_gbs"], "kernels": out}


def profile_kernel(args) -> None:
    """Launch one kernel family a few times for an ncu capture (no JSON contract)."""

    from h3_flash_b200.runtime.attention.dense import packed_attention

    torch.cuda.set_device(0)
    from h3_flash_b200.workloads import CONFIGS

    cfg = CONFIGS[args.config]
    if args.profile_kernel == "attention":
        g = torch.Generator(device="cuda").manual_seed(0)
        packed = torch.randn(cfg.seq, args.heads_per_rank, 3 * cfg.head_dim, device="cuda",
                             generator=g).to(torch.bfloat16)
        for _ in range(args.warmup + args.steps):
            packed_attention(packed, cfg.head_dim)
    elif args.profile_kernel == "elementwise":
        args.steps, args.warmup = max(args.steps, 1), max(args.warmup, 0)
        elementwise_sweep(args)
    elif args.profile_kernel == "qkv_gemm":
        # One rank's QKV projection with the pack epilogue at the SP layout given by
        # --heads-per-rank (3: the SP8 shape, 6400 rows): x 39 MB, W 57 MB, out 118 MB.
        from h3_flash_b200.runtime.kernels.fusions import fused_qkv_gemm_pack
        from h3_flash_b200.workloads import positions, rope_tables

        world = cfg.heads // args.heads_per_rank
        rows = cfg.seq // world
        g = torch.Generator(device="cuda").manual_seed(0)
        x = torch.randn(rows, cfg.dim, device="cuda", generator=g).to(torch.bfloat16)
        w = (0.02 * torch.randn(3 * cfg.heads * cfg.head_dim, cfg.dim, device="cuda", generator=g)).to(torch.bfloat16)
        b = (0.02 * torch.randn(3 * cfg.heads * cfg.head_dim, device="cuda", generator=g)).to(torch.bfloat16)
        norm = torch.ones(cfg.head_dim, device="cuda", dtype=torch.bfloat16)
        cos, sin = (t[:rows].cuda() for t in rope_tables(positions(cfg), cfg.rotary_dim, cfg.theta))
        out = torch.empty((world, rows, args.heads_per_rank, 3 * cfg.head_dim), device="cuda", dtype=torch.bfloat16)
        for _ in range(args.warmup + args.steps):
            fused_qkv_gemm_pack(x, w, b, norm, norm, cos, sin, cfg.heads, world, cfg.eps, cfg.eps, out=out)
    elif args.profile_kernel == "gemm_gated":
        # The FFN output projection with the closing gated residual in the epilogue,
        # one rank's rows at the SP layout given by --heads-per-rank (24: the N=1 shape):
        # x [rows, 12288], W [3072, 12288], residual and output [rows, 3072].
        from h3_flash_b200.runtime.kernels.fusions import fused_linear_gated_residual

        world = cfg.heads // args.heads_per_rank
        rows = cfg.seq // world
        g = torch.Generator(device="cuda").manual_seed(0)
        x = torch.randn(rows, cfg.ffn_inner, device="cuda", generator=g).to(torch.bfloat16)
        w = (0.02 * torch.randn(cfg.dim, cfg.ffn_inner, device="cuda", generator=g)).to(torch.bfloat16)
        b = (0.02 * torch.randn(cfg.dim, device="cuda", generator=g)).to(torch.bfloat16)
        res = torch.randn(rows, cfg.dim, device="cuda", generator=g).to(torch.bfloat16)
        gate = (0.1 * torch.randn(3, cfg.dim, device="cuda", generator=g)).to(torch.bfloat16)
        idx = torch.arange(rows, device="cuda") % 3
        out = torch.empty((rows, cfg.dim), device="cuda", dtype=torch.bfloat16)
        for _ in range(args.warmup + args.steps):
            fused_linear_gated_residual(x, w, b, res, gate, idx, out=out)
    elif args.profile_kernel == "gemm_gelu":
        # The FFN projection with GELU-tanh in the GEMM epilogue, one rank's rows at
        # the SP layout given by --heads-per-rank (24: the N=1 shape).
        from h3_flash_b200.runtime.kernels.fusions import fused_linear

        world = cfg.heads // args.heads_per_rank
        rows = cfg.seq // world
        g = torch.Generator(device="cuda").manual_seed(0)
        x = torch.randn(rows, cfg.dim, device="cuda", generator=g).to(torch.bfloat16)
        w = (0.02 * torch.randn(cfg.ffn_inner, cfg.dim, device="cuda", generator=g)).to(torch.bfloat16)
        b = (0.02 * torch.randn(cfg.ffn_inner, device="cuda", generator=g)).to(torch.bfloat16)
        out = torch.empty((rows, cfg.ffn_inner), device="cuda", dtype=torch.bfloat16)
        for _ in range(args.warmup + args.steps):
            fused_linear(x, w, b, "gelu-tanh", out=out)
    torch.cuda.synchronize()
    from h3_flash_b200 import _lib

    if _lib.device_status():
        raise RuntimeError("h3b device status set")
    print(f"profile-kernel {args.profile_kernel} done")


def exchange_bench(args) -> dict | None:
    """Per-operation timing of the packed-Ulysses row exchange at the config's shape
    (N>1 under torchrun): the peer-store path (pack to the owners, barrier, scatter)
    against NCCL all-to-all of the same rows. CUDA events, max over ranks."""

    rank, world, _ = _dist_setup(args.gpus)
    if world < 2:
        raise SystemExit("--exchange-bench needs N>1 (launch under torchrun)")
    return exchange_timings(args.config, rank, world, args.steps, args.warmup)


def exchange_timings(config: str, rank: int, world: int, steps: int, warmup: int) -> dict | None:
    """The exchange operations of one block at ``config``'s shape on this rank's rows
    (every rank calls it): collective, returns rank 0's line."""

    import torch.distributed as dist

    from h3_flash_b200.runtime.kernels.fusions import fused_qknorm_rope_pack
    from h3_flash_b200.runtime.parallel.packed_ulysses import (
        PackedUlyssesRuntime,
        _packed_output_all_to_all,
        packed_qkv_exchange,
    )
    from h3_flash_b200.runtime.parallel.peer_exchange import PeerExchange
    from h3_flash_b200.workloads import CONFIGS, split_sizes

    cfg = CONFIGS[config]
    heads, dim = cfg.heads, cfg.head_dim
    counts = split_sizes(cfg.seq, world)
    rows = counts[rank]
    g = torch.Generator(device="cuda").manual_seed(rank)
    qkv = torch.randn(rows, 3 * heads * dim, device="cuda", generator=g).to(torch.bfloat16)
    q, k, v = (qkv[:, i * heads * dim:(i + 1) * heads * dim].view(rows, heads, dim) for i in range(3))
    weight = torch.ones(dim, device="cuda", dtype=torch.bfloat16)
    cos = torch.rand(rows, cfg.rotary_dim, device="cuda", generator=g)
    sin = torch.rand(rows, cfg.rotary_dim, device="cuda", generator=g)
    out = torch.randn(cfg.seq, heads // world, dim, device="cuda", generator=g).to(torch.bfloat16)
    peer = PeerExchange(dist.group.WORLD)
    runtime = PackedUlyssesRuntime(dist.group.WORLD)
    runtime.begin_request()
    runtime.row_counts(rows)
    send = fused_qknorm_rope_pack(q, k, v, weight, weight, cos, sin, world, cfg.eps, cfg.eps)

    def timed(fn) -> float:
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        dist.barrier()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        for _ in range(steps):
            fn()
        end.record()
        torch.cuda.synchronize()
        return _max_over_ranks(start.elapsed_time(end) / steps, world)

    def pack_p2p():
        peer.pack(q, k, v, weight, weight, cos, sin, cfg.eps, cfg.eps, counts)
        peer.barrier()

    def scatter_p2p():
        peer.scatter(out, counts)
        peer.barrier()

    ms = {
        "pack_p2p_and_barrier": timed(pack_p2p),
        "barrier": timed(peer.barrier),
        "scatter_p2p_and_barrier": timed(scatter_p2p),
        "pack_local": timed(lambda: fused_qknorm_rope_pack(q, k, v, weight, weight, cos, sin, world,
                                                           cfg.eps, cfg.eps)),
        "nccl_qkv_all_to_all": timed(lambda: packed_qkv_exchange(send, rows, runtime)),
        "nccl_output_all_to_all_and_merge": timed(lambda: _packed_output_all_to_all(out, rows, runtime)),
    }
    qkv_remote = max(counts) * heads * 3 * dim * 2 * (world - 1) / world
    out_remote = cfg.seq * (heads // world) * dim * 2 * (world - 1) / world
    peer.close()
    del send, out, qkv
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    return {
        "exchange_bench": cfg.name, "n_gpus": world, "steps": steps,
        "ms": {key: round(value, 4) for key, value in ms.items()},
        "remote_mb_per_rank": {"qkv": round(qkv_remote / 1e6, 2), "output": round(out_remote / 1e6, 2)},
        "peer_gbs": {
            "pack": round(qkv_remote / ((ms["pack_p2p_and_barrier"] - ms["barrier"]) * 1e-3) / 1e9, 1),
            "scatter": round(out_remote / ((ms["scatter_p2p_and_barrier"] - ms["barrier"]) * 1e-3) / 1e9, 1),
            "peak_measured_peer_copy": NVLINK_PEER_GBS,
        },
    }


def transformer_bench(args) -> dict | None:
    """The whole H3 transformer forward per request (text/timestep embedders, ``--layers``
    blocks, output norm and projections) on the 480p-5s sequence plus 128 text tokens,
    which times the request-level mechanisms. At N=1: the fused model, then the same model
    with the invariant caches (f2) on a repeated timestep. At N>1: packed Ulysses + caches
    with rank-local inputs and the compact output gather (f1), against every rank
    projecting all inputs and gathering all outputs. CUDA events, max over ranks."""

    import torch.distributed as dist

    from h3_flash_b200.runtime.cache import install_h3_invariant_caches
    from h3_flash_b200.runtime.h3_model import H3Transformer, make_inputs
    from h3_flash_b200.runtime.kernels import install_transformer_fusions
    from h3_flash_b200.workloads import CONFIGS

    rank, world, _ = _dist_setup(args.gpus)
    cfg = CONFIGS[args.config]
    text_dim, video_channels, audio_channels, n_text = 4096, 64, 64, 128

    def build():
        torch.manual_seed(0)
        model = H3Transformer(cfg.dim, cfg.heads, cfg.head_dim, cfg.ffn_inner, args.layers, text_dim=text_dim,
                              video_channels=video_channels, audio_channels=audio_channels,
                              freq_dim=256, freqs_per_axis=16)
        with torch.no_grad():
            for name, param in model.named_parameters():
                if name.endswith(("norm.weight", "norm1.weight", "norm2.weight")) or "norm_q" in name \
                        or "norm_k" in name:
                    param.fill_(1.0)
                elif name.endswith("bias"):
                    param.zero_()
                else:
                    param.normal_(0.0, 0.02)
        return model.to("cuda", torch.bfloat16).eval()

    probe = build()
    inputs = make_inputs(probe, n_text=n_text, n_video=cfg.video_tokens, n_audio=cfg.audio_tokens,
                         text_dim=text_dim, grid=cfg.video_grid, n_timesteps=1, seed=1, device="cuda",
                         dtype=torch.bfloat16)
    del probe

    def timed(model, begin) -> float:
        for _ in range(args.warmup):
            begin()
            with torch.no_grad():
                model(**inputs, return_dict=False)
        torch.cuda.synchronize()
        _barrier(world)
        events = []
        for _ in range(args.steps):
            begin()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            with torch.no_grad():
                model(**inputs, return_dict=False)
            end.record()
            events.append((start, end))
        torch.cuda.synchronize()
        _barrier(world)
        return _max_over_ranks(statistics.mean(s.elapsed_time(e) for s, e in events), world)

    results = {}
    if world == 1:
        model = build()
        install_transformer_fusions(model)
        results["fused_ms"] = round(timed(model, lambda: None), 3)
        caches = install_h3_invariant_caches(model)
        results["fused_cached_ms"] = round(timed(model, caches.begin_request), 3)
        results["cache_audit"] = caches.audit()
    else:
        from h3_flash_b200.runtime.parallel import install_packed_ulysses, install_rank_local_io

        for name, (local_inputs, compact) in (("rank_local_io_ms", (True, True)), ("full_io_ms", (False, False))):
            model = build()
            install_transformer_fusions(model)
            ulysses = install_packed_ulysses(model, exchange=args.exchange)
            caches = install_h3_invariant_caches(model)
            install_rank_local_io(model, group=dist.group.WORLD, rank_local_inputs=local_inputs,
                                  compact_output_gather=compact)

            def begin(ulysses=ulysses, caches=caches):
                ulysses.begin_request()
                caches.begin_request()

            results[name] = round(timed(model, begin), 3)
            if ulysses.peer is not None:
                ulysses.peer.close()
            del model
            torch.cuda.empty_cache()
    if rank != 0:
        return None
    return {"transformer_bench": {"config": cfg.name, "layers": args.layers, "n_gpus": world,
                                  "tokens": {"text": n_text, "video": cfg.video_tokens, "audio": cfg.audio_tokens},
                                  "steps": args.steps, "warmup": args.warmup, **results}}


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__.splitlines()[1])
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=10)
    parser.add_argument("--warmup", type=int, default=3)
    parser.add_argument("--impl", choices=["h3b", "reference"], default="h3b")
    parser.add_argument("--config", default="480p-5s")
    parser.add_argument("--output-exchange", choices=["fused", "scatter"], default="fused",
                        help="p2p: attention stores its output rows at their owners (fused) or a "
                             "scatter kernel moves them after attention")
    parser.add_argument("--exchange", choices=["nccl", "p2p"], default="p2p",
                        help="packed-Ulysses row exchange for N>1: NCCL all-to-all or NVLink peer stores")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-gemm-epilogue", action="store_true",
                        help="cuBLAS FFN/out projections with the GELU and the gated residual as separate h3b "
                             "kernels, instead of the h3b GEMM epilogues")
    parser.add_argument("--transformer-bench", action="store_true",
                        help="time the whole H3 transformer per request (f1/f2 mechanisms) instead")
    parser.add_argument("--layers", type=int, default=2, help="blocks in --transformer-bench")
    parser.add_argument("--eager-sp-baseline", action="store_true",
                        help="N>1: also time the unfused block in the reference's packed-Ulysses structure "
                             "with torch ops (gpu_eager_baseline)")
    parser.add_argument("--no-gemm-pack", action="store_true",
                        help="cuBLAS QKV projection + the h3b pack kernel instead of the fused h3b QKV GEMM")
    parser.add_argument("--no-reference-block", action="store_true",
                        help="skip timing the reference's own LOSSLESS GPU block (gpu_reference_block)")
    parser.add_argument("--no-exchange-roofline", action="store_true",
                        help="N>1: skip timing the exchange operations standalone (exchange_standalone)")
    parser.add_argument("--no-side-lines", action="store_true",
                        help="N=1: skip the attention A/B, the 768p-5s block and the elementwise sweep keys")
    parser.add_argument("--no-eager-baseline", action="store_true",
                        help="skip timing the unfused torch block at N=1")
    parser.add_argument("--sweep", choices=["elementwise"], help="print the config-2 kernel sweep instead")
    parser.add_argument("--profile-kernel", choices=["attention", "elementwise", "qkv_gemm", "gemm_gelu",
                                                     "gemm_gated"],
                        help="launch one kernel family for an ncu capture")
    parser.add_argument("--heads-per-rank", type=int, default=3)
    parser.add_argument("--exchange-bench", action="store_true",
                        help="N>1: time the exchange operations alone (peer stores vs NCCL)")
    args = parser.parse_args()
    sys.path.insert(0, str(ROOT))
    from h3_flash_b200.workloads import CONFIGS

    if args.profile_kernel:
        profile_kernel(args)
        return 0
    if args.exchange_bench:
        line = exchange_bench(args)
        if line is not None:
            print(json.dumps(line), flush=True)
        import torch.distributed as dist

        dist.destroy_process_group()
        return 0
    if args.sweep == "elementwise":
        print(json.dumps(elementwise_sweep(args)), flush=True)
        return 0
    if args.transformer_bench:
        line = transformer_bench(args)
        if line is not None:
            print(json.dumps(line), flush=True)
        if args.gpus > 1:
            import torch.distributed as dist

            dist.destroy_process_group()
        return 0

    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        if rank != 0:
            return 0
        steps = max(args.steps, 1)
        base = cpu_reference_block(args.config, steps, steps, max(args.warmup, 0))
        value = round(base["value"], 2)
        line = {
            "metric": METRIC, "impl": "reference", "value": value, "unit": "ms",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": value, "higher_is_better": False, "scaling": "strong",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic: seeded N(0,1) activations, N(0,0.02) weights",
            "config": {"workload": f"{CONFIGS[args.config].name} DiT block forward (CPU port of the reference path, "
                                   f"W=1, every host thread)", "seq": CONFIGS[args.config].seq,
                       "measurement": "the timed steps cover the block's query rows once; value is their sum"},
            "cpu_baseline": {**base, "value": value},
            "e2e": {"value": value, "unit": "ms", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return 0

    result = run_h3b(args)
    if result is not None:
        if args.gpus == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = cpu_reference_block(args.config, 16, 4, 1)
        print(json.dumps(result), flush=True)
    if args.gpus > 1:
        import torch.distributed as dist

        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
