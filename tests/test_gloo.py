"""Multi-rank host logic on CPU: gloo process groups of 2 and 4 ranks.

* the packed-Ulysses row-count protocol and varlen exchange of this package,
  checked bit-for-bit against the reference's own gloo run (tests/golden/ulysses_w2.npz);
* at 4 ranks with uneven rows (one rank empty): the QKV exchange and the output
  exchange's all-to-all (+ merge) against the oracle's restatement, bit for bit;
* the oracle's sharded block equals its single-process block (the CPU/gloo config);
* failure detection: a peer that dies before a collective surfaces as an error
  within the process-group timeout instead of a hang.
"""

from __future__ import annotations

import datetime
import os
import socket
import traceback

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "ulysses_w2.npz")


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world: int, fn, *args, timeout: float = 240.0) -> list:
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_entry, args=(fn, r, world, port, queue, args)) for r in range(world)]
    for p in procs:
        p.start()
    results = [None] * world
    for _ in procs:
        rank, ok, payload = queue.get(timeout=timeout)
        if not ok:
            for p in procs:
                p.kill()
            raise AssertionError(f"rank {rank} failed:\n{payload}")
        results[rank] = payload
    for p in procs:
        p.join(timeout=60)
    return results


def _entry(fn, rank, world, port, queue, args):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=60))
        torch.set_num_threads(2)
        payload = fn(rank, world, *args)
        queue.put((rank, True, payload))
        dist.destroy_process_group()
    except BaseException:  # noqa: BLE001
        queue.put((rank, False, traceback.format_exc()))


# ---------------------------------------------------------------------------


def _exchange_vs_reference(rank, world):
    from h3_flash_b200.runtime.parallel.packed_ulysses import PackedUlyssesRuntime, packed_qkv_exchange
    from oracle import relayout_ref

    g = dict(np.load(GOLDEN))
    q, k, v = g[f"r{rank}_q"], g[f"r{rank}_k"], g[f"r{rank}_v"]
    send = torch.from_numpy(relayout_ref.pack_qkv(q, k, v, world).view(np.int16)).view(torch.bfloat16)
    runtime = PackedUlyssesRuntime(dist.group.WORLD)
    runtime.begin_request()
    recv = packed_qkv_exchange(send, q.shape[0], runtime)
    counts = runtime.row_counts(q.shape[0])
    try:
        runtime.row_counts(q.shape[0] + 1)
        changed = "no error"
    except RuntimeError as error:
        changed = str(error)
    return recv.view(torch.int16).numpy().view(np.uint16), counts, changed, runtime.provenance()["row_count_collectives_per_request"]


def test_packed_exchange_matches_reference_gloo_run():
    g = dict(np.load(GOLDEN))
    results = _run(2, _exchange_vs_reference)
    for rank, (recv, counts, changed, per_request) in enumerate(results):
        np.testing.assert_array_equal(recv, g[f"r{rank}_packed"])
        assert counts == [5, 6]
        assert "row count changed" in changed
        assert per_request == 1


ROWS_W4 = [3, 0, 5, 2]  # uneven, one rank without rows


def _exchange_round_trip_w4(rank, world):
    """QKV exchange and the output exchange's all-to-all at W=4 over gloo, with the
    same seeded inputs on every rank (each rank rebuilds all ranks' inputs)."""

    from h3_flash_b200.runtime.parallel.packed_ulysses import (
        PackedUlyssesRuntime,
        _all_to_all_varlen,
        packed_qkv_exchange,
    )
    from oracle import relayout_ref

    heads, d = 8, 16
    hl = heads // world
    rng = np.random.default_rng(11)
    qkv = [[rng.integers(0, 2 ** 16, size=(n, heads, d), dtype=np.uint16) for _ in range(3)] for n in ROWS_W4]
    sends = [relayout_ref.pack_qkv(q, k, v, world) for q, k, v in qkv]
    total = sum(ROWS_W4)
    outputs = [rng.integers(0, 2 ** 16, size=(total, hl, d), dtype=np.uint16) for _ in range(world)]
    runtime = PackedUlyssesRuntime(dist.group.WORLD)
    runtime.begin_request()
    rows = ROWS_W4[rank]
    recv = packed_qkv_exchange(torch.from_numpy(sends[rank].view(np.int16)).view(torch.bfloat16), rows, runtime)
    counts = runtime.row_counts(rows)
    block = hl * d
    back = _all_to_all_varlen(torch.from_numpy(outputs[rank].view(np.int16)).view(torch.bfloat16),
                              rows * world * block, [c * block for c in counts], [rows * block] * world,
                              runtime.group)
    back = back.view(torch.int16).numpy().view(np.uint16).reshape(world, rows, hl, d)
    want_recv = relayout_ref.exchange(sends, counts)[rank]
    want_back = relayout_ref.exchange_back(outputs, counts)[rank]
    return (bool(np.array_equal(recv.view(torch.int16).numpy().view(np.uint16), want_recv)),
            bool(np.array_equal(relayout_ref.merge_heads(back), want_back)), counts)


def test_exchange_round_trip_at_four_ranks_matches_the_oracle():
    for recv_ok, back_ok, counts in _run(4, _exchange_round_trip_w4):
        assert counts == ROWS_W4
        assert recv_ok and back_ok


def _oracle_block(rank, world, params, hidden, idx, cos, sin, cfg):
    from h3_flash_b200.workloads import split_bounds
    from oracle.block_ref import block_forward

    start, stop = split_bounds(hidden.shape[0], world, rank)
    return block_forward(params, hidden[start:stop], idx[start:stop], cos[start:stop], sin[start:stop],
                         group=dist.group.WORLD, **cfg)


def test_oracle_sharded_block_equals_single_process():
    from h3_flash_b200.runtime.h3_block import H3TransformerBlock
    from h3_flash_b200.workloads import init_block_
    from oracle.block_ref import block_forward, fp32_params

    torch.manual_seed(0)
    block = init_block_(H3TransformerBlock(dim=256, heads=2, head_dim=128, ffn_inner=512), seed=3)
    params = fp32_params(block)
    rows = 37
    hidden = torch.randn(rows, 256)
    idx = torch.randint(0, 3, (rows,))
    ang = torch.randn(rows, 96)
    cos, sin = ang.cos(), ang.sin()
    cfg = dict(heads=2, head_dim=128, eps=1e-6, qk_eps=1e-6)
    full = block_forward(params, hidden, idx, cos, sin, **cfg)
    parts = _run(2, _oracle_block, params, hidden, idx, cos, sin, cfg)
    torch.testing.assert_close(torch.cat(parts), full, rtol=1e-5, atol=1e-5)


def _peer_dies(rank, world):
    from h3_flash_b200.runtime.parallel.packed_ulysses import PackedUlyssesRuntime

    if rank == 1:
        return "left"  # leaves between steps: never joins the row-count collective
    pg = dist.new_group([0, 1], timeout=datetime.timedelta(seconds=3))
    runtime = PackedUlyssesRuntime(pg)
    runtime.begin_request()
    try:
        runtime.row_counts(4)
    except Exception as error:  # noqa: BLE001
        return f"detected: {type(error).__name__}"
    return "no error"


@pytest.mark.timeout(120)
def test_dead_peer_is_detected_not_hung():
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dead_entry, args=(r, 2, port, queue)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in procs:
        rank, payload = queue.get(timeout=100)
        out[rank] = payload
    for p in procs:
        p.join(timeout=30)
        if p.is_alive():
            p.kill()
    assert out[1] == "left"
    assert out[0].startswith("detected"), out[0]


def _dead_entry(rank, world, port, queue):
    try:
        dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                                timeout=datetime.timedelta(seconds=30))
        if rank == 1:
            # participate in group creation (collective), then leave
            dist.new_group([0, 1], timeout=datetime.timedelta(seconds=3))
            queue.put((rank, "left"))
            queue.close()
            queue.join_thread()  # flush before the hard exit
            os._exit(0)
        queue.put((rank, _peer_dies(rank, world)))
    except BaseException as error:  # noqa: BLE001
        queue.put((rank, f"detected: {type(error).__name__}"))
    queue.close()
    queue.join_thread()
    os._exit(0)
