"""Packed-Ulysses exchange over NVLink peer stores (exchange="p2p").

The peer path must reproduce the NCCL path bit for bit:
- the receive buffer after pack_p2p + barrier equals fused_qknorm_rope_pack +
  all_to_all_single;
- the merged buffer after scatter_p2p + barrier equals all_to_all_single + merge_heads;
- the merged buffer after attention_p2p (output exchange in the attention epilogue)
  + barrier equals attention + all_to_all_single + merge_heads;
- a block stack run with exchange="p2p" (fused output exchange) equals the same stack
  run over NCCL.
Single-GPU: attention_p2p routes every row of every 'rank' to the right owner and head
slot, bit-identical to the local attention output (all 'peers' are local buffers).
This holds over several requests of different (uneven) row splits, so the buffers are
reused and regrown, and for one request in which a rank holds no rows. One single-GPU
test makes the barrier's bounded wait run out on a flag that nothing sets, and checks
the status bit it leaves.
"""

from __future__ import annotations

import ctypes
import datetime
import os
import socket
import traceback

import pytest
import torch

pytestmark = pytest.mark.gpu


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
        from h3_flash_b200.runtime.attention.dense import packed_attention
        from h3_flash_b200.runtime.h3_block import H3BlockStack, H3TransformerBlock
        from h3_flash_b200.runtime.kernels import install_transformer_fusions
        from h3_flash_b200.runtime.kernels.fusions import fused_qknorm_rope_pack
        from h3_flash_b200.runtime.parallel import install_packed_ulysses
        from h3_flash_b200.runtime.parallel.packed_ulysses import (
            PackedUlyssesRuntime,
            _packed_output_all_to_all,
            packed_qkv_exchange,
        )
        from h3_flash_b200.workloads import init_block_, rope_tables, split_bounds

        checks = {}
        # 1) exchange equality, uneven rows, two requests (the second larger: regrow)
        nccl_rt = PackedUlyssesRuntime(dist.group.WORLD)
        p2p_rt = PackedUlyssesRuntime(dist.group.WORLD, exchange="p2p")
        heads = 3 * world
        # requests: uneven rows; then larger (the buffers regrow); then rank 0 with no rows
        for request, base in enumerate((37, 301, 5)):
            rows = base + 3 * (world - rank) if request < 2 else (0 if rank == 0 else base)
            g = torch.Generator(device="cuda").manual_seed(100 * request + rank)
            qkv = torch.randn(rows, 3 * heads * 128, device="cuda", generator=g).to(torch.bfloat16)
            q, k, v = (qkv[:, i * heads * 128 : (i + 1) * heads * 128].view(rows, heads, 128) for i in range(3))
            wq = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(torch.bfloat16)
            wk = (1 + 0.1 * torch.randn(128, device="cuda", generator=g)).to(torch.bfloat16)
            cos = torch.rand(rows, 96, device="cuda", generator=g) * 2 - 1
            sin = torch.rand(rows, 96, device="cuda", generator=g) * 2 - 1
            for rt in (nccl_rt, p2p_rt):
                rt.begin_request()
            counts = nccl_rt.row_counts(rows)
            assert p2p_rt.row_counts(rows) == counts
            send = fused_qknorm_rope_pack(q, k, v, wq, wk, cos, sin, world, 1e-6, 1e-5)
            want = packed_qkv_exchange(send, rows, nccl_rt)
            peer = p2p_rt.peer
            peer.pack(q, k, v, wq, wk, cos, sin, 1e-6, 1e-5, counts)
            peer.barrier()
            got = peer.recv_view(sum(counts), heads // world, 128)
            checks[f"qkv_{request}"] = bool(torch.equal(got, want))
            out = want[..., 256:].contiguous()  # any [S, hl, D] tensor will do
            want_back = _packed_output_all_to_all(out, rows, nccl_rt)
            got_back = peer.scatter(out, counts)
            peer.barrier()
            checks[f"out_{request}"] = bool(torch.equal(got_back, want_back))
            # attention with the output exchange in its epilogue vs attention + NCCL + merge
            want_merged = _packed_output_all_to_all(packed_attention(want, 128), rows, nccl_rt)
            peer.barrier()  # the pack's barrier of a call: peers are done reading their merged rows
            got_merged = peer.attention(counts, heads // world, 128)
            peer.barrier()
            checks[f"attn_{request}"] = bool(torch.equal(got_merged, want_merged))
        checks["regrown"] = p2p_rt.peer.reallocations == 2  # the third request fits

        # 2) a two-block stack, NCCL vs p2p, two requests of different splits
        heads, dim = 2 * world, 256 * world
        def stack(exchange):
            blocks = [init_block_(H3TransformerBlock(dim=dim, heads=heads, head_dim=128, ffn_inner=2 * dim),
                                  seed=7 + i).to("cuda", torch.bfloat16) for i in range(2)]
            s = H3BlockStack(blocks)
            install_transformer_fusions(s)
            return s, install_packed_ulysses(s, exchange=exchange)

        nccl_stack, nccl_sp = stack("nccl")
        p2p_stack, p2p_sp = stack("p2p")
        for request, total in enumerate((900, 1333)):
            gh = torch.Generator().manual_seed(50 + request)
            hidden = torch.randn(1, total, dim, generator=gh).to(torch.bfloat16).cuda()
            idx = torch.randint(0, 3, (total,), generator=gh).cuda()
            pos = torch.stack([torch.arange(total) // 100, (torch.arange(total) // 10) % 10,
                               torch.arange(total) % 10], -1)
            cos, sin = (t.cuda() for t in rope_tables(pos, 96))
            start, stop = split_bounds(total, world, rank)
            args = (hidden[:, start:stop].contiguous(), None, idx[start:stop], (cos[start:stop], sin[start:stop]))
            outs = []
            for s, rt in ((nccl_stack, nccl_sp), (p2p_stack, p2p_sp)):
                rt.begin_request()
                with torch.no_grad():
                    outs.append(s(*args))
            checks[f"block_{request}"] = bool(torch.equal(outs[0], outs[1]))
        torch.cuda.synchronize()
        checks["status"] = _lib.device_status() == 0
        checks["calls"] = p2p_sp.attention_calls == 4
        flags = torch.tensor([int(v) for v in checks.values()], dtype=torch.int32, device="cuda")
        dist.all_reduce(flags, op=dist.ReduceOp.MIN)
        result = dict(zip(checks, flags.tolist()))
        p2p_rt.peer.close()
        p2p_sp.peer.close()
        queue.put((rank, True, result))
        dist.barrier()
        dist.destroy_process_group()
    except BaseException:  # noqa: BLE001
        queue.put((rank, False, traceback.format_exc()))


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_p2p_exchange_matches_nccl_bit_exact():
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
            rank, ok, payload = queue.get(timeout=300)
            assert ok, payload
            results[rank] = payload
    finally:
        for p in procs:
            p.join(timeout=60)
            if p.is_alive():
                p.kill()
    failed = [name for name, ok in results[0].items() if not ok]
    assert not failed, f"p2p differs from NCCL in: {failed}"


def test_peer_barrier_gives_up_on_a_missing_peer():
    """world=2 on one GPU: 'peer' 1's flag array is a local buffer nobody writes, so
    the wait for it runs out (10 s), sets status bit 2 and the kernel returns."""

    from h3_flash_b200 import _lib

    flags = torch.zeros(2, 64, dtype=torch.int32, device="cuda")
    ptrs = (ctypes.c_void_p * 2)(flags[0].data_ptr(), flags[1].data_ptr())
    stream = torch.cuda.current_stream().cuda_stream
    _lib.clear_device_status(stream)
    _lib.call("h3b_peer_barrier", ptrs, 2, 0, stream)
    torch.cuda.synchronize()
    try:
        assert _lib.device_status() & 2
        assert int(flags[1, 0]) == 1  # it did announce itself to the missing peer
        assert int(flags[0, 16]) == 1  # and advanced its own epoch
    finally:
        _lib.clear_device_status(stream)
        torch.cuda.synchronize()
    assert _lib.device_status() == 0


@pytest.mark.parametrize("seq,heads_local,counts", [
    (333, 3, [100, 0, 233]),          # split tail (combine kernel), a rank with no rows
    (4096, 2, [1000, 3096]),          # split tail
    (37888, 1, [18944, 18944]),       # 148 whole units: no split
])
def test_attention_p2p_routes_rows_to_owners(seq, heads_local, counts):
    """Every 'rank' r of a world whose merged buffers all live on this GPU: row s of local
    head h must land in owner o's buffer at (s - start_o, r*hl + h), bit-identical to the
    plain attention output (the buffers start as NaN, so a slot nobody wrote fails)."""

    from h3_flash_b200 import _lib
    from h3_flash_b200.runtime.attention.dense import packed_attention, workspace_bytes

    world = len(counts)
    g = torch.Generator(device="cuda").manual_seed(seq)
    packed = torch.randn(seq, heads_local, 384, device="cuda", generator=g).to(torch.bfloat16)
    want = packed_attention(packed, 128)
    heads = world * heads_local
    merged = [torch.full((max(c, 1), heads, 128), float("nan"), dtype=torch.bfloat16, device="cuda")
              for c in counts]
    ptrs = (ctypes.c_void_p * world)(*[m.data_ptr() for m in merged])
    arr = (ctypes.c_int64 * world)(*counts)
    ws_bytes = workspace_bytes(1, seq, seq, heads_local)
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for rank in range(world):
        _lib.call("h3b_attention_p2p", ptrs, arr, world, rank, packed.data_ptr(), heads_local, 128,
                  1.0 / 128 ** 0.5, ws.data_ptr(), ws_bytes, stream)
    torch.cuda.synchronize()
    start = 0
    for owner, c in enumerate(counts):
        got = merged[owner][:c].view(c, world, heads_local, 128)
        expect = want[start : start + c].unsqueeze(1).expand(c, world, heads_local, 128)
        assert torch.equal(got, expect), owner
        start += c
    assert _lib.device_status() == 0

