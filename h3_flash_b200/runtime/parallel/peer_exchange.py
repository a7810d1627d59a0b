"""Packed-Ulysses exchange as NVLink peer stores instead of NCCL all-to-alls.

The reference moves the packed QKV rows and the attention output with two
``all_to_all_single`` calls per attention (src/h3_flash/runtime/parallel/
packed_ulysses.py:67-128), around a pack kernel and a head merge. Here every
rank's receive buffer, merged-output buffer and barrier flags live in one device
allocation that every other rank maps with CUDA IPC (plain peer mappings).
Then, per attention call, on the current stream:

  h3b_qkv_gemm_pack_p2p      the QKV projection GEMM; its epilogue does QK-norm +
                             RoPE and stores each head row straight into the
                             owning rank's receive buffer [S, hl, 3D] (``pack_gemm``;
                             ``pack`` is h3b_qknorm_rope_pack_p2p on a projection
                             made elsewhere)
  h3b_peer_barrier           all peers' rows have landed
  h3b_attention_p2p          attention on the own receive buffer; its epilogue
                             stores each output row into its owner's merged
                             buffer [r, H, D] (exchange + merge_heads inside the
                             attention kernel)
  h3b_peer_barrier           all peers' output rows have landed

``scatter`` is the unfused form of the third step: attention into a local
[S, hl, D] tensor, then h3b_scatter_heads_p2p moves its rows (same bits).

The result is a view of the merged buffer; the next call on this runtime
overwrites it, after the first barrier, so it must be consumed (the output
projection) before then, on the same stream. The buffers are sized from the
request's row counts and regrown collectively when a larger request arrives.
"""

from __future__ import annotations

import ctypes
import math
from typing import Any

import torch
import torch.distributed as dist

from ... import _lib
from ..._torch import call, ptr, stream_of
from ..kernels.fusions import qknorm_rope_pack_args, qkv_gemm_pack_args

_ALIGN = 256
_FLAG_BYTES = 256


def _round_up(value: int, align: int = _ALIGN) -> int:
    return (value + align - 1) // align * align


class PeerExchange:
    """One group's peer-mapped buffers. Every rank of the group must call the
    collective methods (``ensure``, ``close``) at the same points."""

    def __init__(self, group: Any = None) -> None:
        self.group = group or dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        if self.world > 16:
            raise RuntimeError("peer exchange supports at most 16 ranks")
        self.device = torch.device("cuda", torch.cuda.current_device())
        lib = _lib.load()
        if lib.h3b_peer_flags_bytes() > _FLAG_BYTES:
            raise RuntimeError("libh3b flag array larger than the reserved region")
        self._buffer: torch.Tensor | None = None
        self._recv_bytes = 0
        self._merged_bytes = 0
        self._opened: list[tuple[int, int]] = []
        self._recv_ptrs = self._merged_ptrs = self._flag_ptrs = None
        self._counts_key: tuple[int, ...] | None = None
        self._counts_arr = None
        self.reallocations = 0

    # -- buffers -------------------------------------------------------------
    def ensure(self, total_rows: int, max_rows: int, heads: int, head_dim: int) -> None:
        """Collective when it reallocates: size the buffers for a request."""

        hl = heads // self.world
        recv_bytes = _round_up(total_rows * hl * 3 * head_dim * 2)
        merged_bytes = _round_up(max_rows * heads * head_dim * 2)
        if self._buffer is not None and recv_bytes <= self._recv_bytes and merged_bytes <= self._merged_bytes:
            return
        self._release()
        self._recv_bytes = max(recv_bytes, self._recv_bytes)
        self._merged_bytes = max(merged_bytes, self._merged_bytes)
        total = self._recv_bytes + self._merged_bytes + _FLAG_BYTES
        buffer = torch.empty(total, dtype=torch.uint8, device=self.device)
        flags_at = self._recv_bytes + self._merged_bytes
        buffer[flags_at:].zero_()
        torch.cuda.synchronize(self.device)  # flags are zero before any peer can see them
        handle = (ctypes.c_char * _lib.IPC_HANDLE_BYTES)()
        offset = ctypes.c_int64(0)
        call("h3b_ipc_handle", ptr(buffer), handle, ctypes.byref(offset))
        mine = (bytes(handle), int(offset.value))
        gathered: list[Any] = [None] * self.world
        dist.all_gather_object(gathered, mine, group=self.group)
        bases = []
        for peer, (peer_handle, peer_offset) in enumerate(gathered):
            if peer == self.rank:
                bases.append(ptr(buffer))
                continue
            raw = (ctypes.c_char * _lib.IPC_HANDLE_BYTES).from_buffer_copy(peer_handle)
            mapped = ctypes.c_void_p(0)
            call("h3b_ipc_open", raw, peer_offset, ctypes.byref(mapped))
            self._opened.append((int(mapped.value), peer_offset))
            bases.append(int(mapped.value))
        arr = ctypes.c_void_p * self.world
        recv_at, merged_at = 0, self._recv_bytes
        self._recv_ptrs = arr(*[base + recv_at for base in bases])
        self._merged_ptrs = arr(*[base + merged_at for base in bases])
        self._flag_ptrs = arr(*[base + flags_at for base in bases])
        self._buffer = buffer
        self.reallocations += 1
        # No rank stores into a peer before every rank has mapped every buffer.
        dist.barrier(group=self.group)

    def _release(self) -> None:
        if self._buffer is None:
            return
        # Every rank's device is idle before any mapping goes away.
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        for mapped, offset in self._opened:
            call("h3b_ipc_close", mapped, offset)
        self._opened.clear()
        self._buffer = None
        self._recv_ptrs = self._merged_ptrs = self._flag_ptrs = None

    def close(self) -> None:
        """Collective: unmap the peers' buffers and free this rank's."""

        self._release()
        self._recv_bytes = self._merged_bytes = 0

    # -- views ----------------------------------------------------------------
    def recv_view(self, total_rows: int, heads_local: int, head_dim: int) -> torch.Tensor:
        n = total_rows * heads_local * 3 * head_dim
        return self._buffer[: 2 * n].view(torch.bfloat16).view(total_rows, heads_local, 3 * head_dim)

    def merged_view(self, rows: int, heads: int, head_dim: int) -> torch.Tensor:
        start = self._recv_bytes
        n = rows * heads * head_dim
        return self._buffer[start : start + 2 * n].view(torch.bfloat16).view(rows, heads, head_dim)

    def _counts(self, counts: list[int]):
        key = tuple(counts)
        if key != self._counts_key:
            self._counts_arr = (ctypes.c_int64 * self.world)(*counts)
            self._counts_key = key
        return self._counts_arr

    # -- the three steps ------------------------------------------------------
    def pack(self, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_weight: torch.Tensor,
             k_weight: torch.Tensor, cos: torch.Tensor | None, sin: torch.Tensor | None,
             q_eps: float, k_eps: float, counts: list[int]) -> None:
        """QK-norm + RoPE + the QKV exchange: this rank's rows land in every owner's
        receive buffer at their global rows."""

        op = "fused_qknorm_rope_pack_p2p"
        rotary_dim, cos32, sin32 = qknorm_rope_pack_args(op, q, k, v, q_weight, k_weight, cos,
                                                         sin, self.world)
        rows, heads, head_dim = q.shape
        if rows != counts[self.rank]:
            raise ValueError(f"{op}: {rows} local rows, the request says {counts[self.rank]}")
        total = sum(counts)
        self.ensure(total, max(counts), heads, head_dim)
        call("h3b_qknorm_rope_pack_p2p", self._recv_ptrs, self.world, sum(counts[: self.rank]),
             total, ptr(q), ptr(k), ptr(v), q.stride(0), k.stride(0), v.stride(0),
             ptr(q_weight.contiguous()), ptr(k_weight.contiguous()), ptr(cos32), ptr(sin32), rows,
             heads, head_dim, rotary_dim, float(q_eps), float(k_eps), stream_of(q))

    def pack_gemm(self, x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor | None,
                  q_weight: torch.Tensor, k_weight: torch.Tensor, cos: torch.Tensor | None,
                  sin: torch.Tensor | None, q_eps: float, k_eps: float, heads: int,
                  counts: list[int]) -> None:
        """The QKV projection whose epilogue does QK-norm + RoPE and stores each head
        row into its owner's receive buffer: projection, pack and QKV exchange in one
        kernel (the same receive-buffer contents as ``pack`` on the projection,
        except that the projection is not rounded to bf16 before the norm)."""

        op = "fused_qkv_gemm_pack_p2p"
        x2d, weight, bias, rotary_dim, cos32, sin32, workspace = qkv_gemm_pack_args(
            op, x, weight, bias, q_weight, k_weight, cos, sin, heads)
        rows, dim = x2d.shape
        if rows != counts[self.rank]:
            raise ValueError(f"{op}: {rows} local rows, the request says {counts[self.rank]}")
        if heads % self.world:
            raise ValueError(f"heads ({heads}) must divide Ulysses degree ({self.world})")
        total = sum(counts)
        self.ensure(total, max(counts), heads, 128)
        call("h3b_qkv_gemm_pack_p2p", self._recv_ptrs, self.world, sum(counts[: self.rank]), total,
             ptr(x2d), rows, dim, x2d.stride(0), ptr(weight), ptr(bias) if bias is not None else None,
             ptr(q_weight.contiguous()), ptr(k_weight.contiguous()),
             ptr(cos32) if cos32 is not None else None, ptr(sin32) if sin32 is not None else None,
             heads, 128, rotary_dim, float(q_eps), float(k_eps),
             ptr(workspace) if workspace is not None else None,
             workspace.numel() * 4 if workspace is not None else 0, stream_of(x2d))

    def check(self) -> None:
        """Raise if a barrier of an earlier call gave up on a peer (status bit 2,
        set after 10 s): the rows it exchanged are incomplete. Reads the device
        status word (a host sync), so call it at request boundaries."""

        if _lib.device_status() & 2:
            _lib.clear_device_status(torch.cuda.current_stream(self.device).cuda_stream)
            raise RuntimeError(
                "packed Ulysses peer exchange: a peer did not reach the exchange barrier "
                "within 10 s; the previous request's outputs are invalid"
            )

    def barrier(self) -> None:
        call("h3b_peer_barrier", self._flag_ptrs, self.world, self.rank,
             torch.cuda.current_stream(self.device).cuda_stream)

    def attention(self, counts: list[int], heads_local: int, head_dim: int,
                  softmax_scale: float | None = None) -> torch.Tensor:
        """Attention over this rank's receive buffer with the output exchange and
        head merge fused into its epilogue. Returns this rank's merged rows (a
        view of its buffer), complete after the next ``barrier``."""

        from ..attention.dense import workspace_bytes

        total = sum(counts)
        if self._buffer is None or total * heads_local * 3 * head_dim * 2 > self._recv_bytes \
                or max(counts) * heads_local * self.world * head_dim * 2 > self._merged_bytes:
            raise RuntimeError("attention before pack: the exchange buffers are not sized for this request")
        scale = float(softmax_scale) if softmax_scale is not None else 1.0 / math.sqrt(head_dim)
        ws_bytes = workspace_bytes(1, total, total, heads_local, head_dim)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=self.device) if ws_bytes else None
        stream = torch.cuda.current_stream(self.device).cuda_stream
        call("h3b_attention_p2p", self._merged_ptrs, self._counts(counts), self.world, self.rank,
             ptr(self._buffer), heads_local, head_dim, scale, ptr(ws) if ws is not None else None,
             ws_bytes, stream)
        return self.merged_view(counts[self.rank], heads_local * self.world, head_dim)

    def scatter(self, output: torch.Tensor, counts: list[int]) -> torch.Tensor:
        """Output exchange + head merge: [S, hl, D] of this rank's heads -> every owner's
        [r, H, D]. Returns this rank's merged rows (a view of its buffer)."""

        total, heads_local, head_dim = output.shape
        if total != sum(counts) or not output.is_contiguous():
            raise ValueError("scatter needs the contiguous [S, hl, D] attention output")
        if self._buffer is None or max(counts) * heads_local * self.world * head_dim * 2 > self._merged_bytes:
            raise RuntimeError("scatter before pack: the merged buffers are not sized for this request")
        call("h3b_scatter_heads_p2p", self._merged_ptrs, self._counts(counts), ptr(output),
             self.world, self.rank, heads_local, head_dim, stream_of(output))
        return self.merged_view(counts[self.rank], heads_local * self.world, head_dim)
