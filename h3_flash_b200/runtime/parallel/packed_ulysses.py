"""Dense packed-Ulysses attention: one QKV exchange and one output exchange per block.

Drop-in for ``h3_flash.runtime.parallel.packed_ulysses``
(src/h3_flash/runtime/parallel/packed_ulysses.py). Data path per attention call,
W ranks, r local rows, H heads, hl = H/W:

  fused QKV GEMM [r, 3d]                              (cuBLAS via torch)
  -> fused_qknorm_rope_pack  -> send [W, r, hl, 3D]   (h3b: QK-norm + RoPE + destination-major pack, one pass)
  -> NCCL all_to_all_single  -> recv [S, hl, 3D]      (rows arrive in global order)
  -> packed_attention        -> [S, hl, D]            (h3b tcgen05 attention, Q/K/V read in place)
  -> NCCL all_to_all_single  -> [W, r, hl, D] -> merge_heads -> [r, H, D]
  -> to_out GEMM

The reference's separate QK-norm+RoPE launches and its standalone pack kernel
are fused into one kernel. Row counts are exchanged once per request.

With ``exchange="p2p"`` the two NCCL all-to-alls, the send buffer and the
merge are replaced by peer stores over NVLink (peer_exchange.py): the pack
kernel writes each head row into its owner's receive buffer and the attention
kernel's epilogue writes each output row into its owner's merged buffer
(``fuse_output_exchange=False``: a separate scatter kernel after attention).

With ``gemm_pack`` (default) the QKV projection, QK-norm + RoPE and the pack are
one tcgen05 GEMM (h3b_qkv_gemm_pack): its epilogue writes the send buffer, or
with p2p every owner's receive buffer, directly.
"""

from __future__ import annotations

import socket
from typing import Any

import torch
import torch.distributed as dist
import torch.nn.functional as F

from ..attention.dense import packed_attention
from ..kernels.fusions import (
    fused_qknorm_rope,
    fused_qknorm_rope_pack,
    fused_qkv_gemm_pack,
    qkv_gemm_pack_supported,
)
from ..timing import TIMER
from .context import with_context_parallel_reapplied
from .relayout import can_pack_qkv, merge_heads, pack_qkv_destination_major


class PackedUlyssesRuntime:
    """Request-scoped shape metadata and auditable counters (packed_ulysses.py:19-64)."""

    def __init__(self, group: Any, exchange: str = "nccl", fuse_output_exchange: bool = True) -> None:
        if exchange not in ("nccl", "p2p"):
            raise ValueError(f"exchange must be 'nccl' or 'p2p', got {exchange!r}")
        self.fuse_output_exchange = fuse_output_exchange
        self.group = group
        self.world = dist.get_world_size(group)
        self._row_counts: tuple[list[int], int] | None = None
        self.requests = 0
        self.attention_calls = 0
        backend = dist.get_backend(group)
        self._count_device = "cuda" if str(backend) == "nccl" else "cpu"
        self.exchange = exchange
        self.peer = None
        if exchange == "p2p":
            if not torch.cuda.is_available():
                raise RuntimeError("the p2p exchange needs CUDA devices")
            from .peer_exchange import PeerExchange

            self.peer = PeerExchange(group)

    def begin_request(self) -> None:
        # Every rank calls this at the same request boundary; the next attention
        # call gathers the (possibly uneven) shard sizes collectively, once.
        if self.peer is not None:
            self.peer.check()
        self._row_counts = None
        self.requests += 1

    def row_counts(self, rows_local: int) -> list[int]:
        if self._row_counts is not None:
            counts, seen = self._row_counts
            if seen != rows_local:
                raise RuntimeError(
                    f"packed Ulysses row count changed from {seen} to {rows_local} "
                    "inside one request"
                )
            return counts
        buffer = torch.zeros(self.world, dtype=torch.long, device=self._count_device)
        buffer[dist.get_rank(self.group)] = rows_local
        dist.all_reduce(buffer, group=self.group)
        counts = [int(value) for value in buffer.tolist()]
        self._row_counts = (counts, rows_local)
        return counts

    def provenance(self) -> dict[str, Any]:
        return {
            "backend": "packed_ulysses_h3b",
            "degree": self.world,
            "semantics": "dense",
            "exchange": self.exchange,
            "qkv_collectives_per_attention": 1,
            "output_collectives_per_attention": 1,
            "relayout": "cuda_fused_qknorm_rope_pack" if self.peer is None
            else "cuda_fused_qknorm_rope_pack_p2p",
            "output_exchange": "nccl_all_to_all_then_merge" if self.peer is None
            else ("attention_epilogue_p2p" if self.fuse_output_exchange else "scatter_p2p"),
            "attention": "h3b_tcgen05",
            "row_count_collectives_per_request": 1,
            "requests": self.requests,
            "attention_calls": self.attention_calls,
            "origin": "B200-native rebuild of the H3-Flash packed Ulysses path",
        }


def _all_to_all_varlen(x: torch.Tensor, out_numel: int, input_splits: list[int],
                       output_splits: list[int], group: Any) -> torch.Tensor:
    """packed_ulysses.py:67-82: one varlen all_to_all_single over flat buffers."""

    output = torch.empty(out_numel, dtype=x.dtype, device=x.device)
    dist.all_to_all_single(
        output,
        x.reshape(-1),
        output_split_sizes=output_splits,
        input_split_sizes=input_splits,
        group=group,
    )
    return output


def packed_qkv_exchange(packed: torch.Tensor, rows_local: int, runtime: PackedUlyssesRuntime) -> torch.Tensor:
    """Exchange a destination-major send buffer [W, r, hl, 3D] -> [S, hl, 3D]."""

    world, rows, heads_local, width = packed.shape
    if world != runtime.world or rows != rows_local:
        raise ValueError(f"send buffer {tuple(packed.shape)} does not match world {runtime.world}, rows {rows_local}")
    counts = runtime.row_counts(rows_local)
    rows_full = sum(counts)
    block = heads_local * width
    exchanged = _all_to_all_varlen(
        packed, rows_full * block, [rows_local * block] * runtime.world,
        [count * block for count in counts], runtime.group,
    )
    return exchanged.reshape(rows_full, heads_local, width)


def _packed_qkv_all_to_all(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor,
                           runtime: PackedUlyssesRuntime) -> torch.Tensor:
    """Pack (CUDA kernel) + exchange (packed_ulysses.py:85-108). Returns [S, hl, 3D]."""

    rows_local = q.shape[0]
    if not can_pack_qkv(q, k, v):
        raise RuntimeError("packed Ulysses needs CUDA q/k/v of equal shape with unit last stride")
    packed = pack_qkv_destination_major(q, k, v, runtime.world)
    return packed_qkv_exchange(packed, rows_local, runtime)


def _packed_output_all_to_all(output: torch.Tensor, rows_local: int,
                              runtime: PackedUlyssesRuntime) -> torch.Tensor:
    """Inverse exchange + head merge (packed_ulysses.py:111-128). Returns [r, H, D]."""

    _, heads_local, head_dim = output.shape
    counts = runtime.row_counts(rows_local)
    block = heads_local * head_dim
    exchanged = _all_to_all_varlen(
        output, rows_local * runtime.world * block, [count * block for count in counts],
        [rows_local * block] * runtime.world, runtime.group,
    )
    return merge_heads(exchanged.reshape(runtime.world, rows_local, heads_local, head_dim))


def _linear_params(layer: Any) -> tuple[torch.Tensor, torch.Tensor | None]:
    return layer.weight, getattr(layer, "bias", None)


def qkv_weights(attention: Any) -> tuple[torch.Tensor, torch.Tensor | None] | None:
    """The stacked [3d, dim] weight and [3d] bias of to_q/to_k/to_v (or of to_qkv),
    or None when the projections are not plain Linears. The concatenation is cached,
    keyed on the parameters' storage and version counters, so in-place weight
    updates rebuild it."""

    if getattr(attention, "fused_projections", False) and hasattr(attention, "to_qkv"):
        layer = attention.to_qkv
        return (layer.weight, getattr(layer, "bias", None)) if isinstance(layer, torch.nn.Linear) else None
    layers = (attention.to_q, attention.to_k, attention.to_v)
    if not all(isinstance(layer, torch.nn.Linear) for layer in layers):
        return None
    params = [_linear_params(layer) for layer in layers]
    key = tuple((t.data_ptr(), t._version) if t is not None else None for pair in params for t in pair)
    cache = attention.__dict__.get("_h3b_qkv_cache")
    if cache is None or cache[0] != key:
        with torch.no_grad():
            weight = torch.cat([w for w, _ in params], dim=0)
            biases = [b for _, b in params]
            bias = torch.cat(biases) if all(b is not None for b in biases) else None
            if bias is None and any(b is not None for b in biases):
                bias = torch.cat([
                    b if b is not None else torch.zeros(w.shape[0], dtype=w.dtype, device=w.device)
                    for w, b in params
                ])
        attention.__dict__["_h3b_qkv_cache"] = (key, weight, bias)
        cache = attention.__dict__["_h3b_qkv_cache"]
    return cache[1], cache[2]


def qkv_projection(attention: Any, hidden: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """to_q/to_k/to_v as one GEMM against the cached stacked weight (``qkv_weights``).
    Returns q, k, v views [rows, H, D] into one [rows, 3d] buffer."""

    heads, head_dim = attention.heads, attention.head_dim
    rows = hidden.shape[0]
    stacked = qkv_weights(attention)
    if getattr(attention, "fused_projections", False) and hasattr(attention, "to_qkv"):
        qkv = attention.to_qkv(hidden)
    elif stacked is not None:
        qkv = F.linear(hidden, stacked[0], stacked[1])
    else:
        qkv = torch.cat([layer(hidden) for layer in (attention.to_q, attention.to_k, attention.to_v)], dim=-1)
    width = heads * head_dim
    q = qkv[:, :width].view(rows, heads, head_dim)
    k = qkv[:, width : 2 * width].view(rows, heads, head_dim)
    v = qkv[:, 2 * width :].view(rows, heads, head_dim)
    return q, k, v


def _norm_params(norm: Any) -> tuple[torch.Tensor, float] | None:
    weight = getattr(norm, "weight", None)
    eps = getattr(norm, "eps", None)
    if weight is None or eps is None:
        return None
    return weight, float(eps)


def _out_projection(attention: Any, output: torch.Tensor) -> torch.Tensor:
    """``attention.to_out[0](output)`` on the h3b tcgen05 GEMM where it serves the shape
    (bias in the epilogue), else the layer itself (cuBLAS)."""

    from ..kernels.transformer import linear

    return linear(attention.to_out[0], output)


def ulysses_attention_forward(attention: Any, hidden_states: torch.Tensor, rotary_emb: Any = None,
                              attention_mask: Any = None, *, runtime: PackedUlyssesRuntime | None = None,
                              fused_qknorm_rope: bool = True, gemm_pack: bool = True) -> torch.Tensor:
    """The patched ``attn.forward`` body (packed_ulysses.py:150-215). ``runtime=None``
    runs the same data path on one GPU (no exchange). ``gemm_pack``: where the shapes
    allow it, the QKV projection, QK-norm + RoPE and the pack (and, with the p2p
    exchange, the QKV exchange) run as one GEMM kernel."""

    if attention_mask is not None:
        raise RuntimeError("packed Ulysses requires padless dense attention")
    batch, rows_local, _ = hidden_states.shape
    if batch != 1:
        raise RuntimeError("packed Ulysses currently requires batch size one")
    heads, head_dim = attention.heads, attention.head_dim
    world = runtime.world if runtime is not None else 1
    if heads % world:
        raise ValueError(f"heads ({heads}) must divide Ulysses degree ({world})")
    norm_q, norm_k = _norm_params(attention.norm_q), _norm_params(attention.norm_k)
    cos, sin = rotary_emb if rotary_emb is not None else (None, None)
    x2d = hidden_states.reshape(rows_local, -1)
    fused_norms = fused_qknorm_rope and norm_q is not None and norm_k is not None
    stacked = qkv_weights(attention) if (gemm_pack and fused_norms) else None
    use_gemm = stacked is not None and qkv_gemm_pack_supported(x2d, stacked[0], heads, head_dim, cos)
    peer = world > 1 and runtime.peer is not None and fused_norms and _p2p_supported(head_dim, cos)
    if peer:
        if use_gemm:
            output = _peer_attention_gemm(runtime, x2d, stacked, norm_q, norm_k, cos, sin, heads, head_dim)
        else:
            with TIMER.section("gemm"):
                q, k, v = qkv_projection(attention, x2d)
            output = _peer_attention(runtime, q, k, v, norm_q, norm_k, cos, sin, rows_local, head_dim)
        output = output.reshape(batch, rows_local, heads * head_dim).type_as(hidden_states)
        runtime.attention_calls += 1
        with TIMER.section("gemm"):
            return attention.to_out[1](_out_projection(attention, output))
    if use_gemm:
        with TIMER.section("qkv_gemm_pack"):
            send = fused_qkv_gemm_pack(x2d, stacked[0], stacked[1], norm_q[0], norm_k[0], cos, sin,
                                       heads, world, norm_q[1], norm_k[1])
    else:
        with TIMER.section("gemm"):
            q, k, v = qkv_projection(attention, x2d)
        with TIMER.section("qknorm_rope_pack"):
            if fused_norms:
                send = fused_qknorm_rope_pack(q, k, v, norm_q[0], norm_k[0], cos, sin, world,
                                              norm_q[1], norm_k[1])
            else:
                if rotary_emb is not None and norm_q is not None and norm_k is not None:
                    q = fused_qknorm_rope(q.unsqueeze(0), norm_q[0], cos, sin, norm_q[1]).squeeze(0)
                    k = fused_qknorm_rope(k.unsqueeze(0), norm_k[0], cos, sin, norm_k[1]).squeeze(0)
                elif rotary_emb is None:
                    q, k = attention.norm_q(q), attention.norm_k(k)
                else:
                    raise RuntimeError("rotary embedding needs RMSNorm-style norm_q/norm_k modules")
                send = pack_qkv_destination_major(q.contiguous(), k.contiguous(), v.contiguous(), world)
    if world > 1:
        with TIMER.section("all_to_all"):
            packed = packed_qkv_exchange(send, rows_local, runtime)
    else:
        packed = send.view(rows_local, heads, 3 * head_dim)
    with TIMER.section("attention"):
        output = packed_attention(packed, head_dim)
    if world > 1:
        with TIMER.section("all_to_all"):
            output = _packed_output_all_to_all(output, rows_local, runtime)
    output = output.reshape(batch, rows_local, heads * head_dim).type_as(hidden_states)
    if runtime is not None:
        runtime.attention_calls += 1
    with TIMER.section("gemm"):
        return attention.to_out[1](_out_projection(attention, output))


def _p2p_supported(head_dim: int, cos: Any) -> bool:
    rotary_dim = 0 if cos is None else cos.shape[-1]
    return head_dim in (64, 128, 256) and rotary_dim % 16 == 0 and (head_dim - rotary_dim) % 16 == 0


def _peer_attention_gemm(runtime: PackedUlyssesRuntime, x2d, stacked, norm_q, norm_k, cos, sin,
                         heads: int, head_dim: int) -> torch.Tensor:
    """qkv_gemm_pack_p2p (projection + QK-norm + RoPE + QKV exchange) -> barrier ->
    attention_p2p (or attention -> scatter_p2p) -> barrier. Returns [r, H, D]."""

    peer = runtime.peer
    counts = runtime.row_counts(x2d.shape[0])
    with TIMER.section("qkv_gemm_pack"):
        peer.pack_gemm(x2d, stacked[0], stacked[1], norm_q[0], norm_k[0], cos, sin, norm_q[1],
                       norm_k[1], heads, counts)
    return _peer_exchange_rest(runtime, counts, heads // runtime.world, head_dim)


def _peer_exchange_rest(runtime: PackedUlyssesRuntime, counts: list[int], heads_local: int,
                        head_dim: int) -> torch.Tensor:
    """Everything after the pack: barrier, attention with the output exchange, barrier."""

    peer = runtime.peer
    with TIMER.section("all_to_all"):
        peer.barrier()
    if runtime.fuse_output_exchange:
        with TIMER.section("attention"):
            merged = peer.attention(counts, heads_local, head_dim)
        with TIMER.section("all_to_all"):
            peer.barrier()
        return merged
    with TIMER.section("attention"):
        output = packed_attention(peer.recv_view(sum(counts), heads_local, head_dim), head_dim)
    with TIMER.section("all_to_all"):
        merged = peer.scatter(output, counts)
        peer.barrier()
    return merged


def _peer_attention(runtime: PackedUlyssesRuntime, q, k, v, norm_q, norm_k, cos, sin,
                    rows_local: int, head_dim: int) -> torch.Tensor:
    """pack_p2p -> barrier -> attention_p2p (output exchange in its epilogue) ->
    barrier, or with ``fuse_output_exchange=False`` attention -> scatter_p2p in
    place of attention_p2p. Returns [r, H, D]."""

    peer = runtime.peer
    counts = runtime.row_counts(rows_local)
    with TIMER.section("qknorm_rope_pack"):
        peer.pack(q, k, v, norm_q[0], norm_k[0], cos, sin, norm_q[1], norm_k[1], counts)
    return _peer_exchange_rest(runtime, counts, q.shape[1] // runtime.world, head_dim)


def _single_node_cuda_group(group: Any) -> bool:
    """True when every rank of ``group`` is a CUDA process on this host (collective)."""

    if str(dist.get_backend(group)) != "nccl" or not torch.cuda.is_available():
        return False
    names: list[Any] = [None] * dist.get_world_size(group)
    dist.all_gather_object(names, socket.gethostname(), group=group)
    return len(set(names)) == 1


def install_packed_ulysses(transformer: Any, *, group: Any = None, fused_qknorm_rope: bool = True,
                           exchange: str = "auto", fuse_output_exchange: bool = True,
                           gemm_pack: bool = True) -> PackedUlyssesRuntime:
    """Replace each block's attention forward with the packed-Ulysses path (packed_ulysses.py:131-220).

    ``exchange``: ``"p2p"`` moves rows with peer stores over NVLink (one process
    per GPU on one node, CUDA IPC available), ``"nccl"`` with NCCL all-to-alls;
    ``"auto"`` (collective) picks p2p when all ranks are NCCL ranks on one host.
    ``fuse_output_exchange`` (p2p only): the attention kernel stores its output rows
    into the owners' merged buffers itself, instead of a scatter kernel after it.
    ``gemm_pack``: the QKV projection GEMM does QK-norm + RoPE + the pack (and with
    p2p the QKV exchange) in its epilogue, where the shapes allow it."""

    if not (dist.is_available() and dist.is_initialized()):
        raise RuntimeError("packed Ulysses requires an initialized process group")
    group = group or dist.group.WORLD
    if exchange == "auto":
        exchange = "p2p" if _single_node_cuda_group(group) else "nccl"
    runtime = PackedUlyssesRuntime(group, exchange=exchange, fuse_output_exchange=fuse_output_exchange)
    if runtime.world < 2:
        raise RuntimeError("packed Ulysses degree must be at least two")

    def apply() -> None:
        for block in transformer.transformer_blocks:
            attention = block.attn

            def forward(hidden_states, rotary_emb=None, attention_mask=None, *, attention=attention):
                return ulysses_attention_forward(
                    attention, hidden_states, rotary_emb, attention_mask,
                    runtime=runtime, fused_qknorm_rope=fused_qknorm_rope, gemm_pack=gemm_pack,
                )

            attention.forward = forward

    with_context_parallel_reapplied(transformer, apply)
    return runtime
