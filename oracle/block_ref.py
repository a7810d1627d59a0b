"""The LOSSLESS packed-Ulysses DiT block forward in torch fp32 on the CPU (test infrastructure only).

Restates the reference block (src/h3_flash/runtime/kernels/transformer.py:50-126,
unfused branches) with the packed-Ulysses attention
(src/h3_flash/runtime/parallel/packed_ulysses.py:85-215) in plain fp32:

  normed = RMSNorm(h)*w1*(1+scale_msa[idx]) + shift_msa[idx]
  q,k,v  = normed W_{q,k,v}^T + b;  q,k = rope(RMSNorm_D(.)*w_{q,k})
  (W>1)  pack destination-major -> all_to_all_single -> [S, hl, 3D]
  o      = softmax(q k^T / sqrt(D)) v   per local head, full sequence
  (W>1)  all_to_all_single back -> merge_heads -> [r, H*D]
  h      = h + gate_msa[idx] * (o W_o^T + b_o)
  normed = RMSNorm(h)*w2*(1+scale_mlp[idx]) + shift_mlp[idx]
  h      = h + gate_mlp[idx] * (act(normed W_1^T + b_1) W_2^T + b_2)    act = GELU-tanh | SwiGLU

Used as the fp32 reference of the block-level parity tests and as the timed
CPU baseline (benchmark config "CPU/gloo world_size=2").
"""

from __future__ import annotations

import time

import torch
import torch.distributed as dist
import torch.nn.functional as F


def _rms(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * weight


def _rope(x: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
    """x [r, H, D], cos/sin [r, rot]: rotate-half on the first rot columns (fusions.py:149-170)."""

    rot = cos.shape[-1]
    if rot == 0:
        return x
    half = rot // 2
    xr = x[..., :rot]
    rotated = torch.cat([-xr[..., half:], xr[..., :half]], dim=-1)
    out = xr * cos[:, None, :] + rotated * sin[:, None, :]
    return torch.cat([out, x[..., rot:]], dim=-1)


def attention_heads(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, block: int = 2048) -> torch.Tensor:
    """q/k/v [S, h, D] fp32 -> [S, h, D]; query-blocked softmax(q k^T/sqrt(D)) v."""

    s, h, d = q.shape
    scale = d ** -0.5
    out = torch.empty_like(q)
    kt = k.permute(1, 2, 0)  # [h, D, S]
    vh = v.permute(1, 0, 2)  # [h, S, D]
    for start in range(0, s, block):
        qb = q[start : start + block].permute(1, 0, 2)  # [h, b, D]
        scores = torch.matmul(qb, kt) * scale
        probs = torch.softmax(scores, dim=-1)
        out[start : start + block] = torch.matmul(probs, vh).permute(1, 0, 2)
    return out


def _exchange(x: torch.Tensor, in_splits: list[int], out_splits: list[int], group) -> torch.Tensor:
    out = torch.empty(sum(out_splits), dtype=x.dtype)
    dist.all_to_all_single(out, x.reshape(-1).contiguous(), output_split_sizes=out_splits,
                           input_split_sizes=in_splits, group=group)
    return out


def block_forward(p: dict[str, torch.Tensor], hidden: torch.Tensor, idx: torch.Tensor, cos: torch.Tensor,
                  sin: torch.Tensor, *, heads: int, head_dim: int, eps: float, qk_eps: float,
                  activation: str = "gelu-tanh", group=None, timings: dict | None = None) -> torch.Tensor:
    """One block on this rank's rows. ``p`` holds fp32 parameters keyed like
    H3TransformerBlock.state_dict(); hidden [r, d]; idx [r]; cos/sin [r, rot].
    With a gloo ``group`` of W ranks the attention runs packed-Ulysses style."""

    world = dist.get_world_size(group) if group is not None else 1
    rows, d = hidden.shape
    hl = heads // world
    t0 = time.perf_counter()
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = p["adaln_proj.table"].chunk(6, dim=-1)
    pick = lambda t: t.index_select(0, idx)  # noqa: E731
    normed = _rms(hidden, p["norm1.weight"], eps) * (1.0 + pick(scale_msa)) + pick(shift_msa)
    q = F.linear(normed, p["attn.to_q.weight"], p.get("attn.to_q.bias")).view(rows, heads, head_dim)
    k = F.linear(normed, p["attn.to_k.weight"], p.get("attn.to_k.bias")).view(rows, heads, head_dim)
    v = F.linear(normed, p["attn.to_v.weight"], p.get("attn.to_v.bias")).view(rows, heads, head_dim)
    q = _rope(_rms(q, p["attn.norm_q.weight"], qk_eps), cos, sin)
    k = _rope(_rms(k, p["attn.norm_k.weight"], qk_eps), cos, sin)
    if world > 1:
        counts = torch.zeros(world, dtype=torch.long)
        counts[dist.get_rank(group)] = rows
        dist.all_reduce(counts, group=group)
        counts = [int(c) for c in counts.tolist()]
        packed = torch.stack(
            [t.reshape(rows, world, hl, head_dim).permute(1, 0, 2, 3) for t in (q, k, v)], dim=3
        ).reshape(world, rows, hl, 3 * head_dim)
        block = hl * 3 * head_dim
        recv = _exchange(packed, [rows * block] * world, [c * block for c in counts], group)
        recv = recv.view(sum(counts), hl, 3, head_dim)
        qf, kf, vf = recv[:, :, 0], recv[:, :, 1], recv[:, :, 2]
    else:
        qf, kf, vf = q, k, v
    t1 = time.perf_counter()
    o = attention_heads(qf.contiguous(), kf.contiguous(), vf.contiguous())
    t2 = time.perf_counter()
    if world > 1:
        block = hl * head_dim
        back = _exchange(o, [c * block for c in counts], [rows * block] * world, group)
        o = back.view(world, rows, hl, head_dim).permute(1, 0, 2, 3).reshape(rows, heads * head_dim)
    else:
        o = o.reshape(rows, heads * head_dim)
    attn_out = F.linear(o, p["attn.to_out.0.weight"], p.get("attn.to_out.0.bias"))
    hidden = hidden + pick(gate_msa) * attn_out
    normed = _rms(hidden, p["norm2.weight"], eps) * (1.0 + pick(scale_mlp)) + pick(shift_mlp)
    projected = F.linear(normed, p["ff.net.0.proj.weight"], p.get("ff.net.0.proj.bias"))
    if activation == "gelu-tanh":
        activated = F.gelu(projected, approximate="tanh")
    else:
        value, gate = projected.chunk(2, -1)
        activated = value * F.silu(gate)
    ffn = F.linear(activated, p["ff.net.2.weight"], p.get("ff.net.2.bias"))
    out = hidden + pick(gate_mlp) * ffn
    t3 = time.perf_counter()
    if timings is not None:
        timings["attention_s"] = timings.get("attention_s", 0.0) + (t2 - t1)
        timings["other_s"] = timings.get("other_s", 0.0) + (t1 - t0) + (t3 - t2)
    return out


def project_kv(p: dict[str, torch.Tensor], hidden: torch.Tensor, idx: torch.Tensor, cos: torch.Tensor,
               sin: torch.Tensor, *, heads: int, head_dim: int, eps: float, qk_eps: float
               ) -> tuple[torch.Tensor, torch.Tensor]:
    """Keys (normed and rotated) and values [r, H, D] of ``hidden``'s rows, the
    k/v half of the attention projections of ``block_forward`` at W=1."""

    rows = hidden.shape[0]
    shift_msa, scale_msa = p["adaln_proj.table"].chunk(6, dim=-1)[:2]
    normed = _rms(hidden, p["norm1.weight"], eps) * (1.0 + scale_msa.index_select(0, idx)) \
        + shift_msa.index_select(0, idx)
    k = F.linear(normed, p["attn.to_k.weight"], p.get("attn.to_k.bias")).view(rows, heads, head_dim)
    v = F.linear(normed, p["attn.to_v.weight"], p.get("attn.to_v.bias")).view(rows, heads, head_dim)
    return _rope(_rms(k, p["attn.norm_k.weight"], qk_eps), cos, sin), v


def block_forward_rows(p: dict[str, torch.Tensor], hidden: torch.Tensor, idx: torch.Tensor, cos: torch.Tensor,
                       sin: torch.Tensor, k_all: torch.Tensor, v_all: torch.Tensor, start: int, *, heads: int,
                       head_dim: int, eps: float, qk_eps: float, activation: str = "gelu-tanh") -> torch.Tensor:
    """Rows [start, start + r) of one W=1 ``block_forward`` whose keys and values for
    every row of the sequence are in ``k_all`` / ``v_all`` [S, H, D].

    The chunk projects its own q, k and v and stores its k and v into ``k_all`` /
    ``v_all`` at its rows (the same values), then attends over all S keys. A pass over
    consecutive chunks that cover the sequence therefore does exactly the arithmetic of
    one full ``block_forward``: every projection once, every (query, key) pair once."""

    rows, d = hidden.shape
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = p["adaln_proj.table"].chunk(6, dim=-1)
    pick = lambda t: t.index_select(0, idx)  # noqa: E731
    normed = _rms(hidden, p["norm1.weight"], eps) * (1.0 + pick(scale_msa)) + pick(shift_msa)
    q = F.linear(normed, p["attn.to_q.weight"], p.get("attn.to_q.bias")).view(rows, heads, head_dim)
    k = F.linear(normed, p["attn.to_k.weight"], p.get("attn.to_k.bias")).view(rows, heads, head_dim)
    v = F.linear(normed, p["attn.to_v.weight"], p.get("attn.to_v.bias")).view(rows, heads, head_dim)
    q = _rope(_rms(q, p["attn.norm_q.weight"], qk_eps), cos, sin)
    k_all[start:start + rows] = _rope(_rms(k, p["attn.norm_k.weight"], qk_eps), cos, sin)
    v_all[start:start + rows] = v
    o = attention_heads(q.contiguous(), k_all, v_all).reshape(rows, heads * head_dim)
    attn_out = F.linear(o, p["attn.to_out.0.weight"], p.get("attn.to_out.0.bias"))
    hidden = hidden + pick(gate_msa) * attn_out
    normed = _rms(hidden, p["norm2.weight"], eps) * (1.0 + pick(scale_mlp)) + pick(shift_mlp)
    projected = F.linear(normed, p["ff.net.0.proj.weight"], p.get("ff.net.0.proj.bias"))
    if activation == "gelu-tanh":
        activated = F.gelu(projected, approximate="tanh")
    else:
        value, gate = projected.chunk(2, -1)
        activated = value * F.silu(gate)
    return hidden + pick(gate_mlp) * F.linear(activated, p["ff.net.2.weight"], p.get("ff.net.2.bias"))


def fp32_params(module: torch.nn.Module) -> dict[str, torch.Tensor]:
    return {name: value.detach().to("cpu", torch.float32) for name, value in module.state_dict().items()}
