"""Glue between torch tensors and the libh3b C ABI: pointers, strides, streams, checks."""

from __future__ import annotations

import torch

from . import _lib


def stream_of(tensor: torch.Tensor) -> int:
    """Raw cudaStream_t of the current torch stream on the tensor's device."""

    return torch.cuda.current_stream(tensor.device).cuda_stream


def require_cuda(op: str, *tensors: torch.Tensor) -> None:
    """All tensors must be CUDA tensors on one device. There is no CPU path."""

    device = None
    for t in tensors:
        if not isinstance(t, torch.Tensor) or not t.is_cuda:
            raise RuntimeError(
                f"{op}: h3b kernels run on CUDA tensors only (got "
                f"{'a non-tensor' if not isinstance(t, torch.Tensor) else t.device})"
            )
        if device is None:
            device = t.device
        elif t.device != device:
            raise RuntimeError(f"{op}: tensors live on different devices ({device}, {t.device})")


def require_bf16(op: str, *tensors: torch.Tensor) -> None:
    for t in tensors:
        if t.dtype != torch.bfloat16:
            raise TypeError(f"{op}: expected bfloat16 tensors, got {t.dtype}")


def rows_view(t: torch.Tensor) -> torch.Tensor:
    """Flatten to [rows, cols] without copying when the last dim is contiguous and
    the leading dims collapse; otherwise copy (the reference's reshape().contiguous())."""

    cols = t.shape[-1]
    if t.dim() == 2 and t.stride(-1) == 1:
        return t
    try:
        flat = t.view(-1, cols)
        if flat.stride(-1) == 1:
            return flat
    except RuntimeError:
        pass
    return t.reshape(-1, cols).contiguous()


def table_rows(table: torch.Tensor) -> tuple[torch.Tensor, int]:
    """AdaLN table addressed by row: returns (tensor with unit last stride, row stride).
    A 1-D vector is a one-row table (row stride 0)."""

    if table.stride(-1) != 1:
        table = table.contiguous()
    if table.dim() == 1:
        return table, 0
    if table.dim() != 2:
        table = table.reshape(-1, table.shape[-1])
        if table.stride(-1) != 1:
            table = table.contiguous()
    return table, table.stride(0)


def index64(index: torch.Tensor | None, device: torch.device) -> torch.Tensor:
    if index is None:
        return torch.zeros(1, dtype=torch.int64, device=device)
    index = index.reshape(-1)
    if index.dtype != torch.int64:
        index = index.to(torch.int64)
    if index.device != device:
        index = index.to(device)
    return index.contiguous()


def ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


def call(name: str, *args) -> None:
    _lib.call(name, *args)
