"""Dense attention processor for the MiniMax H3 attention modules.

Interface of ``h3_flash.runtime.attention.dense_fa4`` (src/h3_flash/runtime/attention/
dense_fa4.py:14-194): ``load_fa4``, ``fa4_provenance``, ``DenseFA4MiniMaxH3Processor``
(``site_packages``, ``kernel=``, ``.calls``, the Diffusers processor call) and
``install_dense_fa4``, with the same errors.

Design. The processor is three steps over an attention module's own weights:
``_heads`` projects the hidden states to q, k, v in [B, S, H, D]; ``_normalise`` applies
the per-head RMSNorm and, given rotary tables, RoPE (this package's fused QK-norm+RoPE
kernel); ``_attend`` runs the selected dense kernel, directly or, when the transformer
has Diffusers' context parallelism configured, as the forward op of Diffusers'
context-parallel template. The kernel is a ``_Kernel`` choice: this package's tcgen05
attention (``dense.flash_attn_func``) by default, or FlashAttention-4's CuTe kernel
loaded from an isolated site-packages (``site_packages`` or $H3_FA4_SITE_PACKAGES),
which is what the reference plugs in, e.g. to measure the two side by side.
"""

from __future__ import annotations

import functools
import os
import sys
from collections.abc import Callable
from dataclasses import dataclass
from importlib.metadata import distributions
from pathlib import Path
from typing import Any

from .dense import flash_attn_func as h3b_flash_attn_func

FA4_DISTRIBUTION = "flash-attn-4"


def load_fa4(site_packages: Path) -> Callable[..., Any]:
    """FlashAttention-4's ``flash_attn.cute.flash_attn_func`` from an isolated
    site-packages directory, made importable beside any other ``flash_attn``."""

    root = Path(site_packages).expanduser().resolve()
    if not (root / "flash_attn" / "cute" / "__init__.py").is_file():
        raise RuntimeError(f"FlashAttention 4 CuTe package not found below {root}")
    if str(root) not in sys.path:
        sys.path.append(str(root))
    import flash_attn

    extra = str(root / "flash_attn")
    if extra not in flash_attn.__path__:  # the CuTe subpackage lives in this tree only
        flash_attn.__path__.append(extra)
    from flash_attn.cute import flash_attn_func

    return flash_attn_func


def fa4_provenance(site_packages: Path) -> dict[str, Any]:
    """Distribution name, version and location of the FA4 install at ``site_packages``."""

    root = Path(site_packages).expanduser().resolve()
    versions = [d.version for d in distributions(path=[str(root)])
                if d.metadata.get("Name", "").lower().replace("_", "-") == FA4_DISTRIBUTION]
    if not versions:
        raise RuntimeError(f"flash-attn-4 metadata not found below {root}")
    return {"distribution": FA4_DISTRIBUTION, "version": versions[0], "site_packages": str(root)}


def h3b_provenance() -> dict[str, Any]:
    return {"distribution": "h3b", "kernel": "tcgen05/TMEM flash attention, sm_100a", "library": "libh3b.so"}


@dataclass(frozen=True)
class _Kernel:
    """A dense attention kernel with the [B, S, H, D] ``flash_attn_func`` calling
    convention, and where it came from."""

    fn: Callable[..., Any]
    backend: str
    site_packages: Path | None = None

    @classmethod
    def select(cls, site_packages: Path | None) -> _Kernel:
        if site_packages is None:
            return cls(h3b_flash_attn_func, "h3b_tcgen05")
        return cls(load_fa4(site_packages), "flash_attention_4", Path(site_packages))

    def provenance(self) -> dict[str, Any]:
        return fa4_provenance(self.site_packages) if self.site_packages is not None else h3b_provenance()


def _fa4_forward_op(_ctx: Any, query: Any, key: Any, value: Any, attention_mask: Any = None,
                    dropout_p: float = 0.0, is_causal: bool = False, scale: float | None = None,
                    enable_gqa: bool = False, return_lse: bool = False, _save_ctx: bool = False,
                    _parallel_config: Any = None, *, kernel: Callable[..., Any]) -> Any:
    """Forward op handed to Diffusers' context-parallel template (its op signature);
    serves unmasked inference attention only."""

    unsupported = attention_mask is not None or dropout_p != 0.0 or enable_gqa or return_lse
    if unsupported:
        raise RuntimeError("H3 dense FA4 supports only unmasked inference attention")
    result = kernel(query, key, value, softmax_scale=scale, causal=is_causal)
    return result[0] if isinstance(result, tuple) else result


def _inference_only_backward(*_args: Any, **_kwargs: Any) -> Any:
    raise RuntimeError("H3 dense FA4 context parallelism is inference-only")


def _heads(attn: Any, hidden_states: Any) -> tuple[Any, Any, Any]:
    """q, k, v [B, S, H, D] from the module's (fused or separate) projections."""

    if attn.fused_projections:
        projected = attn.to_qkv(hidden_states).chunk(3, dim=-1)
    else:
        projected = (attn.to_q(hidden_states), attn.to_k(hidden_states), attn.to_v(hidden_states))
    return tuple(t.unflatten(-1, (attn.heads, -1)) for t in projected)


def _normalise(attn: Any, query: Any, key: Any, rotary_emb: tuple[Any, Any] | None) -> tuple[Any, Any]:
    """Per-head RMSNorm of q and k, with RoPE when rotary tables are given."""

    if rotary_emb is None:
        return attn.norm_q(query), attn.norm_k(key)
    from ..kernels.fusions import fused_qknorm_rope

    cos, sin = rotary_emb
    return (fused_qknorm_rope(query, attn.norm_q.weight, cos, sin, attn.norm_q.eps),
            fused_qknorm_rope(key, attn.norm_k.weight, cos, sin, attn.norm_k.eps))


class DenseFA4MiniMaxH3Processor:
    """Dense H3 attention processor. ``kernel`` defaults to this package's tcgen05
    attention; ``site_packages`` (or $H3_FA4_SITE_PACKAGES) selects FlashAttention-4."""

    _attention_backend = None
    _parallel_config = None

    def __init__(self, site_packages: Path | None = None, *, kernel: Callable[..., Any] | None = None) -> None:
        if kernel is None:
            configured = site_packages or os.environ.get("H3_FA4_SITE_PACKAGES") or None
            kernel = _Kernel.select(Path(configured) if configured else None).fn
        self.kernel = kernel
        self.calls = 0

    def _attend(self, query: Any, key: Any, value: Any) -> Any:
        if self._parallel_config is None:
            return self.kernel(query, key, value, causal=False)
        from diffusers.models.attention_dispatch import _templated_context_parallel_attention

        return _templated_context_parallel_attention(
            query, key, value, None, 0.0, False, None, False, False,
            forward_op=functools.partial(_fa4_forward_op, kernel=self.kernel),
            backward_op=_inference_only_backward, _parallel_config=self._parallel_config)

    def __call__(self, attn: Any, hidden_states: Any, rotary_emb: tuple[Any, Any] | None = None,
                 attention_mask: Any | None = None) -> Any:
        if attention_mask is not None:
            raise RuntimeError("dense FA4 profile requires the official padless sequence")
        query, key, value = _heads(attn, hidden_states)
        query, key = _normalise(attn, query, key, rotary_emb)
        output = self._attend(query, key, value)
        if isinstance(output, tuple):
            output = output[0]
        self.calls += 1
        projected = attn.to_out[0](output.flatten(2, 3).type_as(query))
        return attn.to_out[1](projected)


def _is_h3_attention(module: Any) -> bool:
    """Diffusers' MiniMaxH3Attention when Diffusers is present, else any module with
    its attribute layout (this package's H3 stand-in)."""

    try:
        from diffusers.models.transformers.transformer_minimax_h3 import MiniMaxH3Attention
    except ImportError:
        MiniMaxH3Attention = None  # noqa: N806
    if MiniMaxH3Attention is not None and isinstance(module, MiniMaxH3Attention):
        return True
    return all(hasattr(module, name) for name in ("to_q", "to_k", "to_v", "norm_q", "norm_k", "to_out", "heads"))


def install_dense_fa4(transformer: Any, site_packages: Path | None = None) -> dict[str, Any]:
    """Give every H3 attention module of ``transformer`` a dense processor sharing one
    kernel (dense_fa4.py:173-194); returns the installation's provenance."""

    choice = _Kernel.select(site_packages)
    processors = []
    for module in filter(_is_h3_attention, transformer.modules()):
        processor = DenseFA4MiniMaxH3Processor(kernel=choice.fn)
        processor._parallel_config = getattr(transformer, "_parallel_config", None)
        setter = getattr(module, "set_processor", None)
        if setter is not None:
            setter(processor)
        else:
            module.processor = processor
        processors.append(processor)
    if not processors:
        raise RuntimeError("no MiniMax H3 attention modules found")
    transformer._h3_flash_dense_fa4_processors = processors
    return {"backend": choice.backend, "semantics": "dense", "processor_count": len(processors),
            **choice.provenance()}
