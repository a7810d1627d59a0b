"""Dense attention processor for the MiniMax H3 attention modules.

Mirror of src/h3_flash/runtime/attention/dense_fa4.py. The reference plugs the
third-party FlashAttention-4 CuTe kernel into Diffusers' attention processor
slot; here the default kernel is this package's own tcgen05 attention
(``dense.flash_attn_func``, same [B, S, H, D] calling convention). An external
FA4 installation can still be selected exactly as in the reference
(``site_packages`` or ``H3_FA4_SITE_PACKAGES``), e.g. to measure it side by side.
"""

from __future__ import annotations

import functools
import os
import sys
from collections.abc import Callable
from importlib.metadata import distributions
from pathlib import Path
from typing import Any

from .dense import flash_attn_func as h3b_flash_attn_func


def load_fa4(site_packages: Path) -> Callable[..., Any]:
    """Load a FlashAttention-4 CuTe kernel from an isolated site-packages (dense_fa4.py:14-31)."""

    site = Path(site_packages).expanduser().resolve()
    package = site / "flash_attn" / "cute" / "__init__.py"
    if not package.is_file():
        raise RuntimeError(f"FlashAttention 4 CuTe package not found below {site}")
    site_text = str(site)
    if site_text not in sys.path:
        sys.path.append(site_text)
    import flash_attn

    fa4_namespace = str(site / "flash_attn")
    if fa4_namespace not in flash_attn.__path__:
        flash_attn.__path__.append(fa4_namespace)
    from flash_attn.cute import flash_attn_func

    return flash_attn_func


def fa4_provenance(site_packages: Path) -> dict[str, Any]:
    """dense_fa4.py:34-50."""

    site = Path(site_packages).expanduser().resolve()
    version = None
    for distribution in distributions(path=[str(site)]):
        name = distribution.metadata.get("Name", "").lower().replace("_", "-")
        if name == "flash-attn-4":
            version = distribution.version
            break
    if version is None:
        raise RuntimeError(f"flash-attn-4 metadata not found below {site}")
    return {"distribution": "flash-attn-4", "version": version, "site_packages": str(site)}


def h3b_provenance() -> dict[str, Any]:
    return {
        "distribution": "h3b",
        "kernel": "tcgen05/TMEM flash attention, sm_100a",
        "library": "libh3b.so",
    }


def _fa4_forward_op(
    _ctx: Any,
    query: Any,
    key: Any,
    value: Any,
    attention_mask: Any = None,
    dropout_p: float = 0.0,
    is_causal: bool = False,
    scale: float | None = None,
    enable_gqa: bool = False,
    return_lse: bool = False,
    _save_ctx: bool = False,
    _parallel_config: Any = None,
    *,
    kernel: Callable[..., Any],
) -> Any:
    """Forward op for Diffusers' context-parallel template (dense_fa4.py:53-81)."""

    del _ctx, _save_ctx, _parallel_config
    if attention_mask is not None or dropout_p != 0.0 or enable_gqa or return_lse:
        raise RuntimeError("H3 dense FA4 supports only unmasked inference attention")
    output = kernel(query, key, value, softmax_scale=scale, causal=is_causal)
    return output[0] if isinstance(output, tuple) else output


def _inference_only_backward(*_args: Any, **_kwargs: Any) -> Any:
    raise RuntimeError("H3 dense FA4 context parallelism is inference-only")


class DenseFA4MiniMaxH3Processor:
    """Dense H3 attention processor (dense_fa4.py:88-170). ``kernel`` defaults to the
    h3b tcgen05 kernel; ``site_packages`` (or H3_FA4_SITE_PACKAGES) selects FA4."""

    _attention_backend = None
    _parallel_config = None

    def __init__(self, site_packages: Path | None = None, *, kernel: Callable[..., Any] | None = None) -> None:
        if kernel is None:
            if site_packages is None:
                configured = os.environ.get("H3_FA4_SITE_PACKAGES")
                site_packages = Path(configured) if configured else None
            kernel = load_fa4(site_packages) if site_packages is not None else h3b_flash_attn_func
        self.kernel = kernel
        self.calls = 0

    def __call__(self, attn: Any, hidden_states: Any, rotary_emb: tuple[Any, Any] | None = None,
                 attention_mask: Any | None = None) -> Any:
        if attention_mask is not None:
            raise RuntimeError("dense FA4 profile requires the official padless sequence")
        if attn.fused_projections:
            query, key, value = attn.to_qkv(hidden_states).chunk(3, dim=-1)
        else:
            query = attn.to_q(hidden_states)
            key = attn.to_k(hidden_states)
            value = attn.to_v(hidden_states)
        query = query.unflatten(-1, (attn.heads, -1))
        key = key.unflatten(-1, (attn.heads, -1))
        value = value.unflatten(-1, (attn.heads, -1))
        if rotary_emb is not None:
            from ..kernels.fusions import fused_qknorm_rope

            cos, sin = rotary_emb
            query = fused_qknorm_rope(query, attn.norm_q.weight, cos, sin, attn.norm_q.eps)
            key = fused_qknorm_rope(key, attn.norm_k.weight, cos, sin, attn.norm_k.eps)
        else:
            query = attn.norm_q(query)
            key = attn.norm_k(key)
        if self._parallel_config is None:
            output = self.kernel(query, key, value, causal=False)
        else:
            from diffusers.models.attention_dispatch import _templated_context_parallel_attention

            output = _templated_context_parallel_attention(
                query, key, value, None, 0.0, False, None, False, False,
                forward_op=functools.partial(_fa4_forward_op, kernel=self.kernel),
                backward_op=_inference_only_backward,
                _parallel_config=self._parallel_config,
            )
        if isinstance(output, tuple):
            output = output[0]
        self.calls += 1
        output = output.flatten(2, 3).type_as(query)
        output = attn.to_out[0](output)
        return attn.to_out[1](output)


def install_dense_fa4(transformer: Any, site_packages: Path | None = None) -> dict[str, Any]:
    """Install one shared kernel on every H3 attention module (dense_fa4.py:173-194).
    Modules are recognised by their H3 attention attribute layout."""

    kernel = load_fa4(site_packages) if site_packages is not None else h3b_flash_attn_func
    processors = []
    for module in transformer.modules():
        if _is_h3_attention(module):
            processor = DenseFA4MiniMaxH3Processor(kernel=kernel)
            processor._parallel_config = getattr(transformer, "_parallel_config", None)
            if hasattr(module, "set_processor"):
                module.set_processor(processor)
            else:
                module.processor = processor
            processors.append(processor)
    if not processors:
        raise RuntimeError("no MiniMax H3 attention modules found")
    transformer._h3_flash_dense_fa4_processors = processors
    provenance = fa4_provenance(site_packages) if site_packages is not None else h3b_provenance()
    return {"backend": "flash_attention_4" if site_packages is not None else "h3b_tcgen05",
            "semantics": "dense", "processor_count": len(processors), **provenance}


def _is_h3_attention(module: Any) -> bool:
    try:
        from diffusers.models.transformers.transformer_minimax_h3 import MiniMaxH3Attention

        if isinstance(module, MiniMaxH3Attention):
            return True
    except ImportError:
        pass
    return all(hasattr(module, name) for name in ("to_q", "to_k", "to_v", "norm_q", "norm_k", "to_out", "heads"))
