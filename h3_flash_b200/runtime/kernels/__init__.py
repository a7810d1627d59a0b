"""Numerically equivalent sm_100a kernels used by the lossless profiles."""

from .transformer import install_transformer_fusions

__all__ = ["install_transformer_fusions"]
