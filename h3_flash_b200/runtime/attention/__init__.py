"""Dense attention backends (h3b tcgen05 kernel; FA4 selectable)."""

from .dense_fa4 import DenseFA4MiniMaxH3Processor, install_dense_fa4

__all__ = ["DenseFA4MiniMaxH3Processor", "install_dense_fa4"]
