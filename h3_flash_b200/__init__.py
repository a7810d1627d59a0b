"""B200-native (sm_100a) rebuild of H3-Flash's LOSSLESS packed-Ulysses DiT block hot path.

Import paths mirror the reference package: ``h3_flash.runtime.X`` becomes
``h3_flash_b200.runtime.X``. Kernels live in ``lib/libh3b.so`` (C ABI in
``include/h3b.h``), loaded through ctypes; there is no CPU fallback.
"""

__version__ = "0.1.0"
