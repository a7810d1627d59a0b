"""Runtime mechanisms: fused kernels, packed Ulysses parallelism, dense attention."""
