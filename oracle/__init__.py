"""CPU oracle for the LOSSLESS packed-Ulysses DiT block — TEST INFRASTRUCTURE ONLY.

This package restates, on the CPU, the arithmetic of the reference
(fluxmatrix/h3-flash) hot path so that the CUDA kernels of ``h3_flash_b200``
can be checked against it:

* ``bf16``           — bfloat16 bit helpers (round-to-nearest-even, ulp distance).
* ``fusions_ref``    — the reference Triton fusions (src/h3_flash/runtime/kernels/fusions.py)
                       and the benchmark eager ops, in numpy fp32/fp64.
* ``relayout_ref``   — pack / merge relayouts (src/h3_flash/runtime/parallel/relayout.py).
* ``attention_ref``  — dense softmax attention in fp32/fp64 (the SDPA call at
                       src/h3_flash/runtime/parallel/packed_ulysses.py:201-209).
* ``block_ref``      — the whole block forward in torch fp32 on CPU, single process or as
                       W gloo ranks with the packed all-to-all
                       (kernels/transformer.py:50-126, packed_ulysses.py:85-215).

It is pinned against golden vectors produced by running the reference's own
Triton kernels through the Triton CPU interpreter (tests/golden/make_golden.py).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import it, and only as the checker or the timed CPU baseline. The product
package never imports it.
"""
