"""CPU oracle for the FP8 attention hot path — TEST INFRASTRUCTURE ONLY.

This package restates, in numpy (and C for the timed CPU port), the
reference's algorithm for the path:

  * ``quantize``  — ``_per_bh_scale`` / ``_quantize``
    (kernels/triton_kernels/fp8_flash_attn_hopper.py:374-398) and the
    per-128-token-block extension of the same formula;
  * ``attention`` — the fused kernel's tile loop
    (fp8_flash_attn_hopper.py:197-338), the fp32 attention over dequantised
    e4m3 inputs that defines the accuracy tolerance, and the shared-prefix
    candidate-decode semantics;
  * ``fp8``       — e4m3fn / bf16 encode and decode.

It is the checker, never the product: only ``tests/``, ``__graft_entry__.smoke``
and ``bench.py``'s CPU-baseline leg may import it.  The pins that tie it to the
reference live in ``tests/golden`` (bytes produced by the reference's own
functions, imported from its source tree by ``tests/golden/make_golden.py``).
"""
