"""CPU oracle for the batch-1 NVFP4 decode hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy, the reference recipe's dequantise-to-fp32
arithmetic for every op on the decode path (NVFP4 format, router + top-k,
SwiGLU experts, deterministic moe_align, q/k-norm + RoPE + paged decode
attention, LM head + argmax / top-k / top-p).  Each function cites the
reference file:line it follows.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline /
``--impl reference`` legs may import it, and only as the checker or as the
timed CPU baseline.  The product (the ``flint-vllm-single-dgx-spark_b200``
package) never imports it and has no CPU fallback.

Parity pinning: the format functions (``dequantize_nvfp4``,
``repack_gguf_nvfp4``) and ``deterministic_align`` are pinned bit-exactly
against fixtures produced by the reference's own Python functions
(``tests/golden/make_golden.py`` extracts them from the reference source and
runs them).  The kernel rounding rules (router, experts, attention, head)
have no golden vectors in the reference (it ships no tests); they are pinned
by the reference's documented rounding points cited in each function.
"""
