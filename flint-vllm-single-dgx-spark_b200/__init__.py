"""B200-native (sm_100a) NVFP4 batch-1 decode hot path for Flint-class MoE models.

Modules mirror the reference recipe's decode entry points:

* ``fast_head``      -- NVFP4 LM head (logits, argmax, top-k/top-p sampling)   [fast/fast_head.py]
* ``fp4moe_decode``  -- router + top-k, SwiGLU experts, weighted sum           [fast/fp4moe_decode.py]
* ``patch_align``    -- deterministic moe_align_block_size                      [fast/patch_align.py]
* ``attn_gemv``      -- fused add+RMSNorm+QKV GEMV+q/k-norm+RoPE+KV write, O GEMV [fast/attn_gemv.py]
* ``decode_attention`` -- paged split-K GQA decode attention                    [PR ops/decode_attention.py]

All compute runs in ``libflint_b200.so`` (hand-written CUDA for sm_100a, C ABI in ``include/flint_b200.h``),
registered as ``torch.ops.flint_b200.*``.  There is no CPU fallback.
"""
from . import _lib  # noqa: F401
from . import ops  # noqa: F401  (registers torch.ops.flint_b200.*)

__all__ = ["_lib", "ops"]
