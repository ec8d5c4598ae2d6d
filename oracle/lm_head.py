"""NVFP4 LM head on the CPU -- test infrastructure only.

Restates the reference's exact head (fast/fast_head.py:95-115, ``_nv4_fma``): logits = gs * sum_k x_k *
(e2m1 * e4m3), the global scale applied to the fp32 sum; greedy = argmax with the lowest index on ties
(torch.argmax semantics, which vLLM's greedy sampler uses).  Dots are evaluated in float64 and rounded
once to fp32, i.e. the exactly rounded fp32 dot; a GPU fp32 accumulation differs from it by a few ulp.
"""
from __future__ import annotations

import numpy as np

from .nvfp4 import dequantize_nvfp4


def lm_head_logits(x: np.ndarray, P: np.ndarray, S: np.ndarray, gs: float, chunk: int = 8192,
                   W: np.ndarray | None = None) -> np.ndarray:
    """x fp32 (bf16 values) [M, K] -> fp32 logits [M, V].  W: optional already dequantised head; the dots then
    run in W's precision (fp32: the reference's dequantise-to-fp32 matmul), else in float64."""
    if W is not None:
        return ((np.asarray(x, W.dtype) @ W.T).astype(np.float32) * np.float32(gs)).astype(np.float32)
    x64 = np.asarray(x, dtype=np.float64)
    V = P.shape[0]
    out = np.empty((x64.shape[0], V), dtype=np.float32)
    for a in range(0, V, chunk):
        w = dequantize_nvfp4(P[a:a + chunk], S[a:a + chunk]).astype(np.float64)
        out[:, a:a + chunk] = (x64 @ w.T).astype(np.float32)
    return (out * np.float32(gs)).astype(np.float32)


def argmax_lowest(logits: np.ndarray) -> np.ndarray:
    """Row argmax, lowest index among equal maxima."""
    return np.argmax(logits, axis=-1).astype(np.int32)


def top2_gap(logits: np.ndarray) -> np.ndarray:
    part = np.partition(logits, -2, axis=-1)
    return (part[..., -1] - part[..., -2]).astype(np.float64)
