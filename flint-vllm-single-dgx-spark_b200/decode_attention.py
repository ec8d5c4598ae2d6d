"""Paged split-K decode attention -- drop-in for the Flint PR's ``flint_decode_attention`` (patch:2539-2605).

``flint_decode_attention(q, kv_cache, block_tables, seq_lens, sinks, window, scale, out) -> out`` with the same
arguments: q bf16 [B, heads, 128]; kv_cache FlashInfer HND bf16 [blocks, kv_heads, 16, 256] (K | V);
block_tables int32 [B, max_blocks]; seq_lens int32 [B] (including the current token; 0 writes zeros);
sinks fp32 [heads] or None; window None for full attention; out bf16 [B, heads, 128].
CUDA-graph safe: the launch shape depends only on the batch size; lengths and tables are read on the device.
"""
from __future__ import annotations

from . import ops as _ops


def flint_decode_attention(q, kv_cache, block_tables, seq_lens, sinks, window, scale, out):
    B = q.shape[0]
    if B == 0:
        return out
    splits = _ops.attention_splits(B, kv_cache.shape[1])
    import torch
    torch.ops.flint_b200.decode_attention(q, kv_cache, block_tables, seq_lens, sinks, int(window or 0), float(scale),
                                          out, splits)
    return out
