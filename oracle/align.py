"""Deterministic moe_align_block_size on the CPU -- test infrastructure only.

Restates ``_deterministic_align`` (reference fast/patch_align.py:11-30): the
outputs of vLLM's ``moe_align_block_size`` with the routes of each expert in
ascending route order instead of atomic-arrival order.
"""
from __future__ import annotations

import numpy as np


def align_sizes(numel: int, num_experts: int, block_size: int) -> tuple[int, int]:
    """Buffer lengths of vLLM's caller (moe_align_block_size.py: max_num_tokens_padded, max_num_m_blocks)."""
    mx = numel + num_experts * (block_size - 1)
    if numel < num_experts:
        mx = min(numel * block_size, mx)
    return mx, -(-mx // block_size)


def deterministic_align(topk_ids: np.ndarray, num_experts: int, block_size: int,
                        n_sorted: int | None = None, n_blocks: int | None = None):
    """-> (sorted_ids i32 [n_sorted], expert_ids i32 [n_blocks], num_tokens_post_pad i32 [1]).

    fast/patch_align.py:11-30 step by step: counts = bincount(ids);
    padded = ceil(count/B)*B; pad_end = cumsum; routes of each expert placed
    in ascending route index at pad_start[e] + rank; unused slots = numel;
    expert_ids[blk] = searchsorted(pad_end, blk*B, right) or -1 past the last
    expert; num_tokens_post_pad = pad_end[-1]."""
    flat = np.asarray(topk_ids).reshape(-1).astype(np.int64)
    n = flat.size
    if n_sorted is None or n_blocks is None:
        n_sorted, n_blocks = align_sizes(n, num_experts, block_size)
    if n and (flat.min() < 0 or flat.max() >= num_experts):
        raise ValueError("expert id out of range")
    counts = np.bincount(flat, minlength=num_experts).astype(np.int64)
    padded = (counts + block_size - 1) // block_size * block_size
    pad_end = np.cumsum(padded)
    pad_start = pad_end - padded
    cnt_start = np.cumsum(counts) - counts
    si = np.argsort(flat, kind="stable")
    sv = flat[si]
    rank = np.arange(n) - cnt_start[sv]
    sorted_ids = np.full(n_sorted, n, dtype=np.int32)
    sorted_ids[pad_start[sv] + rank] = si.astype(np.int32)
    blk_start = np.arange(n_blocks, dtype=np.int64) * block_size
    e = np.searchsorted(pad_end, blk_start, side="right")
    expert_ids = np.where(e >= num_experts, -1, e).astype(np.int32)
    ntp = np.array([pad_end[-1] if num_experts else 0], dtype=np.int32)
    return sorted_ids, expert_ids, ntp
