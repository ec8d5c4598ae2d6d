"""Deterministic ``moe_align_block_size`` -- drop-in for the reference's ``fast/patch_align.py``.

The reference splices a torch implementation (``_deterministic_align``, fast/patch_align.py:11-30) into vLLM's
``moe_align_block_size.py`` and calls it for >= ``VLLM_DET_MOE_ALIGN_MIN_TOKENS`` tokens (lines 32-43).  Here the
same function (same name, arguments and in-place outputs) is one CUDA kernel, and ``moe_align_block_size``
reproduces the vLLM caller's buffer sizing (installed vllm/model_executor/layers/fused_moe/moe_align_block_size.py).
"""
from __future__ import annotations

import os

import torch

from . import ops as _ops  # noqa: F401

DET_ALIGN = os.environ.get("VLLM_DET_MOE_ALIGN", "0") == "1"
DET_MIN_TOKENS = int(os.environ.get("VLLM_DET_MOE_ALIGN_MIN_TOKENS", "9"))


def align_sizes(numel: int, num_experts: int, block_size: int, pad_sorted_ids: bool = False) -> tuple[int, int]:
    """(len(sorted_ids), len(expert_ids)) as vLLM's moe_align_block_size allocates them."""
    mx = numel + num_experts * (block_size - 1)
    if pad_sorted_ids:
        mx = -(-mx // block_size) * block_size
    if numel < num_experts:
        mx = min(numel * block_size, mx)
    return mx, -(-mx // block_size)


def _deterministic_align(topk_ids, num_experts, block_size, sorted_ids, expert_ids, num_tokens_post_pad):
    """Fills sorted_ids, expert_ids and num_tokens_post_pad in place with one kernel launch (no host sync).

    The buffers follow vLLM's moe_align_block_size contract; the one difference is the placement of an expert's
    routes inside its padded span, which is by increasing flat route index here rather than by the order in which
    atomics happened to land, so every run produces identical buffers (fast/patch_align.py:11-30)."""
    torch.ops.flint_b200.moe_align(topk_ids, int(num_experts), int(block_size), sorted_ids, expert_ids,
                                   num_tokens_post_pad)


def moe_align_block_size(topk_ids: torch.Tensor, block_size: int, num_experts: int, pad_sorted_ids: bool = False):
    """-> (sorted_token_ids, expert_ids, num_tokens_post_padded), deterministic, same contract as vLLM's."""
    n_sorted, n_blocks = align_sizes(topk_ids.numel(), num_experts, block_size, pad_sorted_ids)
    dev = topk_ids.device
    sorted_ids = torch.empty((n_sorted,), dtype=torch.int32, device=dev)
    expert_ids = torch.empty((n_blocks,), dtype=torch.int32, device=dev)
    ntp = torch.empty((1,), dtype=torch.int32, device=dev)
    _deterministic_align(topk_ids, num_experts, block_size, sorted_ids, expert_ids, ntp)
    return sorted_ids, expert_ids, ntp
