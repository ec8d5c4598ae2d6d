"""CPU restatement of the multi-GPU exchange of the sharded decode (expert-parallel MoE, vocabulary-sharded head).

TEST INFRASTRUCTURE ONLY: used by tests/ (gloo ranks on CPU) to check the exchange arithmetic the GPU path uses:

* Data-parallel streams (one per rank): the ranks all-gather their tokens, route every token identically, each rank
  produces the rows of the routes whose expert is local (zeros elsewhere) for all tokens, and a reduce-scatter sum
  hands every rank its own token's rows -- exact for the same reason as below -- which it combines in slot order.
* MoE: rank r holds experts [r*E/N, (r+1)*E/N); for one token it produces y_slots [topk, H] with the bf16 output of
  each routed slot whose expert is local and zeros elsewhere; the element-wise sum over ranks has exactly one
  non-zero term per element (exact), and out = bf16(sum_s tw[s] * y[s]) in slot order with fp32 FMAs -- the same
  arithmetic as the single-GPU MoE block (fast/fp4moe_mar.cu:224-231 rounding of the weighted sum).
* Head: rank r holds rows [r*V/N, (r+1)*V/N); its best argmax key is (order-preserving fp32 image << 32 |
  (0xFFFFFFFF - global id)) with the top bit flipped so that a signed int64 MAX over ranks orders keys as the
  unsigned comparison does; the maximum key carries the lowest id among the largest logits (vLLM's greedy pick).
* Sampled head: rank r's shard contributes its own top-k (global ids, fp32 logits, value descending, lowest id first
  on ties); the top-k of the gathered candidates under the same order is the full vocabulary's top-k, since every
  member of the global top-k is in its own shard's top-k, so the draw over them equals the one-GPU draw.
"""
from __future__ import annotations

import numpy as np


def expert_range(rank: int, world: int, E: int) -> tuple[int, int]:
    return rank * E // world, (rank + 1) * E // world


def vocab_range(rank: int, world: int, V: int) -> tuple[int, int]:
    return rank * V // world, (rank + 1) * V // world


def local_slot_rows(y: np.ndarray, ids: np.ndarray, lo: int, hi: int) -> np.ndarray:
    """y [topk, H] (float32 holding bf16 values) with the rows of non-local experts zeroed."""
    out = np.array(y, np.float32, copy=True)
    out[(ids < lo) | (ids >= hi)] = 0.0
    return out


def combine(y: np.ndarray, tw: np.ndarray) -> np.ndarray:
    """bf16(sum_s tw[s] * y[s]) in slot order, fp32 FMA, as float32 bf16 values."""
    import torch
    acc = torch.zeros(y.shape[1], dtype=torch.float32)
    for s in range(y.shape[0]):
        acc = torch.addcmul(acc, torch.from_numpy(np.float32(tw[s]) * np.ones(1, np.float32)), torch.from_numpy(y[s]))
    return acc.to(torch.bfloat16).float().numpy()


def order_key(v: float) -> int:
    u = int(np.float32(v).view(np.uint32))
    return (~u & 0xFFFFFFFF) if u & 0x80000000 else (u | 0x80000000)


def shard_key(logits: np.ndarray, base: int) -> int:
    """Signed-comparable argmax key of one shard's fp32 logits (global ids from base)."""
    best = 0
    for i, v in enumerate(np.asarray(logits, np.float32)):
        k = (order_key(v) << 32) | (0xFFFFFFFF - (base + i))
        best = max(best, k)
    k = best ^ (1 << 63)
    return k - (1 << 64) if k >= (1 << 63) else k


def key_token(k: int) -> int:
    return 0xFFFFFFFF - ((k + (1 << 64)) % (1 << 64) & 0xFFFFFFFF)


def shard_candidates(logits: np.ndarray, base: int, k: int) -> tuple[np.ndarray, np.ndarray]:
    """The k best (global id, fp32 logit) pairs of one vocabulary shard, value descending, lowest id first on ties:
    what lm_head_sample_shard writes for one row."""
    v = np.asarray(logits, np.float32)
    order = np.lexsort((np.arange(v.size), -v.astype(np.float64)))[:k]
    return (order + base).astype(np.int64), v[order]


def merge_candidates(ids: np.ndarray, vals: np.ndarray, k: int) -> tuple[np.ndarray, np.ndarray]:
    """The k best of the gathered candidates of all shards ([R, k] each) under the same order (value descending,
    lowest global id first): what sample_merge selects before its draw.  Every member of the global top-k is in its
    own shard's top-k, so the result equals the top-k of the whole vocabulary."""
    ids, vals = np.asarray(ids).reshape(-1), np.asarray(vals, np.float32).reshape(-1)
    order = np.lexsort((ids, -vals.astype(np.float64)))[:k]
    return ids[order], vals[order]
