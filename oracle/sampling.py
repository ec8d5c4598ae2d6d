"""CPU checker for the sampling LM head: seeded temperature -> top-k -> top-p -> draw.

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's CPU arms, never by the
product path.

The reference hands its fp32 logits (fast/fast_head.py:360-381) to vLLM's sampler, an external dependency (vLLM
0.32.1rc1.dev197 in the reference image, Dockerfile:3) whose random draw is not reproducible outside vLLM.  The
top-p rule below is vLLM's (sort ascending, drop while the cumulative probability is <= 1 - p, always keep the
best); the top-k selection keeps ties at the lowest token id; the draw is this library's own seeded rule
(Philox4x32-10 keyed by the stream's seed, counter {step, row, 0, 0}, inverse CDF over the kept candidates).  So
sampled parity is pinned to this restatement, not to the reference: the Philox stream is pinned to the published
Random123 known-answer vectors (tests/test_oracle_golden.py), and the draw is checked against the kernel's own
candidates, weights and uniform.

Every float step follows the kernel's float32 order (w_i = exp((c_i - c_0) / T), suffix sums from the smallest,
prefix sums from the largest); numpy's float32 exp may differ from CUDA's expf in the last bit, so callers compare
tokens with `margin` (how close the draw and the top-p cut came to a boundary).
"""
from __future__ import annotations

import numpy as np

MASK = 0xFFFFFFFF
PHILOX_M = (0xD2511F53, 0xCD9E8D57)
PHILOX_W = (0x9E3779B9, 0xBB67AE85)


def philox4x32_10(ctr, key) -> list[int]:
    """Philox4x32-10 (Salmon, Moraes, Dror, Shaw, SC'11): counter [4] u32, key [2] u32 -> [4] u32."""
    c = [int(v) & MASK for v in ctr]
    k0, k1 = int(key[0]) & MASK, int(key[1]) & MASK
    for r in range(10):
        if r:
            k0 = (k0 + PHILOX_W[0]) & MASK
            k1 = (k1 + PHILOX_W[1]) & MASK
        p0 = PHILOX_M[0] * c[0]
        p1 = PHILOX_M[1] * c[2]
        c = [((p1 >> 32) ^ c[1] ^ k0) & MASK, p1 & MASK, ((p0 >> 32) ^ c[3] ^ k1) & MASK, p0 & MASK]
    return c


def uniform(seed: int, step: int, row: int) -> np.float32:
    """u in [0, 1): the top 24 bits of the first Philox word, key = the 64 seed bits."""
    s = int(seed) & ((1 << 64) - 1)
    x = philox4x32_10([step, row, 0, 0], [s & MASK, s >> 32])[0]
    return np.float32((x >> 8) * 2.0 ** -24)


def topk_ids(logits: np.ndarray, k: int) -> np.ndarray:
    """Ids of the k largest fp32 logits, value descending, lowest id first on ties."""
    v = np.asarray(logits, np.float32)
    order = np.lexsort((np.arange(v.size), -v.astype(np.float64)))
    return order[:k]


def sample_row(logits: np.ndarray, top_k: int, temperature: float, top_p: float, seed: int, step: int, row: int):
    """The kernel's rule on one row of fp32 logits; returns a dict with the candidates, weights, kept count, the
    uniform, the chosen token and a relative margin to the nearest decision boundary."""
    ids = topk_ids(logits, top_k)
    c = np.asarray(logits, np.float32)[ids]
    T = np.float32(temperature)
    w = np.exp((c - c[0]) / T).astype(np.float32)
    K = len(w)
    S = np.zeros(K, np.float32)
    s = np.float32(0)
    for j in range(K - 1, -1, -1):
        s = np.float32(s + w[j])
        S[j] = s
    thr = np.float32(np.float32(1.0) - np.float32(top_p)) * S[0]
    J = 1
    while J < K and S[J] > thr:
        J += 1
    P = np.float32(0)
    for i in range(J):
        P = np.float32(P + w[i])
    u = uniform(seed, step, row)
    target = np.float32(u * P)
    C = np.float32(0)
    pick = J - 1
    cum = []
    for i in range(J):
        C = np.float32(C + w[i])
        cum.append(C)
        if C > target:
            pick = i
            break
    # how close the decisions were, relative to the total weight
    bounds = [abs(float(x) - float(target)) for x in cum] + [abs(float(S[j]) - float(thr)) for j in range(1, K)]
    margin = min(bounds) / float(S[0]) if bounds else 1.0
    return dict(ids=ids, logits=c, w=w, kept=J, u=u, token=int(ids[pick]), pick=pick, margin=margin)
