"""MoE decode block on the CPU -- test infrastructure only.

Restates, with the rounding points of the reference's dequantise-to-fp32 path (patch:2890-2899, norm numerics
patch:4937-4952, GB10 kernels fast/fp4moe_mar.cu:267,341-366):
  s = x + res (fp32); res_out = bf16(s); xn = bf16(s * rsqrt(mean(s^2) + eps) * w)
  logit[e] = bf16(xn . Wr[e])                                    (fp32 dot)
  top-k on the bf16 logits, ties -> lowest expert index; weights softmax or sigmoid, renormalised and kept in fp32
  (tw = val / sum, the GB10 kernel's rule, fast/fp4moe_mar.cu:297-301; the PR's SM100 decode instead rounds tw to
  bf16, patch:3049-3050 -- this library and this oracle keep the fp32 weights)
  g, u = xn . W13[e] * gs13[e]; act = bf16(silu(g) * u)           (fp32)
  y_e = bf16(act . W2[e] * gs2[e]); out = bf16(sum_slot tw * y_e)  (fp32, slot order)
``router_logits_mirror`` reproduces the GPU router's exact fp32 summation order (lane-strided chains over
uint4 blocks, then an xor butterfly), so routing ids can be compared bit for bit.
"""
from __future__ import annotations

import numpy as np

from .nvfp4 import bf16_round, dequantize_nvfp4


def rmsnorm(x: np.ndarray, res: np.ndarray | None, w: np.ndarray | None, eps: float):
    """-> (xn fp32 of bf16 values, res_out fp32 of bf16 values)."""
    s = x.astype(np.float32) + (res.astype(np.float32) if res is not None else 0)
    res_out = bf16_round(s)
    if w is None:
        return bf16_round(s), res_out
    ms = (s.astype(np.float64) ** 2).mean(-1, keepdims=True)
    rs = (1.0 / np.sqrt(ms + eps)).astype(np.float32)
    return bf16_round((s * rs) * w.astype(np.float32)), res_out


def router_logits_mirror(xn: np.ndarray, wr: np.ndarray) -> np.ndarray:
    """xn [M, H], wr [E, H] (bf16 values as fp32) -> bf16-rounded fp32 logits [M, E], GPU summation order:
    lane l accumulates k = 8*(l + 32*i) + j for i (outer) then j (inner) with fp32 FMAs (the products are exact),
    then lanes combine with an xor butterfly 16, 8, 4, 2, 1."""
    M, H = xn.shape
    E = wr.shape[0]
    NV = H // 256
    xv = xn.astype(np.float32).reshape(M, NV, 32, 8)           # [M, i, lane, j]
    wv = wr.astype(np.float32).reshape(E, NV, 32, 8)
    acc = np.zeros((M, E, 32), dtype=np.float32)
    for i in range(NV):
        for j in range(8):
            acc = acc + (xv[:, None, i, :, j] * wv[None, :, i, :, j])
    lanes = np.arange(32)
    for o in (16, 8, 4, 2, 1):
        acc = acc + acc[..., lanes ^ o]
    return bf16_round(acc[..., 0])


def route_weights(logits: np.ndarray, ids: np.ndarray, score_fn: int) -> np.ndarray:
    """Renormalised routing weights of the chosen experts ids [M, k] (fp32): softmax over the chosen logits
    (score_fn 0) or sigmoid of each, divided by their sum (score_fn 1)."""
    sel = np.take_along_axis(logits.astype(np.float32), ids, -1).astype(np.float64)
    v = 1.0 / (1.0 + np.exp(-sel)) if score_fn == 1 else np.exp(sel - sel.max(-1, keepdims=True))
    return (v / v.sum(-1, keepdims=True)).astype(np.float32)


def topk_route(logits: np.ndarray, topk: int, score_fn: int):
    """-> (ids int32 [M, k], weights fp32 [M, k]); score_fn 0 = softmax (select on logits), 1 = sigmoid."""
    lg = logits.astype(np.float32)
    # selection on the bf16 logits for both score functions (sigmoid is monotone), ties -> lowest expert
    # (patch:3015-3048 and fast/fp4moe_mar.cu:286-290); weights stay fp32 (fast/fp4moe_mar.cu:301)
    order = np.lexsort((np.broadcast_to(np.arange(lg.shape[-1]), lg.shape), -lg), axis=-1)
    ids = order[:, :topk].astype(np.int32)
    return ids, route_weights(lg, ids, score_fn)


def experts_up(xn: np.ndarray, ids: np.ndarray, w13, s13, g13, dense=None) -> np.ndarray:
    """-> act (bf16 values as fp32) [M*k, I], row m*k+s for expert ids[m, s].  dense: optional e -> dequantised
    gate/up weight of expert e; the dots then run in that array's precision (float64 without it)."""
    M, k = ids.shape
    I = w13.shape[1] // 2
    act = np.zeros((M * k, I), dtype=np.float32)
    cache = {}
    for m in range(M):
        for s in range(k):
            e = int(ids[m, s])
            if dense is not None:
                W = dense(e)
            else:
                if e not in cache:
                    cache[e] = dequantize_nvfp4(w13[e], s13[e]).astype(np.float64)
                W = cache[e]
            h = W @ xn[m].astype(W.dtype)
            g = (h[:I].astype(np.float32) * np.float32(g13[e])).astype(np.float32)
            u = (h[I:].astype(np.float32) * np.float32(g13[e])).astype(np.float32)
            silu = (g.astype(np.float64) / (1.0 + np.exp(-g.astype(np.float64)))).astype(np.float32)
            act[m * k + s] = bf16_round(silu * u)
    return act


def experts_down(act: np.ndarray, ids: np.ndarray, tw: np.ndarray, w2, s2, g2, dense=None) -> np.ndarray:
    """-> out (bf16 values as fp32) [M, H].  dense: optional e -> dequantised down weight of expert e (as in
    experts_up)."""
    M, k = ids.shape
    H = w2.shape[1]
    out = np.zeros((M, H), dtype=np.float32)
    cache = {}
    for m in range(M):
        acc = np.zeros(H, dtype=np.float64)
        for s in range(k):
            e = int(ids[m, s])
            if dense is not None:
                W = dense(e)
            else:
                if e not in cache:
                    cache[e] = dequantize_nvfp4(w2[e], s2[e]).astype(np.float64)
                W = cache[e]
            y = bf16_round(((W @ act[m * k + s].astype(W.dtype)).astype(np.float32) * np.float32(g2[e])))
            acc = (acc + np.float64(tw[m, s]) * y.astype(np.float64)).astype(np.float32).astype(np.float64)
        out[m] = bf16_round(acc.astype(np.float32))
    return out
