"""Decode attention block on the CPU -- test infrastructure only.

QKV (fast/attn_gemv2.cu:101-265 rounding points; q/k norm + RoPE numerics patch:5657-5664):
  xn = bf16(s * rsqrt(mean(s^2) + eps) * w), s = x + res; y = bf16(gs * xn . W)
  q/k heads: n = bf16(y * rsqrt(mean(y^2) + eps) * w_head); NeoX RoPE r1 = n1*cos - n2*sin, r2 = n2*cos + n1*sin (fp32)
  v heads: y unchanged
O: y = bf16(gs * a . W)
Decode attention (patch:1444-1464): S = K q (fp32), p = exp2((S - m) * scale * log2 e), P rounded to bf16 for P V,
the denominator sums the unrounded p, plus exp2(sink * log2 e - m * c) when sinks are given.  Evaluated in float64
with the global maximum (the GPU's running-maximum form differs only by rounding).
"""
from __future__ import annotations

import numpy as np

from .moe import rmsnorm
from .nvfp4 import bf16_round, dequantize_nvfp4

LOG2E = 1.4426950408889634


def gemv_nvfp4(x: np.ndarray, P, S, gs, W: np.ndarray | None = None) -> np.ndarray:
    """bf16(gs * x . dequant(P, S)^T): x [M, K] -> [M, N] (bf16 values as fp32).  The dot is float64 unless W, the
    already dequantised weight, is given: then it runs in W's precision (fp32 W = the reference's dequantise-to-fp32
    matmul, fast/fast_head.py:95-115 and patch:295-319)."""
    if W is None:
        W = dequantize_nvfp4(P, S).astype(np.float64)
    acc = (np.asarray(x, W.dtype) @ W.T).astype(np.float32)
    return bf16_round(acc * np.float32(gs))


def rope_cos_sin(max_pos: int, dim: int = 128, theta: float = 1e6) -> np.ndarray:
    """fp32 [max_pos, dim] table: cos | sin of NeoX-style rotary frequencies."""
    inv = 1.0 / (theta ** (np.arange(0, dim, 2, dtype=np.float64) / dim))
    ang = np.arange(max_pos, dtype=np.float64)[:, None] * inv[None, :]
    return np.concatenate([np.cos(ang), np.sin(ang)], axis=1).astype(np.float32)


def qkv_head(x, res, nw, eps, P, S, gs, q_w, k_w, positions, cos_sin, nq, nkv, D=128, W=None):
    """-> (q [M, nq*D], y [M, N] (raw q and v heads, normalised+rotated k heads), res_out, k_new, v_new [M, nkv, D]).
    W: optional dequantised QKV weight (see gemv_nvfp4)."""
    xn, res_out = rmsnorm(x, res, nw, eps)
    y = gemv_nvfp4(xn, P, S, gs, W)
    M = y.shape[0]
    heads = y.reshape(M, nq + 2 * nkv, D).copy()
    out = heads.copy()
    for hd in range(nq + nkv):
        v = heads[:, hd]
        var = (v.astype(np.float64) ** 2).mean(-1, keepdims=True)
        rs = (1.0 / np.sqrt(var + eps)).astype(np.float32)
        w = q_w if hd < nq else k_w
        n = bf16_round((v * rs) * w.astype(np.float32))
        if cos_sin is not None:
            cs = cos_sin[positions]
            c, s = cs[:, :D // 2], cs[:, D // 2:]
            n1, n2 = n[:, :D // 2], n[:, D // 2:]
            n = np.concatenate([n1 * c - n2 * s, n2 * c + n1 * s], axis=1).astype(np.float32)
        out[:, hd] = bf16_round(n)
    q = out[:, :nq].reshape(M, nq * D)
    y_out = heads.copy()
    y_out[:, nq:nq + nkv] = out[:, nq:nq + nkv]          # only the k heads are written back (attn_gemv2.cu:256)
    return q, y_out.reshape(M, -1), res_out, out[:, nq:nq + nkv], out[:, nq + nkv:]


def decode_attention(q, kv_cache, block_tables, seq_lens, sinks, window, scale):
    """q [B, Hq, D]; kv_cache [blocks, Hkv, 16, 2D] (K | V); -> out [B, Hq, D] (bf16 values as fp32)."""
    B, Hq, D = q.shape
    Hkv = kv_cache.shape[1]
    G = Hq // Hkv
    out = np.zeros((B, Hq, D), dtype=np.float32)
    c = scale * LOG2E
    for b in range(B):
        L = int(seq_lens[b])
        if L == 0:
            continue
        start = max(0, L - window) if window else 0
        pages = [int(block_tables[b, p]) for p in range((L + 15) // 16)]
        kv = np.concatenate([kv_cache[p] for p in pages], axis=1)[:, :L]      # [Hkv, L, 2D]
        for h in range(Hkv):
            K = kv[h, start:, :D].astype(np.float64)
            V = kv[h, start:, D:].astype(np.float64)
            for g in range(G):
                qh = h * G + g
                s = K @ q[b, qh].astype(np.float64)
                m = s.max()
                p = np.exp2((s - m) * c)
                den = p.sum()
                if sinks is not None:
                    den += np.exp2(float(sinks[qh]) * LOG2E - m * c)
                pb = bf16_round(p.astype(np.float32)).astype(np.float64)
                out[b, qh] = bf16_round(((pb @ V) / den).astype(np.float32))
    return out
