"""Whole-model greedy decode on the CPU, composed from the per-kernel oracles -- test infrastructure only.

One decode step of the reference's fast path for a BASELINE-shaped layer stack (fast/model.py:734-759 per layer,
compute_logits fast/fast_head.py:360-381 and fast/model.py:924-929 for the head):

    layer l:  q, k, v, res_a = qkv_head(h, res)        add + RMSNorm, NVFP4 QKV, q/k norm, RoPE  (attention.qkv_head)
              cache[l][pos] = k, v; att = decode attention over cache[l][:pos+1]          (attention.decode_attention)
              a = O(att)                                                                  (attention.gemv_nvfp4)
              xn, res_b = RMSNorm(a + res_a); logits = router(xn); ids, tw = top-k       (moe.*)
              h = down(up(xn, ids), ids, tw)                                               (moe.experts_up / down)
    head:     logits = gs * final_norm(h + res_b) . dequant(head)                          (lm_head.lm_head_logits)

Weights are dequantised once to fp32 (exact: e2m1 x e4m3 fits) and every GEMV is the fp32 matmul of the reference's
dequantise-to-fp32 path, with the bf16 rounding points of the per-kernel oracles.  The router logits use the GPU
kernel's fixed summation order (moe.router_logits_mirror), so routing can be compared expert for expert.

Routing of a token is a discrete choice on bf16 logits: when the model's hidden state differs from the GPU's by a bf16
ulp somewhere, two experts whose logits are within an ulp or two may legitimately swap.  ``step`` therefore takes the
GPU's own choice (``gpu_ids``, with its router logits ``gpu_logits``) after checking it: the choice must be the exact
top-k of the GPU's logits, and those must agree with this oracle's within ``route_tol_ulps`` bf16 ulps; anything
else raises ``RoutingMismatch``.  Adoptions and the largest logit difference are recorded.
"""
from __future__ import annotations

import numpy as np

from .attention import decode_attention, gemv_nvfp4, qkv_head
from .lm_head import lm_head_logits
from .moe import experts_down, experts_up, rmsnorm, route_weights, router_logits_mirror, topk_route
from .nvfp4 import dequantize_nvfp4

PAGE = 16


class RoutingMismatch(AssertionError):
    pass


def bf16_ulp(v: float) -> float:
    """Spacing of bf16 values at magnitude |v| (8 significant bits)."""
    v = abs(float(v))
    if v == 0.0:
        return 2.0 ** -133
    return 2.0 ** (np.floor(np.log2(v)) - 7)


class DecodeOracle:
    """CPU decode of one stream.  ``weights``: numpy copies of a model's tensors (bf16 values as fp32, NVFP4 bytes as
    uint8): embed [V, H], final_norm [H], head (P, S, gs), cos_sin [max_pos, D] and per layer ln1, ln2, q_norm,
    k_norm [D], qkv (P, S, gs), o (P, S, gs), gate [E, H], w13, s13, g13, w2, s2, g2.  ``dense`` caches the
    dequantised fp32 weights; share one between oracles of the same model."""

    def __init__(self, cfg, weights: dict, max_pos: int, dense: dict | None = None, route_tol_ulps: float = 4.0):
        if cfg.shared_inter or cfg.mlp_only_layers or cfg.layer_types or cfg.attn_sinks or cfg.no_rope_layers:
            raise ValueError("DecodeOracle covers the BASELINE layer structure only")
        self.c, self.w = cfg, weights
        self.score = 1 if cfg.score == "sigmoid" else 0
        self.dense = dense if dense is not None else {}
        self.tol = route_tol_ulps
        self.npages = (max_pos + PAGE - 1) // PAGE
        nkv, D = cfg.num_kv_heads, cfg.head_dim
        self.kv = [np.zeros((self.npages, nkv, PAGE, 2 * D), np.float32) for _ in range(cfg.layers)]
        self.adopted = 0                 # routing choices taken from the GPU within the tolerance
        self.route_checks = 0
        self.max_logit_ulps = 0.0        # largest router-logit difference seen, in bf16 ulps of the row maximum

    # ---- dequantised weights, computed once per tensor ----
    def _dq(self, key, P, S) -> np.ndarray:
        W = self.dense.get(key)
        if W is None:
            W = self.dense[key] = dequantize_nvfp4(P, S)            # fp32, exact
        return W

    def _expert(self, l: int, which: str, e: int) -> np.ndarray:
        L = self.w["layers"][l]
        P, S = (L["w13"], L["s13"]) if which == "up" else (L["w2"], L["s2"])
        return self._dq((l, which, e), P[e], S[e])

    # ---- routing ----
    def route(self, logits: np.ndarray, gpu_ids: np.ndarray | None, gpu_logits: np.ndarray | None = None):
        """-> (ids [1, k], weights [1, k]) for bf16 logits [1, E]: this oracle's top-k, or the GPU's choice.

        With the GPU's own router logits: its ids must be exactly the top-k of those logits (the kernel's selection
        rule), and those logits must agree with this oracle's within ``route_tol_ulps`` bf16 ulps of the row's
        largest logit; the GPU's choice is then taken.  Without them: the GPU's ids must be a top-k of this oracle's
        logits up to that many ulps at each compared logit.  Anything else raises RoutingMismatch."""
        k = self.c.topk
        ids, tw = topk_route(logits, k, self.score)
        if gpu_ids is None:
            return ids, tw
        self.route_checks += 1
        g = np.asarray(gpu_ids, np.int32).reshape(1, k)
        v = logits[0].astype(np.float64)
        if gpu_logits is not None:
            gl = np.asarray(gpu_logits, np.float32).reshape(1, -1)
            own, _ = topk_route(gl, k, self.score)
            if not np.array_equal(own, g):
                raise RoutingMismatch(f"GPU experts {g[0].tolist()} are not the top-{k} of the GPU's own router logits "
                                      f"({own[0].tolist()})")
            d = float(np.abs(gl[0].astype(np.float64) - v).max())
            unit = bf16_ulp(np.abs(v).max())
            self.max_logit_ulps = max(self.max_logit_ulps, d / unit)
            if d > self.tol * unit:
                raise RoutingMismatch(f"router logits differ from the oracle's by {d:.3g} (> {self.tol} bf16 ulps of "
                                      f"{np.abs(v).max():.3g})")
            if not np.array_equal(g, ids):
                self.adopted += 1
                return g, route_weights(logits, g, self.score)
            return ids, tw
        if np.array_equal(g, ids):
            return ids, tw
        chosen = np.zeros(v.shape[0], bool)
        chosen[g[0]] = True
        near = lambda a, b: self.tol * bf16_ulp(max(abs(a), abs(b)))
        lo, hi = v[chosen].min(), v[~chosen].max()
        sel = v[g[0]]
        ok = (len(set(g[0].tolist())) == k and lo >= hi - near(lo, hi)
              and all(sel[i] >= sel[i + 1] - near(sel[i], sel[i + 1]) for i in range(k - 1)))
        if not ok:
            raise RoutingMismatch(f"GPU experts {g[0].tolist()} are not a top-{k} of the oracle logits "
                                  f"(oracle {ids[0].tolist()}, {self.tol} bf16 ulps)")
        self.adopted += 1
        return g, route_weights(logits, g, self.score)

    # ---- one position ----
    def step(self, token: int, pos: int, gpu_ids: np.ndarray | None = None,
             gpu_logits: np.ndarray | None = None) -> np.ndarray:
        """Run token at position pos through every layer (writing its K/V) and the head; gpu_ids [layers, k] and
        gpu_logits [layers, E] are the GPU's routing and router logits for this position (or None).
        -> fp32 logits [V]."""
        c, W = self.c, self.w
        nq, nkv, D, eps = c.num_heads, c.num_kv_heads, c.head_dim, c.rms_eps
        x, res = W["embed"][token][None, :], None
        pg, off = divmod(pos, PAGE)
        for l in range(c.layers):
            L = W["layers"][l]
            P, S, gs = L["qkv"]
            q, _, res_a, k_new, v_new = qkv_head(x, res, L["ln1"], eps, P, S, gs, L["q_norm"], L["k_norm"],
                                                 np.array([pos]), W["cos_sin"], nq, nkv, D,
                                                 W=self._dq((l, "qkv"), P, S))
            self.kv[l][pg, :, off, :D] = k_new[0]
            self.kv[l][pg, :, off, D:] = v_new[0]
            npg = pg + 1
            att = decode_attention(q.reshape(1, nq, D), self.kv[l][:npg], np.arange(npg)[None, :], [pos + 1], None, 0,
                                   D ** -0.5)
            Po, So, go = L["o"]
            a = gemv_nvfp4(att.reshape(1, -1), Po, So, go, W=self._dq((l, "o"), Po, So))
            xn, res_b = rmsnorm(a, res_a, L["ln2"], eps)
            lg = router_logits_mirror(xn, L["gate"])
            ids, tw = self.route(lg, None if gpu_ids is None else gpu_ids[l],
                                 None if gpu_logits is None else gpu_logits[l])
            act = experts_up(xn, ids, L["w13"], L["s13"], L["g13"], dense=lambda e: self._expert(l, "up", e))
            x = experts_down(act, ids, tw, L["w2"], L["s2"], L["g2"], dense=lambda e: self._expert(l, "down", e))
            res = res_b
        xf, _ = rmsnorm(x, res, W["final_norm"], eps)
        P, S, gs = W["head"]
        return lm_head_logits(xf, P, S, gs, W=self._dq(("head",), P, S))[0]
