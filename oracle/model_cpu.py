"""CPU baseline: the reference's dequantise-to-fp32 torch path for a full decode token -- test infrastructure only.

Used by bench.py (its cpu_baseline leg and ``--impl reference``) to time the reference algorithm on the host cores:
every NVFP4 matrix is dequantised per call exactly as the reference's ``dequantize_nvfp4`` does (LUT decode in chunks
of 8192 rows, patch:295-319) and multiplied in fp32 (the stock path feeding ``compute_logits``, fast/fast_head.py:
360-381, and the GEMVs of fast/attn_gemv2.cu / fp4moe_mar.cu restated on the CPU); attention is a float32 GQA
softmax over the paged context; routing is softmax top-k renormalised.

Two variants, as the reference can run either way: ``predequantized=False`` dequantises every matrix at every call
(the literal path); ``predequantized=True`` dequantises all weights to fp32 once at construction (not timed) and
only multiplies per token (the steady state).

Sample: ``n_tokens`` decode tokens at ``context`` tokens of KV.  To keep host memory bounded the expert tensors of
one layer are shared by all layers (the per-token work -- which experts are dequantised and multiplied -- is the same
as with distinct layers); all other weights and the KV cache are per layer.  Weights are random valid NVFP4 bytes.
Per layer: add + RMSNorm, QKV, q/k RMSNorm and NeoX RoPE (fast/attn_gemv2.cu:170-265), GQA attention over the
context, O, add + RMSNorm, router top-k, the routed experts and their weighted sum; then the final norm and head.
"""
from __future__ import annotations

import os
import time

import torch

_E2M1 = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0, -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0)


def dequantize_nvfp4(P: torch.Tensor, S: torch.Tensor, gs: float, chunk: int = 8192) -> torch.Tensor:
    """Restates patch:295-319: [N, K/2] u8 codes (low nibble first) and E4M3 [N, K/16] -> fp32 [N, K] * gs."""
    lut = torch.tensor(_E2M1, dtype=torch.float32)
    N = P.shape[0]
    out = torch.empty((N, P.shape[1] * 2), dtype=torch.float32)
    for a in range(0, N, chunk):
        w = P[a:a + chunk]
        codes = torch.stack([w & 0x0F, w >> 4], dim=-1).int()
        vals = lut[codes].reshape(w.shape[0], -1, 16)
        vals = vals * S[a:a + chunk].view(torch.float8_e4m3fn).float().unsqueeze(-1)
        out[a:a + chunk] = vals.flatten(-2) * gs
    return out


def _rand_nvfp4(gen, N, K):
    P = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, generator=gen)
    S = torch.randint(0x28, 0x47, (N, K // 16), dtype=torch.uint8, generator=gen)
    return P, S, 0.02 / 3


def _rmsnorm(x, w, eps):
    return (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * w).to(torch.bfloat16).float()


def _rope(t, cos, sin):
    """NeoX rotation of the last dimension (halves rotated against each other)."""
    h = t.shape[-1] // 2
    a, b = t[..., :h], t[..., h:]
    return torch.cat([a * cos - b * sin, b * cos + a * sin], dim=-1)


class CpuFlint:
    def __init__(self, cfg, context: int, seed: int = 0, predequantized: bool = False):
        g = torch.Generator().manual_seed(seed)
        c = self.c = cfg
        self.context = context
        self.layers = []
        E, I, H = c.num_experts, c.moe_inter, c.hidden
        self.experts = [(_rand_nvfp4(g, 2 * I, H), _rand_nvfp4(g, H, I)) for _ in range(E)]
        for _ in range(c.layers):
            self.layers.append(dict(
                qkv=_rand_nvfp4(g, c.qkv_rows, H), o=_rand_nvfp4(g, H, c.num_heads * c.head_dim),
                gate=(torch.randn((E, H), generator=g) * 0.02).to(torch.bfloat16).float(),
                k=(torch.randn((context + 64, c.num_kv_heads, c.head_dim), generator=g)).to(torch.bfloat16).float(),
                v=(torch.randn((context + 64, c.num_kv_heads, c.head_dim), generator=g)).to(torch.bfloat16).float()))
        self.embed = (torch.randn((c.vocab, H), generator=g)).to(torch.bfloat16)
        self.head = _rand_nvfp4(g, c.vocab, H)
        self.ones = torch.ones(H)
        self.fp32 = {}
        if predequantized:                           # steady state: every matrix dequantised once, up front
            for i, L in enumerate(self.layers):
                self.fp32[("qkv", i)] = dequantize_nvfp4(*L["qkv"])
                self.fp32[("o", i)] = dequantize_nvfp4(*L["o"])
            for e, (w13, w2) in enumerate(self.experts):
                self.fp32[("w13", e)] = dequantize_nvfp4(*w13)
                self.fp32[("w2", e)] = dequantize_nvfp4(*w2)
            self.fp32[("head", 0)] = dequantize_nvfp4(*self.head)

    def _w(self, key, idx, nv):
        """fp32 weight: the pre-dequantised copy, or the reference's per-call dequantisation."""
        w = self.fp32.get((key, idx))
        return w if w is not None else dequantize_nvfp4(*nv)

    @torch.no_grad()
    def decode_token(self, token: int, pos: int) -> int:
        c = self.c
        H, D, nq, nkv = c.hidden, c.head_dim, c.num_heads, c.num_kv_heads
        res = self.embed[token].float()[None]
        h = torch.zeros_like(res)
        ang = pos * (1.0 / (c.rope_theta ** (torch.arange(0, D, 2, dtype=torch.float64) / D)))
        cos, sin = torch.cos(ang).float(), torch.sin(ang).float()
        head_ones = torch.ones(D)
        for li, L in enumerate(self.layers):
            res = res + h
            x = _rmsnorm(res, self.ones, c.rms_eps)
            y = (x @ self._w("qkv", li, L["qkv"]).t()).to(torch.bfloat16).float()
            q = _rope(_rmsnorm(y[:, :nq * D].reshape(nq, D), head_ones, c.rms_eps), cos, sin)
            q = q.to(torch.bfloat16).float()
            k_new = _rope(_rmsnorm(y[0, nq * D:(nq + nkv) * D].reshape(nkv, D), head_ones, c.rms_eps), cos, sin)
            L["k"][pos] = k_new.to(torch.bfloat16).float()
            L["v"][pos] = y[0, (nq + nkv) * D:].reshape(nkv, D)
            K, V = L["k"][:pos + 1], L["v"][:pos + 1]
            G = nq // nkv
            s = torch.einsum("hgd,thd->hgt", q.reshape(nkv, G, D), K) * D ** -0.5
            p = torch.softmax(s, dim=-1)
            attn = torch.einsum("hgt,thd->hgd", p, V).reshape(1, nq * D).to(torch.bfloat16).float()
            a = (attn @ self._w("o", li, L["o"]).t()).to(torch.bfloat16).float()
            res = res + a
            xn = _rmsnorm(res, self.ones, c.rms_eps)
            logits = (xn @ L["gate"].t()).to(torch.bfloat16).float()
            top = torch.topk(logits[0], c.topk)
            tw = torch.softmax(top.values, dim=-1)
            out = torch.zeros((1, H))
            for w, e in zip(tw.tolist(), top.indices.tolist()):
                w13, w2 = self.experts[e]
                gu = xn @ self._w("w13", e, w13).t()
                g_, u_ = gu[:, :c.moe_inter], gu[:, c.moe_inter:]
                act = (torch.nn.functional.silu(g_) * u_).to(torch.bfloat16).float()
                out += w * (act @ self._w("w2", e, w2).t()).to(torch.bfloat16).float()
            h = out.to(torch.bfloat16).float()
        x = _rmsnorm(res + h, self.ones, c.rms_eps)
        return int((x @ self._w("head", 0, self.head).t()).argmax())


def time_decode(cfg, n_tokens: int = 1, context: int = 6057, warmup: int = 0, predequantized: bool = False) -> dict:
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    m = CpuFlint(cfg, context, predequantized=predequantized)
    tok = 1
    for i in range(warmup):
        tok = m.decode_token(tok, context + i)
    t0 = time.perf_counter()
    for i in range(n_tokens):
        tok = m.decode_token(tok, context + warmup + i)
    dt = time.perf_counter() - t0
    return {"value": round(n_tokens / dt, 5), "unit": "tok/s", "cores": threads, "kind": "port",
            "tokens": n_tokens, "seconds": round(dt, 2),
            "sample": f"{n_tokens} full-model decode token(s) at {context} tokens of KV context after {warmup} untimed; "
                      + ("weights dequantised to fp32 once (steady state)" if predequantized else
                         "per-call NVFP4 dequantisation") + " + fp32 matmuls (torch CPU), expert tensors shared across "
                      "layers"}
