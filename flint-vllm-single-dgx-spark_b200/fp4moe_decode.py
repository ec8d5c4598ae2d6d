"""Decode-time NVFP4 MoE -- drop-in for the reference's ``fast/fp4moe_decode.py``.

Same entry points, argument order and outputs as the reference (fast/fp4moe_decode.py:61-95):

* ``route(x, gate_w) -> (tw f32 [M, k], ti i32 [M, k])``
* ``route_norm(x, res, nw, eps, gate_w, trigger=0) -> (tw, ti, xn bf16 [M, H], res_out bf16 [M, H])``
* ``moe_up(x, ti, w) -> (act bf16 [M*k, I], sact)``
* ``moe_down(act, sact, ti, tw, w, trigger=0) -> out bf16 [M, H]``

Differences, by design: the kernels read the ModelOpt NVFP4 tensors in place (``DecodeWeights``) instead of the
Marlin repack the GB10 kernels need, run 1..8 tokens instead of 1, and take the expert count / top-k / score
function from the weights instead of hard-coding Flint's 256 / 6 / sigmoid.  ``sact`` (the shared-expert
activation of Flint) is ``None``: the BASELINE model has no shared expert.  ``trigger`` is accepted for
signature compatibility (every launch is stream ordered).
"""
from __future__ import annotations

import os

import torch

from . import _lib
from . import ops as _ops  # noqa: F401  (registers torch.ops.flint_b200.*)

TOPK = int(os.environ.get("FLINT_MOE_TOPK", "6"))
SCORE = os.environ.get("FLINT_MOE_SCORE", "sigmoid")
_SCORE_FN = {"softmax": 0, "sigmoid": 1}


def get_ext():
    return _lib.lib()


def _u8(t):
    return t.view(torch.uint8)


class DecodeWeights:
    """Views (no copies) of an MoE layer's NVFP4 expert tensors in the ModelOpt layout.

    w13 u8 [E, 2I, H/2] (gate rows 0..I-1, up rows I..2I-1), s13 E4M3 [E, 2I, H/16], g13 fp32 [E] (or [E, 2]:
    the first column is used, as fast/fp4moe_decode.py:41 does); w2 u8 [E, H, I/2], s2 E4M3 [E, H, I/16], g2 fp32 [E].
    topk / score select the router (softmax with renormalised top-k, or sigmoid)."""

    def __init__(self, w13, s13, g13, w2, s2, g2, topk: int = TOPK, score: str = SCORE):
        E, I2, Hh = w13.shape
        assert w13.dtype == torch.uint8 and w2.dtype == torch.uint8, (w13.dtype, w2.dtype)
        assert tuple(s13.shape) == (E, I2, Hh // 8) and tuple(w2.shape) == (E, Hh * 2, I2 // 4), (s13.shape, w2.shape)
        assert tuple(s2.shape) == (E, Hh * 2, I2 // 32), s2.shape
        for t in (w13, s13, w2, s2):
            assert t.is_contiguous()
        self.E, self.I, self.H = E, I2 // 2, Hh * 2
        self.w13, self.s13 = w13, _u8(s13)
        self.w2, self.s2 = w2, _u8(s2)
        self.g13 = g13.float().reshape(E, -1)[:, 0].contiguous()
        self.g2 = g2.float().reshape(E, -1)[:, 0].contiguous()
        self.topk = int(topk)
        self.score_fn = _SCORE_FN[score]


def _route_impl(x, res, nw, eps, gate_w, topk, score_fn, want_norm):
    M, H = x.shape
    E = gate_w.shape[0]
    dev = x.device
    ti = torch.empty((M, topk), dtype=torch.int32, device=dev)
    tw = torch.empty((M, topk), dtype=torch.float32, device=dev)
    lg = torch.empty((M, E), dtype=torch.float32, device=dev)
    dummy = torch.empty((0,), dtype=torch.bfloat16, device=dev)
    xn = torch.empty((M, H), dtype=torch.bfloat16, device=dev) if want_norm else dummy
    res_out = torch.empty((M, H), dtype=torch.bfloat16, device=dev) if (want_norm and res is not None) else dummy
    torch.ops.flint_b200.moe_route(x, res, nw, float(eps), gate_w, topk, score_fn, lg, ti, tw, xn, res_out, want_norm,
                                   want_norm and res is not None)
    return tw, ti, xn, res_out, lg


def route(x, gate_w, topk: int = TOPK, score: str = SCORE):
    """Fused router (gate GEMV + top-k + renorm), one launch -> (tw [M,k] f32, ti [M,k] i32)."""
    tw, ti, _, _, _ = _route_impl(x, None, None, 0.0, gate_w, topk, _SCORE_FN[score], False)
    return tw, ti


def route_norm(x, res, nw, eps, gate_w, trigger=0, topk: int = TOPK, score: str = SCORE):
    """Router with the residual add + RMSNorm fused in (one launch): x = attention output, res = residual stream.
    -> (tw [M,k] f32, ti [M,k] i32, xn [M,H] bf16 normalized hidden state, new residual [M,H] bf16)."""
    tw, ti, xn, res_out, _ = _route_impl(x, res, nw, eps, gate_w, topk, _SCORE_FN[score], True)
    return tw, ti, xn, (res_out if res is not None else None)


def moe_up(x, ti, w: DecodeWeights):
    act = torch.empty((x.shape[0] * ti.shape[-1], w.I), dtype=torch.bfloat16, device=x.device)
    torch.ops.flint_b200.moe_up(x, ti, w.w13, w.s13, w.g13, act)
    return act, None


def moe_down(act, sact, ti, tw, w: DecodeWeights, trigger=0):
    """-> sum_j tw_j * expert_{ti_j}(x) (bf16)."""
    M = ti.shape[0]
    out = torch.empty((M, w.H), dtype=torch.bfloat16, device=act.device)
    torch.ops.flint_b200.moe_down(act, ti, tw, w.w2, w.s2, w.g2, out)
    return out


def moe_decode(x, res, nw, eps, gate_w, w: DecodeWeights, fused: bool = True, extras: bool = False,
               impl: str | None = None):
    """The whole decode MoE block: (mlp(norm(x + res)), x + res).  impl "chain" (fused=False): the three launches
    route_norm -> moe_up -> moe_down; "fused" (fused=True): one persistent launch for 1..8 tokens (flint_moe_fused);
    "block": one launch for one token with the down weights prefetched under the gate/up work (flint_moe_block).
    extras=True (fused / block) also returns (xn, logits, topk_ids, topk_weights)."""
    impl = impl or ("fused" if fused else "chain")
    if impl == "block":
        M, H = x.shape
        dev = x.device
        out = torch.empty((M, H), dtype=torch.bfloat16, device=dev)
        res_out = torch.empty((M, H), dtype=torch.bfloat16, device=dev) if res is not None else None
        ex = (torch.empty((M, H), dtype=torch.bfloat16, device=dev), torch.empty((M, w.E), dtype=torch.float32, device=dev),
              torch.empty((M, w.topk), dtype=torch.int32, device=dev), torch.empty((M, w.topk), dtype=torch.float32, device=dev))
        xn, lg, ti, tw = ex if extras else (None, None, None, None)
        torch.ops.flint_b200.moe_block(x, res, nw, float(eps), gate_w, w.topk, w.score_fn, w.w13, w.s13, w.g13, w.w2, w.s2,
                                       w.g2, out, res_out, xn, lg, ti, tw)
        return (out, res_out, ex) if extras else (out, res_out)
    if impl == "chain":
        tw, ti, xn, res_out = route_norm(x, res, nw, eps, gate_w, topk=w.topk,
                                         score=("softmax", "sigmoid")[w.score_fn])
        act, sact = moe_up(xn, ti, w)
        return moe_down(act, sact, ti, tw, w), res_out
    M, H = x.shape
    dev = x.device
    out = torch.empty((M, H), dtype=torch.bfloat16, device=dev)
    res_out = torch.empty((M, H), dtype=torch.bfloat16, device=dev) if res is not None else out
    xn = torch.empty((M, H), dtype=torch.bfloat16, device=dev)
    lg = torch.empty((M, w.E), dtype=torch.float32, device=dev)
    ti = torch.empty((M, w.topk), dtype=torch.int32, device=dev)
    tw = torch.empty((M, w.topk), dtype=torch.float32, device=dev)
    torch.ops.flint_b200.moe_fused(x, res, nw, float(eps), gate_w, w.topk, w.score_fn, w.w13, w.s13, w.g13, w.w2, w.s2,
                                   w.g2, out, res_out, xn, lg, ti, tw, extras)
    if extras:
        return out, (res_out if res is not None else None), (xn, lg, ti, tw)
    return out, (res_out if res is not None else None)
