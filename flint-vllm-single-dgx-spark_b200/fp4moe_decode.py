"""Decode-time NVFP4 MoE -- drop-in for the reference's ``fast/fp4moe_decode.py``.

Same entry points, argument order and outputs as the reference (fast/fp4moe_decode.py:61-95):

* ``route(x, gate_w) -> (tw f32 [M, k], ti i32 [M, k])``
* ``route_norm(x, res, nw, eps, gate_w, trigger=0) -> (tw, ti, xn bf16 [M, H], res_out bf16 [M, H])``
* ``moe_up(x, ti, w) -> (act bf16 [M*k, I], sact)``
* ``moe_down(act, sact, ti, tw, w, trigger=0) -> out bf16 [M, H]``

Differences, by design: the kernels read the ModelOpt NVFP4 layout (``DecodeWeights``, in place); the Marlin
tensors the reference's caller passes to ``MarlinDecodeWeights`` are converted to it once on the GPU
(``unpack_marlin``).  The kernels run 1..8 tokens instead of 1 and take the expert count / top-k / score function
from the weights instead of hard-coding Flint's 256 / 6 / sigmoid.  ``trigger`` is accepted for
signature compatibility (every launch is stream ordered).

Flint's ungated shared expert (``DecodeWeights(..., shared=...)``): ``moe_up`` also returns its activation ``sact``
[M, SI] and ``moe_down`` adds its output, ``out = bf16(routed + shared)`` with ``routed = bf16(sum tw * y_e)`` and
``shared = bf16(sact . W2s * gs)`` -- the PR's combine rule (patch:3391-3397); the GB10 kernels fold the same sum
(fast/fp4moe_mar.cu:224-231).  The shared expert runs on the routed kernels as a one-expert stack that every token
routes to with weight 1; the final add is one bf16 elementwise add.  ``sact`` is ``None`` without a shared expert
(the BASELINE model).  ``dense_mlp`` is Flint's dense SwiGLU layer (``mlp_only_layers``) on the same kernels.
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

    def __init__(self, w13, s13, g13, w2, s2, g2, topk: int = TOPK, score: str = SCORE, shared=None):
        """shared: None, or the shared expert's (w13, s13, g13, w2, s2, g2) -- u8 [2SI, H/2], E4M3 [2SI, H/16],
        fp32 scalar, u8 [H, SI/2], E4M3 [H, SI/16], fp32 scalar (a leading dimension of 1 is accepted)."""
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
        self.shared = None
        if shared is not None:
            sw13, ss13, sg13, sw2, ss2, sg2 = shared
            one = lambda t: t.reshape(1, *t.shape[-2:])
            self.shared = DecodeWeights(one(sw13), one(ss13), sg13.reshape(1), one(sw2), one(ss2), sg2.reshape(1),
                                        topk=1, score="softmax")
            assert self.shared.H == self.H, "shared expert hidden size"

    @classmethod
    def from_layer(cls, w13, s13, g13, w2, s2, g2, sh_gu=None, sh_dn=None, topk: int = TOPK, score: str = SCORE):
        """The reference's argument grouping (MarlinDecodeWeights, fast/fp4moe_decode.py:27-44): the routed experts'
        six tensors, then the shared expert's gate_up and down projections as (weight, weight_scale, global scale)
        tuples -- here the layer's ModelOpt NVFP4 tensors (gate rows before up rows), not the Marlin repack."""
        if (sh_gu is None) != (sh_dn is None):
            raise ValueError("the shared expert needs both its gate_up and its down projection")
        shared = None if sh_gu is None else (sh_gu[0], sh_gu[1], sh_gu[2].float().reshape(-1)[:1], sh_dn[0], sh_dn[1],
                                             sh_dn[2].float().reshape(-1)[:1])
        return cls(w13, s13, g13, w2, s2, g2, topk=topk, score=score, shared=shared)


def unpack_marlin(weight, weight_scale, global_scale):
    """vLLM's Marlin-processed NVFP4 tensors of one projection -> ModelOpt (codes u8 [E, N, K/2], E4M3 scales u8
    [E, N, K/16], global fp32 [E]), on the GPU (flint_marlin_nvfp4_unpack; layout fast/fp4moe_mar.cu:1-7).

    weight int32 [E, K/16, 2N] (or [K/16, 2N] for one matrix, e.g. the shared expert), weight_scale [E, K/16, N]
    processed scale bytes (any 1-byte dtype), global_scale the processed global scale per matrix ([E], [E, 2] -- the
    first column is used, as fast/fp4moe_decode.py:41 does -- or a scalar).  The result reproduces the weights the
    reference's kernels use bit for bit: e2m1 * e4m3 * gs == e2m1 * fp16(h << 7) * g * 2^-126.  Allocates the
    ModelOpt copy (the Marlin tensors are not modified).  ValueError if a scale byte is not a processed scale."""
    single = weight.dim() == 2
    w = weight.unsqueeze(0) if single else weight
    sc = weight_scale.unsqueeze(0) if single else weight_scale
    if w.dtype != torch.int32 or w.dim() != 3:
        raise ValueError(f"unpack_marlin: expected int32 Marlin tiles [E, K/16, 2N], got {weight.dtype} "
                         f"{tuple(weight.shape)}")
    E, KT, W2 = w.shape
    N, K = W2 // 2, KT * 16
    g = global_scale.float().reshape(E, -1)[:, 0].contiguous()
    dev = w.device
    P = torch.empty((E, N, K // 2), dtype=torch.uint8, device=dev)
    S = torch.empty((E, N, K // 16), dtype=torch.uint8, device=dev)
    gs = torch.empty((E,), dtype=torch.float32, device=dev)
    bad = torch.zeros((1,), dtype=torch.int32, device=dev)
    torch.ops.flint_b200.marlin_nvfp4_unpack(w.contiguous(), sc.contiguous().view(torch.uint8), g, P, S, gs, bad)
    if int(bad.item()):
        raise ValueError("unpack_marlin: a scale byte is not a processed NVFP4 scale (0, or 0x80..0xF6)")
    return (P[0], S[0], gs[0]) if single else (P, S, gs)


def grouped_moe(x, topk_ids, topk_weights, w: "DecodeWeights", block_size: int = 64, tensor_cores: bool = True):
    """Prefill MoE of a prompt (the Flint PR's grouped_moe, patch:4093-4212, runs FlashInfer's grouped GEMMs; this
    runs the library's NVFP4 tiles): x bf16 [T, H] (normalised), topk_ids [T, topk], topk_weights fp32 [T, topk] ->
    out bf16 [T, H] = bf16(sum_s tw[t, s] * y[t, s]) in slot order, y the routed expert's output row.  The routes are
    grouped by expert with the deterministic align (blocks of 64), each decoded weight fragment serves a block's 64
    routes; gate/up, SwiGLU and down keep the decode kernels' rounding points (fp32 sums in another order).  The
    routed experts only (a shared expert or dense layer is added by the caller, as for the decode path).
    tensor_cores: the tcgen05 tiles (decoded weights and accumulator in tensor memory; the default, the faster
    form) or, with False, the mma.sync tiles."""
    from .patch_align import align_sizes
    ops = torch.ops.flint_b200
    T, H = x.shape
    k = topk_ids.shape[-1]
    numel = T * k
    dev = x.device
    n_sorted, n_blocks = align_sizes(numel, w.E, block_size, pad_sorted_ids=True)
    sorted_ids = torch.empty((n_sorted,), dtype=torch.int32, device=dev)
    expert_ids = torch.empty((n_blocks,), dtype=torch.int32, device=dev)
    ntp = torch.empty((1,), dtype=torch.int32, device=dev)
    ops.moe_align(topk_ids.reshape(-1), w.E, block_size, sorted_ids, expert_ids, ntp)
    xh = torch.empty((T, H), dtype=torch.float16, device=dev)
    sx = torch.empty((T,), dtype=torch.int32, device=dev)
    ops.rows_to_f16(x, xh, sx)
    act = torch.empty((numel, w.I), dtype=torch.bfloat16, device=dev)
    ops.moe_grouped_up(xh, sx, sorted_ids, expert_ids, ntp, numel, k, w.w13, w.s13, w.g13, act, int(tensor_cores))
    ah = torch.empty((numel, w.I), dtype=torch.float16, device=dev)
    sa = torch.empty((numel,), dtype=torch.int32, device=dev)
    ops.rows_to_f16(act, ah, sa)
    y = torch.empty((numel, H), dtype=torch.bfloat16, device=dev)
    ops.moe_grouped_down(ah, sa, sorted_ids, expert_ids, ntp, numel, k, w.w2, w.s2, w.g2, y, int(tensor_cores))
    out = torch.empty((T, H), dtype=torch.bfloat16, device=dev)
    ops.moe_combine(y, topk_weights.float().contiguous(), out)
    return out


def unpack_flashinfer(w1, w1_sf, w2, w2_sf):
    """The Flint PR's FlashInfer W4A16 expert tensors (the outputs of prepare_weights,
    vllm/models/flint/ops/moe_cute.py:29-59 / patch:4061-4091: gate/up rows interleaved, scales in the 6-D MMA
    layout, returned as permuted views) -> ModelOpt (w13 u8 [E, 2I, H/2], s13 [E, 2I, H/16], w2 u8 [E, H, I/2],
    s2 [E, H, I/16]) for the decode kernels, on the GPU (flint_flashinfer_nvfp4_unpack), bit for bit.  The scales
    may be given as the PR's 6-D views ([32, 4, m, 4, k, E]) or as their stored arrays ([E, m, k, 32, 4, 4]).  The
    global scales are not part of that layout and pass through unchanged."""
    def stored(sf):
        sf = sf.view(torch.uint8) if sf.dtype != torch.uint8 else sf
        if sf.dim() == 6 and sf.shape[0] == 32 and sf.shape[1] == 4:         # the PR's logical view
            sf = sf.permute(5, 2, 4, 0, 1, 3)
        return sf.contiguous()
    w1, w2 = w1.view(torch.uint8).contiguous(), w2.view(torch.uint8).contiguous()
    E, R13, Hh = w1.shape
    dev = w1.device
    w13 = torch.empty((E, R13, Hh), dtype=torch.uint8, device=dev)
    s13 = torch.empty((E, R13, Hh // 8), dtype=torch.uint8, device=dev)
    w2o = torch.empty_like(w2)
    s2 = torch.empty((E, w2.shape[1], w2.shape[2] // 8), dtype=torch.uint8, device=dev)
    torch.ops.flint_b200.flashinfer_nvfp4_unpack(w1, stored(w1_sf), w2, stored(w2_sf), w13, s13, w2o, s2)
    return w13, s13, w2o, s2


class MarlinDecodeWeights(DecodeWeights):
    """The reference's constructor and argument order (fast/fp4moe_decode.py:27-44, called at fast/model.py:277-282):
    the routed experts' six tensors, then the shared expert's gate_up and down as (weight, weight_scale, global
    scale) tuples, with Flint's routing (top-6 sigmoid, or FLINT_MOE_TOPK / FLINT_MOE_SCORE).

    Accepts what fast/model.py hands over -- vLLM's Marlin-processed tensors (int32 tiles, processed scales and
    global scales; layout fast/fp4moe_mar.cu:1-7) -- and converts them once, on the GPU, to the ModelOpt layout these
    kernels read (``unpack_marlin``; a second copy of the expert weights, while vLLM keeps its Marlin tensors for
    prefill).  ModelOpt tensors (uint8 codes) are used in place."""

    def __init__(self, w13, s13, g13, w2, s2, g2, sh_gu, sh_dn):
        if w13.dtype == torch.int32 and w2.dtype == torch.int32:
            w13, s13, g13 = unpack_marlin(w13, s13, g13)
            w2, s2, g2 = unpack_marlin(w2, s2, g2)
            if sh_gu is not None:
                sh_gu, sh_dn = unpack_marlin(*sh_gu), unpack_marlin(*sh_dn)
        elif w13.dtype != torch.uint8 or w2.dtype != torch.uint8:
            raise ValueError(f"MarlinDecodeWeights: expected Marlin int32 tiles or ModelOpt uint8 codes, got "
                             f"{w13.dtype} / {w2.dtype}")
        shared = None
        if sh_gu is not None:
            shared = (sh_gu[0], sh_gu[1], sh_gu[2].float().reshape(-1)[:1], sh_dn[0], sh_dn[1],
                      sh_dn[2].float().reshape(-1)[:1])
        super().__init__(w13, s13, g13, w2, s2, g2, topk=TOPK, score=SCORE, shared=shared)


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


_ONE_ROUTE: dict = {}


def _one_route(M: int, device):
    """(ids int32 [M, 1] = 0, weights fp32 [M, 1] = 1): every token to expert 0 of a one-expert stack, weight 1."""
    key = (M, device)
    r = _ONE_ROUTE.get(key)
    if r is None:
        r = _ONE_ROUTE[key] = (torch.zeros((M, 1), dtype=torch.int32, device=device),
                               torch.ones((M, 1), dtype=torch.float32, device=device))
    return r


def moe_up(x, ti, w: DecodeWeights):
    """-> (act bf16 [M*k, I], sact bf16 [M, SI] of the shared expert or None)."""
    act = torch.empty((x.shape[0] * ti.shape[-1], w.I), dtype=torch.bfloat16, device=x.device)
    torch.ops.flint_b200.moe_up(x, ti, w.w13, w.s13, w.g13, act)
    sact = None
    if w.shared is not None:
        sw = w.shared
        ids0, _ = _one_route(x.shape[0], x.device)
        sact = torch.empty((x.shape[0], sw.I), dtype=torch.bfloat16, device=x.device)
        torch.ops.flint_b200.moe_up(x, ids0, sw.w13, sw.s13, sw.g13, sact)
    return act, sact


def moe_down(act, sact, ti, tw, w: DecodeWeights, trigger=0):
    """-> bf16(sum_j tw_j * expert_{ti_j}(x)) (+ the shared expert's output, then rounded once more when sact is
    given)."""
    M = ti.shape[0]
    out = torch.empty((M, w.H), dtype=torch.bfloat16, device=act.device)
    torch.ops.flint_b200.moe_down(act, ti, tw, w.w2, w.s2, w.g2, out)
    if sact is not None:
        out = out + shared_down(sact, w)
    return out


def shared_down(sact, w: DecodeWeights):
    """The shared expert's output bf16(sact . W2s^T * gs) [M, H] (weight 1 on its one route)."""
    sw = w.shared
    ids0, one = _one_route(sact.shape[0], sact.device)
    ys = torch.empty((sact.shape[0], sw.H), dtype=torch.bfloat16, device=sact.device)
    torch.ops.flint_b200.moe_down(sact, ids0, one, sw.w2, sw.s2, sw.g2, ys)
    return ys


_ZERO_ROUTER: dict = {}


def dense_mlp(x, res, nw, eps, w: DecodeWeights):
    """Flint's dense SwiGLU layer (the PR's FlintMLP on ``mlp_only_layers``): (bf16(down(silu(g) * u)) of
    rmsnorm(x + res), x + res).  w: a one-expert DecodeWeights (w13 [1, 2I, H/2], w2 [1, H, I/2]).  Runs on the
    MoE chain: the route kernel's add + RMSNorm with an all-zero 32-way router (every token's top-1 is expert 0,
    weight exactly 1), then the up and down kernels."""
    if w.E != 1:
        raise ValueError("dense_mlp takes a one-expert DecodeWeights")
    key = (x.device, w.H)
    zr = _ZERO_ROUTER.get(key)
    if zr is None:
        zr = _ZERO_ROUTER[key] = torch.zeros((32, w.H), dtype=torch.bfloat16, device=x.device)
    tw, ti, xn, res_out, _ = _route_impl(x, res, nw, eps, zr, 1, 0, True)
    act, _ = moe_up(xn, ti, w)
    return moe_down(act, None, ti, tw, w), (res_out if res is not None else None)


def moe_decode(x, res, nw, eps, gate_w, w: DecodeWeights, fused: bool = True, extras: bool = False,
               impl: str | None = None, _routed_only: bool = False):
    """The whole decode MoE block: (mlp(norm(x + res)), x + res).  impl "chain" (fused=False): the three launches
    route_norm -> moe_up -> moe_down; "fused" (fused=True): one persistent launch for 1..8 tokens (flint_moe_fused);
    "block": one launch for one token with the down weights prefetched under the gate/up work (flint_moe_block).
    extras=True (fused / block) also returns (xn, logits, topk_ids, topk_weights)."""
    impl = impl or ("fused" if fused else "chain")
    if (w.shared is not None and impl == "block" and not _routed_only and x.shape[0] == 1 and w.shared.I % 256 == 0
            and w.shared.I <= 1024 and w.topk < 8):
        # the shared expert inside the one-launch block (flint_moe_block_shared)
        dev, M, H = x.device, x.shape[0], x.shape[1]
        out = torch.empty((M, H), dtype=torch.bfloat16, device=dev)
        res_out = torch.empty((M, H), dtype=torch.bfloat16, device=dev) if res is not None else None
        ex = (None, torch.empty((M, w.E), dtype=torch.float32, device=dev),
              torch.empty((M, w.topk), dtype=torch.int32, device=dev), torch.empty((M, w.topk), dtype=torch.float32, device=dev))
        _, lg, ti, tw = ex if extras else (None, None, None, None)
        sw = w.shared
        torch.ops.flint_b200.moe_block_shared(x, res, nw, float(eps), gate_w, w.topk, w.score_fn, w.w13, w.s13, w.g13,
                                              w.w2, w.s2, w.g2, sw.w13[0], sw.s13[0], sw.g13, sw.w2[0], sw.s2[0], sw.g2,
                                              out, res_out, lg, ti, tw)
        return (out, res_out, ex) if extras else (out, res_out)
    if w.shared is not None and impl != "chain" and not _routed_only:
        out, res_out, ex = moe_decode(x, res, nw, eps, gate_w, w, impl=impl, extras=True, _routed_only=True)
        sact = torch.empty((x.shape[0], w.shared.I), dtype=torch.bfloat16, device=x.device)
        ids0, _ = _one_route(x.shape[0], x.device)
        torch.ops.flint_b200.moe_up(ex[0], ids0, w.shared.w13, w.shared.s13, w.shared.g13, sact)
        out = out + shared_down(sact, w)
        return (out, res_out, ex) if extras else (out, res_out)
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
