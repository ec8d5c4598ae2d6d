"""torch custom ops (namespace ``flint_b200``) over the C ABI.

Each op checks shapes/dtypes on the host, calls the matching ``flint_*`` entry point on the current CUDA
stream and raises ``FlintError`` on a non-zero status.  Output buffers are caller-owned (``mutates_args``),
as in the reference, whose Python wrappers allocate outputs with ``torch.empty`` and pass them to the
kernels (fast/fp4moe_decode.py:64-65, fast/attn_gemv.py:126-127).  Ops are CUDA-graph capturable once
their workspaces exist (see ``_lib.workspace``).
"""
from __future__ import annotations

import ctypes
import os

import torch

from . import _lib
from ._lib import check, lib, ptr, stream_ptr

NS = "flint_b200"
# Programmatic dependent launch: each kernel starts (barrier setup, weight prefetch) while its predecessor in the
# stream drains, and waits on it (griddepcontrol.wait) before touching its outputs.
PDL = 1 if os.environ.get("FLINT_PDL", "1") == "1" else 0


def _u8(t: torch.Tensor) -> torch.Tensor:
    return t if t.dtype == torch.uint8 else t.view(torch.uint8)


def _check_nvfp4(P: torch.Tensor, S: torch.Tensor, what: str) -> tuple[int, int]:
    if P.dim() != 2 or S.dim() != 2 or P.shape[0] != S.shape[0] or S.shape[1] * 8 != P.shape[1]:
        raise _lib.FlintError(f"{what}: NVFP4 weight {tuple(P.shape)} / scales {tuple(S.shape)} mismatch")
    if not (P.is_contiguous() and S.is_contiguous()):
        raise _lib.FlintError(f"{what}: NVFP4 weight and scales must be contiguous")
    return P.shape[0], P.shape[1] * 2


# ------------------------------------------------------------------------------------------------------------
# (4) LM head
# ------------------------------------------------------------------------------------------------------------
@torch.library.custom_op(f"{NS}::lm_head_nv4", mutates_args=("logits", "tokens"))
def lm_head_nv4(x: torch.Tensor, P: torch.Tensor, S: torch.Tensor, gs: float, logits: torch.Tensor,
                tokens: torch.Tensor, write_logits: bool, write_tokens: bool, res: torch.Tensor | None = None,
                norm_w: torch.Tensor | None = None, eps: float = 0.0) -> None:
    """logits[m] = gs * x[m] @ dequant(P, S)^T (fp32); tokens[m] = argmax (lowest index on ties).  With norm_w the
    final (residual add +) RMSNorm is applied to x first."""
    _lib.require_cuda(x, "lm_head_nv4")
    V, K = _check_nvfp4(P, S, "lm_head_nv4")
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != K or x.stride(1) != 1:
        raise _lib.FlintError(f"lm_head_nv4: x must be bf16 [M, {K}] with unit inner stride, got {x.dtype} {tuple(x.shape)}")
    M = x.shape[0]
    if write_logits and (logits.dtype != torch.float32 or logits.shape[0] < M or logits.shape[1] < V or logits.stride(1) != 1):
        raise _lib.FlintError("lm_head_nv4: logits must be fp32 [M, V]")
    if write_tokens and (tokens.dtype != torch.int32 or tokens.numel() < M):
        raise _lib.FlintError("lm_head_nv4: tokens must be int32 [M]")
    ws = _lib.workspace(x.device, "lm_head", lib().flint_lm_head_workspace_bytes())
    rc = lib().flint_lm_head_nv4_fused(ptr(x), x.stride(0), ptr(res), ptr(norm_w), float(eps), M, ptr(_u8(P)), ptr(_u8(S)),
                                       float(gs), V, K, ptr(logits) if write_logits else None,
                                       logits.stride(0) if write_logits else 0, ptr(tokens) if write_tokens else None,
                                       ptr(ws), PDL, stream_ptr(x.device))
    check(rc, "flint_lm_head_nv4")


@lm_head_nv4.register_fake
def _(x, P, S, gs, logits, tokens, write_logits, write_tokens, res=None, norm_w=None, eps=0.0):
    return None


@torch.library.custom_op(f"{NS}::lm_head_shard", mutates_args=("keys_out",))
def lm_head_shard(x: torch.Tensor, P: torch.Tensor, S: torch.Tensor, gs: float, index_base: int, keys_out: torch.Tensor,
                  res: torch.Tensor | None, norm_w: torch.Tensor | None, eps: float) -> None:
    """One vocabulary shard of the NVFP4 head: per-row argmax keys (int64 [M], global ids from index_base)."""
    _lib.require_cuda(x, "lm_head_shard")
    V, K = _check_nvfp4(P, S, "lm_head_shard")
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != K or keys_out.dtype != torch.int64:
        raise _lib.FlintError("lm_head_shard: x bf16 [M, K], keys_out int64 [M]")
    ws = _lib.workspace(x.device, "lm_head", lib().flint_lm_head_workspace_bytes())
    rc = lib().flint_lm_head_nv4_shard(ptr(x), x.stride(0), ptr(res), ptr(norm_w), float(eps), x.shape[0], ptr(_u8(P)),
                                       ptr(_u8(S)), float(gs), V, K, int(index_base), ptr(keys_out), ptr(ws), PDL,
                                       stream_ptr(x.device))
    check(rc, "flint_lm_head_nv4_shard")


@lm_head_shard.register_fake
def _(x, P, S, gs, index_base, keys_out, res, norm_w, eps):
    return None


@torch.library.custom_op(f"{NS}::keys_to_tokens", mutates_args=("tokens",))
def keys_to_tokens(keys: torch.Tensor, tokens: torch.Tensor) -> None:
    _lib.require_cuda(keys, "keys_to_tokens")
    rc = lib().flint_argmax_keys_to_tokens(ptr(keys), keys.numel(), ptr(tokens), PDL, stream_ptr(keys.device))
    check(rc, "flint_argmax_keys_to_tokens")


@keys_to_tokens.register_fake
def _(keys, tokens):
    return None


@torch.library.custom_op(f"{NS}::lm_head_sample_shard", mutates_args=("cand_ids", "cand_logits", "scratch"))
def lm_head_sample_shard(x: torch.Tensor, P: torch.Tensor, S: torch.Tensor, gs: float, index_base: int, top_k: int,
                         cand_ids: torch.Tensor, cand_logits: torch.Tensor, scratch: torch.Tensor, res: torch.Tensor | None,
                         norm_w: torch.Tensor | None, eps: float) -> None:
    """One vocabulary shard's sorted top-k sampling candidates (global ids) per row (flint_lm_head_nv4_sample_shard)."""
    _lib.require_cuda(x, "lm_head_sample_shard")
    V, K = _check_nvfp4(P, S, "lm_head_sample_shard")
    M = x.shape[0]
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != K or cand_ids.numel() < M * top_k:
        raise _lib.FlintError("lm_head_sample_shard: x bf16 [M, K], candidates [M, top_k]")
    ws = _lib.workspace(x.device, f"lm_head_sample_{M}_{V}", lib().flint_lm_head_sample_workspace_bytes(M, V))
    rc = lib().flint_lm_head_nv4_sample_shard(ptr(x), x.stride(0), ptr(res), ptr(norm_w), float(eps), M, ptr(_u8(P)),
                                              ptr(_u8(S)), float(gs), V, K, int(index_base), int(top_k), ptr(cand_ids),
                                              ptr(cand_logits), ptr(scratch), ptr(ws), PDL, stream_ptr(x.device))
    check(rc, "flint_lm_head_nv4_sample_shard")


@lm_head_sample_shard.register_fake
def _(x, P, S, gs, index_base, top_k, cand_ids, cand_logits, scratch, res, norm_w, eps):
    return None


@torch.library.custom_op(f"{NS}::sample_merge", mutates_args=("tokens",))
def sample_merge(cand_ids: torch.Tensor, cand_logits: torch.Tensor, temperature: float, top_p: float,
                 seeds: torch.Tensor, step: torch.Tensor | None, tokens: torch.Tensor) -> None:
    """Draw from the gathered shard candidates [R, M, top_k] (flint_sample_merge)."""
    _lib.require_cuda(cand_ids, "sample_merge")
    R, M, k = cand_ids.shape
    rc = lib().flint_sample_merge(ptr(cand_ids), ptr(cand_logits), R, M, k, float(temperature), float(top_p), ptr(seeds),
                                  ptr(step), ptr(tokens), None, PDL, stream_ptr(cand_ids.device))
    check(rc, "flint_sample_merge")


@sample_merge.register_fake
def _(cand_ids, cand_logits, temperature, top_p, seeds, step, tokens):
    return None


@torch.library.custom_op(f"{NS}::lm_head_sample", mutates_args=("tokens", "logits", "cand_ids", "cand_logits", "kept"))
def lm_head_sample(x: torch.Tensor, P: torch.Tensor, S: torch.Tensor, gs: float, temperature: float, top_k: int,
                   top_p: float, seeds: torch.Tensor, step: torch.Tensor | None, tokens: torch.Tensor,
                   logits: torch.Tensor | None, cand_ids: torch.Tensor | None, cand_logits: torch.Tensor | None,
                   kept: torch.Tensor | None, res: torch.Tensor | None = None, norm_w: torch.Tensor | None = None,
                   eps: float = 0.0) -> None:
    """Seeded temperature -> top-k -> top-p draw fused into the NVFP4 head (rule: include/flint_b200.h,
    flint_lm_head_nv4_sample).  seeds: int64 [M] (the bits are the Philox key); step: int32 [1] device counter.
    The optional outputs (logits, cand_ids, cand_logits, kept) are positional without defaults: torch drops trailing
    arguments equal to their defaults when it boxes a call, which would hide a mutated argument."""
    _lib.require_cuda(x, "lm_head_sample")
    V, K = _check_nvfp4(P, S, "lm_head_sample")
    if x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != K or x.stride(1) != 1:
        raise _lib.FlintError(f"lm_head_sample: x must be bf16 [M, {K}] with unit inner stride")
    M = x.shape[0]
    if seeds.dtype != torch.int64 or seeds.numel() < M or not seeds.is_contiguous():
        raise _lib.FlintError("lm_head_sample: seeds must be contiguous int64 [M]")
    if step is not None and step.dtype != torch.int32:
        raise _lib.FlintError("lm_head_sample: step must be an int32 device counter")
    if tokens.dtype != torch.int32 or tokens.numel() < M:
        raise _lib.FlintError("lm_head_sample: tokens must be int32 [M]")
    if logits is not None and (logits.dtype != torch.float32 or logits.shape[0] < M or logits.shape[1] < V
                               or logits.stride(1) != 1):
        raise _lib.FlintError("lm_head_sample: logits must be fp32 [M, V]")
    for t, dt, what in ((cand_ids, torch.int32, "cand_ids"), (cand_logits, torch.float32, "cand_logits")):
        if t is not None and (t.dtype != dt or t.numel() < M * top_k or not t.is_contiguous()):
            raise _lib.FlintError(f"lm_head_sample: {what} must be contiguous {dt} [M, top_k]")
    if kept is not None and (kept.dtype != torch.int32 or kept.numel() < M):
        raise _lib.FlintError("lm_head_sample: kept must be int32 [M]")
    nbytes = lib().flint_lm_head_sample_workspace_bytes(M, V)
    ws = _lib.workspace(x.device, f"lm_head_sample_{M}_{V}", nbytes)
    rc = lib().flint_lm_head_nv4_sample(
        ptr(x), x.stride(0), ptr(res), ptr(norm_w), float(eps), M, ptr(_u8(P)), ptr(_u8(S)), float(gs), V, K, ptr(logits),
        logits.stride(0) if logits is not None else 0, float(temperature), int(top_k), float(top_p), ptr(seeds), ptr(step),
        ptr(tokens), ptr(cand_ids), ptr(cand_logits), ptr(kept), ptr(ws), PDL, stream_ptr(x.device))
    check(rc, "flint_lm_head_nv4_sample")


@lm_head_sample.register_fake
def _(x, P, S, gs, temperature, top_k, top_p, seeds, step, tokens, logits, cand_ids, cand_logits, kept, res=None,
      norm_w=None, eps=0.0):
    return None


# ------------------------------------------------------------------------------------------------------------
# (1) MoE decode and (2) deterministic align
# ------------------------------------------------------------------------------------------------------------
def _moe_ws(device: torch.device, H: int) -> torch.Tensor:
    return _lib.workspace(device, "moe", lib().flint_moe_workspace_bytes(H))


def _bf16_2d(t: torch.Tensor, what: str) -> None:
    if t.dtype != torch.bfloat16 or t.dim() != 2 or t.stride(1) != 1:
        raise _lib.FlintError(f"{what}: expected a bf16 matrix with unit inner stride, got {t.dtype} {tuple(t.shape)}")


@torch.library.custom_op(f"{NS}::moe_route", mutates_args=("logits", "topk_ids", "topk_weights", "xn", "res_out"))
def moe_route(x: torch.Tensor, res: torch.Tensor | None, norm_w: torch.Tensor | None, eps: float, gate_w: torch.Tensor,
              topk: int, score_fn: int, logits: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor,
              xn: torch.Tensor, res_out: torch.Tensor, write_xn: bool, write_res: bool) -> None:
    """Router: (residual add +) RMSNorm, bf16 logits, top-k (softmax: score_fn 0, sigmoid: 1), renormalised weights."""
    _lib.require_cuda(x, "moe_route")
    _bf16_2d(x, "moe_route x")
    M, H = x.shape
    E = gate_w.shape[0]
    if gate_w.dtype != torch.bfloat16 or gate_w.shape[1] != H or not gate_w.is_contiguous():
        raise _lib.FlintError("moe_route: gate_w must be contiguous bf16 [E, H]")
    if res is not None and (res.shape != x.shape or res.stride() != x.stride() or res.dtype != torch.bfloat16):
        raise _lib.FlintError("moe_route: res must match x")
    rc = lib().flint_moe_route(ptr(x), x.stride(0), ptr(res), ptr(norm_w), float(eps), ptr(gate_w), M, H, E, topk,
                               score_fn, ptr(logits), ptr(topk_ids), ptr(topk_weights), ptr(xn) if write_xn else None,
                               ptr(res_out) if write_res else None, ptr(_moe_ws(x.device, H)), PDL, stream_ptr(x.device))
    check(rc, "flint_moe_route")


@moe_route.register_fake
def _(x, res, norm_w, eps, gate_w, topk, score_fn, logits, topk_ids, topk_weights, xn, res_out, write_xn, write_res):
    return None


@torch.library.custom_op(f"{NS}::moe_up", mutates_args=("act",))
def moe_up(xn: torch.Tensor, topk_ids: torch.Tensor, w13: torch.Tensor, s13: torch.Tensor, g13: torch.Tensor,
           act: torch.Tensor) -> None:
    """act[m*topk+s] = bf16(silu(g) * u) of expert topk_ids[m, s] (NVFP4 gate/up rows [0:I] / [I:2I])."""
    _lib.require_cuda(xn, "moe_up")
    _bf16_2d(xn, "moe_up xn")
    M, H = xn.shape
    E, I2, Hh = w13.shape
    topk = topk_ids.shape[-1]
    if Hh * 2 != H or s13.shape != (E, I2, H // 16) or g13.numel() != E or act.shape != (M * topk, I2 // 2):
        raise _lib.FlintError("moe_up: weight / activation shapes mismatch")
    rc = lib().flint_moe_up(ptr(xn), xn.stride(0), M, ptr(topk_ids), topk, ptr(_u8(w13)), ptr(_u8(s13)), ptr(g13), E,
                            I2 // 2, H, ptr(act), ptr(_moe_ws(xn.device, H)), PDL, stream_ptr(xn.device))
    check(rc, "flint_moe_up")


@moe_up.register_fake
def _(xn, topk_ids, w13, s13, g13, act):
    return None


@torch.library.custom_op(f"{NS}::moe_down", mutates_args=("out",))
def moe_down(act: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, w2: torch.Tensor, s2: torch.Tensor,
             g2: torch.Tensor, out: torch.Tensor) -> None:
    """out[m] = bf16(sum_s topk_weights[m, s] * bf16(act[m*topk+s] . W2[e] * g2[e]))."""
    _lib.require_cuda(act, "moe_down")
    E, H, Ih = w2.shape
    M, topk = topk_ids.shape
    if act.shape != (M * topk, Ih * 2) or s2.shape != (E, H, Ih // 8) or g2.numel() != E or out.shape != (M, H):
        raise _lib.FlintError("moe_down: weight / activation shapes mismatch")
    rc = lib().flint_moe_down(ptr(act), M, ptr(topk_ids), ptr(topk_weights), topk, ptr(_u8(w2)), ptr(_u8(s2)), ptr(g2), E,
                              Ih * 2, H, ptr(out), ptr(_moe_ws(act.device, H)), PDL, stream_ptr(act.device))
    check(rc, "flint_moe_down")


@moe_down.register_fake
def _(act, topk_ids, topk_weights, w2, s2, g2, out):
    return None


@torch.library.custom_op(f"{NS}::moe_up_ep", mutates_args=("act",))
def moe_up_ep(xn: torch.Tensor, topk_ids: torch.Tensor, w13: torch.Tensor, s13: torch.Tensor, g13: torch.Tensor,
              num_experts: int, expert_lo: int, act: torch.Tensor) -> None:
    """Expert-parallel moe_up (flint_moe_up_ep): act rows of the routes whose expert is local (w13 holds experts
    expert_lo .. expert_lo + n_local - 1 of num_experts)."""
    _lib.require_cuda(xn, "moe_up_ep")
    _bf16_2d(xn, "moe_up_ep xn")
    M, H = xn.shape
    n_local, I2, Hh = w13.shape
    topk = topk_ids.shape[-1]
    if Hh * 2 != H or act.shape != (M * topk, I2 // 2):
        raise _lib.FlintError("moe_up_ep: weight / activation shapes mismatch")
    rc = lib().flint_moe_up_ep(ptr(xn), xn.stride(0), M, ptr(topk_ids), topk, ptr(_u8(w13)), ptr(_u8(s13)), ptr(g13),
                               int(num_experts), I2 // 2, H, int(expert_lo), n_local, ptr(act), ptr(_moe_ws(xn.device, H)),
                               PDL, stream_ptr(xn.device))
    check(rc, "flint_moe_up_ep")


@moe_up_ep.register_fake
def _(xn, topk_ids, w13, s13, g13, num_experts, expert_lo, act):
    return None


@torch.library.custom_op(f"{NS}::moe_down_ep", mutates_args=("y_out",))
def moe_down_ep(act: torch.Tensor, topk_ids: torch.Tensor, w2: torch.Tensor, s2: torch.Tensor, g2: torch.Tensor,
                num_experts: int, expert_lo: int, y_out: torch.Tensor) -> None:
    """Expert-parallel moe_down (flint_moe_down_ep): y_out [M * topk, H] = y of each local route, zero rows for the
    others (sum over ranks, then moe_combine)."""
    _lib.require_cuda(act, "moe_down_ep")
    n_local, H, Ih = w2.shape
    M, topk = topk_ids.shape
    if act.shape != (M * topk, Ih * 2) or y_out.shape != (M * topk, H):
        raise _lib.FlintError("moe_down_ep: weight / activation shapes mismatch")
    rc = lib().flint_moe_down_ep(ptr(act), M, ptr(topk_ids), topk, ptr(_u8(w2)), ptr(_u8(s2)), ptr(g2), int(num_experts),
                                 Ih * 2, H, int(expert_lo), n_local, ptr(y_out), ptr(_moe_ws(act.device, H)), PDL,
                                 stream_ptr(act.device))
    check(rc, "flint_moe_down_ep")


@moe_down_ep.register_fake
def _(act, topk_ids, w2, s2, g2, num_experts, expert_lo, y_out):
    return None


@torch.library.custom_op(f"{NS}::moe_fused", mutates_args=("out", "res_out", "xn_out", "logits_out", "ids_out",
                                                             "tw_out"))
def moe_fused(x: torch.Tensor, res: torch.Tensor | None, norm_w: torch.Tensor, eps: float, gate_w: torch.Tensor, topk: int,
              score_fn: int, w13: torch.Tensor, s13: torch.Tensor, g13: torch.Tensor, w2: torch.Tensor, s2: torch.Tensor,
              g2: torch.Tensor, out: torch.Tensor, res_out: torch.Tensor, xn_out: torch.Tensor, logits_out: torch.Tensor,
              ids_out: torch.Tensor, tw_out: torch.Tensor, write_extras: bool) -> None:
    """The whole decode MoE block in one persistent launch: (add +) RMSNorm, router, top-k, gate/up + SwiGLU, down,
    weighted sum.  res_out always written when res is given; xn / logits / ids / weights when write_extras."""
    _lib.require_cuda(x, "moe_fused")
    _bf16_2d(x, "moe_fused x")
    M, H = x.shape
    E, I2, Hh = w13.shape
    if Hh * 2 != H or gate_w.shape != (E, H) or out.shape != (M, H):
        raise _lib.FlintError("moe_fused: shape mismatch")
    nbytes = lib().flint_moe_fused_workspace_bytes(E, H, I2 // 2)
    ws = _lib.workspace(x.device, f"moe_fused_{E}_{H}_{I2 // 2}", nbytes)
    ex = write_extras
    rc = lib().flint_moe_fused(ptr(x), x.stride(0), ptr(res), ptr(norm_w), float(eps), ptr(gate_w), M, H, E, topk, score_fn,
                               ptr(_u8(w13)), ptr(_u8(s13)), ptr(g13), ptr(_u8(w2)), ptr(_u8(s2)), ptr(g2), I2 // 2,
                               ptr(out), ptr(res_out) if res is not None else None, ptr(xn_out) if ex else None,
                               ptr(logits_out) if ex else None, ptr(ids_out) if ex else None, ptr(tw_out) if ex else None,
                               ptr(ws), PDL, stream_ptr(x.device))
    check(rc, "flint_moe_fused")


@moe_fused.register_fake
def _(x, res, norm_w, eps, gate_w, topk, score_fn, w13, s13, g13, w2, s2, g2, out, res_out, xn_out, logits_out, ids_out,
      tw_out, write_extras):
    return None


@torch.library.custom_op(f"{NS}::moe_fused_ep", mutates_args=("y_out", "res_out", "ids_out", "tw_out"))
def moe_fused_ep(x: torch.Tensor, res: torch.Tensor | None, norm_w: torch.Tensor, eps: float, gate_w: torch.Tensor,
                 topk: int, score_fn: int, w13: torch.Tensor, s13: torch.Tensor, g13: torch.Tensor, w2: torch.Tensor,
                 s2: torch.Tensor, g2: torch.Tensor, num_experts: int, expert_lo: int, y_out: torch.Tensor,
                 res_out: torch.Tensor | None, ids_out: torch.Tensor, tw_out: torch.Tensor) -> None:
    """Expert-parallel fused MoE for 1..8 tokens (flint_moe_fused_ep): per-route rows of the local experts (zero rows
    for the others), the routing of every token and the residual."""
    _lib.require_cuda(x, "moe_fused_ep")
    _bf16_2d(x, "moe_fused_ep x")
    M, H = x.shape
    n_local, I2, Hh = w13.shape
    if Hh * 2 != H or gate_w.shape != (num_experts, H) or y_out.shape != (M * topk, H):
        raise _lib.FlintError("moe_fused_ep: shapes must match the expert weights")
    if res is not None and res.stride() != x.stride():
        raise _lib.FlintError("moe_fused_ep: res must have x's row stride")
    nbytes = lib().flint_moe_fused_workspace_bytes(num_experts, H, I2 // 2)
    ws = _lib.workspace(x.device, f"moe_fused_{num_experts}_{H}_{I2 // 2}", nbytes)
    rc = lib().flint_moe_fused_ep(ptr(x), x.stride(0), ptr(res), ptr(norm_w), float(eps), ptr(gate_w), M, H,
                                  int(num_experts), topk, score_fn, ptr(_u8(w13)), ptr(_u8(s13)), ptr(g13), ptr(_u8(w2)),
                                  ptr(_u8(s2)), ptr(g2), I2 // 2, int(expert_lo), n_local, ptr(y_out), ptr(res_out),
                                  None, ptr(ids_out), ptr(tw_out), ptr(ws), PDL, stream_ptr(x.device))
    check(rc, "flint_moe_fused_ep")


@moe_fused_ep.register_fake
def _(x, res, norm_w, eps, gate_w, topk, score_fn, w13, s13, g13, w2, s2, g2, num_experts, expert_lo, y_out, res_out,
      ids_out, tw_out):
    return None


@torch.library.custom_op(f"{NS}::moe_block", mutates_args=("out", "res_out", "xn_out", "logits_out", "ids_out",
                                                             "tw_out"))
def moe_block(x: torch.Tensor, res: torch.Tensor | None, norm_w: torch.Tensor, eps: float, gate_w: torch.Tensor, topk: int,
              score_fn: int, w13: torch.Tensor, s13: torch.Tensor, g13: torch.Tensor, w2: torch.Tensor, s2: torch.Tensor,
              g2: torch.Tensor, out: torch.Tensor, res_out: torch.Tensor | None, xn_out: torch.Tensor | None,
              logits_out: torch.Tensor | None, ids_out: torch.Tensor | None, tw_out: torch.Tensor | None,
              prefetch: list[int] | None = None) -> None:
    """The decode MoE block of ONE token in one launch (flint_moe_block).  The optional outputs are positional
    without defaults (torch drops trailing default-valued arguments when it boxes a call).  prefetch: optional
    (pointer, bytes) pairs the kernel pulls into L2 for the op that follows (prefetch_ranges)."""
    _lib.require_cuda(x, "moe_block")
    _bf16_2d(x, "moe_block x")
    M, H = x.shape
    E, I2, Hh = w13.shape
    if M != 1 or Hh * 2 != H or gate_w.shape != (E, H) or out.shape != (1, H):
        raise _lib.FlintError("moe_block: one token, shapes must match the expert weights")
    nbytes = lib().flint_moe_block_workspace_bytes(E, I2 // 2)
    ws = _lib.workspace(x.device, f"moe_block_{E}_{I2 // 2}", nbytes)
    pf, pf_arg = _prefetch_arg(prefetch)
    rc = lib().flint_moe_block(ptr(x), x.stride(0), ptr(res), ptr(norm_w), float(eps), ptr(gate_w), H, E, topk, score_fn,
                               ptr(_u8(w13)), ptr(_u8(s13)), ptr(g13), ptr(_u8(w2)), ptr(_u8(s2)), ptr(g2), I2 // 2,
                               ptr(out), ptr(res_out), ptr(xn_out), ptr(logits_out), ptr(ids_out), ptr(tw_out), ptr(ws),
                               pf_arg, PDL, stream_ptr(x.device))
    check(rc, "flint_moe_block")


@moe_block.register_fake
def _(x, res, norm_w, eps, gate_w, topk, score_fn, w13, s13, g13, w2, s2, g2, out, res_out, xn_out, logits_out, ids_out,
      tw_out, prefetch=None):
    return None


@torch.library.custom_op(f"{NS}::moe_block_shared", mutates_args=("out", "res_out", "logits_out", "ids_out", "tw_out"))
def moe_block_shared(x: torch.Tensor, res: torch.Tensor | None, norm_w: torch.Tensor, eps: float, gate_w: torch.Tensor,
                     topk: int, score_fn: int, w13: torch.Tensor, s13: torch.Tensor, g13: torch.Tensor, w2: torch.Tensor,
                     s2: torch.Tensor, g2: torch.Tensor, sw13: torch.Tensor, ss13: torch.Tensor, sg13: torch.Tensor,
                     sw2: torch.Tensor, ss2: torch.Tensor, sg2: torch.Tensor, out: torch.Tensor,
                     res_out: torch.Tensor | None, logits_out: torch.Tensor | None, ids_out: torch.Tensor | None,
                     tw_out: torch.Tensor | None) -> None:
    """moe_block with Flint's ungated shared expert in the same launch (flint_moe_block_shared): shared gate/up
    sw13 u8 [2SI, H/2] + ss13 [2SI, H/16] + sg13 fp32 [1], down sw2 u8 [H, SI/2] + ss2 [H, SI/16] + sg2 fp32 [1];
    out = bf16(bf16(routed) + shared)."""
    _lib.require_cuda(x, "moe_block_shared")
    _bf16_2d(x, "moe_block_shared x")
    M, H = x.shape
    E, I2, Hh = w13.shape
    SI2 = sw13.shape[-2]
    if M != 1 or Hh * 2 != H or gate_w.shape != (E, H) or out.shape != (1, H) or sw13.shape[-1] * 2 != H or \
            sw2.shape[-2] != H or sw2.shape[-1] * 4 != SI2:
        raise _lib.FlintError("moe_block_shared: one token, shapes must match the expert weights")
    nbytes = lib().flint_moe_block_workspace_bytes(E, I2 // 2)
    ws = _lib.workspace(x.device, f"moe_block_{E}_{I2 // 2}", nbytes)
    rc = lib().flint_moe_block_shared(ptr(x), x.stride(0), ptr(res), ptr(norm_w), float(eps), ptr(gate_w), H, E, topk,
                                      score_fn, ptr(_u8(w13)), ptr(_u8(s13)), ptr(g13), ptr(_u8(w2)), ptr(_u8(s2)),
                                      ptr(g2), I2 // 2, ptr(_u8(sw13)), ptr(_u8(ss13)), ptr(sg13), ptr(_u8(sw2)),
                                      ptr(_u8(ss2)), ptr(sg2), SI2 // 2, ptr(out), ptr(res_out), None, ptr(logits_out),
                                      ptr(ids_out), ptr(tw_out), ptr(ws), None, PDL, stream_ptr(x.device))
    check(rc, "flint_moe_block_shared")


@moe_block_shared.register_fake
def _(x, res, norm_w, eps, gate_w, topk, score_fn, w13, s13, g13, w2, s2, g2, sw13, ss13, sg13, sw2, ss2, sg2, out,
      res_out, logits_out, ids_out, tw_out):
    return None


@torch.library.custom_op(f"{NS}::moe_block_ep", mutates_args=("y_out", "tw_out", "res_out"))
def moe_block_ep(x: torch.Tensor, res: torch.Tensor | None, norm_w: torch.Tensor, eps: float, gate_w: torch.Tensor,
                 topk: int, score_fn: int, w13: torch.Tensor, s13: torch.Tensor, g13: torch.Tensor, w2: torch.Tensor,
                 s2: torch.Tensor, g2: torch.Tensor, expert_lo: int, y_out: torch.Tensor, tw_out: torch.Tensor,
                 res_out: torch.Tensor | None, prefetch: list[int] | None = None) -> None:
    """Expert-parallel one-token MoE block (flint_moe_block_ep): the local experts' rows of y_out [topk, H], zeros for
    the other ranks' slots, and the routing weights."""
    _lib.require_cuda(x, "moe_block_ep")
    _bf16_2d(x, "moe_block_ep x")
    M, H = x.shape
    n_local, I2, Hh = w13.shape
    E = gate_w.shape[0]
    if M != 1 or Hh * 2 != H or gate_w.shape[1] != H or y_out.shape != (topk, H) or tw_out.numel() < topk:
        raise _lib.FlintError("moe_block_ep: shapes do not match")
    nbytes = lib().flint_moe_block_workspace_bytes(E, I2 // 2)
    ws = _lib.workspace(x.device, f"moe_block_{E}_{I2 // 2}", nbytes)
    pf, pf_arg = _prefetch_arg(prefetch)
    rc = lib().flint_moe_block_ep(ptr(x), x.stride(0), ptr(res), ptr(norm_w), float(eps), ptr(gate_w), H, E, topk,
                                  score_fn, ptr(_u8(w13)), ptr(_u8(s13)), ptr(g13), ptr(_u8(w2)), ptr(_u8(s2)), ptr(g2),
                                  I2 // 2, int(expert_lo), n_local, ptr(y_out), ptr(tw_out), ptr(res_out), ptr(ws), pf_arg,
                                  PDL, stream_ptr(x.device))
    check(rc, "flint_moe_block_ep")


@moe_block_ep.register_fake
def _(x, res, norm_w, eps, gate_w, topk, score_fn, w13, s13, g13, w2, s2, g2, expert_lo, y_out, tw_out, res_out,
      prefetch=None):
    return None


@torch.library.custom_op(f"{NS}::moe_combine", mutates_args=("out",))
def moe_combine(y: torch.Tensor, tw: torch.Tensor, out: torch.Tensor) -> None:
    """out [M, H] = bf16(sum_s tw[m, s] * y[m * topk + s]) in slot order; y [M * topk, H], tw [M, topk]."""
    _lib.require_cuda(y, "moe_combine")
    M = out.shape[0] if out.dim() == 2 else 1
    R, H = y.shape
    if R % M or tw.numel() != R:
        raise _lib.FlintError("moe_combine: y [M * topk, H], tw [M, topk], out [M, H]")
    rc = lib().flint_moe_combine(ptr(y), ptr(tw), M, R // M, H, ptr(out), PDL, stream_ptr(y.device))
    check(rc, "flint_moe_combine")


@moe_combine.register_fake
def _(y, tw, out):
    return None


class _L2Prefetch(ctypes.Structure):
    """flint_l2_prefetch (include/flint_b200.h)."""
    _fields_ = [("ptr", ctypes.c_void_p * 8), ("bytes", ctypes.c_int64 * 8), ("n", ctypes.c_int32),
                ("kv", ctypes.c_void_p), ("block_bytes", ctypes.c_int64), ("kv_blocks", ctypes.c_int64),
                ("block_tables", ctypes.c_void_p), ("bt_stride", ctypes.c_int64), ("bt_cols", ctypes.c_int64),
                ("seq_lens", ctypes.c_void_p), ("streams", ctypes.c_int32), ("block_tokens", ctypes.c_int32),
                ("max_blocks", ctypes.c_int32)]


_KV_TAG = -1          # starts the paged-KV part of a prefetch spec (prefetch_kv)


def _prefetch_arg(spec: list[int] | None):
    """[ptr0, bytes0, ptr1, bytes1, ...] (+ a prefetch_kv tail) -> (struct kept alive by the caller, pointer
    argument) or (None, None)."""
    if not spec:
        return None, None
    kv = None
    if _KV_TAG in spec:
        i = spec.index(_KV_TAG)
        spec, kv = spec[:i], spec[i + 1:]
        if len(kv) != 10:
            raise _lib.FlintError("prefetch: malformed paged-KV part")
    if len(spec) % 2 or len(spec) > 16:
        raise _lib.FlintError("prefetch: up to 8 (pointer, bytes) pairs")
    pf = _L2Prefetch()
    pf.n = len(spec) // 2
    for i in range(pf.n):
        pf.ptr[i], pf.bytes[i] = spec[2 * i], spec[2 * i + 1]
    if kv is not None:
        (pf.kv, pf.block_bytes, pf.kv_blocks, pf.block_tables, pf.bt_stride, pf.bt_cols, pf.seq_lens, pf.streams,
         pf.block_tokens, pf.max_blocks) = kv
    return pf, ctypes.cast(ctypes.pointer(pf), ctypes.c_void_p)


def prefetch_kv(kv: torch.Tensor, block_tables: torch.Tensor, seq_lens: torch.Tensor, max_blocks: int) -> list[int]:
    """The paged-KV part of a prefetch spec: the pages of kv (HND [blocks, kv_heads, block_tokens, 2 D], whole blocks)
    that streams 0 .. len(seq_lens) - 1 will read, at most max_blocks blocks; append to prefetch_ranges(...)."""
    if kv.dim() != 4 or not kv.is_contiguous() or block_tables.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise _lib.FlintError("prefetch_kv: contiguous HND cache, int32 block tables and sequence lengths")
    blk = kv.stride(0) * kv.element_size()
    return [_KV_TAG, kv.data_ptr(), blk, kv.shape[0], block_tables.data_ptr(), block_tables.stride(0),
            block_tables.shape[1], seq_lens.data_ptr(), seq_lens.numel(), kv.shape[2], int(max_blocks)]


def prefetch_ranges(*tensors: torch.Tensor) -> list[int]:
    """The flattened (pointer, bytes) list of whole tensors, for the ops' `prefetch` argument."""
    out: list[int] = []
    for t in tensors:
        out += [t.data_ptr(), t.numel() * t.element_size()]
    return out


def _peer_array(peers: list[int]):
    return (ctypes.c_void_p * len(peers))(*peers)


@torch.library.custom_op(f"{NS}::moe_block_peer", mutates_args=("out", "res_out"))
def moe_block_peer(x: torch.Tensor, res: torch.Tensor | None, norm_w: torch.Tensor, eps: float, gate_w: torch.Tensor,
                   topk: int, score_fn: int, w13: torch.Tensor, s13: torch.Tensor, g13: torch.Tensor, w2: torch.Tensor,
                   s2: torch.Tensor, g2: torch.Tensor, expert_lo: int, peers: list[int], rank: int, out: torch.Tensor,
                   res_out: torch.Tensor | None, prefetch: list[int] | None = None) -> None:
    """Expert-parallel one-token MoE block with the exchange fused in (flint_moe_block_peer): every rank gets the
    full weighted expert sum in out [1, H].  peers: every rank's exchange buffer as mapped here (PeerBuffers.ptrs)."""
    _lib.require_cuda(x, "moe_block_peer")
    _bf16_2d(x, "moe_block_peer x")
    M, H = x.shape
    n_local, I2, Hh = w13.shape
    E = gate_w.shape[0]
    if M != 1 or Hh * 2 != H or gate_w.shape[1] != H or out.shape[-1] != H:
        raise _lib.FlintError("moe_block_peer: shapes do not match")
    nbytes = lib().flint_moe_block_workspace_bytes(E, I2 // 2)
    ws = _lib.workspace(x.device, f"moe_block_{E}_{I2 // 2}", nbytes)
    pf, pf_arg = _prefetch_arg(prefetch)
    rc = lib().flint_moe_block_peer(ptr(x), x.stride(0), ptr(res), ptr(norm_w), float(eps), ptr(gate_w), H, E, topk,
                                    score_fn, ptr(_u8(w13)), ptr(_u8(s13)), ptr(g13), ptr(_u8(w2)), ptr(_u8(s2)), ptr(g2),
                                    I2 // 2, int(expert_lo), n_local, _peer_array(peers), int(rank), len(peers), ptr(out),
                                    ptr(res_out), ptr(ws), pf_arg, PDL, stream_ptr(x.device))
    check(rc, "flint_moe_block_peer")


@moe_block_peer.register_fake
def _(x, res, norm_w, eps, gate_w, topk, score_fn, w13, s13, g13, w2, s2, g2, expert_lo, peers, rank, out, res_out,
      prefetch=None):
    return None


@torch.library.custom_op(f"{NS}::dp_gather_peer", mutates_args=("out",))
def dp_gather_peer(send: torch.Tensor, peers: list[int], rank: int, out: torch.Tensor) -> None:
    """Every rank's two rows (bf16 [2, H]) into out [world, 2, H] over NVLink peer memory (flint_dp_gather_peer)."""
    _lib.require_cuda(send, "dp_gather_peer")
    H = send.shape[-1]
    if send.dtype != torch.bfloat16 or send.numel() != 2 * H or out.numel() != len(peers) * 2 * H or \
            not send.is_contiguous() or not out.is_contiguous():
        raise _lib.FlintError("dp_gather_peer: send bf16 [2, H], out [world, 2, H], contiguous")
    rc = lib().flint_dp_gather_peer(ptr(send), H, _peer_array(peers), int(rank), len(peers), ptr(out), PDL,
                                    stream_ptr(send.device))
    check(rc, "flint_dp_gather_peer")


@dp_gather_peer.register_fake
def _(send, peers, rank, out):
    return None


@torch.library.custom_op(f"{NS}::dp_combine_peer", mutates_args=("out",))
def dp_combine_peer(y: torch.Tensor, topk_ids: torch.Tensor, topk_weights: torch.Tensor, num_experts: int,
                    peers: list[int], rank: int, out: torch.Tensor) -> None:
    """Each route's row to its token's rank over NVLink peer memory, then this rank's token's slot-order weighted
    sum (flint_dp_combine_peer)."""
    _lib.require_cuda(y, "dp_combine_peer")
    W = len(peers)
    R, H = y.shape
    topk = topk_ids.shape[-1]
    if R != W * topk or topk_ids.numel() != R or topk_weights.numel() != R or out.numel() != H:
        raise _lib.FlintError("dp_combine_peer: y [world * topk, H], ids / weights [world, topk], out [H]")
    rc = lib().flint_dp_combine_peer(ptr(y), ptr(topk_ids), ptr(topk_weights), topk, int(num_experts), H,
                                     _peer_array(peers), int(rank), W, ptr(out), PDL, stream_ptr(y.device))
    check(rc, "flint_dp_combine_peer")


@dp_combine_peer.register_fake
def _(y, topk_ids, topk_weights, num_experts, peers, rank, out):
    return None


@torch.library.custom_op(f"{NS}::dp_combine_peer_recv", mutates_args=("out",))
def dp_combine_peer_recv(topk_ids: torch.Tensor, topk_weights: torch.Tensor, num_experts: int, peers: list[int],
                         rank: int, out: torch.Tensor) -> None:
    """This rank's token's slot-order weighted sum of the rows that flint_moe_fused_dp_peer pushed
    (flint_dp_combine_peer with y NULL)."""
    _lib.require_cuda(out, "dp_combine_peer_recv")
    W, topk = topk_ids.shape
    H = out.numel()
    if W != len(peers) or topk_weights.shape != topk_ids.shape:
        raise _lib.FlintError("dp_combine_peer_recv: ids / weights [world, topk], out [H]")
    rc = lib().flint_dp_combine_peer(None, ptr(topk_ids), ptr(topk_weights), topk, int(num_experts), H,
                                     _peer_array(peers), int(rank), W, ptr(out), PDL, stream_ptr(out.device))
    check(rc, "flint_dp_combine_peer")


@dp_combine_peer_recv.register_fake
def _(topk_ids, topk_weights, num_experts, peers, rank, out):
    return None


@torch.library.custom_op(f"{NS}::moe_fused_dp_peer", mutates_args=("res_out", "ids_out", "tw_out"))
def moe_fused_dp_peer(send: torch.Tensor, norm_w: torch.Tensor, eps: float, gate_w: torch.Tensor, topk: int,
                      score_fn: int, w13: torch.Tensor, s13: torch.Tensor, g13: torch.Tensor, w2: torch.Tensor,
                      s2: torch.Tensor, g2: torch.Tensor, num_experts: int, expert_lo: int, peers: list[int], rank: int,
                      res_out: torch.Tensor, ids_out: torch.Tensor, tw_out: torch.Tensor) -> None:
    """The data-parallel MoE layer with its exchanges inside the launch (flint_moe_fused_dp_peer): this rank's rows
    send bf16 [2, H] in, every rank's residual res_out [world, H] and routing ids_out / tw_out [world, topk] out; the
    local routes' rows go to their tokens' ranks for dp_combine_peer_recv."""
    _lib.require_cuda(send, "moe_fused_dp_peer")
    W = len(peers)
    H = send.shape[-1]
    n_local, I2, Hh = w13.shape
    if send.dtype != torch.bfloat16 or send.numel() != 2 * H or not send.is_contiguous() or Hh * 2 != H or \
            gate_w.shape != (num_experts, H) or res_out.shape != (W, H) or ids_out.shape != (W, topk) or \
            tw_out.shape != (W, topk):
        raise _lib.FlintError("moe_fused_dp_peer: send bf16 [2, H], res_out [world, H], ids / weights [world, topk]")
    nbytes = lib().flint_moe_fused_workspace_bytes(num_experts, H, I2 // 2)
    ws = _lib.workspace(send.device, f"moe_fused_{num_experts}_{H}_{I2 // 2}", nbytes)
    rc = lib().flint_moe_fused_dp_peer(ptr(send), ptr(norm_w), float(eps), ptr(gate_w), H, int(num_experts), int(topk),
                                       int(score_fn), ptr(_u8(w13)), ptr(_u8(s13)), ptr(g13), ptr(_u8(w2)),
                                       ptr(_u8(s2)), ptr(g2), I2 // 2, int(expert_lo), n_local, _peer_array(peers),
                                       int(rank), W, ptr(res_out), None, ptr(ids_out), ptr(tw_out), ptr(ws), PDL,
                                       stream_ptr(send.device))
    check(rc, "flint_moe_fused_dp_peer")


@moe_fused_dp_peer.register_fake
def _(send, norm_w, eps, gate_w, topk, score_fn, w13, s13, g13, w2, s2, g2, num_experts, expert_lo, peers, rank,
      res_out, ids_out, tw_out):
    return None


@torch.library.custom_op(f"{NS}::keys_allmax_peer", mutates_args=("tokens",))
def keys_allmax_peer(keys: torch.Tensor, peers: list[int], rank: int, tokens: torch.Tensor) -> None:
    """Argmax over the vocabulary shards of all ranks (flint_argmax_keys_allmax_peer)."""
    _lib.require_cuda(keys, "keys_allmax_peer")
    rc = lib().flint_argmax_keys_allmax_peer(ptr(keys), keys.numel(), _peer_array(peers), int(rank), len(peers),
                                             ptr(tokens), PDL, stream_ptr(keys.device))
    check(rc, "flint_argmax_keys_allmax_peer")


@keys_allmax_peer.register_fake
def _(keys, peers, rank, tokens):
    return None


@torch.library.custom_op(f"{NS}::moe_align", mutates_args=("sorted_ids", "expert_ids", "num_tokens_post_pad"))
def moe_align(topk_ids: torch.Tensor, num_experts: int, block_size: int, sorted_ids: torch.Tensor,
              expert_ids: torch.Tensor, num_tokens_post_pad: torch.Tensor) -> None:
    """Deterministic moe_align_block_size (routes of an expert in ascending route order)."""
    _lib.require_cuda(topk_ids, "moe_align")
    ids = topk_ids if topk_ids.dtype == torch.int32 and topk_ids.is_contiguous() else topk_ids.contiguous().to(torch.int32)
    status = _lib.workspace(topk_ids.device, "align_status", 4)
    rc = lib().flint_moe_align(ptr(ids), ids.numel(), num_experts, block_size, ptr(sorted_ids), sorted_ids.numel(),
                               ptr(expert_ids), expert_ids.numel(), ptr(num_tokens_post_pad), ptr(status), 0,
                               stream_ptr(topk_ids.device))
    check(rc, "flint_moe_align")


@moe_align.register_fake
def _(topk_ids, num_experts, block_size, sorted_ids, expert_ids, num_tokens_post_pad):
    return None


# ------------------------------------------------------------------------------------------------------------
# (3) attention block
# ------------------------------------------------------------------------------------------------------------
def _proj_ws(device):
    return _lib.workspace(device, "attn_proj", lib().flint_attn_proj_workspace_bytes())


@torch.library.custom_op(f"{NS}::attn_qkv", mutates_args=("q_out", "qkv_out", "res_out", "k_cache", "v_cache"))
def attn_qkv(x: torch.Tensor, res: torch.Tensor | None, norm_w: torch.Tensor, eps: float, W: torch.Tensor,
             S: torch.Tensor, gs: torch.Tensor, num_q_heads: int, num_kv_heads: int, head_mode: bool,
             q_norm_w: torch.Tensor | None, k_norm_w: torch.Tensor | None, eps_head: float,
             positions: torch.Tensor | None, cos_sin: torch.Tensor | None, k_cache: torch.Tensor, v_cache: torch.Tensor,
             slots: torch.Tensor | None, q_out: torch.Tensor, qkv_out: torch.Tensor, res_out: torch.Tensor,
             write_res: bool, tokens: torch.Tensor | None = None) -> None:
    """Fused (add +) RMSNorm + NVFP4 QKV GEMV (+ q/k norm, RoPE and paged KV write when head_mode).  With tokens
    (int32 [M]) x is an embedding table and row m of the input is x[tokens[m]]."""
    _lib.require_cuda(x, "attn_qkv")
    _bf16_2d(x, "attn_qkv x")
    N, K = _check_nvfp4(W, S, "attn_qkv")
    M, H = (x.shape[0], x.shape[1]) if tokens is None else (tokens.numel(), x.shape[1])
    if H != K or qkv_out.shape != (M, N) or (res is not None and res.stride() != x.stride()):
        raise _lib.FlintError("attn_qkv: shape mismatch")
    if head_mode and (k_cache.dim() != 4 or k_cache.stride(3) != 1 or v_cache.stride() != k_cache.stride()):
        raise _lib.FlintError("attn_qkv: caches must be [blocks, block_size, kv_heads, head_dim] views, unit inner stride")
    if head_mode and positions is not None and positions.dtype != torch.int64:
        raise _lib.FlintError("attn_qkv: positions must be int64")
    if head_mode and slots is not None and slots.dtype != torch.int64:
        raise _lib.FlintError("attn_qkv: slots must be int64")
    cs = cos_sin if (head_mode and cos_sin is not None) else None
    rc = lib().flint_attn_qkv(
        ptr(x), x.stride(0), ptr(tokens), ptr(res), ptr(norm_w), float(eps), ptr(_u8(W)), ptr(_u8(S)), ptr(gs), M, H, N, num_q_heads,
        num_kv_heads, 1 if head_mode else 0, ptr(q_norm_w), ptr(k_norm_w), float(eps_head), ptr(positions), ptr(cs),
        cs.stride(0) if cs is not None else 0, ptr(k_cache) if head_mode else None, ptr(v_cache) if head_mode else None,
        k_cache.stride(0) if head_mode else 0, k_cache.stride(1) if head_mode else 0, k_cache.stride(2) if head_mode else 0,
        k_cache.shape[1] if head_mode else 1, ptr(slots), ptr(q_out) if head_mode else None, ptr(qkv_out),
        ptr(res_out) if write_res else None, ptr(_proj_ws(x.device)), PDL, stream_ptr(x.device))
    check(rc, "flint_attn_qkv")


@attn_qkv.register_fake
def _(x, res, norm_w, eps, W, S, gs, num_q_heads, num_kv_heads, head_mode, q_norm_w, k_norm_w, eps_head, positions,
      cos_sin, k_cache, v_cache, slots, q_out, qkv_out, res_out, write_res, tokens=None):
    return None


@torch.library.custom_op(f"{NS}::attn_o", mutates_args=("y",))
def attn_o(a: torch.Tensor, W: torch.Tensor, S: torch.Tensor, gs: torch.Tensor, y: torch.Tensor) -> None:
    """y = bf16(gs * a @ dequant(W, S)^T)."""
    _lib.require_cuda(a, "attn_o")
    _bf16_2d(a, "attn_o a")
    N, K = _check_nvfp4(W, S, "attn_o")
    M = a.shape[0]
    if a.shape[1] != K or y.shape != (M, N):
        raise _lib.FlintError("attn_o: shape mismatch")
    rc = lib().flint_attn_o(ptr(a), a.stride(0), M, ptr(_u8(W)), ptr(_u8(S)), ptr(gs), N, K, ptr(y),
                            ptr(_proj_ws(a.device)), PDL, stream_ptr(a.device))
    check(rc, "flint_attn_o")


@attn_o.register_fake
def _(a, W, S, gs, y):
    return None


@torch.library.custom_op(f"{NS}::attn_block", mutates_args=("kv_cache", "out", "res_out", "q_out", "attn_out"))
def attn_block(x: torch.Tensor, res: torch.Tensor | None, norm_w: torch.Tensor, eps: float, W: torch.Tensor,
               S: torch.Tensor, gs: torch.Tensor, num_q_heads: int, num_kv_heads: int, q_norm_w: torch.Tensor,
               k_norm_w: torch.Tensor, eps_head: float, positions: torch.Tensor, cos_sin: torch.Tensor | None,
               kv_cache: torch.Tensor, block_tables: torch.Tensor, seq_lens: torch.Tensor, slots: torch.Tensor,
               sinks: torch.Tensor | None, window: int, scale: float, Wo: torch.Tensor, So: torch.Tensor,
               gs_o: torch.Tensor, out: torch.Tensor, res_out: torch.Tensor, q_out: torch.Tensor | None,
               attn_out: torch.Tensor | None, tokens: torch.Tensor | None = None) -> None:
    """The fused decode attention block (one launch): add + RMSNorm, QKV, q/k norm + RoPE + KV write, paged attention,
    O projection.  With tokens (int32 [M]) x is the embedding table.  q_out / attn_out: optional outputs (positional,
    no defaults, so that torch never drops them when it boxes the call)."""
    _lib.require_cuda(x, "attn_block")
    _bf16_2d(x, "attn_block x")
    N, K = _check_nvfp4(W, S, "attn_block qkv")
    No, Ko = _check_nvfp4(Wo, So, "attn_block o")
    M = x.shape[0] if tokens is None else tokens.numel()
    H = x.shape[1]
    if H != K or Ko != num_q_heads * 128 or N != (num_q_heads + 2 * num_kv_heads) * 128:
        raise _lib.FlintError("attn_block: weight shapes do not match the head layout")
    if out.shape != (M, No) or res_out.shape != (M, H) or out.stride() != res_out.stride():
        raise _lib.FlintError("attn_block: out / res_out must be [M, N_o] / [M, H] with equal strides")
    if res is not None and (res.shape != (M, H) or res.stride() != out.stride()):
        raise _lib.FlintError("attn_block: res must be [M, H] with the stride of out")
    nblk, hkv, page, d2 = kv_cache.shape
    if hkv != num_kv_heads or page != 16 or d2 != 256 or kv_cache.stride(3) != 1 or kv_cache.stride(2) != 256:
        raise _lib.FlintError("attn_block: kv_cache must be HND bf16 [blocks, kv_heads, 16, 256]")
    if block_tables.dtype != torch.int32 or seq_lens.dtype != torch.int32 or positions.dtype != torch.int64 \
            or slots.dtype != torch.int64:
        raise _lib.FlintError("attn_block: block_tables / seq_lens int32, positions / slots int64")
    nbytes = lib().flint_attn_block_workspace_bytes(N, Ko)
    ws = _lib.workspace(x.device, f"attn_block_{N}_{Ko}", nbytes)
    rc = lib().flint_attn_block(
        ptr(x), x.stride(0), ptr(tokens), ptr(res), out.stride(0), ptr(norm_w), float(eps), M, H, ptr(_u8(W)), ptr(_u8(S)),
        ptr(gs), num_q_heads, num_kv_heads, ptr(q_norm_w), ptr(k_norm_w), float(eps_head), ptr(positions), ptr(cos_sin),
        cos_sin.stride(0) if cos_sin is not None else 0, ptr(kv_cache), nblk, kv_cache.stride(0), kv_cache.stride(1),
        ptr(block_tables), block_tables.stride(0), block_tables.shape[1], ptr(seq_lens), ptr(slots), ptr(sinks),
        int(window), float(scale), ptr(_u8(Wo)), ptr(_u8(So)), ptr(gs_o), No, ptr(out), ptr(res_out), ptr(q_out),
        ptr(attn_out), ptr(ws), PDL, stream_ptr(x.device))
    check(rc, "flint_attn_block")


@attn_block.register_fake
def _(x, res, norm_w, eps, W, S, gs, num_q_heads, num_kv_heads, q_norm_w, k_norm_w, eps_head, positions, cos_sin,
      kv_cache, block_tables, seq_lens, slots, sinks, window, scale, Wo, So, gs_o, out, res_out, q_out, attn_out,
      tokens=None):
    return None


def attention_splits(batch: int, num_kv_heads: int) -> int:
    return int(lib().flint_decode_attention_splits(batch, num_kv_heads))


@torch.library.custom_op(f"{NS}::decode_attention", mutates_args=("out",))
def decode_attention(q: torch.Tensor, kv_cache: torch.Tensor, block_tables: torch.Tensor, seq_lens: torch.Tensor,
                     sinks: torch.Tensor | None, window: int, scale: float, out: torch.Tensor, splits: int) -> None:
    """Paged split-K decode attention (HND bf16 cache [blocks, kv_heads, 16, 2*128])."""
    _lib.require_cuda(q, "decode_attention")
    B, Hq, D = q.shape
    nblk, Hkv, page, D2 = kv_cache.shape
    if D != 128 or page != 16 or D2 != 256 or kv_cache.stride(3) != 1 or kv_cache.stride(2) != 256:
        raise _lib.FlintError("decode_attention: kv_cache must be HND bf16 [blocks, kv_heads, 16, 256]")
    if q.stride(2) != 1 or q.stride(1) != D or out.stride(2) != 1 or out.stride(1) != D:
        raise _lib.FlintError("decode_attention: q / out must be [B, heads, 128] with contiguous heads")
    if block_tables.dtype != torch.int32 or seq_lens.dtype != torch.int32:
        raise _lib.FlintError("decode_attention: block_tables / seq_lens must be int32")
    nbytes = lib().flint_decode_attention_workspace_bytes(B, Hkv, splits)
    ws = _lib.workspace(q.device, "decode_attention", nbytes)
    rc = lib().flint_decode_attention(ptr(q), q.stride(0), ptr(kv_cache), nblk, Hkv, kv_cache.stride(0),
                                      kv_cache.stride(1), ptr(block_tables), block_tables.stride(0),
                                      block_tables.shape[1], ptr(seq_lens), ptr(sinks), int(window), float(scale), B, Hq,
                                      ptr(out), out.stride(0), splits, ptr(ws), PDL, stream_ptr(q.device))
    check(rc, "flint_decode_attention")


@decode_attention.register_fake
def _(q, kv_cache, block_tables, seq_lens, sinks, window, scale, out, splits):
    return None


# ------------------------------------------------------------------------------------------------------------
# device-side decode bookkeeping
# ------------------------------------------------------------------------------------------------------------
@torch.library.custom_op(f"{NS}::decode_advance", mutates_args=("positions", "seq_lens", "slots", "history", "step",
                                                                 "next_tokens"))
def decode_advance(tokens: torch.Tensor, positions: torch.Tensor, seq_lens: torch.Tensor, slots: torch.Tensor,
                   block_tables: torch.Tensor, block_size: int, history: torch.Tensor, step: torch.Tensor,
                   next_tokens: torch.Tensor) -> None:
    """Record tokens in history[:, step], advance positions / seq_lens, next KV slots from the block table."""
    _lib.require_cuda(tokens, "decode_advance")
    M = tokens.numel()
    rc = lib().flint_decode_advance(ptr(tokens), M, ptr(positions), ptr(seq_lens), ptr(slots), ptr(block_tables),
                                    block_tables.stride(0), block_tables.shape[1], block_size,
                                    ptr(history) if history.numel() else None, history.stride(0) if history.dim() else 0,
                                    ptr(step), history.shape[1] if history.dim() == 2 else 0,
                                    ptr(next_tokens) if next_tokens.numel() else None, PDL, stream_ptr(tokens.device))
    check(rc, "flint_decode_advance")


@decode_advance.register_fake
def _(tokens, positions, seq_lens, slots, block_tables, block_size, history, step, next_tokens):
    return None


# ------------------------------------------------------------------------------------------------------------
# checkpoint format: GGUF NVFP4 -> ModelOpt NVFP4, and the exact dequant
# ------------------------------------------------------------------------------------------------------------
@torch.library.custom_op(f"{NS}::gguf_nvfp4_repack", mutates_args=("packed", "scales", "bad_blocks"))
def gguf_nvfp4_repack(blocks: torch.Tensor, n_cols: int, packed: torch.Tensor, scales: torch.Tensor,
                      bad_blocks: torch.Tensor) -> None:
    """GGUF NVFP4 super-blocks u8 [..., n_cols/64*36] -> packed u8 [..., n_cols/2] and E4M3 bits u8
    [..., n_cols/16]; bad_blocks (int32 [1], zeroed by the caller) counts warps that met the scale byte 0xFF."""
    _lib.require_cuda(blocks, "gguf_nvfp4_repack")
    if n_cols % 64 or blocks.shape[-1] != n_cols // 64 * 36:
        raise _lib.FlintError(f"gguf_nvfp4_repack: last dim {blocks.shape[-1]} is not {n_cols}/64*36")
    rows = blocks.numel() // blocks.shape[-1] if blocks.shape[-1] else 0
    if packed.numel() != rows * n_cols // 2 or scales.numel() != rows * n_cols // 16:
        raise _lib.FlintError("gguf_nvfp4_repack: output sizes do not match the input")
    if not (blocks.is_contiguous() and packed.is_contiguous() and scales.is_contiguous()):
        raise _lib.FlintError("gguf_nvfp4_repack: tensors must be contiguous")
    if rows == 0:
        return
    rc = lib().flint_gguf_nvfp4_repack(ptr(blocks), rows, n_cols, ptr(packed), ptr(scales), ptr(bad_blocks), 0,
                                       stream_ptr(blocks.device))
    check(rc, "flint_gguf_nvfp4_repack")


@gguf_nvfp4_repack.register_fake
def _(blocks, n_cols, packed, scales, bad_blocks):
    return None


@torch.library.custom_op(f"{NS}::marlin_nvfp4_unpack", mutates_args=("packed", "scales", "global_out", "bad"))
def marlin_nvfp4_unpack(weight: torch.Tensor, weight_scale: torch.Tensor, global_scale: torch.Tensor,
                        packed: torch.Tensor, scales: torch.Tensor, global_out: torch.Tensor, bad: torch.Tensor) -> None:
    """Marlin-processed NVFP4 (int32 [E, K/16, 2N], processed scale bytes [E, K/16, N], processed global fp32 [E])
    -> ModelOpt packed u8 [E, N, K/2], E4M3 bits u8 [E, N, K/16], global fp32 [E]; bad (int32 [1], zeroed by the
    caller) counts CTAs that met a byte that is not a processed scale."""
    _lib.require_cuda(weight, "marlin_nvfp4_unpack")
    if weight.dtype != torch.int32 or weight.dim() != 3:
        raise _lib.FlintError("marlin_nvfp4_unpack: weight must be int32 [E, K/16, 2N]")
    E, KT, W2 = weight.shape
    N, K = W2 // 2, KT * 16
    if tuple(weight_scale.shape) != (E, KT, N) or tuple(packed.shape) != (E, N, K // 2) or \
            tuple(scales.shape) != (E, N, K // 16) or global_scale.numel() != E or global_out.numel() != E:
        raise _lib.FlintError("marlin_nvfp4_unpack: shapes do not match the weight")
    for t in (weight, weight_scale, global_scale, packed, scales, global_out):
        if not t.is_contiguous():
            raise _lib.FlintError("marlin_nvfp4_unpack: tensors must be contiguous")
    if global_scale.dtype != torch.float32 or global_out.dtype != torch.float32:
        raise _lib.FlintError("marlin_nvfp4_unpack: global scales are fp32")
    rc = lib().flint_marlin_nvfp4_unpack(ptr(weight), ptr(_u8(weight_scale)), ptr(global_scale), E, N, K, ptr(packed),
                                         ptr(scales), ptr(global_out), ptr(bad), 0, stream_ptr(weight.device))
    check(rc, "flint_marlin_nvfp4_unpack")


@marlin_nvfp4_unpack.register_fake
def _(weight, weight_scale, global_scale, packed, scales, global_out, bad):
    return None


@torch.library.custom_op(f"{NS}::flashinfer_nvfp4_unpack", mutates_args=("w13_out", "s13_out", "w2_out", "s2_out"))
def flashinfer_nvfp4_unpack(w1: torch.Tensor, w1_sf: torch.Tensor, w2: torch.Tensor, w2_sf: torch.Tensor,
                            w13_out: torch.Tensor, s13_out: torch.Tensor, w2_out: torch.Tensor,
                            s2_out: torch.Tensor) -> None:
    """FlashInfer W4A16 NVFP4 experts (w1 u8 [E, 2I, H/2] interleaved, w1_sf stored 6-D [E, 2I/128, H/64, 32, 4, 4],
    w2 u8 [E, H, I/2], w2_sf [E, H/128, I/64, 32, 4, 4]) -> ModelOpt codes and scale bytes
    (flint_flashinfer_nvfp4_unpack)."""
    _lib.require_cuda(w1, "flashinfer_nvfp4_unpack")
    E, R13, Hh = w1.shape
    H, I = 2 * Hh, R13 // 2
    if w1.dtype != torch.uint8 or w2.dtype != torch.uint8 or tuple(w2.shape) != (E, H, I // 2) or \
            w1_sf.numel() != E * R13 * (H // 16) or w2_sf.numel() != E * H * (I // 16) or \
            tuple(w13_out.shape) != (E, R13, Hh) or tuple(s13_out.shape) != (E, R13, H // 16) or \
            tuple(w2_out.shape) != (E, H, I // 2) or tuple(s2_out.shape) != (E, H, I // 16):
        raise _lib.FlintError("flashinfer_nvfp4_unpack: shapes do not match w1 [E, 2I, H/2]")
    for t in (w1, w1_sf, w2, w2_sf, w13_out, s13_out, w2_out, s2_out):
        if not t.is_contiguous():
            raise _lib.FlintError("flashinfer_nvfp4_unpack: tensors must be contiguous (scales in their stored order)")
    rc = lib().flint_flashinfer_nvfp4_unpack(ptr(w1), ptr(_u8(w1_sf)), ptr(w2), ptr(_u8(w2_sf)), E, H, I,
                                             ptr(w13_out), ptr(s13_out), ptr(w2_out), ptr(s2_out), 0,
                                             stream_ptr(w1.device))
    check(rc, "flint_flashinfer_nvfp4_unpack")


@flashinfer_nvfp4_unpack.register_fake
def _(w1, w1_sf, w2, w2_sf, w13_out, s13_out, w2_out, s2_out):
    return None


@torch.library.custom_op(f"{NS}::rows_to_f16", mutates_args=("dst", "shift"))
def rows_to_f16(src: torch.Tensor, dst: torch.Tensor, shift: torch.Tensor) -> None:
    """bf16 rows [n, K] -> f16 rows x * 2^shift[row] with the decode kernels' per-row power of two
    (flint_rows_to_f16)."""
    _lib.require_cuda(src, "rows_to_f16")
    _bf16_2d(src, "rows_to_f16 src")
    n, K = src.shape
    if dst.dtype != torch.float16 or tuple(dst.shape) != (n, K) or not dst.is_contiguous() or shift.numel() != n:
        raise _lib.FlintError("rows_to_f16: dst f16 [n, K] contiguous, shift int32 [n]")
    rc = lib().flint_rows_to_f16(ptr(src), src.stride(0), n, K, ptr(dst), ptr(shift), PDL, stream_ptr(src.device))
    check(rc, "flint_rows_to_f16")


@rows_to_f16.register_fake
def _(src, dst, shift):
    return None


def _grouped(fn: str, xh, shift, sorted_ids, expert_ids, ntp, numel, topk, w, s, g, H, I, out, tc):
    _lib.require_cuda(xh, fn)
    ws = _lib.workspace(xh.device, "moe_grouped_status", 4)
    rc = getattr(lib(), f"flint_{fn}")(ptr(xh), ptr(shift), ptr(sorted_ids), ptr(expert_ids), ptr(ntp), int(numel),
                                       int(topk), w.shape[0], ptr(_u8(w)), ptr(_u8(s)), ptr(g), int(H), int(I),
                                       expert_ids.numel(), ptr(out), ptr(ws), int(tc), PDL, stream_ptr(xh.device))
    check(rc, f"flint_{fn}")


@torch.library.custom_op(f"{NS}::moe_grouped_up", mutates_args=("act",))
def moe_grouped_up(xh: torch.Tensor, shift: torch.Tensor, sorted_ids: torch.Tensor, expert_ids: torch.Tensor,
                   num_tokens_post_pad: torch.Tensor, numel: int, topk: int, w13: torch.Tensor, s13: torch.Tensor,
                   g13: torch.Tensor, act: torch.Tensor, tensor_cores: int) -> None:
    """Prefill gate/up + SwiGLU of the aligned routes (flint_moe_grouped_up): act bf16 [numel, I] per route;
    tensor_cores 1: tcgen05, 0: mma.sync."""
    H = xh.shape[1]
    I = w13.shape[1] // 2
    if act.shape != (numel, I) or w13.shape[2] * 2 != H:
        raise _lib.FlintError("moe_grouped_up: act [numel, I], w13 [E, 2I, H/2]")
    _grouped("moe_grouped_up", xh, shift, sorted_ids, expert_ids, num_tokens_post_pad, numel, topk, w13, s13, g13, H,
             I, act, tensor_cores)


@moe_grouped_up.register_fake
def _(xh, shift, sorted_ids, expert_ids, num_tokens_post_pad, numel, topk, w13, s13, g13, act, tensor_cores):
    return None


@torch.library.custom_op(f"{NS}::moe_grouped_down", mutates_args=("y",))
def moe_grouped_down(ah: torch.Tensor, shift: torch.Tensor, sorted_ids: torch.Tensor, expert_ids: torch.Tensor,
                     num_tokens_post_pad: torch.Tensor, numel: int, topk: int, w2: torch.Tensor, s2: torch.Tensor,
                     g2: torch.Tensor, y: torch.Tensor, tensor_cores: int) -> None:
    """Prefill down projection of the aligned routes (flint_moe_grouped_down): y bf16 [numel, H] per route;
    tensor_cores 1: tcgen05, 0: mma.sync."""
    I = ah.shape[1]
    H = w2.shape[1]
    if y.shape != (numel, H) or w2.shape[2] * 2 != I:
        raise _lib.FlintError("moe_grouped_down: y [numel, H], w2 [E, H, I/2]")
    _grouped("moe_grouped_down", ah, shift, sorted_ids, expert_ids, num_tokens_post_pad, numel, topk, w2, s2, g2, H, I,
             y, tensor_cores)


@moe_grouped_down.register_fake
def _(ah, shift, sorted_ids, expert_ids, num_tokens_post_pad, numel, topk, w2, s2, g2, y, tensor_cores):
    return None


@torch.library.custom_op(f"{NS}::nvfp4_dequant", mutates_args=("out",))
def nvfp4_dequant(P: torch.Tensor, S: torch.Tensor, global_scale: torch.Tensor | None, out: torch.Tensor) -> None:
    """out [..., K] (fp32 or bf16) = e2m1(P) * e4m3(S) (* global_scale, one fp32 scalar on the device)."""
    _lib.require_cuda(P, "nvfp4_dequant")
    K = P.shape[-1] * 2
    rows = P.numel() // P.shape[-1] if P.shape[-1] else 0
    if S.numel() != rows * K // 16 or out.numel() != rows * K or out.dtype not in (torch.float32, torch.bfloat16):
        raise _lib.FlintError(f"nvfp4_dequant: weight {tuple(P.shape)}, scales {tuple(S.shape)}, "
                              f"out {tuple(out.shape)} {out.dtype}")
    if not (P.is_contiguous() and S.is_contiguous() and out.is_contiguous()):
        raise _lib.FlintError("nvfp4_dequant: tensors must be contiguous")
    gs = None
    if global_scale is not None:
        if global_scale.numel() != 1 or global_scale.dtype != torch.float32 or global_scale.device != P.device:
            raise _lib.FlintError("nvfp4_dequant: global_scale must be one fp32 value on the weight's device")
        gs = ptr(global_scale)
    if rows == 0:
        return
    rc = lib().flint_nvfp4_dequant(ptr(_u8(P)), ptr(_u8(S)), rows, K, gs, 1 if out.dtype == torch.float32 else 0,
                                   ptr(out), 0, stream_ptr(P.device))
    check(rc, "flint_nvfp4_dequant")


@nvfp4_dequant.register_fake
def _(P, S, global_scale, out):
    return None


# ------------------------------------------------------------------------------------------------------------
# functional fused forms (allocate their outputs): the whole MoE block, the whole attention block, the whole head
# ------------------------------------------------------------------------------------------------------------
@torch.library.custom_op(f"{NS}::moe_decode", mutates_args=())
def moe_decode(x: torch.Tensor, res: torch.Tensor | None, norm_w: torch.Tensor, eps: float, gate_w: torch.Tensor,
               w13: torch.Tensor, s13: torch.Tensor, g13: torch.Tensor, w2: torch.Tensor, s2: torch.Tensor,
               g2: torch.Tensor, topk: int, score_fn: int) -> tuple[torch.Tensor, torch.Tensor]:
    """(mlp(rmsnorm(x + res)), x + res) of the decode MoE block in one launch: flint_moe_block for one token when
    its shape limits allow (H 2048, E <= 256, I <= 1024), else flint_moe_fused (1..8 tokens)."""
    M, H = x.shape
    E, I2, _ = w13.shape
    out = torch.empty((M, H), dtype=torch.bfloat16, device=x.device)
    res_out = torch.empty((M, H), dtype=torch.bfloat16, device=x.device)
    if res is None:
        res_out.copy_(x)
    if M == 1 and H == 2048 and E <= 256 and I2 // 2 <= 1024:
        moe_block(x, res, norm_w, eps, gate_w, topk, score_fn, w13, s13, g13, w2, s2, g2, out,
                  res_out if res is not None else None, None, None, None, None)
    else:
        dev = x.device
        moe_fused(x, res, norm_w, eps, gate_w, topk, score_fn, w13, s13, g13, w2, s2, g2, out, res_out,
                  torch.empty((M, H), dtype=torch.bfloat16, device=dev),
                  torch.empty((M, E), dtype=torch.float32, device=dev),
                  torch.empty((M, topk), dtype=torch.int32, device=dev),
                  torch.empty((M, topk), dtype=torch.float32, device=dev), False)
    return out, res_out


@moe_decode.register_fake
def _(x, res, norm_w, eps, gate_w, w13, s13, g13, w2, s2, g2, topk, score_fn):
    return torch.empty_like(x), torch.empty_like(x)


@torch.library.custom_op(f"{NS}::attn_decode", mutates_args=("kv_cache",))
def attn_decode(x: torch.Tensor, res: torch.Tensor | None, norm_w: torch.Tensor, eps: float, W: torch.Tensor,
                S: torch.Tensor, gs: torch.Tensor, num_q_heads: int, num_kv_heads: int, q_norm_w: torch.Tensor,
                k_norm_w: torch.Tensor, eps_head: float, positions: torch.Tensor, cos_sin: torch.Tensor | None,
                kv_cache: torch.Tensor, block_tables: torch.Tensor, seq_lens: torch.Tensor, slots: torch.Tensor,
                sinks: torch.Tensor | None, window: int, scale: float, Wo: torch.Tensor, So: torch.Tensor,
                gs_o: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """(o_proj(attention(qkv(rmsnorm(x + res)))), x + res) of the decode attention block in one launch
    (flint_attn_block): add + RMSNorm, QKV, q/k norm, RoPE (cos_sin None: none), the KV write at slots, paged GQA
    attention (sinks, window) and the O projection."""
    M = x.shape[0]
    out = torch.empty((M, Wo.shape[0]), dtype=torch.bfloat16, device=x.device)
    res_out = torch.empty((M, x.shape[1]), dtype=torch.bfloat16, device=x.device)
    attn_block(x, res, norm_w, eps, W, S, gs, num_q_heads, num_kv_heads, q_norm_w, k_norm_w, eps_head, positions,
               cos_sin, kv_cache, block_tables, seq_lens, slots, sinks, window, scale, Wo, So, gs_o, out, res_out, None,
               None)
    return out, res_out


@attn_decode.register_fake
def _(x, res, norm_w, eps, W, S, gs, num_q_heads, num_kv_heads, q_norm_w, k_norm_w, eps_head, positions, cos_sin,
      kv_cache, block_tables, seq_lens, slots, sinks, window, scale, Wo, So, gs_o):
    M = x.shape[0]
    return x.new_empty((M, Wo.shape[0])), x.new_empty((M, x.shape[1]))


@torch.library.custom_op(f"{NS}::lm_head", mutates_args=())
def lm_head(x: torch.Tensor, P: torch.Tensor, S: torch.Tensor, gs: float, mode: str, temperature: float, top_k: int,
            top_p: float, seeds: torch.Tensor | None, step: torch.Tensor | None,
            want_logits: bool) -> tuple[torch.Tensor, torch.Tensor]:
    """(tokens int32 [M], logits fp32 [M, V] or an empty tensor) of the NVFP4 head in one pass: mode "greedy" (argmax,
    lowest id on ties) or "sample" (seeded temperature -> top-k -> top-p draw; seeds int64 [M], step int32 [1])."""
    if mode not in ("greedy", "sample"):
        raise _lib.FlintError(f"lm_head: mode must be 'greedy' or 'sample', got {mode!r}")
    M, dev = x.shape[0], x.device
    tokens = torch.empty((M,), dtype=torch.int32, device=dev)
    logits = torch.empty((M, P.shape[0]) if want_logits else (0,), dtype=torch.float32, device=dev)
    if mode == "greedy":
        lm_head_nv4(x, P, S, gs, logits if want_logits else torch.empty((1, 1), dtype=torch.float32, device=dev),
                    tokens, want_logits, True)
    else:
        if seeds is None:
            raise _lib.FlintError("lm_head: mode 'sample' needs one int64 seed per row")
        lm_head_sample(x, P, S, gs, temperature, top_k, top_p, seeds, step, tokens, logits if want_logits else None,
                       None, None, None)
    return tokens, logits


@lm_head.register_fake
def _(x, P, S, gs, mode, temperature, top_k, top_p, seeds, step, want_logits):
    M = x.shape[0]
    return (x.new_empty((M,), dtype=torch.int32),
            x.new_empty((M, P.shape[0]) if want_logits else (0,), dtype=torch.float32))
