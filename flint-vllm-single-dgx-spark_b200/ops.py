"""torch custom ops (namespace ``flint_b200``) over the C ABI.

Each op checks shapes/dtypes on the host, calls the matching ``flint_*`` entry point on the current CUDA
stream and raises ``FlintError`` on a non-zero status.  Output buffers are caller-owned (``mutates_args``),
as in the reference, whose Python wrappers allocate outputs with ``torch.empty`` and pass them to the
kernels (fast/fp4moe_decode.py:64-65, fast/attn_gemv.py:126-127).  Ops are CUDA-graph capturable once
their workspaces exist (see ``_lib.workspace``).
"""
from __future__ import annotations

import torch

from . import _lib
from ._lib import check, lib, ptr, stream_ptr

NS = "flint_b200"


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
                tokens: torch.Tensor, write_logits: bool, write_tokens: bool) -> None:
    """logits[m] = gs * x[m] @ dequant(P, S)^T (fp32); tokens[m] = argmax (lowest index on ties)."""
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
    rc = lib().flint_lm_head_nv4(ptr(x), x.stride(0), M, ptr(_u8(P)), ptr(_u8(S)), float(gs), V, K,
                                 ptr(logits) if write_logits else None, logits.stride(0) if write_logits else 0,
                                 ptr(tokens) if write_tokens else None, ptr(ws), 0, stream_ptr(x.device))
    check(rc, "flint_lm_head_nv4")


@lm_head_nv4.register_fake
def _(x, P, S, gs, logits, tokens, write_logits, write_tokens):
    return None
