"""Batch-1 (1..8 token) NVFP4 attention GEMVs -- drop-in for the reference's ``fast/attn_gemv.py``.

Same entry points, arguments and outputs (fast/attn_gemv.py:24-58):

* ``qkv_gemv(x, res, nw, eps, W, S, gs, pdl=True) -> (qkv [M, N], res_out [M, H])``
* ``qkv_head(x, res, nw, eps, W, S, gs, q_w, k_w, positions, cos_sin, k_cache, v_cache, slots, trigger=True, pdl=True)
  -> (q [M, 32*128], qkv [M, N], res_out)`` -- fused add+RMSNorm, QKV GEMV, per-head q/k RMSNorm (same eps), NeoX RoPE
  from the fp32 cos|sin table, KV-cache write at ``slots``
* ``o_gemv(a, W, S, gs, pdl=True, trigger=0) -> y [M, H]``
* ``counters(device)`` -- the persistent per-device workspace (allocate before CUDA graph capture)

W u8 [N, K/2], S E4M3 [N, K/16] are the raw ModelOpt NVFP4 tensors, gs the fp32 global scale (device tensor).
The head counts default to Flint's / the BASELINE's 32 query and 4 KV heads of dim 128 (``NUM_Q_HEADS`` /
``NUM_KV_HEADS`` or keyword arguments).
"""
from __future__ import annotations

import torch

from . import _lib
from . import ops as _ops

NUM_Q_HEADS = 32
NUM_KV_HEADS = 4
HEAD_DIM = 128


def get_ext():
    return _lib.lib()


def counters(device):
    """Persistent workspace of the projection kernels (zeroed at allocation).  Allocate before CUDA graph capture."""
    return _ops._proj_ws(torch.device(device))


def _gs(gs, dev):
    if isinstance(gs, torch.Tensor):
        return gs.float().reshape(-1)[:1].contiguous()
    return torch.tensor([float(gs)], dtype=torch.float32, device=dev)


def qkv_gemv(x, res, nw, eps, W, S, gs, pdl=True, num_q_heads=None, num_kv_heads=None):
    """x, res [M, H] bf16 (res may be None). Returns (qkv [M, N] bf16 = GEMV(rmsnorm(x + res)), new residual [M, H])."""
    M, H = x.shape
    N = W.shape[0]
    nkv = num_kv_heads or NUM_KV_HEADS
    nq = num_q_heads or (N // HEAD_DIM - 2 * nkv)
    dev = x.device
    y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    res_out = torch.empty((M, H), dtype=torch.bfloat16, device=dev)
    dummy = torch.empty((0,), dtype=torch.bfloat16, device=dev)
    torch.ops.flint_b200.attn_qkv(x, res, nw, float(eps), W, S, _gs(gs, dev), nq, nkv, False, None, None, 0.0, None, None,
                                  dummy, dummy, None, dummy, y, res_out, True)
    return y, res_out


def qkv_head(x, res, nw, eps, W, S, gs, q_w, k_w, positions, cos_sin, k_cache, v_cache, slots, trigger=True, pdl=True,
             num_q_heads=None, num_kv_heads=None):
    """Fused add+RMSNorm + qkv GEMV + per-head q/k RMSNorm + RoPE + KV write. Returns (q [M, nq*128], qkv [M, N], res)."""
    M, H = x.shape
    N = W.shape[0]
    nkv = num_kv_heads or NUM_KV_HEADS
    nq = num_q_heads or (N // HEAD_DIM - 2 * nkv)
    dev = x.device
    y = torch.empty((M, N), dtype=torch.bfloat16, device=dev)
    q = torch.empty((M, nq * HEAD_DIM), dtype=torch.bfloat16, device=dev)
    res_out = torch.empty((M, H), dtype=torch.bfloat16, device=dev)
    torch.ops.flint_b200.attn_qkv(x, res, nw, float(eps), W, S, _gs(gs, dev), nq, nkv, True, q_w, k_w, float(eps),
                                  positions, cos_sin, k_cache, v_cache, slots, q, y, res_out, True)
    return q, y, res_out


def o_gemv(a, W, S, gs, pdl=True, trigger=0):
    y = torch.empty((a.shape[0], W.shape[0]), dtype=torch.bfloat16, device=a.device)
    torch.ops.flint_b200.attn_o(a, W, S, _gs(gs, a.device), y)
    return y
