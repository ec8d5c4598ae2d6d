"""The FlashInfer W4A16 layout of NVFP4 expert weights -- test infrastructure (a CPU restatement used as the checker
of the GPU conversion, never on the product path).

The Flint PR's grouped MoE (vllm/models/flint/ops/moe_cute.py, `prepare_weights`, patch:4061-4091) hands
FlashInfer's SM100 NVFP4-weight GEMMs the ModelOpt expert tensors rearranged:

* gate/up codes and scales: the rows [gate; up] become [up; gate] and are then interleaved in 64-row groups: row
  block b (128 rows) holds up rows 64 b .. 64 b + 63 followed by gate rows 64 b .. 64 b + 63;
* block scales (after that row order for gate/up): [E, rows, groups] bytes viewed as
  [E, rows / 128, 4, 32, groups / 4, 4] and stored as [E, rows / 128, groups / 4, 32, 4, 4]
  ("the 6-D MMA layout"), returned as a permuted (logical) view [32, 4, rows / 128, 4, groups / 4, E];
* down codes are unchanged, down scales take the 6-D layout.

`to_flashinfer` restates that arrangement in numpy and `from_flashinfer` inverts it; both are pinned to fixtures
made with the PR's own function (tests/golden/make_flashinfer_golden.py).
"""
from __future__ import annotations

import numpy as np


def _interleave_rows(x: np.ndarray) -> np.ndarray:
    """[gate; up] rows -> per 128-row block: 64 up rows, then 64 gate rows (patch:4073-4077)."""
    e, rows = x.shape[:2]
    half = rows // 2
    y = np.concatenate([x[:, half:], x[:, :half]], axis=1)
    y = y.reshape(e, 2, rows // 128, 64, *x.shape[2:]).swapaxes(1, 2)
    return np.ascontiguousarray(y).reshape(x.shape)


def _deinterleave_rows(y: np.ndarray) -> np.ndarray:
    e, rows = y.shape[:2]
    half = rows // 2
    x = y.reshape(e, rows // 128, 2, 64, *y.shape[2:]).swapaxes(1, 2).reshape(y.shape)
    return np.ascontiguousarray(np.concatenate([x[:, half:], x[:, :half]], axis=1))


def mma_scales_physical(s: np.ndarray) -> np.ndarray:
    """[E, rows, groups] scale bytes -> the stored 6-D layout [E, rows/128, groups/4, 32, 4, 4] (patch:4079-4086)."""
    e, rows, groups = s.shape
    assert rows % 128 == 0 and groups % 4 == 0
    return np.ascontiguousarray(s.reshape(e, rows // 128, 4, 32, groups // 4, 4).transpose(0, 1, 4, 3, 2, 5))


def mma_scales_linear(p: np.ndarray) -> np.ndarray:
    """Inverse of mma_scales_physical."""
    e, mt, kt = p.shape[:3]
    return np.ascontiguousarray(p.transpose(0, 1, 4, 3, 2, 5)).reshape(e, mt * 128, kt * 4)


def to_flashinfer(w13, s13, w2, s2):
    """ModelOpt (codes uint8 [E, 2I, H/2], scales uint8 [E, 2I, H/16], down [E, H, I/2], [E, H, I/16]) ->
    (w1, w1_sf physical 6-D, w2, w2_sf physical 6-D)."""
    return (_interleave_rows(w13), mma_scales_physical(_interleave_rows(s13)), np.ascontiguousarray(w2),
            mma_scales_physical(s2))


def from_flashinfer(w1, w1_sf, w2, w2_sf):
    """Inverse of to_flashinfer: back to the ModelOpt tensors the decode kernels read."""
    return (_deinterleave_rows(w1), _deinterleave_rows(mma_scales_linear(w1_sf)), np.ascontiguousarray(w2),
            mma_scales_linear(w2_sf))


def logical_to_physical(sf_logical: np.ndarray) -> np.ndarray:
    """The PR returns the scales as a permuted view [32, 4, m, 4, k, E] of the stored [E, m, k, 32, 4, 4]."""
    return np.ascontiguousarray(sf_logical.transpose(5, 2, 4, 0, 1, 3))
