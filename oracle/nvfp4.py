"""NVFP4 (E2M1 values, E4M3 per-16 block scales, fp32 tensor scale) on the CPU.

Test infrastructure only (see ``oracle/__init__.py``).

Layout ("ModelOpt"): packed codes ``P`` uint8 [..., N, K/2] with the even k in
the low nibble; block scales ``S`` uint8 (E4M3 bit patterns) [..., N, K/16];
one fp32 global scale per tensor (per expert for stacked experts).
value = e2m1(code) * e4m3(scale) * global_scale.
"""
from __future__ import annotations

import numpy as np

# patch:291-292 (vllm/models/flint/gguf_nvfp4.py:_E2M1_POS/_E2M1)
E2M1_POS = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
E2M1 = np.array(E2M1_POS + tuple(-v for v in E2M1_POS), dtype=np.float32)

_GGUF_QK = 64          # values per GGUF NVFP4 super-block (patch:212)
_GGUF_BLOCK_BYTES = 36  # 4 scale bytes + 32 code bytes (patch:213)


def e4m3_to_f32(b: np.ndarray) -> np.ndarray:
    """E4M3 (fn variant: bias 7, no inf, 0x7F/0xFF = NaN) bit patterns -> fp32."""
    b = np.asarray(b, dtype=np.uint8).astype(np.int32)
    s = np.where(b & 0x80, -1.0, 1.0).astype(np.float32)
    e = (b >> 3) & 0xF
    m = (b & 0x7).astype(np.float32)
    sub = m / 8.0 * np.float32(2.0 ** -6)
    nrm = (1.0 + m / 8.0) * np.exp2((e - 7).astype(np.float32))
    v = np.where(e == 0, sub, nrm).astype(np.float32) * s
    return np.where((b & 0x7F) == 0x7F, np.float32(np.nan), v).astype(np.float32)


_E4M3_TABLE = e4m3_to_f32(np.arange(256, dtype=np.uint8))


def dequantize_nvfp4(weight: np.ndarray, weight_scale: np.ndarray,
                     global_scale: float | np.ndarray | None = None) -> np.ndarray:
    """ModelOpt NVFP4 [..., N, K/2] u8 + E4M3 [..., N, K/16] -> fp32 [..., N, K].

    Restates patch:295-319 (gguf_nvfp4.dequantize_nvfp4): LUT decode of the
    low then high nibble, times the block scale, optionally times the global
    scale.  ``e2m1 * e4m3`` is exact in fp32 (and in bf16/fp16)."""
    w = np.asarray(weight, dtype=np.uint8)
    codes = np.stack([w & 0x0F, w >> 4], axis=-1).reshape(*w.shape[:-1], -1)
    vals = E2M1[codes].reshape(*w.shape[:-1], -1, 16)
    sc = _E4M3_TABLE[np.asarray(weight_scale, dtype=np.uint8)]
    vals = (vals * sc[..., None]).reshape(*w.shape[:-1], -1)
    if global_scale is not None:
        gs = np.asarray(global_scale, dtype=np.float32)
        if gs.ndim > 0:
            gs = gs.reshape(gs.shape + (1,) * (vals.ndim - gs.ndim))
        vals = vals * gs
    return vals.astype(np.float32)


def repack_gguf_nvfp4(blocks: np.ndarray, n_cols: int) -> tuple[np.ndarray, np.ndarray]:
    """GGUF NVFP4 super-blocks [..., n_cols/64*36] u8 -> (P [..., n_cols/2], S [..., n_cols/16]).

    Restates patch:269-288 (gguf_nvfp4._repack_nvfp4): each 36-byte block is 4
    UE4M3 scale bytes (0x7F decodes to zero, 0xFF is rejected, the sign bit is
    cleared) then 4 sub-blocks of 8 code bytes whose low nibbles are values
    0..7 and high nibbles values 8..15 of the sub-block."""
    blocks = np.asarray(blocks, dtype=np.uint8)
    lead = blocks.shape[:-1]
    blocks = blocks.reshape(*lead, n_cols // _GGUF_QK, _GGUF_BLOCK_BYTES)
    scales = blocks[..., :4]
    if (scales == 0xFF).any():
        raise ValueError("NVFP4 GGUF block scale 0xFF is not supported")
    scales = np.where(scales == 0x7F, 0, scales & 0x7F).astype(np.uint8)
    qs = blocks[..., 4:].reshape(*lead, n_cols // _GGUF_QK, 4, 8)
    codes = np.concatenate([qs & 0x0F, qs >> 4], axis=-1)
    packed = codes[..., 0::2] | (codes[..., 1::2] << 4)
    return (packed.reshape(*lead, n_cols // 2).astype(np.uint8),
            scales.reshape(*lead, n_cols // 16).astype(np.uint8))


# ---------------------------------------------------------------------------------------------
# rounding helpers
# ---------------------------------------------------------------------------------------------
def bf16_round(x: np.ndarray) -> np.ndarray:
    """fp32 -> nearest-even bf16, returned as fp32 (NaN kept)."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = r.view(np.float32)
    return np.where(np.isnan(x), x, out).astype(np.float32)


def bf16_bits(x: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns (uint16), nearest-even."""
    return (bf16_round(x).view(np.uint32) >> 16).astype(np.uint16)


def bf16_from_bits(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def f32_to_e4m3(x: np.ndarray) -> np.ndarray:
    """fp32 -> E4M3 bits, nearest-even with saturation to +-448 (positive inputs in practice)."""
    x = np.asarray(x, dtype=np.float32)
    pos = _E4M3_TABLE[:0x7F]                      # 0x00..0x7E, ascending
    a = np.minimum(np.abs(x), np.float32(448.0))
    idx = np.searchsorted(pos, a, side="left")
    idx = np.clip(idx, 1, len(pos) - 1)
    lo, hi = pos[idx - 1], pos[idx]
    pick_hi = (hi - a < a - lo) | ((hi - a == a - lo) & ((idx & 1) == 0))
    code = np.where(pick_hi, idx, idx - 1).astype(np.uint8)
    code = np.where(a >= pos[-1], 0x7E, code).astype(np.uint8)
    return np.where(x < 0, code | 0x80, code).astype(np.uint8)


_E2M1_MID = np.array([0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0], dtype=np.float32)


def f32_to_e2m1(x: np.ndarray) -> np.ndarray:
    """fp32 (already divided by the block scale) -> E2M1 codes 0..15, nearest-even, saturating at 6."""
    x = np.asarray(x, dtype=np.float32)
    a = np.abs(x)
    # searchsorted(left) maps a midpoint to the lower code; ties go to the even code (mantissa bit 0)
    mag = np.searchsorted(_E2M1_MID, a, side="left").astype(np.uint8)
    tie_up = np.isin(a, _E2M1_MID) & ((mag & 1) == 1)
    mag = np.minimum(np.where(tie_up, mag + 1, mag), 7).astype(np.uint8)
    return np.where((x < 0) & (mag != 0), mag | 8, mag).astype(np.uint8)


def quantize_nvfp4(w: np.ndarray) -> tuple[np.ndarray, np.ndarray, np.float32]:
    """fp32 [N, K] -> (P u8 [N, K/2], S u8 E4M3 [N, K/16], gs fp32).

    Our seeded quantiser (the reference ships none): gs = amax / (448 * 6);
    block scale = e4m3(amax_block / (6 * gs)); code = e2m1(w / (scale * gs))."""
    w = np.asarray(w, dtype=np.float32)
    n, k = w.shape
    amax = np.float32(np.abs(w).max())
    gs = np.float32(amax / np.float32(448.0 * 6.0)) if amax > 0 else np.float32(1.0)
    blk = w.reshape(n, k // 16, 16)
    bmax = np.abs(blk).max(-1)
    s = f32_to_e4m3(bmax / (np.float32(6.0) * gs))
    sf = _E4M3_TABLE[s] * gs
    q = np.where(sf[..., None] > 0, blk / np.where(sf[..., None] > 0, sf[..., None], 1), 0)
    codes = f32_to_e2m1(q.astype(np.float32)).reshape(n, k)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    return packed, s.astype(np.uint8), gs
