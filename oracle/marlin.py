"""vLLM's Marlin-processed NVFP4 layout on the CPU -- test infrastructure only.

The reference's GB10 MoE kernels read the expert tensors in the form vLLM leaves them after its Marlin preparation
(handed over at fast/model.py:271-282, layout documented at fast/fp4moe_mar.cu:1-7).  The preparation is vLLM's
(third party, not under the reference: ``prepare_moe_fp4_layer_for_marlin`` / ``nvfp4_marlin_process_scales`` /
``nvfp4_marlin_process_global_scale`` in vllm/model_executor/layers/quantization/utils/marlin_utils_fp4.py,
``marlin_permute_scales`` / ``get_scale_perms`` in marlin_utils.py, and the CUDA op ``gptq_marlin_repack``; the
reference pins vLLM 0.32.1rc1, README.md:146, this image has 0.22).  Restated here:

pack (ModelOpt -> Marlin-processed), per expert:
  codes:  tile (kt, nt) of 16 k x 64 n, 128 int32 words; nibble j of word w holds the e2m1 code at
          k = 16 kt + 2c + 8 (j & 1) + ((j >> 2) & 1), n = 64 nt + q + 16 g + 8 ((j >> 1) & 1), where l = w / 4,
          g = w % 4, q = l / 4, c = l % 4 (fast/fp4moe_mar.cu:3-4); words stored [kt][nt][w].
  scales: [K/16][N]; scale value v (E4M3) -> fp16(v * sf * 2^7), values below 2 flushed to 0, stored as the byte
          (fp16 bits >> 7) & 0xFF; inside each 64-column group the scale of n = 64 nt + 8 s + q sits at byte
          64 nt + 8 q + (s & 4) + [0, 2, 1, 3][s & 3] (fast/fp4moe_mar.cu:5-6; vLLM's scale_perm followed by the
          [0, 2, 1, 3] swap of process_scales).
  sf:     one power of two per layer (shared by all experts): the largest 2^m with max(v) * 2^m <= 448, or 1 when
          max(v) * 2^7 >= 448 * 2^7 (vLLM's _nvfp4_compute_scale_factor for bf16 activations).
  global: g = gs * 2^119 / sf (bf16 activations: 2^(126 - 7)).
  A weight is then e2m1 * fp16(byte << 7) * g * 2^-126 (fast/fp4moe_mar.cu:6).

unpack (what flint_marlin_nvfp4_unpack computes): codes back to [N][K/2] (even k low nibble); scale byte b -> E4M3
byte b - 0x78 (0 stays 0), i.e. the E4M3 value fp16(b << 7) * 2^-7 = v * sf; global gs' = g * 2^-119 = gs / sf.
e2m1 * (v * sf) * (gs / sf) is the reference's weight exactly.
"""
from __future__ import annotations

import numpy as np

from .nvfp4 import _E4M3_TABLE

_SWAP = np.array([0, 2, 1, 3])


def _tile_maps():
    """(k, n) offsets inside a 16 x 64 tile of nibble j of word w: two int arrays [128, 8]."""
    w = np.arange(128)[:, None]
    j = np.arange(8)[None, :]
    lane, g = w // 4, w % 4
    q, c = lane // 4, lane % 4
    k = 2 * c + 8 * (j & 1) + ((j >> 2) & 1)
    n = q + 16 * g + 8 * ((j >> 1) & 1)
    return k, n


def pack_codes(P: np.ndarray) -> np.ndarray:
    """ModelOpt codes u8 [N, K/2] -> Marlin words int32 [K/16, N/64 * 128]."""
    N, Kh = P.shape
    K, KT, NT = 2 * Kh, Kh // 8, N // 64
    codes = np.stack([P & 0xF, P >> 4], axis=-1).reshape(N, K)
    tiles = codes.reshape(NT, 64, KT, 16).transpose(2, 0, 1, 3)              # [KT, NT, 64 n, 16 k]
    k, n = _tile_maps()
    nib = tiles[:, :, n, k].astype(np.uint32)                                 # [KT, NT, 128, 8]
    words = np.zeros(nib.shape[:3], np.uint32)
    for j in range(8):
        words |= nib[..., j] << np.uint32(4 * j)
    return words.reshape(KT, NT * 128).view(np.int32)


def unpack_codes(words: np.ndarray, N: int, K: int) -> np.ndarray:
    """Marlin words int32 [K/16, N/64 * 128] -> ModelOpt codes u8 [N, K/2]."""
    KT, NT = K // 16, N // 64
    w = words.view(np.uint32).reshape(KT, NT, 128)
    nib = np.stack([(w >> np.uint32(4 * j)) & 0xF for j in range(8)], axis=-1).astype(np.uint8)
    tiles = np.zeros((KT, NT, 64, 16), np.uint8)
    k, n = _tile_maps()
    tiles[:, :, n, k] = nib
    codes = tiles.transpose(1, 2, 0, 3).reshape(N, K)
    return (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)


def scale_positions(N: int) -> np.ndarray:
    """Byte position, inside a [N] row of processed scales, of the scale of each column n."""
    n = np.arange(N)
    grp, r = n // 64, n % 64
    s, q = r // 8, r % 8
    return 64 * grp + 8 * q + (s & 4) + _SWAP[s & 3]


def scale_factor(S_layer: np.ndarray) -> float:
    """The layer's power-of-two rescale of its E4M3 scales (all experts together)."""
    v = _E4M3_TABLE[np.asarray(S_layer, np.uint8)].astype(np.float64) * 2.0 ** 7
    nz = v[v > 0]
    if nz.size and nz.max() < 448 * 2.0 ** 7:
        return float(2.0 ** np.floor(np.log2(448 * 2.0 ** 7 / nz.max())))
    return 1.0


def pack_scales(S: np.ndarray, sf: float) -> np.ndarray:
    """ModelOpt E4M3 bytes [N, K/16] -> processed, permuted scale bytes u8 [K/16, N]."""
    N = S.shape[0]
    h = (_E4M3_TABLE[np.asarray(S, np.uint8)].astype(np.float32).T * np.float32(sf * 2.0 ** 7)).astype(np.float16)
    h[h < 2] = 0
    b = ((h.view(np.uint16) >> 7) & 0xFF).astype(np.uint8)
    out = np.zeros_like(b)
    out[:, scale_positions(N)] = b
    return out


def unpack_scales(Sm: np.ndarray, N: int) -> np.ndarray:
    """Processed scale bytes u8 [K/16, N] -> E4M3 bytes u8 [N, K/16] (b -> b - 0x78, 0 stays 0)."""
    b = np.asarray(Sm, np.uint8)[:, scale_positions(N)].astype(np.int32)
    return np.where(b == 0, 0, b - 0x78).astype(np.uint8).T.copy()


def pack_layer(P: np.ndarray, S: np.ndarray, gs: np.ndarray):
    """A layer's stacked experts P [E, N, K/2], S [E, N, K/16], gs [E] -> (words int32 [E, K/16, 2N],
    scale bytes u8 [E, K/16, N], processed globals fp32 [E], sf)."""
    sf = scale_factor(S)
    words = np.stack([pack_codes(p) for p in P])
    sc = np.stack([pack_scales(s, sf) for s in S])
    g = (np.asarray(gs, np.float32) * np.float32(2.0 ** 119) / np.float32(sf)).astype(np.float32)
    return words, sc, g, sf


def unpack_layer(words: np.ndarray, Sm: np.ndarray, g: np.ndarray):
    """Inverse of pack_layer up to the scale factor: -> (P [E, N, K/2], S [E, N, K/16] holding v * sf, gs / sf)."""
    E, KT, W2 = words.shape
    N, K = W2 // 2, KT * 16
    P = np.stack([unpack_codes(w, N, K) for w in words])
    S = np.stack([unpack_scales(s, N) for s in Sm])
    return P, S, (np.asarray(g, np.float32) * np.float32(2.0 ** -119)).astype(np.float32)
