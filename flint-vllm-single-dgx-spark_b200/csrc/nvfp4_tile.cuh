// Shared-memory stage ring for NVFP4 weight streaming (TMA producer warp, mma.sync consumer warps).
//
// A stage holds a ROWS x 256-k slice of an NVFP4 matrix: codes ROWS x 128 B (128B-swizzled: 16-byte unit u of row r
// is stored at unit u ^ (r & 7)) and block scales ROWS x 16 B.  Consumer warp w owns stage rows [16w, 16w+16) and
// runs 2 chunks x 8 m16n8k16 steps per stage.  Tile row g (= lane/4) of a warp is stage row 16w + phi(g) (and + 8)
// with phi(g) = (g >> 1) | ((g & 1) << 2): the two rows a quarter-warp reads differ in bit 2 of the swizzle key, so
// every 128-bit fragment read is bank-conflict free.
#pragma once
#include "common.cuh"
#include "tma.cuh"

namespace flint {

constexpr int kSliceK = 256;   // k per stage (128 code bytes per row)

template <int ROWS>
struct StageGeom {
  static constexpr int code_bytes = ROWS * 128;
  static constexpr int scale_bytes = ROWS * 16;
  static constexpr int bytes = code_bytes + scale_bytes;
};

__device__ __forceinline__ int tile_phi(int g) { return (g >> 1) | ((g & 1) << 2); }

__device__ __forceinline__ uint4 lds128(const void* p) {
  uint4 r;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "r"(smem_u32(p)));
  return r;
}
__device__ __forceinline__ uint32_t lds_u16(const void* p) {
  unsigned short r;
  asm volatile("ld.shared.u16 %0, [%1];" : "=h"(r) : "r"(smem_u32(p)));
  return r;
}

// One 128-k chunk of a 16-row tile.  qg / qg8: this lane's 16 code bytes (k = 32t .. 32t+31 of the chunk) of rows
// g / g+8; s2: their two block-scale bytes each (row g in the low 16 bits); ch: chunk index along K.
// acc[4][4]: four independent accumulator chains (mma step j -> acc[j & 3]).
__device__ __forceinline__ void mma_chunk(const uint4& qg, const uint4& qg8, uint32_t s2, const __half* xrow, bool active,
                                          int ch, int t, float (&acc)[4][4]) {
  const uint32_t sc_g = e4m3x2_to_f16x2(s2 & 0xFFFFu);
  const uint32_t sc_g8 = e4m3x2_to_f16x2(s2 >> 16);
  const uint32_t sa_g = bcast_lo(sc_g), sb_g = bcast_hi(sc_g);
  const uint32_t sa_g8 = bcast_lo(sc_g8), sb_g8 = bcast_hi(sc_g8);
  const uint32_t wg[4] = {qg.x, qg.y, qg.z, qg.w};
  const uint32_t wg8[4] = {qg8.x, qg8.y, qg8.z, qg8.w};
  const __half* xq = xrow + ch * 128 + 32 * t;
  const int qswz = (t >> 1) << 1;
#pragma unroll
  for (int q = 0; q < 4; ++q) {                     // word q: values 8q .. 8q+7 -> mma steps 2q, 2q+1
    uint4 b = make_uint4(0u, 0u, 0u, 0u);
    if (active) b = lds128(xq + 8 * (q ^ qswz));
    uint32_t dg[4], dg8[4];
    e2m1x8_to_f16x2(wg[q], dg);
    e2m1x8_to_f16x2(wg8[q], dg8);
    const uint32_t s_g = q < 2 ? sa_g : sb_g;       // scale block 2t for values 0..15, 2t+1 for 16..31
    const uint32_t s_g8 = q < 2 ? sa_g8 : sb_g8;
#pragma unroll
    for (int h = 0; h < 2; ++h) {                   // step j = 2q + h: bytes 2h, 2h+1 of the word
      uint32_t a[4];
      a[0] = hmul2(dg[2 * h], s_g);
      a[1] = hmul2(dg8[2 * h], s_g8);
      a[2] = hmul2(dg[2 * h + 1], s_g);
      a[3] = hmul2(dg8[2 * h + 1], s_g8);
      mma_f16(acc[(2 * q + h) & 3], a, h ? b.z : b.x, h ? b.w : b.y);
    }
  }
}

// Consume one stage (2 chunks) for warp `warp`; ks = slice index along K.
__device__ __forceinline__ void consume_stage(const uint8_t* codes, const uint8_t* scales, int warp, int g, int t, int ks,
                                              const __half* xrow, bool active, float (&acc)[4][4]) {
  const int pr0 = 16 * warp + tile_phi(g), pr1 = pr0 + 8;
  const int key = pr0 & 7;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int phys = (4 * c + t) ^ key;
    const uint4 qg = lds128(codes + pr0 * 128 + phys * 16);
    const uint4 qg8 = lds128(codes + pr1 * 128 + phys * 16);
    const uint32_t s2 = lds_u16(scales + pr0 * 16 + 8 * c + 2 * t) | (lds_u16(scales + pr1 * 16 + 8 * c + 2 * t) << 16);
    mma_chunk(qg, qg8, s2, xrow, active, ks * 2 + c, t, acc);
  }
}

__device__ __forceinline__ void zero_acc(float (&acc)[4][4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[i][e] = 0.f;
}
__device__ __forceinline__ void sum_acc(float (&acc)[4][4], float (&d)[4]) {
#pragma unroll
  for (int e = 0; e < 4; ++e) d[e] = (acc[0][e] + acc[1][e]) + (acc[2][e] + acc[3][e]);
}

}  // namespace flint
