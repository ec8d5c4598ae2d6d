// Epoch-tagged words: data one CTA publishes and the others poll, without a grid barrier.
//
// A word is (epoch << 32) | 32 data bits, written with one 64-bit store (single-copy atomic), so a reader that sees
// the current epoch in a word also sees that word's data; no fence or flag is involved.  Epochs count launches on the
// device, so stale words from an earlier launch are never taken.  (The same idea as the 8-byte flag+data words of
// low-latency collective protocols.)  Every poll is bounded: after FLINT_WAIT_LIMIT rounds the reader records
// STATUS_WAIT_TIMEOUT and goes on with what it has.
#pragma once
#include "common.cuh"
#include "timeline.cuh"
#include "tma.cuh"

namespace flint {

__device__ __forceinline__ void st_tagged(unsigned long long* p, unsigned epoch, uint32_t data) {
  asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(((unsigned long long)epoch << 32) | data) : "memory");
}
__device__ __forceinline__ unsigned long long ld_tagged(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ ulonglong2 ld_tagged2(const unsigned long long* p) {    // two words, each one atomic unit
  ulonglong2 v;
  asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(v.x), "=l"(v.y) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ bool tag_is(unsigned long long w, unsigned epoch) { return (unsigned)(w >> 32) == epoch; }

// One warp stages one row published as tagged words (src[k / 2] carries the bf16 pair (k, k+1), k in the low half):
// polls its 16-byte units (8 consecutive k = four words) until they carry `epoch`, takes the row's max |value|
// (unsigned max over the float bits), derives the power-of-two shift of stage_rows_f16 and writes the f16 row into
// the stage_rows_f16 layout.  K <= 1024.
__device__ __forceinline__ void stage_row_f16_tagged_warp(const unsigned long long* __restrict__ src, int K,
                                                          unsigned epoch, __half* xs_row, int* shift_out, int lane,
                                                          unsigned* status) {
  const int K8 = K >> 3;
  constexpr int kU = 4;
  uint32_t w[kU][4];
  unsigned need = 0, got = 0;
#pragma unroll
  for (int i = 0; i < kU; ++i) {
    w[i][0] = w[i][1] = w[i][2] = w[i][3] = 0u;
    if (lane + 32 * i < K8) need |= 1u << i;
  }
#pragma unroll 1
  for (unsigned it = 0; got != need; ++it) {
    if (it == FLINT_WAIT_LIMIT) {
      atomicOr(status, STATUS_WAIT_TIMEOUT);
      break;
    }
#pragma unroll
    for (int i = 0; i < kU; ++i) {
      if ((need & ~got) & (1u << i)) {
        const unsigned long long* p = src + (int64_t)(lane + 32 * i) * 4;
        const ulonglong2 a = ld_tagged2(p), b = ld_tagged2(p + 2);
        if (tag_is(a.x, epoch) && tag_is(a.y, epoch) && tag_is(b.x, epoch) && tag_is(b.y, epoch)) {
          w[i][0] = (uint32_t)a.x;
          w[i][1] = (uint32_t)a.y;
          w[i][2] = (uint32_t)b.x;
          w[i][3] = (uint32_t)b.y;
          got |= 1u << i;
        }
      }
    }
    if (got != need) poll_pause();
  }
  unsigned mxb = 0u;
#pragma unroll
  for (int i = 0; i < kU; ++i) {
    float f[8];
    bf16x8_to_f32(make_uint4(w[i][0], w[i][1], w[i][2], w[i][3]), f);
#pragma unroll
    for (int j = 0; j < 8; ++j) mxb = max(mxb, __float_as_uint(fabsf(f[j])));
  }
  mxb = __reduce_max_sync(0xffffffffu, mxb);
  const float mx = __uint_as_float(mxb);
  int s = 0;
  if (mx > 0.f && !(mx != mx) && mx <= 3.0e38f) s = 14 - ((int)((mxb >> 23) & 0xFF) - 127);
  if (lane == 0) *shift_out = s;
#pragma unroll
  for (int i = 0; i < kU; ++i) {
    if (!((need >> i) & 1u)) continue;
    float f[8];
    bf16x8_to_f32(make_uint4(w[i][0], w[i][1], w[i][2], w[i][3]), f);
    uint32_t h[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __half2 v = __floats2half2_rn(scale_pow2(f[2 * j], s), scale_pow2(f[2 * j + 1], s));
      h[j] = *reinterpret_cast<uint32_t*>(&v);
    }
    *reinterpret_cast<uint4*>(xs_row + xs_perm((lane + 32 * i) * 8)) = make_uint4(h[0], h[1], h[2], h[3]);
  }
  __syncwarp();
}

}  // namespace flint
