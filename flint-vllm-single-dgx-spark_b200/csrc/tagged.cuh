// Epoch-tagged words: data one CTA publishes and the others poll, without a grid barrier.
//
// A word is (epoch << 32) | 32 data bits, written with one 64-bit store (single-copy atomic), so a reader that sees
// the current epoch in a word also sees that word's data; no fence or flag is involved.  Epochs count launches on the
// device, so stale words from an earlier launch are never taken.  (The same idea as the 8-byte flag+data words of
// low-latency collective protocols.)  Every poll is bounded: after FLINT_WAIT_LIMIT rounds the reader records
// STATUS_WAIT_TIMEOUT and goes on with what it has.
#pragma once
#include "common.cuh"
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

// stage_rows_f16 for rows published as tagged words: src[r * K/2 + k/2] carries the bf16 pair (k, k+1) (k in the low
// half).  Each thread polls its own 16-byte units (8 consecutive k = four words; up to 4 units per round of
// 4 * nthreads) until all carry `epoch`, then the rows are rescaled exactly as stage_rows_f16 does (same shift rule,
// same f16 values).  rowmap (optional): the r-th staged row is row rowmap[r] of src, of xs and of shift.
__device__ __forceinline__ void stage_rows_f16_tagged(const unsigned long long* __restrict__ src, int rows, int K,
                                                      unsigned epoch, __half* xs, int* shift, float* red, int nthreads,
                                                      int bar, unsigned* status, const int* rowmap = nullptr) {
  const int tid = threadIdx.x;
  const int K8 = K >> 3, n = rows * K8;
  auto sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthreads) : "memory"); };
  auto row_of = [&](int r) { return rowmap ? rowmap[r] : r; };
  int* redi = reinterpret_cast<int*>(red);
  for (int r = tid; r < rows; r += nthreads) redi[r] = 0;
  sync();
  constexpr int kB = 4;
#pragma unroll 1
  for (int base = 0; base < n; base += kB * nthreads) {
    uint32_t w[kB][4];
    unsigned need = 0, got = 0;
#pragma unroll
    for (int i = 0; i < kB; ++i)
      if (base + tid + i * nthreads < n) need |= 1u << i;
#pragma unroll 1
    for (unsigned it = 0; got != need; ++it) {
      if (it == FLINT_WAIT_LIMIT) {
        atomicOr(status, STATUS_WAIT_TIMEOUT);
        break;
      }
#pragma unroll
      for (int i = 0; i < kB; ++i) {
        if ((need & ~got) & (1u << i)) {
          const int idx = base + tid + i * nthreads, r = idx / K8;
          const unsigned long long* p = src + ((int64_t)row_of(r) * K8 + (idx - r * K8)) * 4;   // words of unit k8
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
    }
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      if ((need >> i) & 1u) {
        const int idx = base + tid + i * nthreads, r = idx / K8, k8 = idx - r * K8;
        const uint4 v = make_uint4(w[i][0], w[i][1], w[i][2], w[i][3]);
        float f[8];
        bf16x8_to_f32(v, f);
        float mx = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fabsf(f[j]));
        atomicMax(&redi[r], __float_as_int(mx));
        *reinterpret_cast<uint4*>(xs + row_of(r) * xs_stride(K) + xs_perm(k8 * 8)) = v;
      }
    }
  }
  sync();
  for (int r = tid; r < rows; r += nthreads) {
    const float mx = __int_as_float(redi[r]);
    int s = 0;
    if (mx > 0.f && !(mx != mx) && mx <= 3.0e38f) s = 14 - ((int)((__float_as_uint(mx) >> 23) & 0xFF) - 127);
    shift[row_of(r)] = s;
  }
  sync();
#pragma unroll 1
  for (int idx = tid; idx < n; idx += nthreads) {
    const int r = idx / K8, k8 = idx - r * K8, rr = row_of(r);
    uint4* p = reinterpret_cast<uint4*>(xs + rr * xs_stride(K) + xs_perm(k8 * 8));
    float f[8];
    bf16x8_to_f32(*p, f);
    const int s = shift[rr];
    uint32_t h[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __half2 v = __floats2half2_rn(scale_pow2(f[2 * j], s), scale_pow2(f[2 * j + 1], s));
      h[j] = *reinterpret_cast<uint32_t*>(&v);
    }
    *p = make_uint4(h[0], h[1], h[2], h[3]);
  }
  sync();
}

// One warp stages one row published as tagged words (the pair layout of stage_rows_f16_tagged): polls its 16-byte
// units until they carry `epoch`, takes the row's max |value| (unsigned max over the float bits, as the block-wide
// form's atomicMax does), derives the same power-of-two shift and writes the f16 row.  K <= 1024.
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
