// Shared device helpers for the sm_100a NVFP4 decode kernels.
//
// NVFP4 (ModelOpt layout): codes P u8 [N, K/2] (even k in the low nibble), block scales S (E4M3 bits)
// [N, K/16], one fp32 global scale per tensor.  value = e2m1 * e4m3 * gs.
//
// Weights are decoded exactly to f16: cvt.rn.f16x2.e2m1x2 gives the E2M1 pair, cvt.rn.f16x2.e4m3x2 the block
// scale, and mul.rn.f16x2 their product (<= 6 significant bits, 2^-10 .. 2688: exact in f16).  Activations are
// staged in shared memory as f16 after an exact per-token power-of-two rescale that puts max|x| in [2^14, 2^15),
// so the bf16 -> f16 conversion is exact for every element within 2^29 of the row maximum and never overflows.
// Products are accumulated in fp32 by mma.sync m16n8k16 (weight rows = M, tokens = N, 1..8 tokens per tile).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "../../include/flint_b200.h"

namespace flint {

typedef __nv_bfloat16 bf16;

__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// read-once weight streams: non-coherent, no L1 allocation, L2 evict-first
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 r;
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ uint32_t ldg_stream_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}

// 4 E2M1 pairs of a 32-bit word -> 4 f16x2 (byte b -> out[b]; low nibble -> low half)
__device__ __forceinline__ void e2m1x8_to_f16x2(uint32_t w, uint32_t (&o)[4]) {
  asm("{\n.reg .b8 b0, b1, b2, b3;\n"
      "mov.b32 {b0, b1, b2, b3}, %4;\n"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n}"
      : "=r"(o[0]), "=r"(o[1]), "=r"(o[2]), "=r"(o[3]) : "r"(w));
}
// two E4M3 bytes (low 16 bits) -> f16x2 (low byte -> low half)
__device__ __forceinline__ uint32_t e4m3x2_to_f16x2(uint32_t two) {
  uint32_t r;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"((unsigned short)(two & 0xFFFFu)));
  return r;
}
__device__ __forceinline__ uint32_t hmul2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bcast_lo(uint32_t h2) { return __byte_perm(h2, 0, 0x1010); }
__device__ __forceinline__ uint32_t bcast_hi(uint32_t h2) { return __byte_perm(h2, 0, 0x3232); }

// D += A * B, m16n8k16, f16 inputs, fp32 accumulate
__device__ __forceinline__ void mma_f16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// D += A * B, m16n8k16, bf16 inputs, fp32 accumulate
__device__ __forceinline__ void mma_bf16(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float bf16_bits_to_f32(uint32_t b) { return __uint_as_float(b << 16); }
__device__ __forceinline__ float bf16r(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
__device__ __forceinline__ void bf16x8_to_f32(uint4 u, float* f) {
  const uint32_t a[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(a[i] << 16);
    f[2 * i + 1] = __uint_as_float(a[i] & 0xFFFF0000u);
  }
}

// order-preserving u32 image of an fp32 (larger float -> larger key; NaN above +inf)
__device__ __forceinline__ uint32_t f32_order_key(float v) {
  const uint32_t u = __float_as_uint(v);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
__device__ __forceinline__ float f32_from_order_key(uint32_t k) {
  return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}
// argmax key: value, then the LOWEST index on ties
__device__ __forceinline__ unsigned long long argmax_key(float v, uint32_t idx) {
  return ((unsigned long long)f32_order_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}
__device__ __forceinline__ uint32_t argmax_key_index(unsigned long long k) { return 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull); }
__device__ __forceinline__ float argmax_key_value(unsigned long long k) { return f32_from_order_key((uint32_t)(k >> 32)); }

__device__ __forceinline__ unsigned long long shfl_xor_u64(unsigned long long v, int o) {
  uint32_t lo = (uint32_t)v, hi = (uint32_t)(v >> 32);
  lo = __shfl_xor_sync(0xffffffffu, lo, o);
  hi = __shfl_xor_sync(0xffffffffu, hi, o);
  return ((unsigned long long)hi << 32) | lo;
}

// ------------------------------------------------------------------------------------------------------------
// Activation staging: x bf16 [M, K] (row stride ldx) -> f16 in shared memory, rescaled per token by 2^shift[m].
// Lane quad t of a warp consumes k = 128*c + 32*t + v (v = 0..31) of chunk c as four 16-byte units q = v/8; unit q of
// lanes t = 2, 3 is stored at q ^ 2, and rows are K + 8 halves apart, so each 128-bit B-fragment read of a warp
// (up to 2 token rows per quarter-warp) is bank-conflict free.  Rows M..7 are never read.
// ------------------------------------------------------------------------------------------------------------
__host__ __device__ constexpr int xs_stride(int K) { return K + 8; }

__device__ __forceinline__ int xs_perm(int k) {
  const int t = (k >> 5) & 3, q = (k >> 3) & 3;
  return (k & ~31) + ((q ^ ((t >> 1) << 1)) << 3) + (k & 7);
}

// x * 2^s for |s| <= 252 as two exact power-of-two products.  Equal to ldexpf(x, s) whenever the product is a
// normal float; below that (|x * 2^s| < 2^-126) it may round differently, which no f16 conversion of the result can
// see (f16 flushes everything below 2^-25 to zero).  A short multiply instead of the library routine keeps the
// staging loops small.
__device__ __forceinline__ float scale_pow2(float x, int s) {
  const int a = s >> 1, b = s - a;
  return (x * __int_as_float((127 + a) << 23)) * __int_as_float((127 + b) << 23);
}

// atomicMax of a non-negative float's bits into the shared word *p, reduced first across the calling lanes that name
// the same word (one atomic per word and warp instead of one per lane contending on it).  Every lane of the calling
// set must reach the call.
__device__ __forceinline__ void smem_max_grouped(int* p, float v) {
  const unsigned act = __activemask();
  const unsigned grp = __match_any_sync(act, (unsigned long long)p);
  const unsigned m = __reduce_max_sync(grp, __float_as_uint(v));
  if ((int)(threadIdx.x & 31) == __ffs(grp) - 1) atomicMax(p, (int)m);
}

// smem_max_grouped for callers whose active lanes all name the same word (a norm's row loop): one warp reduction,
// no lane matching.
__device__ __forceinline__ void smem_max_warp(int* p, float v) {
  const unsigned act = __activemask();
  const unsigned m = __reduce_max_sync(act, __float_as_uint(v));
  if ((int)(threadIdx.x & 31) == __ffs(act) - 1) atomicMax(p, (int)m);
}

// Stage `rows` activation rows (src + r*ld, bf16, K columns, 16-byte aligned rows) as f16 into xs (row stride
// xs_stride(K)) with a per-row power-of-two rescale shift[r].  Called by threads [0, nthreads) of the block (a multiple
// of 32), which synchronise on named barrier `bar` (0 = __syncthreads when nthreads == blockDim.x).
// One global pass: raw bf16 goes to its permuted place in xs while the row maxima accumulate (one shared atomicMax
// per row and warp on the non-negative float bits), then each element is converted in place.  red: >= rows floats.
// stage_rows_f16_map stages source row row_of(i) (i < rows; entries < 0 are skipped) into slot i of xs / shift;
// stage_rows_f16 is the identity map.
template <class RowOf>
__device__ __forceinline__ void stage_rows_f16_map(const bf16* __restrict__ src, int64_t ld, int rows, int K, __half* xs,
                                                   int* shift, float* red, int nthreads, int bar, bool cg, RowOf row_of) {
  const int tid = threadIdx.x;
  const int K8 = K >> 3, n = rows * K8;
  auto sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthreads) : "memory"); };
  int* redi = reinterpret_cast<int*>(red);
  for (int i = tid; i < rows; i += nthreads) redi[i] = 0;
  sync();
  // up to kB 16-byte loads per thread are issued back to back (one memory round trip per kB * nthreads units)
  constexpr int kB = 4;
  for (int base = 0; base < n; base += kB * nthreads) {
    uint4 v[kB];
    int rr[kB], kk[kB];                               // rr: the slot (-1: nothing to stage)
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int idx = base + i * nthreads + tid;
      const int ri = idx / K8;
      kk[i] = idx - ri * K8;
      const int sr = idx < n ? row_of(ri) : -1;
      rr[i] = sr >= 0 ? ri : -1;
      if (sr >= 0) {
        const uint4* vp = reinterpret_cast<const uint4*>(src + sr * ld) + kk[i];
        v[i] = cg ? __ldcg(vp) : *vp;                 // cg: rows written by other CTAs of this kernel
      }
    }
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int r = rr[i];
      float mx = 0.f;
      if (r >= 0) {
        float f[8];
        bf16x8_to_f32(v[i], f);
#pragma unroll
        for (int j = 0; j < 8; ++j) mx = fmaxf(mx, fabsf(f[j]));
        *reinterpret_cast<uint4*>(xs + r * xs_stride(K) + xs_perm(kk[i] * 8)) = v[i];   // 8 consecutive k: one 16-byte unit
      }
      // the lanes of a warp hold consecutive units (one to three rows): one atomic per row and warp
      const unsigned grp = __match_any_sync(0xffffffffu, r);
      const unsigned gmx = __reduce_max_sync(grp, __float_as_uint(mx));
      if (r >= 0 && (tid & 31) == __ffs(grp) - 1) atomicMax(&redi[r], (int)gmx);
    }
  }
  sync();
  for (int i = tid; i < rows; i += nthreads) {
    if (row_of(i) < 0) continue;
    const float mx = __int_as_float(redi[i]);
    int s = 0;
    if (mx > 0.f && !(mx != mx) && mx <= 3.0e38f) s = 14 - ((int)((__float_as_uint(mx) >> 23) & 0xFF) - 127);
    shift[i] = s;
  }
  sync();
  for (int idx = tid; idx < n; idx += nthreads) {
    const int r = idx / K8, k8 = idx - r * K8;
    if (row_of(r) < 0) continue;
    uint4* p = reinterpret_cast<uint4*>(xs + r * xs_stride(K) + xs_perm(k8 * 8));
    float f[8];
    bf16x8_to_f32(*p, f);
    const int s = shift[r];
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

struct RowIdentity {
  __device__ __forceinline__ int operator()(int i) const { return i; }
};

__device__ __forceinline__ void stage_rows_f16(const bf16* __restrict__ src, int64_t ld, int rows, int K, __half* xs,
                                               int* shift, float* red, int nthreads, int bar, bool cg = false) {
  stage_rows_f16_map(src, ld, rows, K, xs, shift, red, nthreads, bar, cg, RowIdentity{});
}

// s = x (+ res) in fp32; res_out = bf16(s) (global, optional); xn = bf16(s * rsqrt(mean(s^2) + eps) * w) into shared
// memory (w == nullptr: xn = bf16(s)).  Threads [0, nthreads) with named barrier `bar`.  The sum of squares is
// reduced in a fixed order (per-thread chains, xor butterfly, warps in order), identical in every CTA that runs it.
// sbuf: fp32 shared scratch [M][H]; red: >= (nthreads/32) * 8 floats; M <= 8; rows of x / res 16-byte aligned.
__device__ __forceinline__ void add_rmsnorm_smem(const bf16* x, int64_t ldx, const bf16* res, const bf16* __restrict__ w,
                                                 float eps, int M, int H, float* sbuf, bf16* xn, bf16* res_out, float* red,
                                                 int nthreads, int bar) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = nthreads >> 5, H8 = H >> 3;
  auto sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthreads) : "memory"); };
  float ss[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    ss[m] = 0.f;
    if (m < M) {
      for (int k8 = tid; k8 < H8; k8 += nthreads) {
        float a[8];
        bf16x8_to_f32(reinterpret_cast<const uint4*>(x + m * ldx)[k8], a);
        if (res) {
          float b[8];
          bf16x8_to_f32(reinterpret_cast<const uint4*>(res + m * ldx)[k8], b);
#pragma unroll
          for (int j = 0; j < 8; ++j) a[j] += b[j];
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) ss[m] = fmaf(a[j], a[j], ss[m]);
        float4* d = reinterpret_cast<float4*>(sbuf + m * H + k8 * 8);
        d[0] = make_float4(a[0], a[1], a[2], a[3]);
        d[1] = make_float4(a[4], a[5], a[6], a[7]);
      }
    }
  }
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    float v = ss[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp * 8 + m] = v;
  }
  sync();
  for (int idx = tid; idx < M * H8; idx += nthreads) {
    const int m = idx / H8, k8 = idx - m * H8;
    float rs = 1.f;
    if (w) {
      float tot = 0.f;
      for (int ww = 0; ww < nw; ++ww) tot += red[ww * 8 + m];
      rs = rsqrtf(tot / (float)H + eps);
    }
    const float4* sp = reinterpret_cast<const float4*>(sbuf + m * H + k8 * 8);
    const float4 s0 = sp[0], s1 = sp[1];
    const float a[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    float wf[8];
    if (w) bf16x8_to_f32(reinterpret_cast<const uint4*>(w)[k8], wf);
    uint32_t pk[4], rk[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_bfloat162 n2 = w ? __floats2bfloat162_rn(a[2 * j] * rs * wf[2 * j], a[2 * j + 1] * rs * wf[2 * j + 1])
                            : __floats2bfloat162_rn(a[2 * j], a[2 * j + 1]);
      pk[j] = *reinterpret_cast<uint32_t*>(&n2);
      __nv_bfloat162 r2 = __floats2bfloat162_rn(a[2 * j], a[2 * j + 1]);
      rk[j] = *reinterpret_cast<uint32_t*>(&r2);
    }
    reinterpret_cast<uint4*>(xn + m * H)[k8] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    if (res_out) reinterpret_cast<uint4*>(res_out + m * H)[k8] = make_uint4(rk[0], rk[1], rk[2], rk[3]);
  }
  sync();
}

// Two-pass variant without fp32 scratch (for kernels whose shared memory is taken by their weight ring):
// pass 1 reduces sum(s^2) per row, pass 2 re-reads x (+ res) and writes xn = bf16(s * rsqrt(mean + eps) * w).
__device__ __forceinline__ void add_rmsnorm_2pass(const bf16* x, int64_t ldx, const bf16* res, const bf16* __restrict__ w,
                                                  float eps, int M, int H, bf16* xn, float* red, int nthreads, int bar) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = nthreads >> 5, H8 = H >> 3;
  auto sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthreads) : "memory"); };
  auto load = [&](int m, int k8, float* a) {
    bf16x8_to_f32(reinterpret_cast<const uint4*>(x + m * ldx)[k8], a);
    if (res) {
      float b[8];
      bf16x8_to_f32(reinterpret_cast<const uint4*>(res + m * ldx)[k8], b);
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] += b[j];
    }
  };
  float ss[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    ss[m] = 0.f;
    if (m < M)
      for (int k8 = tid; k8 < H8; k8 += nthreads) {
        float a[8];
        load(m, k8, a);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss[m] = fmaf(a[j], a[j], ss[m]);
      }
  }
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    float v = ss[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp * 8 + m] = v;
  }
  sync();
  for (int idx = tid; idx < M * H8; idx += nthreads) {
    const int m = idx / H8, k8 = idx - m * H8;
    float tot = 0.f;
    for (int ww = 0; ww < nw; ++ww) tot += red[ww * 8 + m];
    const float rs = rsqrtf(tot / (float)H + eps);
    float a[8], wf[8];
    load(m, k8, a);
    bf16x8_to_f32(reinterpret_cast<const uint4*>(w)[k8], wf);
    uint32_t pk[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_bfloat162 n2 = __floats2bfloat162_rn(a[2 * j] * rs * wf[2 * j], a[2 * j + 1] * rs * wf[2 * j + 1]);
      pk[j] = *reinterpret_cast<uint32_t*>(&n2);
    }
    reinterpret_cast<uint4*>(xn + m * H)[k8] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  }
  sync();
}

// add_rmsnorm_2pass + stage_rows_f16 without the bf16 staging buffer: s = x (+ res) (row m of x at x + rows[m] * ldx
// when rows is given: an embedding gather), res_out = bf16(s) (optional), xn = bf16(s * rsqrt(mean(s^2) + eps) * w)
// written straight to its permuted place in xs and then rescaled to f16 by 2^shift[m] in place.  The same per-thread
// fmaf chains and warp order as add_rmsnorm_2pass, so every CTA running it with the same thread count gets identical
// bits.  res and res_out rows are ldr elements apart.  red: >= (nthreads/32) * 8 + 8 floats.
__device__ __forceinline__ void norm_stage_f16(const bf16* x, int64_t ldx, const int* rows, const bf16* res, int64_t ldr,
                                               const bf16* __restrict__ w, float eps, int M, int H, __half* xs, int* shift,
                                               float* red, bf16* res_out, int nthreads, int bar) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = nthreads >> 5, H8 = H >> 3;
  auto sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthreads) : "memory"); };
  auto xrow = [&](int m) { return x + (rows ? (int64_t)rows[m] : (int64_t)m) * ldx; };
  auto load = [&](int m, int k8, float* a) {
    bf16x8_to_f32(reinterpret_cast<const uint4*>(xrow(m))[k8], a);
    if (res) {
      float b[8];
      bf16x8_to_f32(reinterpret_cast<const uint4*>(res + m * ldr)[k8], b);
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] += b[j];
    }
  };
  int* rmax = reinterpret_cast<int*>(red + nw * 8);
  float ss[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    ss[m] = 0.f;
    if (m < M)
      for (int k8 = tid; k8 < H8; k8 += nthreads) {
        float a[8];
        load(m, k8, a);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss[m] = fmaf(a[j], a[j], ss[m]);
      }
  }
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    float v = ss[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp * 8 + m] = v;
  }
  if (tid < 8) rmax[tid] = 0;
  sync();
  for (int idx = tid; idx < M * H8; idx += nthreads) {
    const int m = idx / H8, k8 = idx - m * H8;
    float tot = 0.f;
    for (int ww = 0; ww < nw; ++ww) tot += red[ww * 8 + m];
    const float rs = rsqrtf(tot / (float)H + eps);
    float a[8], wf[8];
    load(m, k8, a);
    if (res_out) {
      uint32_t pr[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 r2 = __floats2bfloat162_rn(a[2 * j], a[2 * j + 1]);
        pr[j] = *reinterpret_cast<uint32_t*>(&r2);
      }
      reinterpret_cast<uint4*>(res_out + m * ldr)[k8] = make_uint4(pr[0], pr[1], pr[2], pr[3]);
    }
    bf16x8_to_f32(reinterpret_cast<const uint4*>(w)[k8], wf);
    uint32_t pk[4];
    float mx = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_bfloat162 n2 = __floats2bfloat162_rn(a[2 * j] * rs * wf[2 * j], a[2 * j + 1] * rs * wf[2 * j + 1]);
      mx = fmaxf(mx, fmaxf(fabsf(__low2float(n2)), fabsf(__high2float(n2))));
      pk[j] = *reinterpret_cast<uint32_t*>(&n2);
    }
    smem_max_grouped(&rmax[m], mx);   // lanes may span rows here
    *reinterpret_cast<uint4*>(xs + m * xs_stride(H) + xs_perm(k8 * 8)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  }
  sync();
  for (int r = tid; r < M; r += nthreads) {
    const float mx = __int_as_float(rmax[r]);
    int s = 0;
    if (mx > 0.f && !(mx != mx) && mx <= 3.0e38f) s = 14 - ((int)((__float_as_uint(mx) >> 23) & 0xFF) - 127);
    shift[r] = s;
  }
  sync();
  for (int idx = tid; idx < M * H8; idx += nthreads) {
    const int r = idx / H8, k8 = idx - r * H8;
    uint4* p = reinterpret_cast<uint4*>(xs + r * xs_stride(H) + xs_perm(k8 * 8));
    float f[8];
    bf16x8_to_f32(*p, f);
    const int s = shift[r];
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

// add + RMSNorm of M <= 8 rows for H / 8 <= nthreads (one 8-wide chunk per thread and row) writing both the bf16
// result xn (shared memory, rows H apart; optional global copies xn_out and res_out = bf16(x + res), rows H apart)
// and its f16 staging in xs with the per-row power-of-two shift[m]: add_rmsnorm_1pass_w followed by
// stage_rows_f16(xn, ...), with the same bits, in one pass -- every row's loads are issued before any arithmetic,
// and the staging converts the registers instead of re-reading xn.  x and res rows are ldx apart; wchunk: this
// thread's 8 norm weights.  red: >= (nthreads/32) * 8 + 8 floats.
__device__ __forceinline__ void norm_xn_stage_f16(const bf16* x, int64_t ldx, const bf16* res, uint4 wchunk, float eps,
                                                  int M, int H, bf16* xn, bf16* xn_out, bf16* res_out, __half* xs,
                                                  int* shift, float* red, int nthreads, int bar, bool cg = false) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = nthreads >> 5, H8 = H >> 3;
  auto sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthreads) : "memory"); };
  const bool own = tid < H8;
  int* rmax = reinterpret_cast<int*>(red + nw * 8);
  uint4 xv[8], rv[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    xv[m] = make_uint4(0u, 0u, 0u, 0u);
    rv[m] = xv[m];
    if (m < M && own) {                       // cg: rows another GPU stored into this one's memory
      const uint4* xp = reinterpret_cast<const uint4*>(x + m * ldx) + tid;
      xv[m] = cg ? __ldcg(xp) : *xp;
      if (res) {
        const uint4* rp = reinterpret_cast<const uint4*>(res + m * ldx) + tid;
        rv[m] = cg ? __ldcg(rp) : *rp;
      }
    }
  }
  float a[8][8], ss[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    ss[m] = 0.f;
    if (m < M && own) {
      bf16x8_to_f32(xv[m], a[m]);
      if (res) {
        float b[8];
        bf16x8_to_f32(rv[m], b);
#pragma unroll
        for (int j = 0; j < 8; ++j) a[m][j] += b[j];
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss[m] = fmaf(a[m][j], a[m][j], ss[m]);
    }
  }
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    float v = ss[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp * 8 + m] = v;
  }
  if (tid < 8) rmax[tid] = 0;
  sync();
  float wf[8], rsv[8];
  bf16x8_to_f32(wchunk, wf);
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    float tot = 0.f;
    for (int ww = 0; ww < nw; ++ww) tot += red[ww * 8 + m];
    rsv[m] = rsqrtf(tot / (float)H + eps);
  }
  uint32_t pk[8][4];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    if (m < M && own) {
      uint32_t pr[4];
      float mx = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 n2 = __floats2bfloat162_rn(a[m][2 * j] * rsv[m] * wf[2 * j], a[m][2 * j + 1] * rsv[m] * wf[2 * j + 1]);
        mx = fmaxf(mx, fmaxf(fabsf(__low2float(n2)), fabsf(__high2float(n2))));
        pk[m][j] = *reinterpret_cast<uint32_t*>(&n2);
        __nv_bfloat162 r2 = __floats2bfloat162_rn(a[m][2 * j], a[m][2 * j + 1]);
        pr[j] = *reinterpret_cast<uint32_t*>(&r2);
      }
      const uint4 nv = make_uint4(pk[m][0], pk[m][1], pk[m][2], pk[m][3]);
      reinterpret_cast<uint4*>(xn + m * H)[tid] = nv;
      if (xn_out) reinterpret_cast<uint4*>(xn_out + (int64_t)m * H)[tid] = nv;
      if (res_out) reinterpret_cast<uint4*>(res_out + (int64_t)m * H)[tid] = make_uint4(pr[0], pr[1], pr[2], pr[3]);
      smem_max_warp(&rmax[m], mx);
    }
  }
  sync();
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    if (m < M) {
      const float mx = __int_as_float(rmax[m]);
      int s = 0;
      if (mx > 0.f && !(mx != mx) && mx <= 3.0e38f) s = 14 - ((int)((__float_as_uint(mx) >> 23) & 0xFF) - 127);
      if (tid == 0) shift[m] = s;
      if (own) {
        uint32_t h[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          __half2 v = __floats2half2_rn(scale_pow2(bf16_bits_to_f32(pk[m][j] & 0xFFFFu), s),
                                        scale_pow2(bf16_bits_to_f32(pk[m][j] >> 16), s));
          h[j] = *reinterpret_cast<uint32_t*>(&v);
        }
        *reinterpret_cast<uint4*>(xs + m * xs_stride(H) + xs_perm(tid * 8)) = make_uint4(h[0], h[1], h[2], h[3]);
      }
    }
  }
  sync();
}

// norm_xn_stage_f16 for nthreads = 2 (H / 8) (two halves of the block): thread t owns chunk c = t % (H / 8) of rows
// 4 h .. 4 h + 3, h = t / (H / 8) -- half the registers of the one-half form.  Per row the same per-thread chains,
// the same butterfly over the 32 chunks of a warp and the same order over the chunk warps, so the same bits.
// H / 8 a multiple of 32; wchunk: the norm weights of chunk c.  red: >= (H / 256) * 8 + 8 floats.
__device__ __forceinline__ void norm_xn_stage_f16_halves(const bf16* x, int64_t ldx, const bf16* res, uint4 wchunk,
                                                         float eps, int M, int H, bf16* xn, bf16* xn_out,
                                                         bf16* res_out, __half* xs, int* shift, float* red,
                                                         int nthreads, int bar, bool cg) {
  const int tid = threadIdx.x, lane = tid & 31, H8 = H >> 3, half = tid / H8, c = tid - half * H8;
  const int cw = c >> 5, ncw = H8 >> 5;
  auto sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthreads) : "memory"); };
  int* rmax = reinterpret_cast<int*>(red + ncw * 8);
  uint4 xv[4], rv[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = 4 * half + i;
    xv[i] = make_uint4(0u, 0u, 0u, 0u);
    rv[i] = xv[i];
    if (m < M) {                              // cg: rows another GPU stored into this one's memory
      const uint4* xp = reinterpret_cast<const uint4*>(x + m * ldx) + c;
      xv[i] = cg ? __ldcg(xp) : *xp;
      if (res) {
        const uint4* rp = reinterpret_cast<const uint4*>(res + m * ldx) + c;
        rv[i] = cg ? __ldcg(rp) : *rp;
      }
    }
  }
  float a[4][8], ss[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    ss[i] = 0.f;
    if (4 * half + i < M) {
      bf16x8_to_f32(xv[i], a[i]);
      if (res) {
        float b[8];
        bf16x8_to_f32(rv[i], b);
#pragma unroll
        for (int j = 0; j < 8; ++j) a[i][j] += b[j];
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss[i] = fmaf(a[i][j], a[i][j], ss[i]);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float v = ss[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[cw * 8 + 4 * half + i] = v;
  }
  if (tid < 8) rmax[tid] = 0;
  sync();
  float wf[8], rsv[4];
  bf16x8_to_f32(wchunk, wf);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float tot = 0.f;
    for (int ww = 0; ww < ncw; ++ww) tot += red[ww * 8 + 4 * half + i];
    rsv[i] = rsqrtf(tot / (float)H + eps);
  }
  uint32_t pk[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = 4 * half + i;
    if (m < M) {
      uint32_t pr[4];
      float mx = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 n2 = __floats2bfloat162_rn(a[i][2 * j] * rsv[i] * wf[2 * j], a[i][2 * j + 1] * rsv[i] * wf[2 * j + 1]);
        mx = fmaxf(mx, fmaxf(fabsf(__low2float(n2)), fabsf(__high2float(n2))));
        pk[i][j] = *reinterpret_cast<uint32_t*>(&n2);
        __nv_bfloat162 r2 = __floats2bfloat162_rn(a[i][2 * j], a[i][2 * j + 1]);
        pr[j] = *reinterpret_cast<uint32_t*>(&r2);
      }
      const uint4 nv = make_uint4(pk[i][0], pk[i][1], pk[i][2], pk[i][3]);
      reinterpret_cast<uint4*>(xn + m * H)[c] = nv;
      if (xn_out) reinterpret_cast<uint4*>(xn_out + (int64_t)m * H)[c] = nv;
      if (res_out) reinterpret_cast<uint4*>(res_out + (int64_t)m * H)[c] = make_uint4(pr[0], pr[1], pr[2], pr[3]);
      smem_max_warp(&rmax[m], mx);
    }
  }
  sync();
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = 4 * half + i;
    if (m < M) {
      const float mx = __int_as_float(rmax[m]);
      int s = 0;
      if (mx > 0.f && !(mx != mx) && mx <= 3.0e38f) s = 14 - ((int)((__float_as_uint(mx) >> 23) & 0xFF) - 127);
      if (c == 0) shift[m] = s;
      uint32_t h[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __half2 v = __floats2half2_rn(scale_pow2(bf16_bits_to_f32(pk[i][j] & 0xFFFFu), s),
                                      scale_pow2(bf16_bits_to_f32(pk[i][j] >> 16), s));
        h[j] = *reinterpret_cast<uint32_t*>(&v);
      }
      *reinterpret_cast<uint4*>(xs + m * xs_stride(H) + xs_perm(c * 8)) = make_uint4(h[0], h[1], h[2], h[3]);
    }
  }
  sync();
}

// 16-byte global -> shared copy that does not wait (L2 only: also right for rows another GPU stored here).
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;"
               ::"r"(static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst))), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// norm_xn_stage_f16_halves with little code: the same arithmetic, bits and outputs, but every loop over the rows
// is rolled (a kernel that runs this once per launch pays for each new instruction it fetches, so an unrolled
// 4-row body costs more than the arithmetic).  All rows' x / res chunks are first copied into `scratch` (shared
// memory, >= 2 M H bf16) with asynchronous copies issued back to back; x + res is recomputed from them where the
// unrolled form kept it in registers.
__device__ __forceinline__ void norm_xn_stage_f16_compact(const bf16* x, int64_t ldx, const bf16* res, uint4 wchunk,
                                                          float eps, int M, int H, bf16* xn, bf16* xn_out,
                                                          bf16* res_out, __half* xs, int* shift, float* red,
                                                          int nthreads, int bar, bf16* scratch) {
  const int tid = threadIdx.x, lane = tid & 31, H8 = H >> 3, half = tid / H8, c = tid - half * H8;
  const int cw = c >> 5, ncw = H8 >> 5, m0 = 4 * half, m1 = min(M, m0 + 4);
  auto sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthreads) : "memory"); };
  int* rmax = reinterpret_cast<int*>(red + ncw * 8);
  bf16* sx = scratch;                                       // [M][H]
  bf16* sr = scratch + (size_t)M * H;                       // [M][H]
#pragma unroll 1
  for (int m = m0; m < m1; ++m) {
    cp_async16(reinterpret_cast<uint4*>(sx + m * H) + c, reinterpret_cast<const uint4*>(x + m * ldx) + c);
    if (res) cp_async16(reinterpret_cast<uint4*>(sr + m * H) + c, reinterpret_cast<const uint4*>(res + m * ldx) + c);
  }
  cp_async_wait_all();                                      // each thread reads back only its own chunks
  auto load_s = [&](int m, float (&a)[8]) {                 // s = x (+ res) in fp32, the unrolled form's sums
    bf16x8_to_f32(reinterpret_cast<const uint4*>(sx + m * H)[c], a);
    if (res) {
      float b[8];
      bf16x8_to_f32(reinterpret_cast<const uint4*>(sr + m * H)[c], b);
#pragma unroll
      for (int j = 0; j < 8; ++j) a[j] += b[j];
    }
  };
#pragma unroll 1
  for (int m = m0; m < m0 + 4; ++m) {
    float v = 0.f;
    if (m < M) {
      float a[8];
      load_s(m, a);
#pragma unroll
      for (int j = 0; j < 8; ++j) v = fmaf(a[j], a[j], v);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[cw * 8 + m] = v;
  }
  if (tid < 8) rmax[tid] = 0;
  sync();
  float wf[8];
  bf16x8_to_f32(wchunk, wf);
#pragma unroll 1
  for (int m = m0; m < m1; ++m) {
    float tot = 0.f;
    for (int ww = 0; ww < ncw; ++ww) tot += red[ww * 8 + m];
    const float rs = rsqrtf(tot / (float)H + eps);
    float a[8];
    load_s(m, a);
    uint32_t pk[4], pr[4];
    float mx = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_bfloat162 n2 = __floats2bfloat162_rn(a[2 * j] * rs * wf[2 * j], a[2 * j + 1] * rs * wf[2 * j + 1]);
      mx = fmaxf(mx, fmaxf(fabsf(__low2float(n2)), fabsf(__high2float(n2))));
      pk[j] = *reinterpret_cast<uint32_t*>(&n2);
      __nv_bfloat162 r2 = __floats2bfloat162_rn(a[2 * j], a[2 * j + 1]);
      pr[j] = *reinterpret_cast<uint32_t*>(&r2);
    }
    const uint4 nv = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    reinterpret_cast<uint4*>(xn + m * H)[c] = nv;
    if (xn_out) reinterpret_cast<uint4*>(xn_out + (int64_t)m * H)[c] = nv;
    if (res_out) reinterpret_cast<uint4*>(res_out + (int64_t)m * H)[c] = make_uint4(pr[0], pr[1], pr[2], pr[3]);
    smem_max_warp(&rmax[m], mx);
  }
  sync();
#pragma unroll 1
  for (int m = m0; m < m1; ++m) {
    const float mx = __int_as_float(rmax[m]);
    int s = 0;
    if (mx > 0.f && !(mx != mx) && mx <= 3.0e38f) s = 14 - ((int)((__float_as_uint(mx) >> 23) & 0xFF) - 127);
    if (c == 0) shift[m] = s;
    const uint4 nv = reinterpret_cast<const uint4*>(xn + m * H)[c];
    const uint32_t pk[4] = {nv.x, nv.y, nv.z, nv.w};
    uint32_t h[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __half2 v = __floats2half2_rn(scale_pow2(bf16_bits_to_f32(pk[j] & 0xFFFFu), s),
                                    scale_pow2(bf16_bits_to_f32(pk[j] >> 16), s));
      h[j] = *reinterpret_cast<uint32_t*>(&v);
    }
    *reinterpret_cast<uint4*>(xs + m * xs_stride(H) + xs_perm(c * 8)) = make_uint4(h[0], h[1], h[2], h[3]);
  }
  sync();
}

// norm_stage_f16 with ONE global pass, for H / 8 <= nthreads: each thread owns one 8-wide chunk of every row and keeps
// x (+ res) in registers between the sum of squares and the normalisation (same fmaf chains, same bits).
// (norm_stage_f16_1w: the thread's 8 norm weights, w[8 tid .. 8 tid + 7], are passed in, loaded before the PDL wait.)
__device__ __forceinline__ void norm_stage_f16_1w(const bf16* x, int64_t ldx, const int* rows, const bf16* res, int64_t ldr,
                                                  uint4 wchunk, float eps, int M, int H, __half* xs, int* shift, float* red,
                                                  bf16* res_out, int nthreads, int bar) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = nthreads >> 5, H8 = H >> 3;
  auto sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthreads) : "memory"); };
  const bool own = tid < H8;
  int* rmax = reinterpret_cast<int*>(red + nw * 8);
  float a[8][8], ss[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    ss[m] = 0.f;
    if (m < M && own) {
      bf16x8_to_f32(reinterpret_cast<const uint4*>(x + (rows ? (int64_t)rows[m] : (int64_t)m) * ldx)[tid], a[m]);
      if (res) {
        float b[8];
        bf16x8_to_f32(reinterpret_cast<const uint4*>(res + m * ldr)[tid], b);
#pragma unroll
        for (int j = 0; j < 8; ++j) a[m][j] += b[j];
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss[m] = fmaf(a[m][j], a[m][j], ss[m]);
    }
  }
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    float v = ss[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp * 8 + m] = v;
  }
  if (tid < 8) rmax[tid] = 0;
  sync();
  float wf[8];
  bf16x8_to_f32(wchunk, wf);
  uint32_t pk[8][4];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    if (m < M && own) {
      float tot = 0.f;
      for (int ww = 0; ww < nw; ++ww) tot += red[ww * 8 + m];
      const float rs = rsqrtf(tot / (float)H + eps);
      if (res_out) {
        uint32_t pr[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          __nv_bfloat162 r2 = __floats2bfloat162_rn(a[m][2 * j], a[m][2 * j + 1]);
          pr[j] = *reinterpret_cast<uint32_t*>(&r2);
        }
        reinterpret_cast<uint4*>(res_out + m * ldr)[tid] = make_uint4(pr[0], pr[1], pr[2], pr[3]);
      }
      float mx = 0.f;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 n2 = __floats2bfloat162_rn(a[m][2 * j] * rs * wf[2 * j], a[m][2 * j + 1] * rs * wf[2 * j + 1]);
        mx = fmaxf(mx, fmaxf(fabsf(__low2float(n2)), fabsf(__high2float(n2))));
        pk[m][j] = *reinterpret_cast<uint32_t*>(&n2);
      }
      smem_max_warp(&rmax[m], mx);
    }
  }
  sync();
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    if (m < M) {
      const float mx = __int_as_float(rmax[m]);
      int s = 0;
      if (mx > 0.f && !(mx != mx) && mx <= 3.0e38f) s = 14 - ((int)((__float_as_uint(mx) >> 23) & 0xFF) - 127);
      if (tid == 0) shift[m] = s;
      if (own) {
        uint32_t h[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          __half2 v = __floats2half2_rn(scale_pow2(bf16_bits_to_f32(pk[m][j] & 0xFFFFu), s),
                                        scale_pow2(bf16_bits_to_f32(pk[m][j] >> 16), s));
          h[j] = *reinterpret_cast<uint32_t*>(&v);
        }
        *reinterpret_cast<uint4*>(xs + m * xs_stride(H) + xs_perm(tid * 8)) = make_uint4(h[0], h[1], h[2], h[3]);
      }
    }
  }
  sync();
}

__device__ __forceinline__ void norm_stage_f16_1(const bf16* x, int64_t ldx, const int* rows, const bf16* res, int64_t ldr,
                                                 const bf16* __restrict__ w, float eps, int M, int H, __half* xs,
                                                 int* shift, float* red, bf16* res_out, int nthreads, int bar) {
  const uint4 wc = (int)threadIdx.x < (H >> 3) ? reinterpret_cast<const uint4*>(w)[threadIdx.x] : make_uint4(0u, 0u, 0u, 0u);
  norm_stage_f16_1w(x, ldx, rows, res, ldr, wc, eps, M, H, xs, shift, red, res_out, nthreads, bar);
}

// add_rmsnorm_2pass with ONE global pass, for H / 8 <= nthreads (one 8-wide chunk per thread and row, kept in
// registers): the same per-thread chains, butterfly and warp order, so xn has the same bits.  xn: bf16 [M][H] in
// shared memory; res_out / xn_out: optional global copies (rows H apart).  red: >= (nthreads/32) * 8 floats.
// (add_rmsnorm_1pass_w: the thread's 8 norm weights w[8 tid .. 8 tid + 7] passed in, e.g. loaded before a PDL wait.)
__device__ __forceinline__ void add_rmsnorm_1pass_w(const bf16* x, int64_t ldx, const bf16* res, uint4 wchunk,
                                                    float eps, int M, int H, bf16* xn, bf16* res_out, bf16* xn_out,
                                                    float* red, int nthreads, int bar) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, nw = nthreads >> 5, H8 = H >> 3;
  auto sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthreads) : "memory"); };
  const bool own = tid < H8;
  float a[8][8], ss[8];
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    ss[m] = 0.f;
    if (m < M && own) {
      bf16x8_to_f32(reinterpret_cast<const uint4*>(x + m * ldx)[tid], a[m]);
      if (res) {
        float b[8];
        bf16x8_to_f32(reinterpret_cast<const uint4*>(res + m * ldx)[tid], b);
#pragma unroll
        for (int j = 0; j < 8; ++j) a[m][j] += b[j];
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss[m] = fmaf(a[m][j], a[m][j], ss[m]);
    }
  }
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    float v = ss[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp * 8 + m] = v;
  }
  sync();
  float wf[8];
  bf16x8_to_f32(wchunk, wf);
#pragma unroll
  for (int m = 0; m < 8; ++m) {
    if (m < M && own) {
      float tot = 0.f;
      for (int ww = 0; ww < nw; ++ww) tot += red[ww * 8 + m];
      const float rs = rsqrtf(tot / (float)H + eps);
      uint32_t pk[4], pr[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __nv_bfloat162 n2 = __floats2bfloat162_rn(a[m][2 * j] * rs * wf[2 * j], a[m][2 * j + 1] * rs * wf[2 * j + 1]);
        pk[j] = *reinterpret_cast<uint32_t*>(&n2);
        __nv_bfloat162 r2 = __floats2bfloat162_rn(a[m][2 * j], a[m][2 * j + 1]);
        pr[j] = *reinterpret_cast<uint32_t*>(&r2);
      }
      const uint4 nv = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      reinterpret_cast<uint4*>(xn + m * H)[tid] = nv;
      if (xn_out) reinterpret_cast<uint4*>(xn_out + (int64_t)m * H)[tid] = nv;
      if (res_out) reinterpret_cast<uint4*>(res_out + (int64_t)m * H)[tid] = make_uint4(pr[0], pr[1], pr[2], pr[3]);
    }
  }
  sync();
}

__device__ __forceinline__ void add_rmsnorm_1pass(const bf16* x, int64_t ldx, const bf16* res, const bf16* __restrict__ w,
                                                  float eps, int M, int H, bf16* xn, bf16* res_out, bf16* xn_out,
                                                  float* red, int nthreads, int bar) {
  const uint4 wc = (int)threadIdx.x < (H >> 3) ? reinterpret_cast<const uint4*>(w)[threadIdx.x] : make_uint4(0u, 0u, 0u, 0u);
  add_rmsnorm_1pass_w(x, ldx, res, wc, eps, M, H, xn, res_out, xn_out, red, nthreads, bar);
}

// Whole-block variant (the LM head): all threads, __syncthreads.
__device__ __forceinline__ void stage_x_f16(const bf16* __restrict__ x, int64_t ldx, int M, int K, __half* xs,
                                            int* shift, float* red) {
  stage_rows_f16(x, ldx, M, K, xs, shift, red, blockDim.x, 0);
}

}  // namespace flint
