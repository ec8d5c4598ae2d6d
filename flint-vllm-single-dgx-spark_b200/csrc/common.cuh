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

// read-once weight streams: non-coherent, no L1 allocation
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
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

// All threads of the block call this.  red must hold >= blockDim/32 * 8 floats.
__device__ __forceinline__ void stage_x_f16(const bf16* __restrict__ x, int64_t ldx, int M, int K, __half* xs,
                                            int* shift, float* red) {
  const int tid = threadIdx.x, nt = blockDim.x, lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
  for (int m = 0; m < M; ++m) {
    float mx = 0.f;
    for (int k = tid; k < K; k += nt) mx = fmaxf(mx, fabsf(__bfloat162float(x[m * ldx + k])));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    if (lane == 0) red[warp * 8 + m] = mx;
  }
  __syncthreads();
  if (tid < M) {
    float mx = 0.f;
    for (int w = 0; w < nw; ++w) mx = fmaxf(mx, red[w * 8 + tid]);
    int s = 0;
    if (mx > 0.f && !(mx != mx) && mx <= 3.0e38f) {
      const int e = (int)((__float_as_uint(mx) >> 23) & 0xFF) - 127;   // bf16 inputs are never subnormal here
      s = 14 - e;
    }
    shift[tid] = s;
  }
  __syncthreads();
  for (int m = 0; m < M; ++m) {
    const int s = shift[m];
    __half* row = xs + m * xs_stride(K);
    for (int k = tid; k < K; k += nt) row[xs_perm(k)] = __float2half_rn(ldexpf(__bfloat162float(x[m * ldx + k]), s));
  }
  __syncthreads();
}

}  // namespace flint
