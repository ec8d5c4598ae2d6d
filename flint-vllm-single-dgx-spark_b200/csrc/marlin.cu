// vLLM's Marlin-processed NVFP4 expert tensors -> the ModelOpt NVFP4 layout the decode kernels read.
//
// The reference's GB10 MoE kernels read the tensors vLLM holds after its Marlin repack (fast/fp4moe_mar.cu:1-7,
// handed over by fast/model.py:271-282).  That layout, restated:
//   codes   int32 [K/16][N/64][128 words] per expert; word w of tile (kt, nt) belongs to lane l = w / 4 (q = l / 4,
//           c = l % 4) as word g = w % 4; its nibble j (E2M1 code, same bits as ModelOpt's) holds the value at
//           k = 16 kt + 2c + 8 (j & 1) + ((j >> 2) & 1),  n = 64 nt + q + 16 g + 8 ((j >> 1) & 1);
//   scales  u8 [K/16][N] per expert; inside each 64-column group the byte at 64 nt + 8 q + b holds the scale of
//           n = 64 nt + 8 s + q with s = (b & 4) + [0, 2, 1, 3][b & 3]; the byte is the processed S0E5M3 form h,
//           read as fp16(byte << 7), with 0 meaning a zero scale;
//   global  fp32 per expert, the processed global scale g; a weight is e2m1 * h * g * 2^-126.
// ModelOpt keeps e2m1 codes [N][K/2] (even k in the low nibble), E4M3 block scales [N][K/16] and an fp32 global
// scale, weight = e2m1 * e4m3 * gs.  Since h * 2^-7 is always a normal E4M3 value (vLLM rescales the scales so every
// non-zero h is at least 2 and at most 448 * 2^7), the conversion is exact: E4M3 byte = h_byte - 0x78 (0 stays 0)
// and gs = g * 2^-119, so e2m1 * e4m3 * gs equals the reference kernel's e2m1 * h * g * 2^-126 bit for bit.  A
// non-zero scale byte below 0x80 or above 0xF6 is not a processed NVFP4 scale: it is counted in `bad` and written
// as 0.
//
// Kernel: one CTA per (64-column group, expert), 256 threads, looping over chunks of 64 k-tiles (1024 k): each chunk's
// 128-word tiles are read with coalesced 32-bit loads (512 contiguous bytes per k-tile) and scattered as whole
// ModelOpt bytes (the two nibbles of one byte come from nibbles j and j + 4 of one word) into a shared [64 rows][512 B]
// stage, the scales into a [64][64] stage; the stage is then written out row by row with 8-byte stores.  One-time
// weight preparation: (K/2 + K/16) B read and written per row.
#include "common.cuh"
#include "runtime.cuh"

namespace flint {

constexpr int kMuThreads = 256;
constexpr int kMuChunk = 64;          // k-tiles (of 16 k) per chunk

__device__ __forceinline__ uint32_t marlin_scale_to_e4m3(uint32_t b, bool* bad) {
  if (b == 0u) return 0u;
  if (b < 0x80u || b > 0xF6u) {       // not a processed scale: exponent below 16 or a value above 448 * 2^7
    *bad = true;
    return 0u;
  }
  return b - 0x78u;                   // fp16 exponent e5 (bias 15), value * 2^-7 -> E4M3 exponent e5 - 15
}

__global__ void __launch_bounds__(kMuThreads) marlin_nvfp4_unpack_kernel(
    const uint32_t* __restrict__ wm, const uint8_t* __restrict__ sm, const float* __restrict__ gm, int N, int K,
    uint8_t* __restrict__ P, uint8_t* __restrict__ S, float* __restrict__ gs, int* __restrict__ bad) {
  __shared__ __align__(16) uint8_t code_stage[64][kMuChunk * 8];
  __shared__ __align__(16) uint8_t scale_stage[64][kMuChunk];
  pdl_wait();
  const int nt = blockIdx.x, e = blockIdx.y, NT = N / 64, KT = K / 16;
  const int tid = threadIdx.x;
  const uint32_t* wexp = wm + (int64_t)e * KT * NT * 128;
  const uint8_t* sexp = sm + (int64_t)e * KT * N;
  uint8_t* pexp = P + (int64_t)e * N * (K / 2);
  uint8_t* srow = S + (int64_t)e * N * (K / 16);
  bool saw_bad = false;
  if (nt == 0 && tid == 0) gs[e] = gm[e] * 0x1p-119f;   // exact: a power of two, the result stays normal
#pragma unroll 1
  for (int kt0 = 0; kt0 < KT; kt0 += kMuChunk) {
    const int nk = KT - kt0 < kMuChunk ? KT - kt0 : kMuChunk;
    // codes: nk tiles of 128 words
#pragma unroll 1
    for (int i = tid; i < nk * 128; i += kMuThreads) {
      const int ktl = i >> 7, w = i & 127;
      const uint32_t word = __ldg(wexp + ((int64_t)(kt0 + ktl) * NT + nt) * 128 + w);
      const int l = w >> 2, g = w & 3, q = l >> 2, c = l & 3;
#pragma unroll
      for (int j = 0; j < 4; ++j) {                    // nibble j: k even; nibble j + 4: k + 1 (the high nibble)
        const uint32_t lo = (word >> (4 * j)) & 0xFu, hi = (word >> (4 * j + 16)) & 0xFu;
        const int n = q + 16 * g + 8 * ((j >> 1) & 1);
        const int kb = ktl * 8 + c + 4 * (j & 1);      // byte column: (16 ktl + 2c + 8 (j & 1)) / 2
        code_stage[n][kb] = (uint8_t)(lo | (hi << 4));
      }
    }
    // scales: nk rows of 64 bytes
#pragma unroll 1
    for (int i = tid; i < nk * 64; i += kMuThreads) {
      const int ktl = i >> 6, p = i & 63;
      const uint32_t b = sexp[(int64_t)(kt0 + ktl) * N + nt * 64 + p];
      const int q = p >> 3, bb = p & 7;
      const int s = (bb & 4) + ((bb & 3) == 1 ? 2 : (bb & 3) == 2 ? 1 : (bb & 3));
      scale_stage[8 * s + q][ktl] = (uint8_t)marlin_scale_to_e4m3(b, &saw_bad);
    }
    __syncthreads();
    // rows out: nk * 8 code bytes (8-byte stores) and nk scale bytes per row
    const int cw = nk;                                 // 8-byte words per row of this chunk
#pragma unroll 1
    for (int i = tid; i < 64 * cw; i += kMuThreads) {
      const int r = i / cw, u = i - r * cw;
      const uint2 v = *reinterpret_cast<const uint2*>(&code_stage[r][u * 8]);
      *reinterpret_cast<uint2*>(pexp + (int64_t)(nt * 64 + r) * (K / 2) + kt0 * 8 + u * 8) = v;
    }
#pragma unroll 1
    for (int i = tid; i < 64 * nk; i += kMuThreads) {
      const int r = i / nk, u = i - r * nk;
      srow[(int64_t)(nt * 64 + r) * (K / 16) + kt0 + u] = scale_stage[r][u];
    }
    __syncthreads();
  }
  if (__syncthreads_or(saw_bad) && tid == 0) atomicAdd(bad, 1);
  pdl_trigger();
}

}  // namespace flint

extern "C" int flint_marlin_nvfp4_unpack(const void* weight, const void* weight_scale, const float* global_scale,
                                         int64_t E, int64_t N, int64_t K, void* packed, void* scales,
                                         float* global_out, int32_t* bad, int pdl, void* stream) {
  using namespace flint;
  if (!weight || !weight_scale || !global_scale || !packed || !scales || !global_out || !bad) return FLINT_ERR_ARGUMENT;
  if (E < 1 || E > 65535 || N < 64 || N % 64 != 0 || K < 16 || K % 16 != 0 || N > (1 << 20) || K > (1 << 20))
    return FLINT_ERR_SHAPE;
  if (!aligned(weight, 4) || !aligned(packed, 8) || !aligned(global_scale, 4) || !aligned(global_out, 4))
    return FLINT_ERR_ALIGN;
  if (num_sms() <= 0) return FLINT_ERR_DEVICE;
  return launch(marlin_nvfp4_unpack_kernel, dim3((unsigned)(N / 64), (unsigned)E), dim3(kMuThreads), 0, stream, pdl,
                static_cast<const uint32_t*>(weight), static_cast<const uint8_t*>(weight_scale), global_scale, (int)N,
                (int)K, static_cast<uint8_t*>(packed), static_cast<uint8_t*>(scales), global_out, (int*)bad);
}
