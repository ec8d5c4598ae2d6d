// GGUF NVFP4 checkpoint tensors -> the ModelOpt NVFP4 layout the decode kernels read, and the exact NVFP4 dequant.
//
// GGUF NVFP4 (ggml type 40) stores 64 values per 36-byte super-block: four UE4M3 scale bytes (one per 16-value
// sub-block), then four sub-blocks of 8 code bytes whose low nibbles are the sub-block's values 0..7 and whose high
// nibbles are values 8..15.  ModelOpt packs consecutive values into one byte (even value in the low nibble) with the
// E4M3 block scales in a separate [N, K/16] array.  The conversion (patch:269-288, gguf_nvfp4._repack_nvfp4) is a
// lossless byte shuffle: scale byte 0x7F (the E4M3 NaN, decoded by ggml as zero) becomes 0, the sign bit of every
// other scale byte is cleared, and 0xFF (480, not representable in E4M3) is an error.
//
// Repack kernel: one warp per chunk of 32 consecutive super-blocks (1152 contiguous input bytes, 1024 + 128 output
// bytes).  The chunk is loaded with coalesced 16-byte loads into a per-warp shared stage, each lane then shuffles
// its own super-block in registers (nibble pairs joined by shifts, bytes gathered by byte_perm) and writes 32 code
// bytes as two 16-byte stores and its 4 scale bytes as one 32-bit store; every global access of a warp is
// contiguous.  Pure HBM streaming: 36 B read + 36 B written per 64 values.
//
// Dequant kernel (patch:295-319, gguf_nvfp4.dequantize_nvfp4): one thread per 16-value group; value =
// e2m1 * e4m3 (exact), times the optional fp32 global scale (one fp32 multiply, round to nearest), stored as fp32 or
// rounded once to bf16.  Write-bound: 9 B read per 16 values, 32 B (bf16) or 64 B (fp32) written.
#include "common.cuh"
#include "runtime.cuh"

namespace flint {

constexpr int kRpWarps = 8;          // warps per CTA
constexpr int kRpWords = 9;          // 32-bit words per 36-byte super-block

__global__ void __launch_bounds__(kRpWarps * 32) gguf_nvfp4_repack_kernel(const uint32_t* __restrict__ in,
                                                                          int64_t nsb, uint4* __restrict__ packed,
                                                                          uint32_t* __restrict__ scales,
                                                                          int* __restrict__ bad) {
  __shared__ __align__(16) uint32_t stage[kRpWarps][32 * kRpWords];
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t nchunk = (nsb + 31) >> 5;
  uint32_t* st = stage[warp];
  bool seen_ff = false;
#pragma unroll 1
  for (int64_t c = (int64_t)blockIdx.x * kRpWarps + warp; c < nchunk; c += (int64_t)gridDim.x * kRpWarps) {
    const int64_t sb0 = c << 5;
    const int nvalid = nsb - sb0 < 32 ? (int)(nsb - sb0) : 32;
    const uint32_t* src = in + sb0 * kRpWords;
    if (nvalid == 32) {                                // 72 aligned 16-byte units (the chunk starts at c * 1152)
      const uint4* s4 = reinterpret_cast<const uint4*>(src);
      uint4* d4 = reinterpret_cast<uint4*>(st);
      const uint4 a = ldg_stream_v4(s4 + lane), b = ldg_stream_v4(s4 + 32 + lane);
      uint4 t = make_uint4(0, 0, 0, 0);
      if (lane < 8) t = ldg_stream_v4(s4 + 64 + lane);
      d4[lane] = a;
      d4[32 + lane] = b;
      if (lane < 8) d4[64 + lane] = t;
    } else {                                           // the ragged last chunk: word loads
      for (int w = lane; w < nvalid * kRpWords; w += 32) st[w] = ldg_stream_u32(src + w);
    }
    __syncwarp();
    if (lane < nvalid) {
      const uint32_t* b = st + lane * kRpWords;        // stride 9 words: conflict-free across the warp
      const uint32_t sc = b[0];
      seen_ff |= __vcmpeq4(sc, 0xFFFFFFFFu) != 0u;
      scales[sb0 + lane] = sc & 0x7F7F7F7Fu & ~__vcmpeq4(sc, 0x7F7F7F7Fu);
      uint32_t o[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t w0 = b[1 + 2 * j], w1 = b[2 + 2 * j];
        const uint32_t l0 = w0 & 0x0F0F0F0Fu, l1 = w1 & 0x0F0F0F0Fu;
        const uint32_t h0 = (w0 >> 4) & 0x0F0F0F0Fu, h1 = (w1 >> 4) & 0x0F0F0F0Fu;
        // byte 2i of (n | n >> 4) = nibble 2i | nibble 2i+1 << 4; gather bytes 0, 2 of each word
        o[2 * j] = __byte_perm(l0 | (l0 >> 4), l1 | (l1 >> 4), 0x6420);       // values 0..7 of sub-block j
        o[2 * j + 1] = __byte_perm(h0 | (h0 >> 4), h1 | (h1 >> 4), 0x6420);   // values 8..15
      }
      uint4* dst = packed + (sb0 + lane) * 2;
      dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
      dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
    }
    __syncwarp();
  }
  if (__any_sync(0xffffffffu, seen_ff) && lane == 0) atomicAdd(bad, 1);
  pdl_trigger();
}

__global__ void __launch_bounds__(256) nvfp4_dequant_kernel(const uint2* __restrict__ P, const uint8_t* __restrict__ S,
                                                            int64_t ngroups, const float* __restrict__ gsp,
                                                            int out_f32, void* __restrict__ out) {
  pdl_wait();
  const float gs = gsp ? *gsp : 1.0f;
#pragma unroll 1
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < ngroups; g += (int64_t)gridDim.x * blockDim.x) {
    const uint2 codes = __ldcs(P + g);
    const float sf = __half2float(__ushort_as_half((unsigned short)(e4m3x2_to_f16x2(S[g]) & 0xFFFFu)));
    uint32_t h[8];
    e2m1x8_to_f16x2(codes.x, *reinterpret_cast<uint32_t(*)[4]>(&h[0]));
    e2m1x8_to_f16x2(codes.y, *reinterpret_cast<uint32_t(*)[4]>(&h[4]));
    float v[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const __half2 p = *reinterpret_cast<const __half2*>(&h[i]);
      v[2 * i] = __half2float(__low2half(p)) * sf;     // exact: <= 5 significant bits
      v[2 * i + 1] = __half2float(__high2half(p)) * sf;
      if (gsp) {
        v[2 * i] = __fmul_rn(v[2 * i], gs);
        v[2 * i + 1] = __fmul_rn(v[2 * i + 1], gs);
      }
    }
    if (out_f32) {
      float4* d = reinterpret_cast<float4*>(out) + g * 4;
#pragma unroll
      for (int i = 0; i < 4; ++i) __stcs(d + i, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
    } else {
      uint32_t w[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const __nv_bfloat162 p = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&p);
      }
      uint4* d = reinterpret_cast<uint4*>(out) + g * 2;
      __stcs(d, make_uint4(w[0], w[1], w[2], w[3]));
      __stcs(d + 1, make_uint4(w[4], w[5], w[6], w[7]));
    }
  }
  pdl_trigger();
}

}  // namespace flint

using namespace flint;

extern "C" int flint_gguf_nvfp4_repack(const void* blocks, int64_t rows, int64_t n_cols, void* packed, void* scales,
                                       int32_t* bad_blocks, int pdl, void* stream) {
  if (!blocks || !packed || !scales || !bad_blocks) return FLINT_ERR_ARGUMENT;
  if (rows < 0 || n_cols < 64 || n_cols % 64 != 0) return FLINT_ERR_SHAPE;
  if (!aligned(blocks, 16) || !aligned(packed, 16) || !aligned(scales, 4)) return FLINT_ERR_ALIGN;
  const int64_t nsb = rows * (n_cols / 64);
  if (nsb == 0) return FLINT_OK;
  const int sms = num_sms();
  if (sms < 1) return FLINT_ERR_DEVICE;
  const int64_t nchunk = (nsb + 31) / 32;
  const int64_t want = (nchunk + kRpWarps - 1) / kRpWarps;
  const int grid = (int)(want < (int64_t)sms * 8 ? want : (int64_t)sms * 8);
  return launch(gguf_nvfp4_repack_kernel, dim3(grid), dim3(kRpWarps * 32), 0, stream, pdl,
                reinterpret_cast<const uint32_t*>(blocks), nsb, reinterpret_cast<uint4*>(packed),
                reinterpret_cast<uint32_t*>(scales), (int*)bad_blocks);
}

extern "C" int flint_nvfp4_dequant(const void* P, const void* S, int64_t rows, int64_t n_cols,
                                   const float* global_scale, int out_f32, void* out, int pdl, void* stream) {
  if (!P || !S || !out) return FLINT_ERR_ARGUMENT;
  if (rows < 0 || n_cols < 16 || n_cols % 16 != 0) return FLINT_ERR_SHAPE;
  if (!aligned(P, 8) || !aligned(out, 16)) return FLINT_ERR_ALIGN;
  const int64_t ng = rows * (n_cols / 16);
  if (ng == 0) return FLINT_OK;
  const int sms = num_sms();
  if (sms < 1) return FLINT_ERR_DEVICE;
  // 4 CTAs of 256 threads per SM: measured 1.35x faster on this write-bound stream than a full-occupancy grid
  const int64_t want = (ng + 255) / 256;
  const int grid = (int)(want < (int64_t)sms * 4 ? want : (int64_t)sms * 4);
  return launch(nvfp4_dequant_kernel, dim3(grid), dim3(256), 0, stream, pdl, reinterpret_cast<const uint2*>(P),
                reinterpret_cast<const uint8_t*>(S), ng, global_scale, out_f32 ? 1 : 0, out);
}
