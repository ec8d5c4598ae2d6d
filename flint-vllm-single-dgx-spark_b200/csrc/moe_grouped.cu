// Prefill-side grouped MoE (replaces the Flint PR's FlashInfer grouped GEMMs for prompts, grouped_moe at
// patch:4093-4212): the routes of a prompt, grouped by expert in blocks of 64 by the deterministic align
// (flint_moe_align), run through the NVFP4 gate/up + SwiGLU and down projections with each decoded weight fragment
// reused across the block's 64 routes (the decode kernels use it for at most 8 tokens).  Two tile forms, selected
// by the entry points' tensor_cores argument: tcgen05 (decoded weights and accumulator in tensor memory, further
// below; the faster one) and mma.sync (8 n-groups per decoded A fragment, described here).
//
//   flint_rows_to_f16      any bf16 rows -> f16 rows scaled by the decode kernels' per-row power of two (exact)
//   flint_moe_grouped_up   act[route] = bf16(silu(g) * u), g / u = (xh[token] . W13[e] rows) * g13[e] * 2^-shift
//   flint_moe_grouped_down y[route]   = bf16((ah[route] . W2[e] rows) * g2[e] * 2^-shift)
// then flint_moe_combine over the prompt's tokens gives out[t] = bf16(sum_s tw[t][s] y[t topk + s]) in slot order.
//
// mma.sync form: CTA = (align block of 64 routes, 128 weight rows: 64 gate + 64 up rows of one 64-column slice of
// the intermediate, or 128 down rows); 8 warps, each 16 weight rows x 64 routes.  K goes in stages of 256: the
// stage's codes (128 B per row, 16-byte units swizzled by row as the decode kernels' TMA boxes are), scales and the
// 64 routes' f16 activations are copied to shared memory, then each warp decodes its A fragments once per 16 k and
// issues one m16n8k16 MMA per group of 8 routes.  Products are exact in f16 (e2m1 x e4m3 x the rescaled activation),
// sums fp32 with one chain per route group, so results match the decode kernels within fp32 summation order.
#include "common.cuh"
#include "nvfp4_tile.cuh"
#include "runtime.cuh"

namespace flint {

constexpr int kGB = 64;                     // routes per align block
constexpr int kGW = 8;                      // warps
constexpr int kGT = kGW * 32;
constexpr int kGRows = kGW * 16;            // weight rows per CTA
constexpr int kGXS = kSliceK + 8;           // f16 stride of a staged activation row (256 k)
constexpr int kGSmem = kGRows * 128 + kGRows * 16 + kGB * kGXS * 2;   // codes + scales + activations (the
                                                                      // activation region also takes the fp32
                                                                      // results [128][64] at the end)
static_assert(kGB * kGXS * 2 >= kGRows * kGB * 4, "result tile must fit over the activations");

// one warp per row: f16(x * 2^s), s from the row's largest |x| (the decode kernels' staging rule), unpermuted.
// Two passes over the row (the second from L1 / L2), 16-byte accesses when the row and K allow them.
__global__ void __launch_bounds__(256) rows_to_f16_kernel(const bf16* __restrict__ src, int64_t ld, int rows, int K,
                                                          __half* __restrict__ dst, int* __restrict__ shift) {
  pdl_wait();
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  if (r < rows) {
    const bf16* row = src + (int64_t)r * ld;
    __half* out = dst + (int64_t)r * K;
    const bool vec = (K % 8) == 0 && (reinterpret_cast<uintptr_t>(row) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    float mx = 0.f;
    if (vec) {
      for (int k = lane * 8; k < K; k += 256) {
        const uint4 u = *reinterpret_cast<const uint4*>(row + k);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
          mx = fmaxf(mx, fmaxf(fabsf(f.x), fabsf(f.y)));
        }
      }
    } else {
      for (int k = lane; k < K; k += 32) mx = fmaxf(mx, fabsf(__bfloat162float(row[k])));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    int s = 0;
    if (mx > 0.f && !(mx != mx) && mx <= 3.0e38f) s = 14 - ((int)((__float_as_uint(mx) >> 23) & 0xFF) - 127);
    if (lane == 0) shift[r] = s;
    if (vec) {
      for (int k = lane * 8; k < K; k += 256) {
        const uint4 u = *reinterpret_cast<const uint4*>(row + k);
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
        uint32_t h[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&w[i]));
          const __half2 v = __floats2half2_rn(scale_pow2(f.x, s), scale_pow2(f.y, s));
          h[i] = *reinterpret_cast<const uint32_t*>(&v);
        }
        *reinterpret_cast<uint4*>(out + k) = make_uint4(h[0], h[1], h[2], h[3]);
      }
    } else {
      for (int k = lane; k < K; k += 32) out[k] = __float2half_rn(scale_pow2(__bfloat162float(row[k]), s));
    }
  }
  pdl_trigger();
}

struct GroupedArgs {
  const __half* xh;          // f16 rows: the tokens [T][K] (up) or the routes [R][K] (down)
  const int* shift;          // per row of xh
  const int* sorted_ids;     // align: routes grouped by expert, blocks of 64, padding = numel
  const int* expert_ids;     // align: expert of each block
  const int* ntp;            // align: num_tokens_post_pad (device)
  int numel, topk, E;
  const uint8_t* W;          // codes [E][N][K/2]
  const uint8_t* S;          // E4M3 scales [E][N][K/16]
  const float* g;            // global scale [E]
  int K, N, I;               // N = 2I (up) or H (down)
  bf16* out;                 // act [R][I] (up) or y [R][H] (down)
  int ldo;
  unsigned* status;
};

template <bool UP>
__global__ void __launch_bounds__(kGT) moe_grouped_kernel(const GroupedArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  uint8_t* codes = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* scales = codes + kGRows * 128;
  __half* xa = reinterpret_cast<__half*>(scales + kGRows * 16);
  float* res = reinterpret_cast<float*>(xa);                      // [128 rows][64 routes] after the last stage
  __shared__ int s_route[kGB], s_row[kGB];

  pdl_wait();
  // tiles fastest: the CTAs of one align block run together and share its route rows in L2
  const int blk = blockIdx.y, tile = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (blk * kGB >= __ldg(a.ntp)) return;                            // past the padded routes
  const int e = a.expert_ids[blk];
  if (e < 0 || e >= a.E) {
    if (tid == 0) atomicOr(a.status, 2u);
    return;
  }
  if (tid < kGB) {
    const int route = a.sorted_ids[blk * kGB + tid];
    const bool ok = route >= 0 && route < a.numel;
    s_route[tid] = ok ? route : -1;
    s_row[tid] = ok ? (UP ? route / a.topk : route) : -1;
  }
  // weight row of CTA row r: up -- gate rows tile*64 + r (r < 64), up rows I + tile*64 + r - 64; down -- tile*128 + r
  auto wrow = [&](int r) {
    return UP ? (r < 64 ? tile * 64 + r : a.I + tile * 64 + (r - 64)) : tile * kGRows + r;
  };
  const int g = lane >> 2, t = lane & 3;
  const int pr0 = 16 * warp + tile_phi(g), pr1 = pr0 + 8, key = pr0 & 7;
  float acc[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[j][i] = 0.f;
  const int nks = a.K / kSliceK, cb = a.K / 2, sb = a.K / 16;
  const uint8_t* We = a.W + (int64_t)e * a.N * cb;
  const uint8_t* Se = a.S + (int64_t)e * a.N * sb;

#pragma unroll 1
  for (int ks = 0; ks < nks; ++ks) {
    __syncthreads();                                                // the previous stage is consumed
    for (int i = tid; i < kGRows * 8; i += kGT) {                   // codes: 128 rows x 8 units of 16 B
      const int r = i >> 3, u = i & 7;
      *reinterpret_cast<uint4*>(codes + r * 128 + ((u ^ (r & 7)) << 4)) =
          *reinterpret_cast<const uint4*>(We + (int64_t)wrow(r) * cb + ks * 128 + u * 16);
    }
    for (int r = tid; r < kGRows; r += kGT)                         // scales: 16 B per row
      *reinterpret_cast<uint4*>(scales + r * 16) = *reinterpret_cast<const uint4*>(Se + (int64_t)wrow(r) * sb + ks * 16);
    for (int i = tid; i < kGB * 32; i += kGT) {                     // activations: 64 rows x 32 units of 8 halves
      const int rr = i >> 5, u = i & 31, row = s_row[rr];
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      if (row >= 0) v = *reinterpret_cast<const uint4*>(a.xh + (int64_t)row * a.K + ks * kSliceK + u * 8);
      *reinterpret_cast<uint4*>(xa + rr * kGXS + xs_perm(u * 8)) = v;
    }
    __syncthreads();
#pragma unroll 1
    for (int c = 0; c < 2; ++c) {
      const int phys = (4 * c + t) ^ key;
      const uint4 qg = lds128(codes + pr0 * 128 + phys * 16);
      const uint4 qg8 = lds128(codes + pr1 * 128 + phys * 16);
      const uint32_t s2 = lds_u16(scales + pr0 * 16 + 8 * c + 2 * t) | (lds_u16(scales + pr1 * 16 + 8 * c + 2 * t) << 16);
      const uint32_t sc_g = e4m3x2_to_f16x2(s2 & 0xFFFFu), sc_g8 = e4m3x2_to_f16x2(s2 >> 16);
      const uint32_t wg[4] = {qg.x, qg.y, qg.z, qg.w}, wg8[4] = {qg8.x, qg8.y, qg8.z, qg8.w};
      const int qswz = (t >> 1) << 1;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint32_t dg[4], dg8[4];
        e2m1x8_to_f16x2(wg[q], dg);
        e2m1x8_to_f16x2(wg8[q], dg8);
        const uint32_t s_g = q < 2 ? bcast_lo(sc_g) : bcast_hi(sc_g), s_g8 = q < 2 ? bcast_lo(sc_g8) : bcast_hi(sc_g8);
        const uint32_t a0[4] = {hmul2(dg[0], s_g), hmul2(dg8[0], s_g8), hmul2(dg[1], s_g), hmul2(dg8[1], s_g8)};
        const uint32_t a1[4] = {hmul2(dg[2], s_g), hmul2(dg8[2], s_g8), hmul2(dg[3], s_g), hmul2(dg8[3], s_g8)};
#pragma unroll
        for (int j = 0; j < 8; ++j) {                               // route group j: routes 8 j .. 8 j + 7
          const uint4 b = lds128(xa + (8 * j + g) * kGXS + c * 128 + 32 * t + 8 * (q ^ qswz));
          mma_f16(acc[j], a0, b.x, b.y);
          mma_f16(acc[j], a1, b.z, b.w);
        }
      }
    }
  }
  __syncthreads();                                                  // results go over the activations
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    res[pr0 * kGB + 8 * j + 2 * t] = acc[j][0];
    res[pr0 * kGB + 8 * j + 2 * t + 1] = acc[j][1];
    res[pr1 * kGB + 8 * j + 2 * t] = acc[j][2];
    res[pr1 * kGB + 8 * j + 2 * t + 1] = acc[j][3];
  }
  __syncthreads();
  const float ge = a.g[e];
  if (UP) {
    for (int idx = tid; idx < 64 * kGB; idx += kGT) {               // 64 columns x 64 routes
      const int i = idx / 64, col = idx - i * 64, route = s_route[i];
      if (route < 0) continue;
      const float sc = ldexpf(ge, -a.shift[s_row[i]]);
      const float gv = res[col * kGB + i] * sc, uv = res[(64 + col) * kGB + i] * sc;
      const float silu = gv / (1.0f + expf(-gv));
      a.out[(int64_t)route * a.ldo + tile * 64 + col] = __float2bfloat16_rn(silu * uv);
    }
  } else {
    for (int idx = tid; idx < kGRows * kGB; idx += kGT) {           // 128 rows x 64 routes
      const int i = idx / kGRows, r = idx - i * kGRows, route = s_route[i];
      if (route < 0) continue;
      a.out[(int64_t)route * a.ldo + tile * kGRows + r] =
          __float2bfloat16_rn(res[r * kGB + i] * ldexpf(ge, -a.shift[route]));
    }
  }
  pdl_trigger();
}

// ---- the same tile on the 5th-generation tensor cores (tcgen05: decoded weights and accumulator in tensor memory) ----
// 8 consumer warps, a TMA warp and an MMA warp; K goes in stages of 64.
//   TMA warp (one lane): the stage's code bytes of the CTA's 128 weight rows, 2 TMA boxes of 64 rows x 32 B with the
//     32-byte swizzle, into a 3-slot ring (full / empty mbarriers, bounded waits);
//   consumer thread (warp w, lane l): weight row r = 32 (w % 4) + l, k half h = w / 4 of the stage.  It reads its 16
//     code bytes (conflict-free under the swizzle) and its 2 E4M3 scales (loaded once per CTA into a padded array),
//     decodes them to 16 f16 pairs and writes them with one tcgen05.st into its own tensor-memory lane (warp w owns
//     lanes 32 (w % 4) ..): the MMA's A operand, two stage buffers of 32 columns.  The 64 routes' f16 activations
//     are copied by cp.async (one stage ahead, zeros for padding routes) into one of three shared-memory buffers in
//     the K-major no-swizzle canonical layout (8-row x 16-byte core matrices: route group i at i * 1024 B, 16-k step
//     s at s * 256 B, k half j at j * 128 B); lane l takes route l % 8 of an 8-route group, so each 8-lane phase of a
//     16-byte copy fills one 128-byte line; each warp then arrives on the stage's ready mbarrier;
//   MMA warp (one lane): waits for the stage's 8 arrivals, issues its 4 tcgen05.mma kind::f16 (A from tensor memory,
//     B from shared memory; M = 128 weight rows, N = 64 routes, K = 16) into the 128 x 64 fp32 accumulator
//     (tensor-memory columns 0..63) and commits them to the stage's done mbarrier.  One wait per stage, on the MMAs
//     of two stages back, frees both the A buffer and the B buffer that the stage rewrites.
// 128 tensor-memory columns, <= 53 KB of shared memory (K <= 2048) and <= 48 registers per thread: four CTAs per
// SM.  The
// epilogue reads the accumulator with tcgen05.ld.  Each product is exact; the tensor core's fp32 sums run in their
// own order (within the activation tolerance of the mma.sync tile and of the oracle).
constexpr int kTcK = 64;                            // k per stage
constexpr int kTcSbo = (kTcK / 16) * 256;           // B: bytes between 8-route groups
constexpr int kTcB = kGB * kTcK * 2;                // 8 KB activations per buffer
constexpr int kTcNB = 2;                            // A stage buffers (tensor memory); ready / done mbarriers
constexpr int kTcNBB = 3;                           // B stage buffers (shared memory)
constexpr int kTcNS = 3;                            // code ring slots
constexpr int kTcSlot = kGRows * (kTcK / 2);        // 4 KB of codes per slot (two 2 KB boxes)
constexpr int kTcACols = kTcK / 2;                  // tensor-memory columns of one A buffer (f16 pairs)
constexpr int kTcXU = kGB * (kTcK / 8) / kGT;       // activation units of 8 k per thread per stage
constexpr int kTcRS = kGB + 1;                      // fp32 stride of a result row (conflict-free column walks)
constexpr int kTcThreads = kGT + 64;                // + the TMA warp and the MMA warp
constexpr int kTcCols = 128;                        // tensor memory: accumulator 0..63, A buffers at 64 and 96
static_assert(64 + kTcACols * kTcNB <= kTcCols, "A buffers fit the allocation");
static_assert(kTcXU == 2 && kGW == 8 && kGRows == 128, "lane maps: 8 routes x 4 units per warp, 2 threads per row");
static_assert(kTcNS * kTcSlot + kTcNBB * kTcB >= kGRows * kTcRS * 4, "result tile must fit over the ring and B buffers");

// scale bytes per row in shared memory: K/16 + 4 (an odd number of words, so 32 rows read in one wavefront)
__host__ __device__ constexpr int tc_scale_stride(int K) { return K / 16 + 4; }
static int tc_smem(int K) {
  return kTcNS * kTcSlot + kTcNBB * kTcB + ((kGRows * tc_scale_stride(K) + 15) / 16) * 16;
}

// canonical-layout byte offset of 8 k (16 B) at route r, unit v (of kTcK / 8) within a B buffer
__device__ __forceinline__ int tc_off(int r, int v) { return (r >> 3) * kTcSbo + (v >> 1) * 256 + (v & 1) * 128 + (r & 7) * 16; }
__device__ __forceinline__ uint64_t tc_desc(const void* p) {      // K-major, no swizzle, LBO 128 B, SBO kTcSbo
  return (uint64_t)((smem_u32(p) >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(kTcSbo >> 4) << 32) |
         (1ull << 46);
}
// D (tensor memory) += A (tensor memory) x B (shared memory descriptor)
__device__ __forceinline__ void tc_mma_f16_ta(uint32_t d, uint32_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n.reg .pred p;\nsetp.ne.b32 p, %4, 0;\n"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d), "r"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tc_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// 16-byte global -> shared copy that fills zeros when `valid` is false (src-size 0: nothing is read)
__device__ __forceinline__ void tc_cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void tc_cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void tc_cp_async_wait1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// 2-D TMA tile load without an L2 hint: the weight rows are read again by the expert's other align blocks
__device__ __forceinline__ void tc_tma_load(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

template <bool UP>
__global__ void __launch_bounds__(kTcThreads, 4)
moe_grouped_tc_kernel(const __grid_constant__ CUtensorMap mc, const GroupedArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* Bs = ring + kTcNS * kTcSlot;                           // buffer b at Bs + b kTcB
  uint8_t* scales = Bs + kTcNBB * kTcB;                           // [128 rows][tc_scale_stride(K)]
  float* res = reinterpret_cast<float*>(ring);                    // [128 rows][kTcRS] after the last stage
  __shared__ int s_route[kGB], s_row[kGB];
  __shared__ uint32_t s_taddr;
  __shared__ __align__(8) uint64_t s_full[kTcNS], s_empty[kTcNS], s_ready[kTcNB], s_mma[kTcNB];

  pdl_wait();
  // tiles fastest: the CTAs of one align block run together and share its route rows in L2
  const int blk = blockIdx.y, tile = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (blk * kGB >= __ldg(a.ntp)) return;
  const int e = a.expert_ids[blk];
  if (e < 0 || e >= a.E) {
    if (tid == 0) atomicOr(a.status, 2u);
    return;
  }
  if (tid < kGB) {
    const int route = a.sorted_ids[blk * kGB + tid];
    const bool ok = route >= 0 && route < a.numel;
    s_route[tid] = ok ? route : -1;
    s_row[tid] = ok ? (UP ? route / a.topk : route) : -1;
  }
  auto wrow = [&](int r) {
    return UP ? (r < 64 ? tile * 64 + r : a.I + tile * 64 + (r - 64)) : tile * kGRows + r;
  };
  const int nks = a.K / kTcK, sb = a.K / 16, sst = tc_scale_stride(a.K);
  const uint8_t* Se = a.S + (int64_t)e * a.N * sb;
  const int y0 = e * a.N + (UP ? tile * 64 : tile * kGRows), y1 = e * a.N + (UP ? a.I + tile * 64 : tile * kGRows + 64);
  const int npre = nks < kTcNS ? nks : kTcNS;
  auto produce = [&](int ks) {                                     // one stage's two code boxes
    const int slot = ks % kTcNS;
    uint8_t* dst = ring + slot * kTcSlot;
    mbar_arrive_expect_tx(&s_full[slot], (unsigned)kTcSlot);
    tc_tma_load(dst, &mc, ks * (kTcK / 2), y0, &s_full[slot]);
    tc_tma_load(dst + kTcSlot / 2, &mc, ks * (kTcK / 2), y1, &s_full[slot]);
  };
  if (warp == kGW && lane == 0) {                                  // barriers, then the first stages right away
    for (int i = 0; i < kTcNS; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], kGW);
    }
    for (int i = 0; i < kTcNB; ++i) {
      mbar_init(&s_ready[i], kGW);
      mbar_init(&s_mma[i], 1);
    }
    fence_mbar_init();
    for (int ks = 0; ks < npre; ++ks) produce(ks);
  }
  if (warp == 0) {                                                 // accumulator + two A buffers
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&s_taddr)),
                 "r"((uint32_t)kTcCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  // consumers' activation units: unit j at route 8 ((warp + 8 j) % 8) + lane % 8, 8-k unit 4 ((warp + 8 j) / 8) +
  // lane / 8; the route rows come straight from the align output, so the first stage's loads start now
  const int l8 = lane & 7, c = lane >> 3;
  int xrow[kTcXU];
  auto fetch = [&](int ks) {                                       // one cp.async group per stage
    uint8_t* Bb = Bs + (ks % kTcNBB) * kTcB;
#pragma unroll
    for (int j = 0; j < kTcXU; ++j) {
      const int v = 4 * ((warp + 8 * j) >> 3) + c;
      const __half* src = a.xh + (xrow[j] >= 0 ? (int64_t)xrow[j] * a.K + ks * kTcK + v * 8 : 0);
      tc_cp_async16(Bb + tc_off(8 * ((warp + 8 * j) & 7) + l8, v), src, xrow[j] >= 0);
    }
    tc_cp_async_commit();
  };
  if (warp < kGW) {
#pragma unroll
    for (int j = 0; j < kTcXU; ++j) {
      const int route = __ldg(a.sorted_ids + blk * kGB + 8 * ((warp + 8 * j) & 7) + l8);
      xrow[j] = route >= 0 && route < a.numel ? (UP ? route / a.topk : route) : -1;
    }
    fetch(0);
    // this CTA's scale rows, once
    const int wpr = sb / 4;
    for (int idx = tid; idx < kGRows * wpr; idx += kGT) {
      const int r = idx / wpr, wd = idx - r * wpr;
      *reinterpret_cast<uint32_t*>(scales + r * sst + wd * 4) =
          __ldg(reinterpret_cast<const unsigned int*>(Se + (uint32_t)(wrow(r) * sb + wd * 4)));
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = s_taddr;
  bool ok = true;

  if (warp == kGW) {
    // ---- producer: code boxes into the ring ----
    if (lane == 0) {
#pragma unroll 1
      for (int ks = npre; ks < nks; ++ks) {
        if (!mbar_wait(&s_empty[ks % kTcNS], (unsigned)(((ks / kTcNS) - 1) & 1), a.status)) break;
        produce(ks);
      }
    }
    __syncwarp();
  } else if (warp == kGW + 1) {
    // ---- MMA issue: one lane, each stage after its buffer's 8 consumer-warp arrivals ----
    if (lane == 0) {
      const uint32_t idesc = (1u << 4) | ((uint32_t)(kGB >> 3) << 17) | ((uint32_t)(kGRows >> 4) << 24);
#pragma unroll 1
      for (int ks = 0; ks < nks; ++ks) {
        const int b = ks % kTcNB;
        if (!mbar_wait(&s_ready[b], (unsigned)((ks / kTcNB) & 1), a.status)) break;
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint8_t* Bb = Bs + (ks % kTcNBB) * kTcB;
#pragma unroll 1
        for (int s16 = 0; s16 < kTcK / 16; ++s16)
          tc_mma_f16_ta(tmem, tmem + (uint32_t)(64 + kTcACols * b + 8 * s16), tc_desc(Bb + s16 * 256), idesc,
                        (ks > 0 || s16 > 0) ? 1u : 0u);
        tc_commit(&s_mma[b]);
      }
    }
    __syncwarp();
  } else {
    // ---- consumers ----
    // decode: row r = 32 (warp % 4) + lane, k half h = warp / 4
    const int r = 32 * (warp & 3) + lane, h = warp >> 2, sw = (r >> 2) & 1;
    const uint32_t a_lane = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
#pragma unroll 1
    for (int ks = 0; ks < nks; ++ks) {
      const int slot = ks % kTcNS, b = ks % kTcNB;
      // buffers: B of stage ks + 1 and A of stage ks were last read by the MMAs of stages ks - 2 and ks - 3; the
      // commit of stage ks - 2 covers both (bounded wait)
      if (ks >= 2 && ok && !mbar_wait(&s_mma[(ks - 2) % kTcNB], (unsigned)(((ks - 2) / kTcNB) & 1), a.status)) ok = false;
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      if (ks + 1 < nks) fetch(ks + 1);                             // the next stage's rows fly during this one
      else tc_cp_async_commit();                                   // (an empty group keeps the count uniform)
      if (ok && !mbar_wait(&s_full[slot], (unsigned)((ks / kTcNS) & 1), a.status)) ok = false;
      const uint8_t* cs = ring + slot * kTcSlot + r * 32;
      const uint4 q0 = *reinterpret_cast<const uint4*>(cs + ((h ^ sw) << 4));
      const uint32_t s2 = *reinterpret_cast<const unsigned short*>(scales + r * sst + ks * (kTcK / 16) + 2 * h);
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_empty[slot]);                  // this warp is done with the slot
      uint32_t d[16];
      {
        const uint32_t s01 = e4m3x2_to_f16x2(s2);
        const uint32_t wq[4] = {q0.x, q0.y, q0.z, q0.w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {                              // 8 k per word; 16-k scale group q / 2
          const uint32_t sg = q < 2 ? bcast_lo(s01) : bcast_hi(s01);
          uint32_t o[4];
          e2m1x8_to_f16x2(wq[q], o);
#pragma unroll
          for (int i = 0; i < 4; ++i) d[4 * q + i] = hmul2(o[i], sg);
        }
      }
      tc_st16(a_lane + (uint32_t)(64 + kTcACols * b + 16 * h), d);
      tc_cp_async_wait1();                                         // this stage's rows are in place
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); // generic-proxy stores -> the tensor core
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_ready[b]);                     // this warp's share of the stage is in place
    }
    // the last commit covers every MMA of the tile (bounded wait)
    if (ok && !mbar_wait(&s_mma[(nks - 1) % kTcNB], (unsigned)(((nks - 1) / kTcNB) & 1), a.status)) ok = false;
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  }
  __syncthreads();
  // accumulator -> registers: thread (warp, lane) holds weight row 32 (warp % 4) + lane for routes 32 (warp / 4) ..
  const float ge = a.g[e];
  if (warp < kGW) {
    const int row = 32 * (warp & 3) + lane;
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {                         // 16 accumulator columns at a time
      const int col0 = 32 * (warp >> 2) + 16 * half;
      float v[16];
      tc_ld16(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)col0, v);
      if (UP) {                                                    // gate and up rows meet through shared memory
#pragma unroll
        for (int i = 0; i < 16; ++i) res[row * kTcRS + col0 + i] = ok ? v[i] : 0.f;
      } else {                                                     // down: straight out, 64 B per warp store
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int route = s_route[col0 + i];
          if (route >= 0)
            a.out[(int64_t)route * a.ldo + tile * kGRows + row] =
                __float2bfloat16_rn((ok ? v[i] : 0.f) * ldexpf(ge, -a.shift[route]));
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)kTcCols) : "memory");
  if (warp < kGW) {
    if (UP) {
      for (int idx = tid; idx < 64 * kGB; idx += kGT) {
        const int i = idx / 64, col = idx - i * 64, route = s_route[i];
        if (route < 0) continue;
        const float sc = ldexpf(ge, -a.shift[s_row[i]]);
        const float gv = res[col * kTcRS + i] * sc, uv = res[(64 + col) * kTcRS + i] * sc;
        const float silu = gv / (1.0f + expf(-gv));
        a.out[(int64_t)route * a.ldo + tile * 64 + col] = __float2bfloat16_rn(silu * uv);
      }
    }
  }
  pdl_trigger();
}

template <bool UP>
static int grouped_launch_mma(const GroupedArgs& a, int max_blocks, int tiles, int pdl, void* stream) {
  auto kern = moe_grouped_kernel<UP>;
  const int smem = kGSmem + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return FLINT_ERR_LAUNCH;
  return launch(kern, dim3((unsigned)tiles, (unsigned)max_blocks), dim3(kGT), smem, stream, pdl, a);
}

template <bool UP>
static int grouped_launch_tc(const GroupedArgs& a, int max_blocks, int tiles, int pdl, void* stream) {
  CUtensorMap mc;                                                  // codes [E N rows][K/2 B], boxes of 64 rows x 32 B
  int rc = encode_u8_2d_swz(&mc, a.W, (uint64_t)(a.K / 2), (uint64_t)a.E * a.N, (uint64_t)(a.K / 2), 64u, kTcK / 2);
  if (rc) return rc;
  auto kern = moe_grouped_tc_kernel<UP>;
  const int smem = tc_smem(a.K) + 1024;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return FLINT_ERR_LAUNCH;
  return launch(kern, dim3((unsigned)tiles, (unsigned)max_blocks), dim3(kTcThreads), smem, stream, pdl, mc, a);
}

}  // namespace flint

using namespace flint;

extern "C" int flint_rows_to_f16(const void* src, int64_t ld, int64_t rows, int64_t K, void* dst, int32_t* shift,
                                 int pdl, void* stream) {
  if (!src || !dst || !shift) return FLINT_ERR_ARGUMENT;
  if (rows < 1 || rows > (1 << 30) || K < 1 || ld < K) return FLINT_ERR_SHAPE;
  return launch(rows_to_f16_kernel, dim3((unsigned)((rows + 7) / 8)), dim3(256), 0, stream, pdl, (const bf16*)src, ld,
                (int)rows, (int)K, (__half*)dst, (int*)shift);
}

static int grouped_entry(bool up, int tc, const void* xh, const int32_t* shift, const int32_t* sorted_ids,
                         const int32_t* expert_ids, const int32_t* num_tokens_post_pad, int64_t numel, int64_t topk,
                         int64_t E, const void* W, const void* S, const float* g, int64_t H, int64_t I,
                         int64_t max_blocks, void* out, void* workspace, int pdl, void* stream) {
  if (tc != 0 && tc != 1) return FLINT_ERR_ARGUMENT;
  if (!xh || !shift || !sorted_ids || !expert_ids || !num_tokens_post_pad || !W || !S || !g || !out || !workspace)
    return FLINT_ERR_ARGUMENT;
  if (numel < 1 || topk < 1 || topk > 32 || E < 1 || max_blocks < 1 || max_blocks > 65535 || H < kSliceK ||
      H % kSliceK != 0 || I < kSliceK || I % kSliceK != 0 || I * H >= (int64_t(1) << 31))
    return FLINT_ERR_SHAPE;                                         // one expert's 2I x H/2 code bytes in 32 bits
  if (!aligned(xh, 16) || !aligned(W, 16) || !aligned(S, 16) || !aligned(workspace, 4)) return FLINT_ERR_ALIGN;
  GroupedArgs a;
  a.xh = (const __half*)xh; a.shift = shift; a.sorted_ids = sorted_ids; a.expert_ids = expert_ids;
  a.ntp = num_tokens_post_pad; a.numel = (int)numel; a.topk = (int)topk; a.E = (int)E;
  a.W = (const uint8_t*)W; a.S = (const uint8_t*)S; a.g = g; a.I = (int)I; a.out = (bf16*)out;
  a.status = (unsigned*)workspace;
  if (up) {
    a.K = (int)H; a.N = (int)(2 * I); a.ldo = (int)I;
    return tc ? grouped_launch_tc<true>(a, (int)max_blocks, (int)(I / 64), pdl, stream)
              : grouped_launch_mma<true>(a, (int)max_blocks, (int)(I / 64), pdl, stream);
  }
  a.K = (int)I; a.N = (int)H; a.ldo = (int)H;
  return tc ? grouped_launch_tc<false>(a, (int)max_blocks, (int)(H / kGRows), pdl, stream)
            : grouped_launch_mma<false>(a, (int)max_blocks, (int)(H / kGRows), pdl, stream);
}

extern "C" int flint_moe_grouped_up(const void* xh, const int32_t* shift, const int32_t* sorted_ids,
                                    const int32_t* expert_ids, const int32_t* num_tokens_post_pad, int64_t numel,
                                    int64_t topk, int64_t E, const void* w13, const void* s13, const float* g13,
                                    int64_t H, int64_t I, int64_t max_blocks, void* act, void* workspace,
                                    int tensor_cores, int pdl, void* stream) {
  return grouped_entry(true, tensor_cores, xh, shift, sorted_ids, expert_ids, num_tokens_post_pad, numel, topk, E, w13, s13, g13,
                       H, I, max_blocks, act, workspace, pdl, stream);
}

extern "C" int flint_moe_grouped_down(const void* ah, const int32_t* shift, const int32_t* sorted_ids,
                                      const int32_t* expert_ids, const int32_t* num_tokens_post_pad, int64_t numel,
                                      int64_t topk, int64_t E, const void* w2, const void* s2, const float* g2,
                                      int64_t H, int64_t I, int64_t max_blocks, void* y, void* workspace,
                                      int tensor_cores, int pdl, void* stream) {
  return grouped_entry(false, tensor_cores, ah, shift, sorted_ids, expert_ids, num_tokens_post_pad, numel, topk, E, w2, s2, g2, H,
                       I, max_blocks, y, workspace, pdl, stream);
}
