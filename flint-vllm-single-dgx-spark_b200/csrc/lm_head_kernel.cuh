// NVFP4 LM-head kernel (instantiated by lm_head.cu).
//
// One persistent CTA per SM: warp NW is the TMA producer, warps 0..NW-1 consume.  The CTA owns a contiguous
// range of (16*NW)-row groups; each group is streamed as K/256 stages through an NS-deep shared-memory ring, so up to
// NS stages of weights are in flight per SM without holding any of it in registers.  Products accumulate with
// mma.sync (16 rows x up to 8 tokens per warp).  Epilogue: logits = D * 2^-shift[token] * gs (optionally stored),
// then a (value, lowest index) argmax folded per warp, per CTA (shared memory) and across CTAs (64-bit atomicMax
// in the workspace; the last CTA to arrive writes the token ids and zeroes the workspace).
#pragma once
#include "nvfp4_tile.cuh"

namespace flint {

struct HeadWorkspace {
  unsigned long long best[8];
  unsigned counter;
  unsigned status;
  unsigned pad[14];
};

template <int NS, int NW>
__global__ void __launch_bounds__((NW + 1) * 32, 1)
lm_head_kernel(const __grid_constant__ CUtensorMap map_codes, const __grid_constant__ CUtensorMap map_scales,
               const bf16* __restrict__ x, int64_t ldx, const bf16* __restrict__ res, const bf16* __restrict__ norm_w,
               float eps, int M, float gs, int V, int K, float* __restrict__ logits, int64_t ldl, int* __restrict__ tokens,
               HeadWorkspace* ws) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  using G = StageGeom<NW * 16>;
  constexpr int ROWS = NW * 16;
  uint8_t* ring_codes = smem;
  uint8_t* ring_scales = smem + NS * G::code_bytes;
  __half* xs = reinterpret_cast<__half*>(smem + NS * G::bytes);
  __shared__ uint64_t bar_full[NS], bar_empty[NS];
  __shared__ float red[(NW + 1) * 8];   // norm / staging scratch: warps x tokens
  __shared__ int shift[8];
  __shared__ unsigned long long wbest[NW][8];
  __shared__ int s_last;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ngroups = (V + ROWS - 1) / ROWS;
  const int per_cta = (ngroups + gridDim.x - 1) / gridDim.x;
  const int g0 = blockIdx.x * per_cta, g1 = min(ngroups, g0 + per_cta);
  const int nks = K / kSliceK;
  const int total = g1 > g0 ? (g1 - g0) * nks : 0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&bar_full[i], 1);
      mbar_init(&bar_empty[i], NW);
    }
    fence_mbar_init();
  }
  __syncthreads();

  // producer state (only warp NW lane 0 uses it)
  int p_s = 0, p_grp = g0, p_ks = 0, p_slot = 0;
  unsigned p_phase = 0;
  auto produce_one = [&]() {
    mbar_arrive_expect_tx(&bar_full[p_slot], G::bytes);
    tma_load_2d(ring_codes + p_slot * G::code_bytes, &map_codes, p_ks * 128, p_grp * ROWS, &bar_full[p_slot]);
    tma_load_2d(ring_scales + p_slot * G::scale_bytes, &map_scales, p_ks * 16, p_grp * ROWS, &bar_full[p_slot]);
    ++p_s;
    if (++p_ks == nks) { p_ks = 0; ++p_grp; }
    if (++p_slot == NS) { p_slot = 0; p_phase ^= 1u; }
  };
  if (warp == NW && lane == 0) {
    tma_prefetch_desc(&map_codes);
    tma_prefetch_desc(&map_scales);
    while (p_s < total && p_s < NS) produce_one();       // weights do not depend on the previous kernel
  }
  pdl_wait();
  if (norm_w) {                                          // fused final (residual add +) RMSNorm of the hidden state
    bf16* xnb = reinterpret_cast<bf16*>(xs + M * xs_stride(K));
    add_rmsnorm_2pass(x, ldx, res, norm_w, eps, M, K, xnb, red, blockDim.x, 0);
    stage_x_f16(xnb, K, M, K, xs, shift, red);
  } else {
    stage_x_f16(x, ldx, M, K, xs, shift, red);
  }

  if (warp == NW) {
    if (lane == 0) {
      while (p_s < total) {
        if (!mbar_wait(&bar_empty[p_slot], p_phase ^ 1u, &ws->status)) break;
        produce_one();
      }
    }
    pdl_trigger();
  } else {
    const int g = lane >> 2, t = lane & 3;
    const bool active = g < M;
    const __half* xrow = xs + (active ? g : 0) * xs_stride(K);
    float acc[4][4];
    zero_acc(acc);
    unsigned long long kbest[2] = {0ull, 0ull};
    const int n0 = 2 * t, n1 = 2 * t + 1;
    const float inv0 = n0 < M ? ldexpf(1.0f, -shift[n0]) : 0.f;
    const float inv1 = n1 < M ? ldexpf(1.0f, -shift[n1]) : 0.f;
    const int prow = 16 * warp + tile_phi(g);

    int slot = 0, grp = g0, ks = 0;
    unsigned phase = 0;
    for (int s = 0; s < total; ++s) {
      if (!mbar_wait(&bar_full[slot], phase, &ws->status)) break;
      consume_stage(ring_codes + slot * G::code_bytes, ring_scales + slot * G::scale_bytes, warp, g, t, ks, xrow, active, acc);
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_empty[slot]);
      if (++ks == nks) {
        const int r0 = grp * ROWS + prow, r1 = r0 + 8;
        float d[4];
        sum_acc(acc, d);
        zero_acc(acc);
        const float v00 = (d[0] * inv0) * gs, v01 = (d[1] * inv1) * gs;
        const float v10 = (d[2] * inv0) * gs, v11 = (d[3] * inv1) * gs;
        if (r0 < V) {
          if (n0 < M) { if (logits) logits[n0 * ldl + r0] = v00; kbest[0] = max(kbest[0], argmax_key(v00, r0)); }
          if (n1 < M) { if (logits) logits[n1 * ldl + r0] = v01; kbest[1] = max(kbest[1], argmax_key(v01, r0)); }
        }
        if (r1 < V) {
          if (n0 < M) { if (logits) logits[n0 * ldl + r1] = v10; kbest[0] = max(kbest[0], argmax_key(v10, r1)); }
          if (n1 < M) { if (logits) logits[n1 * ldl + r1] = v11; kbest[1] = max(kbest[1], argmax_key(v11, r1)); }
        }
        ks = 0;
        ++grp;
      }
      if (++slot == NS) { slot = 0; phase ^= 1u; }
    }
    pdl_trigger();
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      kbest[0] = max(kbest[0], shfl_xor_u64(kbest[0], o));
      kbest[1] = max(kbest[1], shfl_xor_u64(kbest[1], o));
    }
    if (g == 0) {
      wbest[warp][n0] = kbest[0];
      wbest[warp][n1] = kbest[1];
    }
  }
  if (tokens == nullptr) return;

  // ---- argmax across warps, then across CTAs ----
  __syncthreads();
  if (threadIdx.x < M) {
    unsigned long long k = 0ull;
#pragma unroll
    for (int w = 0; w < NW; ++w) k = max(k, wbest[w][threadIdx.x]);
    atomicMax(&ws->best[threadIdx.x], k);
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = (atomicAdd(&ws->counter, 1u) == gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (threadIdx.x < M) {
    const unsigned long long k = atomicExch(&ws->best[threadIdx.x], 0ull);
    tokens[threadIdx.x] = (int)argmax_key_index(k);
  }
  if (threadIdx.x == 0) atomicExch(&ws->counter, 0u);
}

}  // namespace flint
