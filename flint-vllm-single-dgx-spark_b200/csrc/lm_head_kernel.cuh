// NVFP4 LM-head kernel (instantiated by lm_head.cu).
//
// One persistent CTA per SM: warp NW is the TMA producer, warps 0..NW-1 consume.  The CTA owns a contiguous
// range of (16*NW)-row groups; each group is streamed as K/256 stages through an NS-deep shared-memory ring, so up to
// NS stages of weights are in flight per SM without holding any of it in registers.  Products accumulate with
// mma.sync (16 rows x up to 8 tokens per warp).  Epilogue: logits = D * 2^-shift[token] * gs (optionally stored),
// then a (value, lowest index) argmax folded per warp, per CTA (shared memory) and across CTAs (64-bit atomicMax
// in the workspace; the last CTA to arrive writes the token ids and zeroes the workspace).  The SAMPLE instantiation
// replaces the argmax with the seeded top-k -> top-p -> draw of sampling.cuh over the logits the CTAs just wrote.
#pragma once
#include "nvfp4_tile.cuh"
#include "sampling.cuh"

namespace flint {

struct HeadWorkspace {
  unsigned long long best[8];
  unsigned counter;
  unsigned status;
  unsigned pad[14];
};

// Sampling parameters and buffers of the SAMPLE instantiation (see sampling.cuh for the rule).
struct SampleParams {
  float temperature, top_p;
  int top_k;
  const unsigned long long* seeds;   // [M] (null: seed 0)
  const int* step;                   // device step counter (the Philox counter's first word); null -> 0
  unsigned long long* cand;          // workspace: per row, per CTA, its top_k keys sorted [M][grid][top_k]
  int* cand_ids;                     // optional [M, top_k]: the candidates' token ids (-1 past the vocabulary)
  float* cand_logits;                // optional [M, top_k]: their logits
  int* kept;                         // optional [M]: candidates left after top-p
  unsigned id_base;                  // global id of row 0 (a vocabulary shard's first row; 0 for the whole head)
};

// Tail of the SAMPLE instantiation: per-CTA top_k of the rows it owns, then (last CTA) the global top_k, top-p and
// the draw.  smem is the drained stage ring (at least 8 * kSampleSurvivors * 8 + 3 KB).
template <int ROWS>
__device__ __forceinline__ void head_sample_tail(uint8_t* smem, const float* logits, int64_t ldl, int M, int V, int g0,
                                                 int g1, const SampleParams& sp, HeadWorkspace* ws, int* tokens,
                                                 int* s_last) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int K = sp.top_k, G = gridDim.x;
  unsigned long long* surv = reinterpret_cast<unsigned long long*>(smem);          // [8][kSampleSurvivors]
  unsigned long long* tops = surv + 8 * kSampleSurvivors;                          // [8][kSampleMaxK]
  float* wbuf = reinterpret_cast<float*>(tops + 8 * kSampleMaxK);                  // [8][kSampleMaxK]
  unsigned long long* s_T = reinterpret_cast<unsigned long long*>(wbuf + 8 * kSampleMaxK);  // [8]
  int* s_n = reinterpret_cast<int*>(s_T + 8);                                      // [8]

  __syncthreads();                       // this CTA's logits are written and its stage ring is drained
  if (warp < M) {
    const int m = warp;
    const float* lrow = logits + (int64_t)m * ldl;
    const int r0 = min(g0 * ROWS, V), r1 = min(g1 * ROWS, V);
    unsigned long long* buf = surv + m * kSampleSurvivors;
    unsigned long long lm = 0ull;
    for (int r = r0 + lane; r < r1; r += 32) lm = max(lm, argmax_key(lrow[r], sp.id_base + r));
    const unsigned long long T = warp_kth_largest(lm, K);
    int n = 0;
    for (int rb = r0; rb < r1; rb += 32) {
      const int r = rb + lane;
      n = warp_compact_ge(r < r1 ? argmax_key(lrow[r], sp.id_base + r) : 0ull, T, buf, n, kSampleSurvivors, lane);
    }
    __syncwarp();
    unsigned long long* out = sp.cand + ((int64_t)m * G + blockIdx.x) * K;
    if (n <= kSampleSurvivors) {
      warp_select_sorted(buf, n, K, out, lane);
    } else {                             // heavy ties above the bound: K rounds straight over the logits
      unsigned long long ceil = ~0ull;
      for (int k = 0; k < K; ++k) {
        unsigned long long best = 0ull;
        for (int r = r0 + lane; r < r1; r += 32) {
          const unsigned long long v = argmax_key(lrow[r], sp.id_base + r);
          if (v < ceil && v > best) best = v;
        }
        best = warp_max_u64(best);
        if (lane == 0) out[k] = best;
        ceil = best;
      }
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) *s_last = (atomicAdd(&ws->counter, 1u) == (unsigned)G - 1u);
  __syncthreads();
  if (!*s_last) return;
  __threadfence();

  // last CTA: a lower bound on each row's global top_k-th key from the CTA maxima
  if (warp < M) {
    const int m = warp;
    unsigned long long lm = 0ull;
    for (int c = lane; c < G; c += 32) lm = max(lm, __ldcg(sp.cand + ((int64_t)m * G + c) * K));
    const unsigned long long T = warp_kth_largest(lm, K);
    if (lane == 0) {
      s_T[m] = T;
      s_n[m] = 0;
    }
  }
  __syncthreads();
  const int per_row = G * K;
  for (int e = threadIdx.x; e < M * per_row; e += blockDim.x) {
    const int m = e / per_row;
    const unsigned long long key = __ldcg(sp.cand + e);
    if (key != 0ull && key >= s_T[m]) {
      const int pos = atomicAdd(&s_n[m], 1);
      if (pos < kSampleSurvivors) surv[m * kSampleSurvivors + pos] = key;
    }
  }
  __syncthreads();
  if (warp < M) {
    const int m = warp;
    unsigned long long* top = tops + m * kSampleMaxK;
    const int n = s_n[m];
    if (n <= kSampleSurvivors) {
      warp_select_sorted(surv + m * kSampleSurvivors, n, K, top, lane);
    } else {                             // heavy ties: K rounds over the row's candidate lists
      unsigned long long ceil = ~0ull;
      for (int k = 0; k < K; ++k) {
        unsigned long long best = 0ull;
        for (int i = lane; i < per_row; i += 32) {
          const unsigned long long v = __ldcg(sp.cand + (int64_t)m * per_row + i);
          if (v < ceil && v > best) best = v;
        }
        best = warp_max_u64(best);
        if (lane == 0) top[k] = best;
        ceil = best;
      }
      __syncwarp();
    }
    const int step = sp.step ? *sp.step : 0;
    const float u = sample_uniform(sp.seeds ? sp.seeds[m] : 0ull, (uint32_t)step, (uint32_t)m);
    int kept = 1;
    const int pick = sample_sorted(top, K, sp.temperature, sp.top_p, u, wbuf + m * kSampleMaxK, lane, &kept);
    if (lane == 0) {
      tokens[m] = (int)argmax_key_index(top[pick]);
      if (sp.kept) sp.kept[m] = kept;
    }
    if (lane < K) {
      const unsigned long long v = top[lane];
      if (sp.cand_ids) sp.cand_ids[m * K + lane] = v ? (int)argmax_key_index(v) : -1;
      if (sp.cand_logits) sp.cand_logits[m * K + lane] = v ? argmax_key_value(v) : -INFINITY;
    }
  }
  if (threadIdx.x == 0) atomicExch(&ws->counter, 0u);
}

template <int NS, int NW, bool SAMPLE>
__global__ void __launch_bounds__((NW + 1) * 32, 1)
lm_head_kernel(const __grid_constant__ CUtensorMap map_codes, const __grid_constant__ CUtensorMap map_scales,
               const bf16* __restrict__ x, int64_t ldx, const bf16* __restrict__ res, const bf16* __restrict__ norm_w,
               float eps, int M, float gs, int V, int K, float* __restrict__ logits, int64_t ldl, int* __restrict__ tokens,
               HeadWorkspace* ws, const SampleParams sp, uint32_t index_base, unsigned long long* keys_out) {
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
        const uint32_t k0 = index_base + (uint32_t)r0, k1 = index_base + (uint32_t)r1;   // global row ids
        if (r0 < V) {
          if (n0 < M) { if (logits) logits[n0 * ldl + r0] = v00; kbest[0] = max(kbest[0], argmax_key(v00, k0)); }
          if (n1 < M) { if (logits) logits[n1 * ldl + r0] = v01; kbest[1] = max(kbest[1], argmax_key(v01, k0)); }
        }
        if (r1 < V) {
          if (n0 < M) { if (logits) logits[n0 * ldl + r1] = v10; kbest[0] = max(kbest[0], argmax_key(v10, k1)); }
          if (n1 < M) { if (logits) logits[n1 * ldl + r1] = v11; kbest[1] = max(kbest[1], argmax_key(v11, k1)); }
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
  if constexpr (SAMPLE) {
    static_assert(NS * G::bytes >= 8 * kSampleSurvivors * 8 + 8 * kSampleMaxK * 12 + 8 * 12, "stage ring too small");
    head_sample_tail<ROWS>(smem, logits, ldl, M, V, g0, g1, sp, ws, tokens, &s_last);
    return;
  }
  if (tokens == nullptr && keys_out == nullptr) return;

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
    // vocabulary shard: the (value, lowest id) key with its top bit flipped, so that a signed int64 MAX over the
    // shards orders keys as the unsigned comparison does (the id in the low half is unchanged)
    if (keys_out) keys_out[threadIdx.x] = k ^ 0x8000000000000000ull;
    else tokens[threadIdx.x] = (int)argmax_key_index(k);
  }
  if (threadIdx.x == 0) atomicExch(&ws->counter, 0u);
}

}  // namespace flint
