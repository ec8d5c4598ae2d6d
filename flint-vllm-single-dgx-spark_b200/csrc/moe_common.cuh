// MoE device helpers shared by the per-op kernels (moe.cu) and the fused decode kernel (moe_fused.cu).
#pragma once
#include "engine.cuh"

namespace flint {

constexpr int kMaxTokens = 8;
constexpr int kMaxRoutes = 64;      // tokens x top-k
constexpr int kMaxExperts = 512;

// top-k key: order-preserving image of the bf16 logit in the high half, 0xFFFF - expert in the low half
// (larger logit first, then the lower expert index)
__device__ __forceinline__ uint32_t route_key(float bf16_logit, int e) {
  const uint32_t b = __float_as_uint(bf16_logit) >> 16;
  const uint32_t o = (b & 0x8000u) ? (~b & 0xFFFFu) : (b | 0x8000u);
  return (o << 16) | (0xFFFFu - (uint32_t)e);
}

// Top-k of one token's E logits by one warp: packed (bf16 logit, expert) keys, redux.sync max per round
// (larger logit first, lower expert on ties).  Weights: softmax over the chosen logits (score_fn 0) or sigmoid
// scores (1), renormalised.  Lane t < topk ends with (ids[t], weights[t]).
__device__ __forceinline__ void warp_topk(const float* logits, int E, int topk, int score_fn, int lane, int& my_e,
                                          float& my_w) {
  constexpr int PER = kMaxExperts / 32;
  const int per = E / 32;
  uint32_t key[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) key[j] = j < per ? route_key(__ldcg(logits + lane + 32 * j), lane + 32 * j) : 0u;
  float l_top = 0.f, sum = 0.f, my_p = 0.f;
  my_e = 0;
  for (int t = 0; t < topk; ++t) {
    uint32_t best = 0u;
#pragma unroll
    for (int j = 0; j < PER; ++j) best = max(best, key[j]);
    best = __reduce_max_sync(0xffffffffu, best);
#pragma unroll
    for (int j = 0; j < PER; ++j)
      if (key[j] == best) key[j] = 0u;
    const int eb = (int)(0xFFFFu - (best & 0xFFFFu));
    const uint32_t ob = best >> 16;
    const float l = __uint_as_float(((ob & 0x8000u) ? (ob & 0x7FFFu) : (~ob & 0xFFFFu)) << 16);
    if (t == 0) l_top = l;
    const float p = score_fn == 1 ? 1.0f / (1.0f + expf(-l)) : expf(l - l_top);
    sum += p;
    if (lane == t) { my_p = p; my_e = eb; }
  }
  my_w = my_p / sum;
}

// warp_topk for logits already in registers (lane holds lv[j] = logit of expert lane + 32 j, j < per <= PER), with
// the same keys, order, weights and bits: each lane sorts its keys once, then every round is one redux.sync max over
// the lane heads and a pop on the winning lane; the scores are evaluated afterwards in parallel and summed in round
// order (the sequential sum of warp_topk).
template <int PER>
__device__ __forceinline__ void warp_topk_regs(const float (&lv)[PER], int per, int topk, int score_fn, int lane,
                                               int& my_e, float& my_w) {
  uint32_t key[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) key[j] = j < per ? route_key(lv[j], lane + 32 * j) : 0u;
#pragma unroll
  for (int i = 1; i < PER; ++i)                       // insertion network, descending
#pragma unroll
    for (int j = i; j > 0; --j) {
      const uint32_t hi = max(key[j - 1], key[j]), lo = min(key[j - 1], key[j]);
      key[j - 1] = hi;
      key[j] = lo;
    }
  float my_l = 0.f;
  my_e = 0;
#pragma unroll 1
  for (int t = 0; t < topk; ++t) {
    const uint32_t best = __reduce_max_sync(0xffffffffu, key[0]);
    if (key[0] == best) {                             // keys are unique (the expert id is part of the key)
#pragma unroll
      for (int j = 0; j + 1 < PER; ++j) key[j] = key[j + 1];
      key[PER - 1] = 0u;
    }
    if (lane == t) {
      my_e = (int)(0xFFFFu - (best & 0xFFFFu));
      const uint32_t ob = best >> 16;
      my_l = __uint_as_float(((ob & 0x8000u) ? (ob & 0x7FFFu) : (~ob & 0xFFFFu)) << 16);
    }
  }
  const float l_top = __shfl_sync(0xffffffffu, my_l, 0);
  const float my_p = lane < topk ? (score_fn == 1 ? 1.0f / (1.0f + expf(-my_l)) : expf(my_l - l_top)) : 0.f;
  float sum = 0.f;
#pragma unroll 1
  for (int t = 0; t < topk; ++t) sum += __shfl_sync(0xffffffffu, my_p, t);
  my_w = my_p / sum;
}

// ------------------------------------------------------------------------------------------------------------
// Route grouping (both expert kernels): groups of routes sharing an expert, experts ascending.
// ------------------------------------------------------------------------------------------------------------
struct Groups {
  int n;                         // number of groups (distinct experts)
  int exp[kMaxRoutes];
  int cnt[kMaxRoutes];
  int route[kMaxRoutes][8];      // route index m*topk + slot
  int tok[kMaxRoutes][8];
};

// Threads [0, nthreads) of the block call it and synchronise on named barrier `bar` (0 with nthreads == blockDim.x
// is __syncthreads).  Expert parallel: only routes whose expert is in [e_lo, e_hi) are grouped, G.exp holds the
// local expert index e - e_lo, and the other routes end with ids[r] = kNotLocal.
// Groups are the routes of one expert in route order, experts ascending, at most 8 routes each (an expert with more
// routes takes several consecutive groups).  Built in parallel, one thread per route: its place among its expert's
// routes and the number of groups of the experts below it (two passes over the R <= 64 routes in shared memory).
// scratch: int[kMaxRoutes] of shared memory.
constexpr int kNotLocal = 0x7fffffff;
__device__ __forceinline__ void build_groups(const int* ids_g, int R, int topk, int E, Groups& G, int* scratch, int* ids,
                                             unsigned* status, int nthreads, int bar, int e_lo = 0,
                                             int e_hi = kNotLocal) {
  const int tid = threadIdx.x;
  auto sync = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthreads) : "memory"); };
  if (tid < R) {
    const int e = ids_g[tid];
    if ((e < 0 || e >= E) && status) atomicOr(status, 2u);
    const int ec = min(max(e, 0), E - 1);
    ids[tid] = ec >= e_lo && ec < e_hi ? ec : kNotLocal;
  }
  sync();
  int e = kNotLocal, before = 0, total = 0;
  if (tid < R) {
    e = ids[tid];
#pragma unroll 4
    for (int r = 0; r < R; ++r) {
      const int f = ids[r];
      before += (f == e) & (r < tid);
      total += f == e;
    }
    // the expert's first route records how many groups the expert takes
    scratch[tid] = before == 0 && e != kNotLocal ? (total + 7) >> 3 : 0;
  }
  sync();
  if (tid < R && e != kNotLocal) {
    int n = before >> 3;
#pragma unroll 4
    for (int r = 0; r < R; ++r) n += ids[r] < e ? scratch[r] : 0;
    const int pos = before & 7;
    G.route[n][pos] = tid;
    G.tok[n][pos] = tid / topk;
    if (pos == 0) {
      G.exp[n] = e - e_lo;
      G.cnt[n] = min(8, total - before);
    }
  }
  if (tid < 32) {                                       // the group count: one warp sums the R <= 64 entries
    const int v = (tid < R ? scratch[tid] : 0) + (tid + 32 < R ? scratch[tid + 32] : 0);
    const int ng = __reduce_add_sync(0xffffffffu, v);
    if (tid == 0) G.n = ng;
  }
  sync();
}

}  // namespace flint
