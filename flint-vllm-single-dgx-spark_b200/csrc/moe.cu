// (1) MoE decode: router + top-k, NVFP4 gate/up GEMV + SwiGLU, NVFP4 down GEMV + weighted expert sum.
// Replaces the reference's fast/fp4moe_mar.cu (route_kernel 243-303, route_norm_kernel 311-417, up_mar 67-152,
// down_mar 157-233) for 1..8 tokens, any (E, top-k, I, H) with E % 32 == 0, H % 256 == 0, I % 256 == 0.
//
// Numerics (the dequantise-to-fp32 path, patch:2890-2899 rounding points):
//   router: s = x + res (fp32), res_out = bf16(s), xn = bf16(s * rsqrt(mean(s^2) + eps) * w)       [norm optional]
//           logit[e] = bf16(sum_k xn[k] * Wr[e, k])  (fp32, fixed order: lane-strided FMA chains + xor butterfly)
//           top-k on the bf16 logits (softmax) or fp32 sigmoid scores, ties -> lowest expert index;
//           tw = softmax / sigmoid scores renormalised over the chosen experts (fp32)
//   up:     g = acc_g * gs13[e], u = acc_u * gs13[e] (fp32); act = bf16(silu(g) * u), silu(g) = g / (1 + exp(-g))
//   down:   y_e = bf16(acc * gs2[e]); out = bf16(sum_slot tw[slot] * y_slot) in slot order (fp32)
//
// Routes of the same expert are grouped (experts ascending, routes ascending inside an expert) so each expert's
// weights stream once per step for all tokens routed to it (mma N dimension = up to 8 routes).
#include "moe_common.cuh"
#include "runtime.cuh"

namespace flint {

struct MoeWorkspace {
  unsigned route_counter;
  unsigned status;
  unsigned pad[14];
  unsigned down_counter[256];       // per 64-row output tile (H <= 16384)
  // followed by y scratch: bf16 [kMaxRoutes, H]
};
static size_t moe_ws_bytes(int H) { return sizeof(MoeWorkspace) + (size_t)kMaxRoutes * H * sizeof(bf16); }

// ------------------------------------------------------------------------------------------------------------
// Router
// ------------------------------------------------------------------------------------------------------------
constexpr int kRouteWarps = 8;

template <int NV>   // H / 256 (uint4 of weights per lane)
__global__ void __launch_bounds__(kRouteWarps * 32)
route_kernel(const bf16* x, int64_t ldx, const bf16* res, const bf16* __restrict__ nw, float eps,
             const bf16* __restrict__ gw, int M, int E, int topk, int score_fn, float* __restrict__ logits, int* __restrict__ ids,
             float* __restrict__ tw, bf16* __restrict__ xn_out, bf16* __restrict__ res_out, MoeWorkspace* ws) {
  constexpr int H = NV * 256, H8 = H / 8, NT = kRouteWarps * 32;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  float* ssum = reinterpret_cast<float*>(smem_raw);                       // [M][H] fp32 x + res
  bf16* xs = reinterpret_cast<bf16*>(smem_raw + (size_t)M * H * 4);      // [M][H] normalised activations
  __shared__ float red[kRouteWarps][kMaxTokens];
  __shared__ int s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, tid = threadIdx.x;
  const int e = blockIdx.x * kRouteWarps + warp;
  uint4 wv[NV];
  if (e < E) {
    const uint4* wp = reinterpret_cast<const uint4*>(gw + (int64_t)e * H);
#pragma unroll
    for (int i = 0; i < NV; ++i) wv[i] = ldg_stream_v4(wp + lane + 32 * i);
  }
  pdl_wait();
  pdl_trigger();

  // ---- s = x (+ res) in one pass over all tokens; per-thread partial sums of s^2 in registers ----
  float ss[kMaxTokens];
#pragma unroll
  for (int m = 0; m < kMaxTokens; ++m) {
    ss[m] = 0.f;
    if (m < M) {
      for (int k8 = tid; k8 < H8; k8 += NT) {
        float a[8];
        bf16x8_to_f32(reinterpret_cast<const uint4*>(x + m * ldx)[k8], a);
        if (res) {
          float bb[8];
          bf16x8_to_f32(reinterpret_cast<const uint4*>(res + m * ldx)[k8], bb);
#pragma unroll
          for (int j = 0; j < 8; ++j) a[j] += bb[j];
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) ss[m] = fmaf(a[j], a[j], ss[m]);
        float4* d = reinterpret_cast<float4*>(ssum + m * H + k8 * 8);
        d[0] = make_float4(a[0], a[1], a[2], a[3]);
        d[1] = make_float4(a[4], a[5], a[6], a[7]);
      }
    }
  }
#pragma unroll
  for (int m = 0; m < kMaxTokens; ++m) {
    float v = ss[m];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp][m] = v;
  }
  __syncthreads();
  for (int idx = tid; idx < M * H8; idx += NT) {
    const int m = idx / H8, k8 = idx - m * H8;
    float rs = 1.f;
    if (nw) {
      float tot = 0.f;
#pragma unroll
      for (int w = 0; w < kRouteWarps; ++w) tot += red[w][m];
      rs = rsqrtf(tot / (float)H + eps);
    }
    const float4* sp = reinterpret_cast<const float4*>(ssum + m * H + k8 * 8);
    const float4 s0 = sp[0], s1 = sp[1];
    const float a[8] = {s0.x, s0.y, s0.z, s0.w, s1.x, s1.y, s1.z, s1.w};
    float wf[8];
    if (nw) bf16x8_to_f32(reinterpret_cast<const uint4*>(nw)[k8], wf);
    uint32_t pk[4], rk[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      __nv_bfloat162 n2 = nw ? __floats2bfloat162_rn(a[2 * j] * rs * wf[2 * j], a[2 * j + 1] * rs * wf[2 * j + 1])
                             : __floats2bfloat162_rn(a[2 * j], a[2 * j + 1]);
      pk[j] = *reinterpret_cast<uint32_t*>(&n2);
      __nv_bfloat162 r2 = __floats2bfloat162_rn(a[2 * j], a[2 * j + 1]);
      rk[j] = *reinterpret_cast<uint32_t*>(&r2);
    }
    reinterpret_cast<uint4*>(xs + m * H)[k8] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    if (blockIdx.x == 0) {
      if (xn_out) reinterpret_cast<uint4*>(xn_out + m * H)[k8] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      if (res_out) reinterpret_cast<uint4*>(res_out + m * H)[k8] = make_uint4(rk[0], rk[1], rk[2], rk[3]);
    }
  }
  __syncthreads();

  // ---- logits: lane-strided FMA chains (uint4 i, element j), then an xor butterfly; rounded to bf16 ----
  if (e < E) {
    for (int m = 0; m < M; ++m) {
      const uint4* xp = reinterpret_cast<const uint4*>(xs + m * H);
      float acc = 0.f;
#pragma unroll
      for (int i = 0; i < NV; ++i) {
        float xf[8], wf[8];
        bf16x8_to_f32(xp[lane + 32 * i], xf);
        bf16x8_to_f32(wv[i], wf);
#pragma unroll
        for (int j = 0; j < 8; ++j) acc = fmaf(wf[j], xf[j], acc);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) __stcg(logits + m * E + e, bf16r(acc));
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = (atomicAdd(&ws->route_counter, 1u) == gridDim.x - 1);
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // ---- last CTA: top-k per token (one warp per token) ----
  for (int m = warp; m < M; m += kRouteWarps) {
    int my_e;
    float my_w;
    warp_topk(logits + m * E, E, topk, score_fn, lane, my_e, my_w);
    if (lane < topk) {
      ids[m * topk + lane] = my_e;
      tw[m * topk + lane] = my_w;
    }
  }
  if (tid == 0) atomicExch(&ws->route_counter, 0u);
}

// ------------------------------------------------------------------------------------------------------------
// Gate/up + SwiGLU: tile = 64 gate rows + the 64 matching up rows of one expert, full K (= H)
// ------------------------------------------------------------------------------------------------------------
constexpr int kUpWarps = 8, kUpStages = 4, kUpBox = 64;
using UpL = EngineSmem<kUpWarps, kUpStages, kUpBox>;

struct UpPlan {
  const CUtensorMap* mc;
  const CUtensorMap* ms;
  const Groups* G;
  const __half* xs;
  const int* shift;
  const float* g13;
  bf16* act;
  int I, H, tpg, n_local, first, stride;
  __device__ int ntiles() const { return n_local; }
  __device__ int nks() const { return H / kSliceK; }
  __device__ int kslice0(int) const { return 0; }
  __device__ const CUtensorMap* map_codes() const { return mc; }
  __device__ const CUtensorMap* map_scales() const { return ms; }
  __device__ void decode(int tile, int& u, int& j) const {
    const int gt = first + tile * stride;
    u = gt / tpg;
    j = gt - u * tpg;
  }
  __device__ void box(int tile, int b, int& y) const {
    int u, j;
    decode(tile, u, j);
    y = G->exp[u] * 2 * I + (b == 0 ? 0 : I) + j * kUpBox;
  }
  __device__ const __half* xrow(int tile, int n, bool& active) const {
    int u, j;
    decode(tile, u, j);
    active = n < G->cnt[u];
    return xs + (active ? G->tok[u][n] : 0) * xs_stride(H);
  }
  __device__ void epilogue(int tile, const float* dt, int tid, int nthreads) {
    int u, j;
    decode(tile, u, j);
    const int cnt = G->cnt[u], e = G->exp[u];
    for (int idx = tid; idx < kUpBox * 8; idx += nthreads) {
      const int n = idx / kUpBox, r = idx - n * kUpBox;
      if (n >= cnt) continue;
      const float sc = ldexpf(g13[e], -shift[G->tok[u][n]]);
      const float gv = dt[r * 8 + n] * sc, uv = dt[(kUpBox + r) * 8 + n] * sc;
      const float silu = gv / (1.0f + expf(-gv));
      act[(int64_t)G->route[u][n] * I + j * kUpBox + r] = __float2bfloat16_rn(silu * uv);
    }
  }
};

__global__ void __launch_bounds__((kUpWarps + 1) * 32)
moe_up_kernel(const __grid_constant__ CUtensorMap mc, const __grid_constant__ CUtensorMap ms, const bf16* x, int64_t ldx,
              const int* ids, int M, int topk, int E, int I, int H, const float* __restrict__ g13, bf16* act, MoeWorkspace* ws,
              int e_lo, int e_hi) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* dtile = reinterpret_cast<float*>(smem + UpL::ring_bytes);
  __half* xs = reinterpret_cast<__half*>(smem + UpL::ring_bytes + UpL::dtile_bytes);
  __shared__ uint64_t bars[2 * kUpStages];
  __shared__ Groups G;
  __shared__ int sorted[kMaxRoutes], ids_s[kMaxRoutes];
  __shared__ int shift[kMaxTokens];
  __shared__ float red[kMaxTokens];
  engine_init_bars<kUpWarps, kUpStages>(bars);
  pdl_wait();
  build_groups(ids, M * topk, topk, E, G, sorted, ids_s, &ws->status, blockDim.x, 0, e_lo, e_hi);
  const int tpg = I / kUpBox;
  const int total = G.n * tpg;
  UpPlan plan{&mc, &ms, &G, xs, shift, g13, act, I, H, tpg, 0, (int)blockIdx.x, (int)gridDim.x};
  plan.n_local = blockIdx.x < total ? (total - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  if (threadIdx.x >= kUpWarps * 32) {
    engine_produce<kUpWarps, kUpStages, kUpBox>(plan, smem, bars, &ws->status);
  } else {
    if (plan.n_local > 0) stage_rows_f16(x, ldx, M, H, xs, shift, red, kUpWarps * 32, 2);
    engine_consume<kUpWarps, kUpStages, kUpBox>(plan, smem, dtile, bars, &ws->status);
  }
  pdl_trigger();
}

// ------------------------------------------------------------------------------------------------------------
// Down + weighted sum: tile = 64 output rows of one expert, full K (= I); the last tile of a row range to finish sums
// the routes of each token in slot order.
// ------------------------------------------------------------------------------------------------------------
constexpr int kDnWarps = 4, kDnStages = 4, kDnBox = 64;
using DnL = EngineSmem<kDnWarps, kDnStages, kDnBox>;

struct DownPlan {
  const CUtensorMap* mc;
  const CUtensorMap* ms;
  const Groups* G;
  const __half* xs;
  const int* shift;
  const float* g2;
  const float* tw;
  bf16* ybuf;
  bf16* out;                         // null in expert-parallel mode (the per-route rows in ybuf are the output)
  unsigned* counters;
  int* s_last;
  int M, topk, I, H, tpg, n_local, first, stride;
  __device__ int ntiles() const { return n_local; }
  __device__ int nks() const { return I / kSliceK; }
  __device__ int kslice0(int) const { return 0; }
  __device__ const CUtensorMap* map_codes() const { return mc; }
  __device__ const CUtensorMap* map_scales() const { return ms; }
  __device__ void decode(int tile, int& u, int& j) const {
    const int gt = first + tile * stride;
    u = gt / tpg;
    j = gt - u * tpg;
  }
  __device__ void box(int tile, int, int& y) const {
    int u, j;
    decode(tile, u, j);
    y = G->exp[u] * H + j * kDnBox;
  }
  __device__ const __half* xrow(int tile, int n, bool& active) const {
    int u, j;
    decode(tile, u, j);
    active = n < G->cnt[u];
    return xs + (active ? G->route[u][n] : 0) * xs_stride(I);
  }
  __device__ void epilogue(int tile, const float* dt, int tid, int nthreads) {
    int u, j;
    decode(tile, u, j);
    const int cnt = G->cnt[u], e = G->exp[u];
    for (int idx = tid; idx < kDnBox * 8; idx += nthreads) {
      const int n = idx / kDnBox, r = idx - n * kDnBox;
      if (n >= cnt) continue;
      const int route = G->route[u][n];
      const float y = dt[r * 8 + n] * ldexpf(g2[e], -shift[route]);
      ybuf[(int64_t)route * H + j * kDnBox + r] = __float2bfloat16_rn(y);
    }
    if (!out) return;                                 // expert parallel: the rows are summed over ranks elsewhere
    __threadfence();
    named_bar_sync(1, nthreads);
    if (tid == 0) {
      const unsigned prev = atomicAdd(&counters[j], 1u);
      *s_last = (prev == (unsigned)G->n - 1);
      if (*s_last) atomicExch(&counters[j], 0u);
    }
    named_bar_sync(1, nthreads);
    if (!*s_last) return;
    __threadfence();
    for (int idx = tid; idx < kDnBox * M; idx += nthreads) {
      const int m = idx / kDnBox, r = idx - m * kDnBox;
      float acc = 0.f;
      for (int s = 0; s < topk; ++s) {
        const unsigned short b = __ldcg(reinterpret_cast<const unsigned short*>(ybuf + (int64_t)(m * topk + s) * H + j * kDnBox + r));
        acc = fmaf(tw[m * topk + s], bf16_bits_to_f32(b), acc);
      }
      out[(int64_t)m * H + j * kDnBox + r] = __float2bfloat16_rn(acc);
    }
  }
};

__global__ void __launch_bounds__((kDnWarps + 1) * 32)
moe_down_kernel(const __grid_constant__ CUtensorMap mc, const __grid_constant__ CUtensorMap ms, const bf16* act,
                const int* ids, const float* tw, int M, int topk, int E, int I, int H, const float* __restrict__ g2, bf16* out,
                MoeWorkspace* ws, int e_lo, int e_hi, bf16* y_out) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* dtile = reinterpret_cast<float*>(smem + DnL::ring_bytes);
  __half* xs = reinterpret_cast<__half*>(smem + DnL::ring_bytes + DnL::dtile_bytes);
  __shared__ uint64_t bars[2 * kDnStages];
  __shared__ Groups G;
  __shared__ int sorted[kMaxRoutes], ids_s[kMaxRoutes];
  __shared__ int shift[kMaxRoutes];
  __shared__ float red[kMaxRoutes];
  __shared__ int s_last;
  engine_init_bars<kDnWarps, kDnStages>(bars);
  pdl_wait();
  const int R = M * topk;
  build_groups(ids, R, topk, E, G, sorted, ids_s, &ws->status, blockDim.x, 0, e_lo, e_hi);
  const int tpg = H / kDnBox;
  const int total = G.n * tpg;
  bf16* ybuf = y_out ? y_out : reinterpret_cast<bf16*>(ws + 1);
  if (y_out) {                                        // expert parallel: the other ranks' routes get zero rows
    const int H8 = H / 8;
    for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < R * H8; idx += gridDim.x * blockDim.x) {
      const int r = idx / H8;
      if (ids_s[r] == kNotLocal) reinterpret_cast<uint4*>(y_out)[idx] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  DownPlan plan{&mc, &ms, &G, xs, shift, g2, tw, ybuf, y_out ? nullptr : out, ws->down_counter, &s_last, M, topk, I, H, tpg, 0,
                (int)blockIdx.x, (int)gridDim.x};
  plan.n_local = blockIdx.x < total ? (total - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  if (threadIdx.x >= kDnWarps * 32) {
    engine_produce<kDnWarps, kDnStages, kDnBox>(plan, smem, bars, &ws->status);
  } else {
    if (plan.n_local > 0) stage_rows_f16(act, I, R, I, xs, shift, red, kDnWarps * 32, 2);
    engine_consume<kDnWarps, kDnStages, kDnBox>(plan, smem, dtile, bars, &ws->status);
  }
  pdl_trigger();
}

// ------------------------------------------------------------------------------------------------------------
// Deterministic moe_align_block_size (fast/patch_align.py:11-30): one CTA of 1024 threads.  Warp w owns the w-th
// of 32 contiguous route segments: it counts its segment per expert (warp match masks), one exclusive scan over the
// warps per expert gives each warp its start within every expert's run, and each warp then places its segment
// 32 routes at a time with no block barrier.  A route's slot is its rank among the routes of its expert in index
// order, as in the reference.
// ------------------------------------------------------------------------------------------------------------
constexpr int kAlignThreads = 1024;

__global__ void __launch_bounds__(kAlignThreads)
moe_align_kernel(const int* __restrict__ topk_ids, int n, int E, int B, int* __restrict__ sorted_ids, int n_sorted,
                 int* __restrict__ expert_ids, int n_blocks, int* __restrict__ ntp, int* __restrict__ status) {
  extern __shared__ int sm[];
  int* cnt = sm;                    // [E]
  int* pad_end = cnt + E;           // [E]
  int* wc = pad_end + E;            // [32][E] per-warp counts of its segment (then its running start)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();
  for (int e = tid; e < E; e += kAlignThreads) cnt[e] = 0;
  for (int i = tid; i < 32 * E; i += kAlignThreads) wc[i] = 0;
  __syncthreads();
  int bad = 0;
  for (int base = 0; base < n; base += 4 * kAlignThreads) {      // 4 loads in flight per thread
    int ev[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int r = base + q * kAlignThreads + tid;
      ev[q] = r < n ? topk_ids[r] : 0;
      if (r < n && (ev[q] < 0 || ev[q] >= E)) { bad = 1; ev[q] = -1; }
      if (r >= n) ev[q] = -1;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q)
      if (ev[q] >= 0) atomicAdd(&cnt[ev[q]], 1);
  }
  if (bad) atomicOr(status, 1);
  __syncthreads();
  if (tid == 0) {
    int acc = 0;
    for (int e = 0; e < E; ++e) {
      acc += (cnt[e] + B - 1) / B * B;
      pad_end[e] = acc;
    }
    ntp[0] = acc;
  }
  for (int i = tid; i < n_sorted; i += kAlignThreads) sorted_ids[i] = n;
  __syncthreads();
  for (int blk = tid; blk < n_blocks; blk += kAlignThreads) {
    const int start = blk * B;
    int lo = 0, hi = E;                          // first e with pad_end[e] > start
    while (lo < hi) {
      const int mid = (lo + hi) >> 1;
      if (pad_end[mid] <= start) lo = mid + 1; else hi = mid;
    }
    expert_ids[blk] = lo >= E ? -1 : lo;
  }
  const int seg = (n + 31) / 32, r0 = warp * seg, r1 = min(n, r0 + seg);
  int* mine = wc + warp * E;                     // this warp's counts, then its running start per expert
  auto load4 = [&](int base, int (&ev)[4]) {    // 4 x 32 routes of the segment, loads in flight together
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int r = base + 32 * q + lane;
      ev[q] = r < r1 ? topk_ids[r] : -1;
      if (ev[q] >= E) ev[q] = -1;
    }
  };
  for (int base = r0; base < r1; base += 128) {  // pass 1: per-warp counts
    int ev[4];
    load4(base, ev);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int e = ev[q];
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      if (e >= 0 && __popc(peers & ((1u << lane) - 1u)) == 0) mine[e] += __popc(peers);
      __syncwarp();
    }
  }
  __syncthreads();
  for (int ee = tid; ee < E; ee += kAlignThreads) {              // exclusive scan over the warps, per expert
    int acc = ee == 0 ? 0 : pad_end[ee - 1];
    for (int w = 0; w < 32; ++w) {
      const int c = wc[w * E + ee];
      wc[w * E + ee] = acc;
      acc += c;
    }
  }
  __syncthreads();
  for (int base = r0; base < r1; base += 128) {  // pass 2: placement, in index order within the segment
    int ev[4];
    load4(base, ev);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int e = ev[q], r = base + 32 * q + lane;
      const unsigned peers = __match_any_sync(0xffffffffu, e);
      const int rank = __popc(peers & ((1u << lane) - 1u));
      if (e >= 0) {
        const int pos = mine[e] + rank;
        if (pos < n_sorted) sorted_ids[pos] = r; else atomicOr(status, 1);
      }
      __syncwarp();
      if (e >= 0 && rank == 0) mine[e] += __popc(peers);
      __syncwarp();
    }
  }
  pdl_trigger();
}

}  // namespace flint

// ============================================================================================================
// C ABI
// ============================================================================================================
using namespace flint;

extern "C" int64_t flint_moe_workspace_bytes(int64_t H) { return (int64_t)moe_ws_bytes((int)H); }
int64_t flint::status_offset_moe() { return (int64_t)offsetof(MoeWorkspace, status); }

extern "C" int flint_moe_route(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps, const void* gate_w,
                               int64_t M, int64_t H, int64_t E, int64_t topk, int score_fn, float* logits, int32_t* topk_ids,
                               float* topk_weights, void* xn_out, void* res_out, void* workspace, int pdl, void* stream) {
  if (!x || !gate_w || !logits || !topk_ids || !topk_weights || !workspace) return FLINT_ERR_ARGUMENT;
  if (M < 1 || M > kMaxTokens || E < 32 || E % 32 != 0 || E > kMaxExperts || topk < 1 || topk > 32 || topk > E ||
      M * topk > kMaxRoutes || (H != 2048 && H != 4096) || ldx < H || ldx % 8 != 0 || (score_fn != 0 && score_fn != 1))
    return FLINT_ERR_SHAPE;
  if (!aligned(x, 16) || !aligned(gate_w, 16) || (res && !aligned(res, 16)) || (norm_w && !aligned(norm_w, 16)) ||
      (xn_out && !aligned(xn_out, 16)) || (res_out && !aligned(res_out, 16)))
    return FLINT_ERR_ALIGN;
  if (res_out && !res) return FLINT_ERR_ARGUMENT;
  const int grid = (int)((E + kRouteWarps - 1) / kRouteWarps);
  const size_t smem = (size_t)M * H * (sizeof(bf16) + sizeof(float));
  auto* ws = static_cast<MoeWorkspace*>(workspace);
  if (H == 2048) {
    if (cudaFuncSetAttribute(route_kernel<8>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return FLINT_ERR_LAUNCH;
    return launch(route_kernel<8>, dim3(grid), dim3(kRouteWarps * 32), smem, stream, pdl, (const bf16*)x, ldx,
                  (const bf16*)res, (const bf16*)norm_w, eps, (const bf16*)gate_w, (int)M, (int)E, (int)topk, score_fn, logits,
                  (int*)topk_ids, topk_weights, (bf16*)xn_out, (bf16*)res_out, ws);
  }
  if (cudaFuncSetAttribute(route_kernel<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return FLINT_ERR_LAUNCH;
  return launch(route_kernel<16>, dim3(grid), dim3(kRouteWarps * 32), smem, stream, pdl, (const bf16*)x, ldx,
                (const bf16*)res, (const bf16*)norm_w, eps, (const bf16*)gate_w, (int)M, (int)E, (int)topk, score_fn, logits,
                (int*)topk_ids, topk_weights, (bf16*)xn_out, (bf16*)res_out, ws);
}

static bool moe_shapes_ok(int64_t M, int64_t topk, int64_t E, int64_t I, int64_t H) {
  return M >= 1 && M <= kMaxTokens && topk >= 1 && M * topk <= kMaxRoutes && E >= 1 && E <= (1 << 16) && I >= kSliceK &&
         I % kSliceK == 0 && I <= 8192 && H >= kSliceK && H % kSliceK == 0 && H <= 16384 && H / 64 <= 256;
}

static int moe_up_launch(const void* xn, int64_t ldx, int64_t M, const int32_t* topk_ids, int64_t topk, const void* w13,
                         const void* s13, const float* g13, int64_t E, int64_t I, int64_t H, int64_t e_lo, int64_t n_local,
                         void* act, void* workspace, int pdl, void* stream) {
  if (!xn || !topk_ids || !w13 || !s13 || !g13 || !act || !workspace) return FLINT_ERR_ARGUMENT;
  if (!moe_shapes_ok(M, topk, E, I, H) || ldx < H || ldx % 8 != 0) return FLINT_ERR_SHAPE;
  if (e_lo < 0 || n_local < 1 || e_lo + n_local > E) return FLINT_ERR_ARGUMENT;
  if (!aligned(xn, 16) || !aligned(w13, 16) || !aligned(s13, 16)) return FLINT_ERR_ALIGN;
  const int sms = num_sms();
  if (sms <= 0) return FLINT_ERR_DEVICE;
  CUtensorMap mc, ms;
  int rc = encode_u8_2d(&mc, w13, H / 2, n_local * 2 * I, H / 2, 128, kUpBox, true);
  if (rc) return rc;
  rc = encode_u8_2d(&ms, s13, H / 16, n_local * 2 * I, H / 16, 16, kUpBox, false);
  if (rc) return rc;
  const size_t smem = 1024 + UpL::ring_bytes + UpL::dtile_bytes + (size_t)M * xs_stride((int)H) * 2;
  if (cudaFuncSetAttribute(moe_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return FLINT_ERR_LAUNCH;
  const int tiles = (int)(M * topk * (I / kUpBox));
  const int grid = tiles < 2 * sms ? tiles : 2 * sms;
  return launch(moe_up_kernel, dim3(grid), dim3((kUpWarps + 1) * 32), smem, stream, pdl, mc, ms, (const bf16*)xn, ldx,
                (const int*)topk_ids, (int)M, (int)topk, (int)E, (int)I, (int)H, g13, (bf16*)act,
                static_cast<MoeWorkspace*>(workspace), (int)e_lo, (int)(e_lo + n_local));
}

extern "C" int flint_moe_up(const void* xn, int64_t ldx, int64_t M, const int32_t* topk_ids, int64_t topk, const void* w13,
                            const void* s13, const float* g13, int64_t E, int64_t I, int64_t H, void* act, void* workspace,
                            int pdl, void* stream) {
  return moe_up_launch(xn, ldx, M, topk_ids, topk, w13, s13, g13, E, I, H, 0, E, act, workspace, pdl, stream);
}

extern "C" int flint_moe_up_ep(const void* xn, int64_t ldx, int64_t M, const int32_t* topk_ids, int64_t topk,
                               const void* w13, const void* s13, const float* g13, int64_t E, int64_t I, int64_t H,
                               int64_t expert_lo, int64_t n_local, void* act, void* workspace, int pdl, void* stream) {
  return moe_up_launch(xn, ldx, M, topk_ids, topk, w13, s13, g13, E, I, H, expert_lo, n_local, act, workspace, pdl,
                       stream);
}

static int moe_down_launch(const void* act, int64_t M, const int32_t* topk_ids, const float* topk_weights, int64_t topk,
                           const void* w2, const void* s2, const float* g2, int64_t E, int64_t I, int64_t H, int64_t e_lo,
                           int64_t n_local, void* out, void* y_out, void* workspace, int pdl, void* stream) {
  if (!act || !topk_ids || !w2 || !s2 || !g2 || (!out && !y_out) || !workspace || (out && !topk_weights))
    return FLINT_ERR_ARGUMENT;
  if (!moe_shapes_ok(M, topk, E, I, H)) return FLINT_ERR_SHAPE;
  if (e_lo < 0 || n_local < 1 || e_lo + n_local > E) return FLINT_ERR_ARGUMENT;
  if (y_out && !aligned(y_out, 16)) return FLINT_ERR_ALIGN;
  if (!aligned(act, 16) || !aligned(w2, 16) || !aligned(s2, 16)) return FLINT_ERR_ALIGN;
  const int sms = num_sms();
  if (sms <= 0) return FLINT_ERR_DEVICE;
  CUtensorMap mc, ms;
  int rc = encode_u8_2d(&mc, w2, I / 2, n_local * H, I / 2, 128, kDnBox, true);
  if (rc) return rc;
  rc = encode_u8_2d(&ms, s2, I / 16, n_local * H, I / 16, 16, kDnBox, false);
  if (rc) return rc;
  const size_t smem = 1024 + DnL::ring_bytes + DnL::dtile_bytes + (size_t)M * topk * xs_stride((int)I) * 2;
  if (smem > 227 * 1024) return FLINT_ERR_SHAPE;
  if (cudaFuncSetAttribute(moe_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return FLINT_ERR_LAUNCH;
  const int per_sm = smem <= 56 * 1024 ? 4 : smem <= 112 * 1024 ? 2 : 1;
  const int tiles = (int)(M * topk * (H / kDnBox));
  const int grid = tiles < per_sm * sms ? tiles : per_sm * sms;
  return launch(moe_down_kernel, dim3(grid), dim3((kDnWarps + 1) * 32), smem, stream, pdl, mc, ms, (const bf16*)act,
                (const int*)topk_ids, topk_weights, (int)M, (int)topk, (int)E, (int)I, (int)H, g2, (bf16*)out,
                static_cast<MoeWorkspace*>(workspace), (int)e_lo, (int)(e_lo + n_local), (bf16*)y_out);
}

extern "C" int flint_moe_down(const void* act, int64_t M, const int32_t* topk_ids, const float* topk_weights, int64_t topk,
                              const void* w2, const void* s2, const float* g2, int64_t E, int64_t I, int64_t H, void* out,
                              void* workspace, int pdl, void* stream) {
  return moe_down_launch(act, M, topk_ids, topk_weights, topk, w2, s2, g2, E, I, H, 0, E, out, nullptr, workspace, pdl,
                         stream);
}

extern "C" int flint_moe_down_ep(const void* act, int64_t M, const int32_t* topk_ids, int64_t topk, const void* w2,
                                 const void* s2, const float* g2, int64_t E, int64_t I, int64_t H, int64_t expert_lo,
                                 int64_t n_local, void* y_out, void* workspace, int pdl, void* stream) {
  return moe_down_launch(act, M, topk_ids, nullptr, topk, w2, s2, g2, E, I, H, expert_lo, n_local, nullptr, y_out,
                         workspace, pdl, stream);
}

extern "C" int flint_moe_align(const int32_t* topk_ids, int64_t numel, int64_t num_experts, int64_t block_size,
                               int32_t* sorted_ids, int64_t n_sorted, int32_t* expert_ids, int64_t n_blocks,
                               int32_t* num_tokens_post_pad, int32_t* status, int pdl, void* stream) {
  if ((numel > 0 && !topk_ids) || (n_sorted > 0 && !sorted_ids) || (n_blocks > 0 && !expert_ids) || !num_tokens_post_pad ||
      !status)
    return FLINT_ERR_ARGUMENT;
  if (numel < 0 || numel > (1 << 24) || num_experts < 1 || num_experts > 1024 || block_size < 1 || block_size > 4096)
    return FLINT_ERR_SHAPE;
  // the caller's buffers must be at least as large as vLLM's moe_align_block_size allocates
  int64_t need = numel + num_experts * (block_size - 1);
  if (numel < num_experts && numel * block_size < need) need = numel * block_size;
  if (n_sorted < need || n_blocks < (need + block_size - 1) / block_size) return FLINT_ERR_SHAPE;
  const size_t smem = (size_t)(2 + 32) * num_experts * sizeof(int);
  if (smem > 227 * 1024) return FLINT_ERR_SHAPE;
  if (cudaFuncSetAttribute(moe_align_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return FLINT_ERR_LAUNCH;
  return launch(moe_align_kernel, dim3(1), dim3(kAlignThreads), smem, stream, pdl, (const int*)topk_ids, (int)numel,
                (int)num_experts, (int)block_size, (int*)sorted_ids, (int)n_sorted, (int*)expert_ids, (int)n_blocks,
                (int*)num_tokens_post_pad, (int*)status);
}
