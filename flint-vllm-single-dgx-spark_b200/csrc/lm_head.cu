// (4) NVFP4 LM head: logits and the greedy argmax in one pass over the head (fast/fast_head.py:95-121,200-207).
//
// Persistent grid (2 CTAs per SM, 8 warps each).  Each CTA owns a contiguous range of 16-row blocks; each warp
// streams whole 16-row x K blocks through a 2-deep register ring (CPS 128-k chunks per stage, 128-bit
// non-allocating loads) and accumulates with mma.sync (rows = M, tokens = N).  Tokens 1..8 share the stream.
// The epilogue scales by 2^-shift[token] * gs, optionally stores fp32 logits and folds (value, lowest index)
// argmax keys; CTAs publish with one 64-bit atomicMax per token, and the last CTA to arrive writes the token
// ids and zeroes the workspace (deterministic: max is order independent, ties resolve to the lowest index).
#include "common.cuh"
#include "runtime.cuh"

namespace flint {

struct HeadWorkspace {
  unsigned long long best[8];
  unsigned counter;
  unsigned pad[15];
};

template <int CPS, int NW>
__global__ void __launch_bounds__(NW * 32, 2)
lm_head_kernel(const bf16* __restrict__ x, int64_t ldx, int M, const uint8_t* __restrict__ W, const uint8_t* __restrict__ S,
               float gs, int V, int K, float* __restrict__ logits, int64_t ldl, int* __restrict__ tokens, HeadWorkspace* ws) {
  extern __shared__ __align__(16) unsigned char smem_raw[];
  __half* xs = reinterpret_cast<__half*>(smem_raw);
  __shared__ float red[NW * 8];
  __shared__ int shift[8];
  __shared__ unsigned long long wbest[NW][8];
  __shared__ int s_last;

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int nblk = (V + 15) >> 4;
  const int per_cta = (nblk + gridDim.x - 1) / gridDim.x;
  const int b0 = blockIdx.x * per_cta;
  const int b1 = min(nblk, b0 + per_cta);
  const int nch = K >> 7;
  const int spb = nch / CPS;                       // stages per 16-row block
  const int my_blocks = (b1 - b0 > warp) ? (b1 - b0 - warp + NW - 1) / NW : 0;
  const int total = my_blocks * spb;
  const int64_t wrow = K >> 1, srow = K >> 4;

  auto rows_of = [&](int s, const uint8_t*& wg, const uint8_t*& wg8, const uint8_t*& sg, const uint8_t*& sg8) {
    const int blk = b0 + warp + NW * (s / spb);
    const int r0 = min(blk * 16 + g, V - 1), r1 = min(blk * 16 + g + 8, V - 1);
    wg = W + (int64_t)r0 * wrow;
    wg8 = W + (int64_t)r1 * wrow;
    sg = S + (int64_t)r0 * srow;
    sg8 = S + (int64_t)r1 * srow;
  };

  WStage<CPS> st0, st1;
  if (total > 0) {
    const uint8_t *a, *b, *c, *d;
    rows_of(0, a, b, c, d);
    load_stage<CPS>(st0, a, b, c, d, 0, t);
  }
  pdl_wait();
  stage_x_f16(x, ldx, M, K, xs, shift, red);

  const bool active = g < M;
  const __half* xrow = xs + (active ? g : 0) * xs_stride(K);
  float acc[2][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[i][e] = 0.f;
  unsigned long long kbest[2] = {0ull, 0ull};
  const int n0 = 2 * t, n1 = 2 * t + 1;
  const float inv0 = n0 < M ? ldexpf(1.0f, -shift[n0]) : 0.f;
  const float inv1 = n1 < M ? ldexpf(1.0f, -shift[n1]) : 0.f;

  auto epilogue = [&](int s) {
    const int blk = b0 + warp + NW * (s / spb);
    const int r0 = blk * 16 + g, r1 = r0 + 8;
    float d[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      d[e] = acc[0][e] + acc[1][e];
      acc[0][e] = 0.f;
      acc[1][e] = 0.f;
    }
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
  };

  for (int s = 0; s < total; s += 2) {
    if (s + 1 < total) {
      const uint8_t *a, *b, *c, *d;
      rows_of(s + 1, a, b, c, d);
      load_stage<CPS>(st1, a, b, c, d, ((s + 1) % spb) * CPS, t);
    }
    compute_stage<CPS>(st0, xrow, active, (s % spb) * CPS, t, acc);
    if ((s % spb) == spb - 1) epilogue(s);
    if (s + 1 < total) {
      if (s + 2 < total) {
        const uint8_t *a, *b, *c, *d;
        rows_of(s + 2, a, b, c, d);
        load_stage<CPS>(st0, a, b, c, d, ((s + 2) % spb) * CPS, t);
      }
      compute_stage<CPS>(st1, xrow, active, ((s + 1) % spb) * CPS, t, acc);
      if (((s + 1) % spb) == spb - 1) epilogue(s + 1);
    }
  }
  pdl_trigger();
  if (tokens == nullptr) return;

  // ---- argmax: lanes of equal t hold the same tokens; reduce over g, then over warps, then over CTAs ----
#pragma unroll
  for (int o = 4; o < 32; o <<= 1) {
    kbest[0] = max(kbest[0], shfl_xor_u64(kbest[0], o));
    kbest[1] = max(kbest[1], shfl_xor_u64(kbest[1], o));
  }
  if (g == 0) {
    wbest[warp][n0] = kbest[0];
    wbest[warp][n1] = kbest[1];
  }
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

template <int CPS>
static int launch_head(const void* x, int64_t ldx, int M, const void* P, const void* S, float gs, int V, int K, float* logits,
                       int64_t ldl, int32_t* tokens, void* ws, int pdl, void* stream) {
  constexpr int NW = 8;
  const int sms = num_sms();
  if (sms <= 0) return FLINT_ERR_DEVICE;
  const int nblk = (V + 15) / 16;
  int grid = 2 * sms;
  const int min_per_cta = NW;                         // at least one block per warp
  if ((nblk + min_per_cta - 1) / min_per_cta < grid) grid = (nblk + min_per_cta - 1) / min_per_cta;
  const size_t smem = (size_t)M * xs_stride(K) * sizeof(__half);
  return launch(lm_head_kernel<CPS, NW>, dim3(grid), dim3(NW * 32), smem, stream, pdl, (const bf16*)x, ldx, M,
                (const uint8_t*)P, (const uint8_t*)S, gs, V, K, logits, ldl, (int*)tokens, (HeadWorkspace*)ws);
}

}  // namespace flint

extern "C" int64_t flint_lm_head_workspace_bytes(void) { return sizeof(flint::HeadWorkspace); }

extern "C" int flint_lm_head_nv4(const void* x, int64_t ldx, int64_t M, const void* P, const void* S, float gs, int64_t V,
                                 int64_t K, float* logits, int64_t ld_logits, int32_t* token_ids, void* workspace, int pdl,
                                 void* stream) {
  using namespace flint;
  if (!x || !P || !S) return FLINT_ERR_ARGUMENT;
  if (M < 1 || M > 8 || V < 1 || V > (1ll << 30) || K < 128 || K % 128 != 0 || K > 8192 || ldx < K) return FLINT_ERR_SHAPE;
  if (logits && ld_logits < V) return FLINT_ERR_SHAPE;
  if (!aligned(P, 16) || !aligned(S, 2) || !aligned(x, 2)) return FLINT_ERR_ALIGN;
  if (token_ids && !workspace) return FLINT_ERR_WORKSPACE;
  if (workspace && !aligned(workspace, 8)) return FLINT_ERR_ALIGN;
  if (K % 512 == 0)
    return launch_head<4>(x, ldx, (int)M, P, S, gs, (int)V, (int)K, logits, ld_logits, token_ids, workspace, pdl, stream);
  return launch_head<1>(x, ldx, (int)M, P, S, gs, (int)V, (int)K, logits, ld_logits, token_ids, workspace, pdl, stream);
}
