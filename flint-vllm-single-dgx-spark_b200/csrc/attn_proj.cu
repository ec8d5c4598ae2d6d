// (3) Attention projections around the decode attention.  Replaces the reference's fast/attn_gemv2.cu
// (qkv_gemv_kernel 101-150, qkv_head_kernel 170-265, o_gemv_kernel 268-289) for 1..8 tokens.
//
// QKV: one thread-block cluster of kQkvCL CTAs per attention head (128 rows of the fused [q; k; v] weight); the CTAs
// split K and reduce through distributed shared memory into rank 0, which then owns the whole head and finishes it:
//   y = bf16(acc * gs)                                             (the qkv output)
//   q / k heads: n = bf16(y * rsqrt(mean(y^2) + eps_head) * w), NeoX RoPE in fp32 from the fp32 cos|sin table,
//                r1 = n1*cos - n2*sin, r2 = n2*cos + n1*sin, rounded to bf16 (q out; k into y and the KV cache)
//   v heads:     y into the KV cache unchanged
// The add + RMSNorm of the hidden state (s = x + res, res_out = bf16(s), xn = bf16(s*rsqrt(mean s^2+eps)*w)) is
// recomputed by every CTA in the same fixed order (identical results); the head with index 0 publishes res_out.
// O: 64-row tiles, K split over a cluster of kOCL CTAs, y = bf16(acc * gs).
#include "engine.cuh"
#include "runtime.cuh"

namespace flint {

constexpr int kQkvWarps = 8, kQkvStages = 4, kQkvBox = 64, kQkvCL = 2, kHeadDim = 128;
constexpr int kOWarps = 4, kOStages = 4, kOBox = 64, kOCL = 4;
using QkvL = EngineSmem<kQkvWarps, kQkvStages, kQkvBox>;
using OL = EngineSmem<kOWarps, kOStages, kOBox>;

struct ProjWorkspace {
  unsigned status;
  unsigned pad[31];
};

struct QkvArgs {
  const bf16* x;
  int64_t ldx;
  const int* tokens;            // optional: row m of x is x + tokens[m] * ldx (embedding gather)
  const bf16* res;
  const bf16* nw;
  float eps;
  const float* gs;
  int M, H, N, nq, nkv;
  int head_mode;               // 0: plain GEMV (qkv_gemv); 1: + q/k norm, RoPE, KV write (qkv_head)
  const bf16* q_w;
  const bf16* k_w;
  float eps_head;
  const int64_t* positions;
  const float* cos_sin;        // [max_pos, 128] (cos | sin) or nullptr (no RoPE)
  int64_t cs_stride;
  bf16* k_cache;
  bf16* v_cache;
  int64_t st_block, st_slot, st_head;
  int block_size;
  const int64_t* slots;
  bf16* q_out;
  bf16* y_out;
  bf16* res_out;
  unsigned* status;
};

struct QkvPlan {
  const CUtensorMap* mc;
  const CUtensorMap* ms;
  const __half* xs;
  const int* shift;
  const QkvArgs* a;
  int head, rank, nks_part;
  __device__ int ntiles() const { return 1; }
  __device__ int nks() const { return nks_part; }
  __device__ int kslice0(int) const { return rank * nks_part; }
  __device__ const CUtensorMap* map_codes() const { return mc; }
  __device__ const CUtensorMap* map_scales() const { return ms; }
  __device__ void box(int, int b, int& y) const { y = head * kHeadDim + b * kQkvBox; }
  __device__ const __half* xrow(int, int n, bool& active) const {
    active = n < a->M;
    return xs + (active ? n : 0) * xs_stride(a->H);
  }
  __device__ void epilogue(int, const float* dt, int tid, int) {
    const int lane = tid & 31, m = tid >> 5;      // one warp per token
    const QkvArgs& A = *a;
    if (m >= A.M) return;
    const float sc = ldexpf(A.gs[0], -shift[m]);
    float y[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int r = lane + 32 * i;
      y[i] = bf16r(dt[r * 8 + m] * sc);
      A.y_out[(int64_t)m * A.N + head * kHeadDim + r] = __float2bfloat16_rn(y[i]);
    }
    if (!A.head_mode) return;
    const bool is_q = head < A.nq, is_v = head >= A.nq + A.nkv;
    float o[4] = {y[0], y[1], y[2], y[3]};
    if (!is_v) {
      float v2 = y[0] * y[0] + y[1] * y[1] + y[2] * y[2] + y[3] * y[3];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v2 += __shfl_xor_sync(0xffffffffu, v2, off);
      const float rs = rsqrtf(v2 / (float)kHeadDim + A.eps_head);
      const bf16* wq = is_q ? A.q_w : A.k_w;
#pragma unroll
      for (int i = 0; i < 4; ++i) o[i] = bf16r(y[i] * rs * __bfloat162float(wq[lane + 32 * i]));
      if (A.cos_sin) {
        const float* cs = A.cos_sin + A.positions[m] * A.cs_stride;
#pragma unroll
        for (int i = 0; i < 2; ++i) {             // pairs (r, r + 64): r = lane + 32 i
          const int r = lane + 32 * i;
          const float c = cs[r], s = cs[64 + r];
          const float n1 = o[i], n2 = o[i + 2];
          o[i] = fmaf(n1, c, -(n2 * s));
          o[i + 2] = fmaf(n2, c, n1 * s);
        }
      }
    }
    if (is_q) {
#pragma unroll
      for (int i = 0; i < 4; ++i)
        A.q_out[(int64_t)m * A.nq * kHeadDim + head * kHeadDim + lane + 32 * i] = __float2bfloat16_rn(o[i]);
      return;
    }
    if (!is_v) {
#pragma unroll
      for (int i = 0; i < 4; ++i) A.y_out[(int64_t)m * A.N + head * kHeadDim + lane + 32 * i] = __float2bfloat16_rn(o[i]);
    }
    const int64_t slot = A.slots ? A.slots[m] : -1;
    if (slot < 0) return;
    const int kvh = is_v ? head - A.nq - A.nkv : head - A.nq;
    const int64_t dst = (slot / A.block_size) * A.st_block + (slot % A.block_size) * A.st_slot + (int64_t)kvh * A.st_head;
    bf16* cache = (is_v ? A.v_cache : A.k_cache) + dst;
#pragma unroll
    for (int i = 0; i < 4; ++i) cache[lane + 32 * i] = __float2bfloat16_rn(o[i]);
  }
};

__global__ void __cluster_dims__(kQkvCL, 1, 1) __launch_bounds__((kQkvWarps + 1) * 32, 1)
qkv_kernel(const __grid_constant__ CUtensorMap mc, const __grid_constant__ CUtensorMap ms, const QkvArgs args) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* dtile = reinterpret_cast<float*>(smem + QkvL::ring_bytes);
  float* pslot = dtile + QkvL::ROWS * 8;                                           // (CL-1) partial tiles
  __half* xs = reinterpret_cast<__half*>(pslot + (kQkvCL - 1) * QkvL::ROWS * 8);   // f16 staged activations
  bf16* xnb = reinterpret_cast<bf16*>(xs + args.M * xs_stride(args.H));            // bf16 normalised hidden state
  float* sbuf = reinterpret_cast<float*>(xnb + args.M * args.H);                   // fp32 x + res
  __shared__ uint64_t bars[2 * kQkvStages];
  __shared__ uint64_t clbar;
  __shared__ int shift[8];
  __shared__ float red[kQkvWarps * 8];
  const unsigned rank = cluster_rank();
  if (threadIdx.x == 0) {
    for (int i = 0; i < kQkvStages; ++i) {
      mbar_init(&bars[i], 1);
      mbar_init(&bars[kQkvStages + i], kQkvWarps);
    }
    mbar_init(&clbar, kQkvCL - 1);
    fence_mbar_init();
  }
  __syncthreads();
  cluster_sync_all();
  const int head = blockIdx.x / kQkvCL;
  QkvPlan plan{&mc, &ms, xs, shift, &args, head, (int)rank, args.H / kSliceK / kQkvCL};
  if (threadIdx.x >= kQkvWarps * 32) {
    engine_produce<kQkvWarps, kQkvStages, kQkvBox>(plan, smem, bars, args.status);   // weights: before the PDL wait
    return;
  }
  pdl_wait();
  pdl_trigger();
  const bf16* xin = args.x;
  int64_t ldx = args.ldx;
  if (args.tokens) {                 // gather the (<= 8) embedding rows into a contiguous staging area first
    bf16* gxe = reinterpret_cast<bf16*>(xs);   // the f16 staging area is written only after the norm read it
    for (int idx = threadIdx.x; idx < args.M * (args.H / 8); idx += kQkvWarps * 32) {
      const int m = idx / (args.H / 8), k8 = idx - m * (args.H / 8);
      reinterpret_cast<uint4*>(gxe + m * args.H)[k8] =
          reinterpret_cast<const uint4*>(args.x + (int64_t)args.tokens[m] * args.ldx)[k8];
    }
    named_bar_sync(2, kQkvWarps * 32);
    xin = gxe;
    ldx = args.H;
  }
  add_rmsnorm_smem(xin, ldx, args.res, args.nw, args.eps, args.M, args.H, sbuf, xnb,
                   (head == 0 && rank == 0) ? args.res_out : nullptr, red, kQkvWarps * 32, 2);
  stage_rows_f16(xnb, args.H, args.M, args.H, xs, shift, red, kQkvWarps * 32, 2);
  engine_consume_cluster<kQkvWarps, kQkvStages, kQkvBox, kQkvCL>(plan, smem, dtile, pslot, &clbar, bars, args.status);
}

static size_t qkv_smem(int M, int H) {   // ring, dtile + partials, f16 x (or gathered rows), bf16 xn, fp32 scratch
  return 1024 + QkvL::ring_bytes + (size_t)kQkvCL * QkvL::ROWS * 8 * 4 + (size_t)M * xs_stride(H) * 2 + (size_t)M * H * 2 +
         (size_t)M * H * 4;
}

// ---- O projection ----
struct OArgs {
  const bf16* a;
  int64_t lda;
  const float* gs;
  int M, K, N;
  bf16* y;
  unsigned* status;
};

struct OPlan {
  const CUtensorMap* mc;
  const CUtensorMap* ms;
  const __half* xs;
  const int* shift;
  const OArgs* a;
  int tile, rank, nks_part;
  __device__ int ntiles() const { return 1; }
  __device__ int nks() const { return nks_part; }
  __device__ int kslice0(int) const { return rank * nks_part; }
  __device__ const CUtensorMap* map_codes() const { return mc; }
  __device__ const CUtensorMap* map_scales() const { return ms; }
  __device__ void box(int, int, int& y) const { y = tile * kOBox; }
  __device__ const __half* xrow(int, int n, bool& active) const {
    active = n < a->M;
    return xs + (active ? n : 0) * xs_stride(a->K);
  }
  __device__ void epilogue(int, const float* dt, int tid, int nthreads) {
    const OArgs& A = *a;
    for (int idx = tid; idx < kOBox * A.M; idx += nthreads) {
      const int m = idx / kOBox, r = idx - m * kOBox;
      A.y[(int64_t)m * A.N + tile * kOBox + r] = __float2bfloat16_rn(dt[r * 8 + m] * ldexpf(A.gs[0], -shift[m]));
    }
  }
};

__global__ void __cluster_dims__(kOCL, 1, 1) __launch_bounds__((kOWarps + 1) * 32, 1)
o_kernel(const __grid_constant__ CUtensorMap mc, const __grid_constant__ CUtensorMap ms, const OArgs args) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* dtile = reinterpret_cast<float*>(smem + OL::ring_bytes);
  float* pslot = dtile + OL::ROWS * 8;
  __half* xs = reinterpret_cast<__half*>(pslot + (kOCL - 1) * OL::ROWS * 8);
  __shared__ uint64_t bars[2 * kOStages];
  __shared__ uint64_t clbar;
  __shared__ int shift[8];
  __shared__ float red[8];
  const unsigned rank = cluster_rank();
  if (threadIdx.x == 0) {
    for (int i = 0; i < kOStages; ++i) {
      mbar_init(&bars[i], 1);
      mbar_init(&bars[kOStages + i], kOWarps);
    }
    mbar_init(&clbar, kOCL - 1);
    fence_mbar_init();
  }
  __syncthreads();
  cluster_sync_all();
  OPlan plan{&mc, &ms, xs, shift, &args, (int)(blockIdx.x / kOCL), (int)rank, args.K / kSliceK / kOCL};
  if (threadIdx.x >= kOWarps * 32) {
    engine_produce<kOWarps, kOStages, kOBox>(plan, smem, bars, args.status);
    return;
  }
  pdl_wait();
  pdl_trigger();
  stage_rows_f16(args.a, args.lda, args.M, args.K, xs, shift, red, kOWarps * 32, 2);
  engine_consume_cluster<kOWarps, kOStages, kOBox, kOCL>(plan, smem, dtile, pslot, &clbar, bars, args.status);
}

static size_t o_smem(int M, int K) { return 1024 + OL::ring_bytes + (size_t)kOCL * OL::ROWS * 8 * 4 + (size_t)M * xs_stride(K) * 2; }

}  // namespace flint

using namespace flint;

extern "C" int64_t flint_attn_proj_workspace_bytes(void) { return sizeof(ProjWorkspace); }
int64_t flint::status_offset_attn_proj() { return (int64_t)offsetof(ProjWorkspace, status); }

extern "C" int flint_attn_qkv(const void* x, int64_t ldx, const int32_t* tokens, const void* res, const void* norm_w, float eps, const void* W,
                              const void* S, const float* gs, int64_t M, int64_t H, int64_t N, int64_t num_q_heads,
                              int64_t num_kv_heads, int head_mode, const void* q_norm_w, const void* k_norm_w, float eps_head,
                              const int64_t* positions, const float* cos_sin, int64_t cos_sin_stride, void* k_cache,
                              void* v_cache, int64_t stride_block, int64_t stride_slot, int64_t stride_head,
                              int64_t block_size, const int64_t* slots, void* q_out, void* qkv_out, void* res_out,
                              void* workspace, int pdl, void* stream) {
  if (!x || !norm_w || !W || !S || !gs || !qkv_out || !workspace) return FLINT_ERR_ARGUMENT;
  if (tokens && res) return FLINT_ERR_ARGUMENT;
  if (M < 1 || M > 8 || H % kSliceK != 0 || (H / kSliceK) % kQkvCL != 0 || H > 8192 || ldx < H || ldx % 8 != 0 ||
      N != (num_q_heads + 2 * num_kv_heads) * kHeadDim || num_q_heads < 1 || num_kv_heads < 1)
    return FLINT_ERR_SHAPE;
  if (head_mode && (!q_norm_w || !k_norm_w || !q_out || !k_cache || !v_cache || !slots || block_size < 1 ||
                    (cos_sin && !positions)))
    return FLINT_ERR_ARGUMENT;
  if (!aligned(x, 16) || (res && !aligned(res, 16)) || !aligned(norm_w, 16) || !aligned(W, 16) || !aligned(S, 16))
    return FLINT_ERR_ALIGN;
  if (num_sms() <= 0) return FLINT_ERR_DEVICE;
  CUtensorMap mc, ms;
  int rc = encode_u8_2d(&mc, W, H / 2, N, H / 2, 128, kQkvBox, true);
  if (rc) return rc;
  rc = encode_u8_2d(&ms, S, H / 16, N, H / 16, 16, kQkvBox, false);
  if (rc) return rc;
  QkvArgs a;
  a.x = (const bf16*)x; a.ldx = ldx; a.tokens = (const int*)tokens; a.res = (const bf16*)res; a.nw = (const bf16*)norm_w; a.eps = eps; a.gs = gs;
  a.M = (int)M; a.H = (int)H; a.N = (int)N; a.nq = (int)num_q_heads; a.nkv = (int)num_kv_heads; a.head_mode = head_mode;
  a.q_w = (const bf16*)q_norm_w; a.k_w = (const bf16*)k_norm_w; a.eps_head = eps_head; a.positions = positions;
  a.cos_sin = cos_sin; a.cs_stride = cos_sin_stride; a.k_cache = (bf16*)k_cache; a.v_cache = (bf16*)v_cache;
  a.st_block = stride_block; a.st_slot = stride_slot; a.st_head = stride_head; a.block_size = (int)block_size;
  a.slots = slots; a.q_out = (bf16*)q_out; a.y_out = (bf16*)qkv_out; a.res_out = (bf16*)res_out;
  a.status = &static_cast<ProjWorkspace*>(workspace)->status;
  const size_t smem = qkv_smem((int)M, (int)H);
  if (smem > 227 * 1024) return FLINT_ERR_SHAPE;
  if (cudaFuncSetAttribute(qkv_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return FLINT_ERR_LAUNCH;
  const int heads = (int)(N / kHeadDim);
  return launch_cluster(qkv_kernel, dim3(heads * kQkvCL), dim3((kQkvWarps + 1) * 32), smem, stream, pdl, kQkvCL, mc, ms, a);
}

extern "C" int flint_attn_o(const void* a, int64_t lda, int64_t M, const void* W, const void* S, const float* gs, int64_t N,
                            int64_t K, void* y, void* workspace, int pdl, void* stream) {
  if (!a || !W || !S || !gs || !y || !workspace) return FLINT_ERR_ARGUMENT;
  if (M < 1 || M > 8 || K % kSliceK != 0 || (K / kSliceK) % kOCL != 0 || K > 16384 || N % kOBox != 0 || lda < K ||
      lda % 8 != 0)
    return FLINT_ERR_SHAPE;
  if (!aligned(a, 16) || !aligned(W, 16) || !aligned(S, 16)) return FLINT_ERR_ALIGN;
  if (num_sms() <= 0) return FLINT_ERR_DEVICE;
  CUtensorMap mc, ms;
  int rc = encode_u8_2d(&mc, W, K / 2, N, K / 2, 128, kOBox, true);
  if (rc) return rc;
  rc = encode_u8_2d(&ms, S, K / 16, N, K / 16, 16, kOBox, false);
  if (rc) return rc;
  OArgs o;
  o.a = (const bf16*)a; o.lda = lda; o.gs = gs; o.M = (int)M; o.K = (int)K; o.N = (int)N; o.y = (bf16*)y;
  o.status = &static_cast<ProjWorkspace*>(workspace)->status;
  const size_t smem = o_smem((int)M, (int)K);
  if (smem > 227 * 1024) return FLINT_ERR_SHAPE;
  if (cudaFuncSetAttribute(o_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return FLINT_ERR_LAUNCH;
  return launch_cluster(o_kernel, dim3((int)(N / kOBox) * kOCL), dim3((kOWarps + 1) * 32), smem, stream, pdl, kOCL, mc, ms, o);
}
