// (4) NVFP4 LM head: logits and the greedy argmax, or the seeded top-k -> top-p draw, in one pass over the head.
// Replaces the reference's Triton _nv4_fma / _nv4_head (fast/fast_head.py:68-121) and the pick of vLLM's sampler
// that follows compute_logits (fast/fast_head.py:360-381).  Kernel design: lm_head_kernel.cuh, sampling.cuh.
#include <atomic>
#include <cstddef>

#include "lm_head_kernel.cuh"
#include "runtime.cuh"

namespace flint {

constexpr int kHeadStages = 4;
constexpr int kHeadWarps = 16;
constexpr int kHeadRows = kHeadWarps * 16;

static size_t head_smem(int M, int K, bool norm) {
  return 1024 + (size_t)kHeadStages * StageGeom<kHeadRows>::bytes + (size_t)M * xs_stride(K) * 2 +
         (norm ? (size_t)M * K * 2 : 0);
}

}  // namespace flint

extern "C" int64_t flint_lm_head_workspace_bytes(void) { return sizeof(flint::HeadWorkspace); }
int64_t flint::status_offset_lm_head() { return (int64_t)offsetof(flint::HeadWorkspace, status); }

namespace flint {

// Argument, shape and alignment checks of the greedy head (everything but the workspace), shared by the entry
// points that take a workspace and the allocation-free one, which must refuse a call before it touches its scratch.
static int head_check_args(const void* x, int64_t ldx, const void* res, const void* norm_w, int64_t M, const void* P,
                           const void* S, int64_t V, int64_t K, const float* logits, int64_t ld_logits) {
  if (!x || !P || !S || (res && !norm_w)) return FLINT_ERR_ARGUMENT;
  if (M < 1 || M > 8 || V < 1 || V > (1ll << 30) || K < kSliceK || K % kSliceK != 0 || K > 8192 || ldx < K)
    return FLINT_ERR_SHAPE;
  if (logits && ld_logits < V) return FLINT_ERR_SHAPE;
  if (!aligned(P, 16) || !aligned(S, 16) || !aligned(x, 16) || ldx % 8 != 0 || (res && !aligned(res, 16)) ||
      (norm_w && !aligned(norm_w, 16)))
    return FLINT_ERR_ALIGN;
  return FLINT_OK;
}

}  // namespace flint

extern "C" int flint_lm_head_nv4_fused(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps, int64_t M,
                                       const void* P, const void* S, float gs, int64_t V, int64_t K, float* logits,
                                       int64_t ld_logits, int32_t* token_ids, void* workspace, int pdl, void* stream) {
  using namespace flint;
  const int arg_rc = head_check_args(x, ldx, res, norm_w, M, P, S, V, K, logits, ld_logits);
  if (arg_rc != FLINT_OK) return arg_rc;
  if (!workspace) return FLINT_ERR_WORKSPACE;
  if (!aligned(workspace, 8)) return FLINT_ERR_ALIGN;
  const int sms = num_sms();
  if (sms <= 0) return FLINT_ERR_DEVICE;
  CUtensorMap mc, ms;
  int rc = encode_u8_2d(&mc, P, K / 2, V, K / 2, 128, kHeadRows, true);
  if (rc) return rc;
  rc = encode_u8_2d(&ms, S, K / 16, V, K / 16, 16, kHeadRows, false);
  if (rc) return rc;
  auto kern = lm_head_kernel<kHeadStages, kHeadWarps, false>;
  const size_t smem = head_smem((int)M, (int)K, norm_w != nullptr);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return FLINT_ERR_LAUNCH;
  const int ngroups = (int)((V + kHeadRows - 1) / kHeadRows);
  const int grid = ngroups < sms ? ngroups : sms;
  return launch(kern, dim3(grid), dim3((kHeadWarps + 1) * 32), smem, stream, pdl, mc, ms, (const bf16*)x, ldx,
                (const bf16*)res, (const bf16*)norm_w, eps, (int)M, gs, (int)V, (int)K, logits, ld_logits, (int*)token_ids,
                (HeadWorkspace*)workspace, SampleParams{}, 0u, (unsigned long long*)nullptr);
}

// Vocabulary shard of the head (rows index_base .. index_base + V - 1 of the full vocabulary): the per-row argmax
// key (order-preserving value, then the lowest global id) of this shard goes to keys_out; the maximum of the keys
// over all shards (an integer MAX all-reduce) is the full-vocabulary argmax key (flint_argmax_keys_to_tokens).
extern "C" int flint_lm_head_nv4_shard(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps,
                                       int64_t M, const void* P, const void* S, float gs, int64_t V, int64_t K,
                                       int64_t index_base, uint64_t* keys_out, void* workspace, int pdl, void* stream) {
  using namespace flint;
  if (!x || !P || !S || (res && !norm_w) || !keys_out) return FLINT_ERR_ARGUMENT;
  if (M < 1 || M > 8 || V < 1 || V > (1ll << 30) || K < kSliceK || K % kSliceK != 0 || K > 8192 || ldx < K ||
      index_base < 0 || index_base + V > (1ll << 31))
    return FLINT_ERR_SHAPE;
  if (!aligned(P, 16) || !aligned(S, 16) || !aligned(x, 16) || ldx % 8 != 0 || (res && !aligned(res, 16)) ||
      (norm_w && !aligned(norm_w, 16)))
    return FLINT_ERR_ALIGN;
  if (!workspace) return FLINT_ERR_WORKSPACE;
  if (!aligned(workspace, 8)) return FLINT_ERR_ALIGN;
  const int sms = num_sms();
  if (sms <= 0) return FLINT_ERR_DEVICE;
  CUtensorMap mc, ms;
  int rc = encode_u8_2d(&mc, P, K / 2, V, K / 2, 128, kHeadRows, true);
  if (rc) return rc;
  rc = encode_u8_2d(&ms, S, K / 16, V, K / 16, 16, kHeadRows, false);
  if (rc) return rc;
  auto kern = lm_head_kernel<kHeadStages, kHeadWarps, false>;
  const size_t smem = head_smem((int)M, (int)K, norm_w != nullptr);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return FLINT_ERR_LAUNCH;
  const int ngroups = (int)((V + kHeadRows - 1) / kHeadRows);
  const int grid = ngroups < sms ? ngroups : sms;
  return launch(kern, dim3(grid), dim3((kHeadWarps + 1) * 32), smem, stream, pdl, mc, ms, (const bf16*)x, ldx,
                (const bf16*)res, (const bf16*)norm_w, eps, (int)M, gs, (int)V, (int)K, (float*)nullptr, (int64_t)0,
                (int*)nullptr, (HeadWorkspace*)workspace, SampleParams{}, (uint32_t)index_base,
                reinterpret_cast<unsigned long long*>(keys_out));
}

namespace flint {

static size_t sample_cand_bytes() { return (size_t)8 * kSampleMaxCtas * kSampleMaxK * 8; }
static size_t sample_logits_offset() { return (sizeof(HeadWorkspace) + sample_cand_bytes() + 255) & ~size_t(255); }

}  // namespace flint

extern "C" int64_t flint_lm_head_sample_workspace_bytes(int64_t M, int64_t V) {
  using namespace flint;
  if (M < 1 || M > 8 || V < 1) return -1;
  return (int64_t)(sample_logits_offset() + (size_t)M * (size_t)V * 4);
}

static int lm_head_sample_launch(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps, int64_t M,
                                 const void* P, const void* S, float gs, int64_t V, int64_t K, float* logits,
                                 int64_t ld_logits, float temperature, int64_t top_k, float top_p, const uint64_t* seeds,
                                 const int32_t* step, int32_t* token_ids, int32_t* cand_ids, float* cand_logits,
                                 int32_t* kept, void* workspace, int pdl, void* stream, int64_t id_base) {
  using namespace flint;
  if (!x || !P || !S || (res && !norm_w) || !token_ids) return FLINT_ERR_ARGUMENT;
  if (!(temperature > 0.f) || !(temperature < INFINITY) || !(top_p > 0.f) || !(top_p <= 1.f)) return FLINT_ERR_ARGUMENT;
  if (M < 1 || M > 8 || V < 1 || V > (1ll << 30) || K < kSliceK || K % kSliceK != 0 || K > 8192 || ldx < K)
    return FLINT_ERR_SHAPE;
  if (top_k < 1 || top_k > kSampleMaxK || top_k > V) return FLINT_ERR_ARGUMENT;
  if (id_base < 0 || id_base + V > (1ll << 31)) return FLINT_ERR_ARGUMENT;
  if (logits && ld_logits < V) return FLINT_ERR_SHAPE;
  if (!aligned(P, 16) || !aligned(S, 16) || !aligned(x, 16) || ldx % 8 != 0 || (res && !aligned(res, 16)) ||
      (norm_w && !aligned(norm_w, 16)) || (logits && !aligned(logits, 4)))
    return FLINT_ERR_ALIGN;
  if (!workspace) return FLINT_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return FLINT_ERR_ALIGN;
  const int sms = num_sms();
  if (sms <= 0) return FLINT_ERR_DEVICE;
  CUtensorMap mc, ms;
  int rc = encode_u8_2d(&mc, P, K / 2, V, K / 2, 128, kHeadRows, true);
  if (rc) return rc;
  rc = encode_u8_2d(&ms, S, K / 16, V, K / 16, 16, kHeadRows, false);
  if (rc) return rc;
  auto kern = lm_head_kernel<kHeadStages, kHeadWarps, true>;
  const size_t smem = head_smem((int)M, (int)K, norm_w != nullptr);
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return FLINT_ERR_LAUNCH;
  const int ngroups = (int)((V + kHeadRows - 1) / kHeadRows);
  int grid = ngroups < sms ? ngroups : sms;
  if (grid > kSampleMaxCtas) grid = kSampleMaxCtas;
  uint8_t* wsb = static_cast<uint8_t*>(workspace);
  SampleParams sp;
  sp.temperature = temperature;
  sp.top_p = top_p;
  sp.top_k = (int)top_k;
  sp.seeds = reinterpret_cast<const unsigned long long*>(seeds);
  sp.step = step;
  sp.cand = reinterpret_cast<unsigned long long*>(wsb + sizeof(HeadWorkspace));
  sp.cand_ids = cand_ids;
  sp.cand_logits = cand_logits;
  sp.kept = kept;
  sp.id_base = (unsigned)id_base;
  float* lg = logits ? logits : reinterpret_cast<float*>(wsb + sample_logits_offset());
  const int64_t ldl = logits ? ld_logits : V;
  return launch(kern, dim3(grid), dim3((kHeadWarps + 1) * 32), smem, stream, pdl, mc, ms, (const bf16*)x, ldx,
                (const bf16*)res, (const bf16*)norm_w, eps, (int)M, gs, (int)V, (int)K, lg, ldl, (int*)token_ids,
                (HeadWorkspace*)workspace, sp, 0u, (unsigned long long*)nullptr);
}

namespace flint {

// Sampled decoding over vocabulary shards: cand_ids / cand_logits [R][M][K] hold each shard's sorted top K (global
// ids, -1 padding).  One warp per row re-selects the top K of their union by (logit desc, id asc) -- the global top
// K, since every entry of the global top K is in its shard's top K -- and applies the sampling rule of
// flint_lm_head_nv4_sample with the same uniform, so the token is the one-GPU token.
__global__ void sample_merge_kernel(const int* __restrict__ cand_ids, const float* __restrict__ cand_logits, int R, int M,
                                    int K, float temperature, float top_p, const unsigned long long* __restrict__ seeds,
                                    const int* step, int* tokens, int* kept_out) {
  __shared__ unsigned long long buf[8][8 * kSampleMaxK];
  __shared__ unsigned long long top[8][kSampleMaxK];
  __shared__ float w[8][kSampleMaxK];
  pdl_wait();
  const int lane = threadIdx.x & 31, m = threadIdx.x >> 5;
  if (m < M) {
    const int n = R * K;
    for (int i = lane; i < n; i += 32) {
      const int r = i / K, k = i - r * K;
      const int64_t at = ((int64_t)r * M + m) * K + k;
      const int id = cand_ids[at];
      buf[m][i] = id >= 0 ? argmax_key(cand_logits[at], (uint32_t)id) : 0ull;
    }
    __syncwarp();
    warp_select_sorted(buf[m], n, K, top[m], lane);
    const int st = step ? *step : 0;
    const float u = sample_uniform(seeds[m], (uint32_t)st, (uint32_t)m);
    int kept = 1;
    const int pick = sample_sorted(top[m], K, temperature, top_p, u, w[m], lane, &kept);
    if (lane == 0) {
      tokens[m] = (int)argmax_key_index(top[m][pick]);
      if (kept_out) kept_out[m] = kept;
    }
  }
  pdl_trigger();
}

}  // namespace flint

extern "C" int flint_sample_merge(const int32_t* cand_ids, const float* cand_logits, int64_t R, int64_t M, int64_t top_k,
                                  float temperature, float top_p, const uint64_t* seeds, const int32_t* step,
                                  int32_t* token_ids, int32_t* kept, int pdl, void* stream) {
  using namespace flint;
  if (!cand_ids || !cand_logits || !seeds || !token_ids) return FLINT_ERR_ARGUMENT;
  if (!(temperature > 0.f) || !(temperature < INFINITY) || !(top_p > 0.f) || !(top_p <= 1.f)) return FLINT_ERR_ARGUMENT;
  if (R < 1 || R > 8 || M < 1 || M > 8 || top_k < 1 || top_k > kSampleMaxK) return FLINT_ERR_SHAPE;
  return launch(sample_merge_kernel, dim3(1), dim3((unsigned)(32 * M)), 0, stream, pdl, cand_ids, cand_logits, (int)R,
                (int)M, (int)top_k, temperature, top_p, reinterpret_cast<const unsigned long long*>(seeds), step,
                (int*)token_ids, (int*)kept);
}

extern "C" int flint_lm_head_nv4_sample(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps,
                                        int64_t M, const void* P, const void* S, float gs, int64_t V, int64_t K,
                                        float* logits, int64_t ld_logits, float temperature, int64_t top_k, float top_p,
                                        const uint64_t* seeds, const int32_t* step, int32_t* token_ids, int32_t* cand_ids,
                                        float* cand_logits, int32_t* kept, void* workspace, int pdl, void* stream) {
  if (!seeds) return FLINT_ERR_ARGUMENT;
  return lm_head_sample_launch(x, ldx, res, norm_w, eps, M, P, S, gs, V, K, logits, ld_logits, temperature, top_k, top_p,
                               seeds, step, token_ids, cand_ids, cand_logits, kept, workspace, pdl, stream, 0);
}

extern "C" int flint_lm_head_nv4_sample_shard(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps,
                                              int64_t M, const void* P, const void* S, float gs, int64_t V, int64_t K,
                                              int64_t index_base, int64_t top_k, int32_t* cand_ids, float* cand_logits,
                                              int32_t* scratch_tokens, void* workspace, int pdl, void* stream) {
  if (!cand_ids || !cand_logits || !scratch_tokens) return FLINT_ERR_ARGUMENT;
  // the shard's own draw (seed 0, step 0) is discarded; its sorted candidates are the output
  return lm_head_sample_launch(x, ldx, res, norm_w, eps, M, P, S, gs, V, K, nullptr, 0, 1.0f, top_k, 1.0f, nullptr,
                               nullptr, scratch_tokens, cand_ids, cand_logits, nullptr, workspace, pdl, stream, index_base);
}

extern "C" int flint_lm_head_nv4(const void* x, int64_t ldx, int64_t M, const void* P, const void* S, float gs, int64_t V,
                                 int64_t K, float* logits, int64_t ld_logits, int32_t* token_ids, void* workspace, int pdl,
                                 void* stream) {
  return flint_lm_head_nv4_fused(x, ldx, nullptr, nullptr, 0.f, M, P, S, gs, V, K, logits, ld_logits, token_ids, workspace,
                                 pdl, stream);
}

// -------------------------------------------------------------------------------------------------------------------
// Allocation-free variant of flint_lm_head_nv4.
//
// Some callers cannot allocate device memory when they call the head: an inference engine that has handed all free
// HBM to its KV-cache pool up front (a cudaMalloc then fails or evicts cache pages), or a host runtime that reaches
// this library only through a C FFI and owns no CUDA allocator of its own.  For them the argmax scratch (the per-row
// best keys, the CTA arrival counter and the status word) lives in the file-scope array below, one copy per device,
// held by every GPU that loads the library until the process exits.  The caller still provides x, the weights and
// the outputs.
//
// Limits: at most kNoAllocMaxRows = 8 rows per call (the scratch holds 8 argmax slots; larger requests are refused
// with FLINT_ERR_SCRATCH).  Every call uses the same scratch and it keeps the last call's contents: each call clears
// the argmax slots and the counter before its kernel, but not the status word, which stays set until
// flint_lm_head_noalloc_status clears it.  Calls that overlap on the GPU (different streams on one device) race on
// the scratch, so issue them in one stream per device.  A call the argument checks refuse enqueues nothing.  The
// first call on a device looks up the array's device address (cudaGetSymbolAddress with that device current); make
// that first call before any stream capture.
// -------------------------------------------------------------------------------------------------------------------
namespace flint {

constexpr int kNoAllocMaxRows = 8;
constexpr int kNoAllocMaxDevices = 64;
static __device__ __align__(256) unsigned char g_head_noalloc_scratch[256];
static_assert(sizeof(HeadWorkspace) <= sizeof(g_head_noalloc_scratch), "scratch too small for the argmax workspace");
static std::atomic<void*> g_head_noalloc_ptr[kNoAllocMaxDevices];

// Device address of this device's copy of the scratch array (host code cannot use the symbol itself: on the host it
// names a stand-in, not device memory).  Racing first calls from several host threads store the same value.
static void* head_noalloc_scratch() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kNoAllocMaxDevices) return nullptr;
  void* p = g_head_noalloc_ptr[dev].load(std::memory_order_acquire);
  if (p == nullptr) {
    if (cudaGetSymbolAddress(&p, g_head_noalloc_scratch) != cudaSuccess) return nullptr;
    g_head_noalloc_ptr[dev].store(p, std::memory_order_release);
  }
  return p;
}

}  // namespace flint

extern "C" int flint_lm_head_nv4_noalloc(const void* x, int64_t ldx, int64_t M, const void* P, const void* S, float gs,
                                         int64_t V, int64_t K, float* logits, int64_t ld_logits, int32_t* token_ids,
                                         int pdl, void* stream) {
  using namespace flint;
  if (M > kNoAllocMaxRows) return FLINT_ERR_SCRATCH;
  const int arg_rc = head_check_args(x, ldx, nullptr, nullptr, M, P, S, V, K, logits, ld_logits);
  if (arg_rc != FLINT_OK) return arg_rc;                 // refused before anything is enqueued
  if (num_sms() <= 0) return FLINT_ERR_DEVICE;
  void* scratch = head_noalloc_scratch();
  if (scratch == nullptr) return FLINT_ERR_DEVICE;
  // clear the argmax slots and the arrival counter; the status word (after them) keeps any earlier time-out
  if (cudaMemsetAsync(scratch, 0, offsetof(HeadWorkspace, status), static_cast<cudaStream_t>(stream)) != cudaSuccess)
    return FLINT_ERR_LAUNCH;
  return flint_lm_head_nv4(x, ldx, M, P, S, gs, V, K, logits, ld_logits, token_ids, scratch, pdl, stream);
}

extern "C" int flint_lm_head_noalloc_status(uint32_t* status, int clear) {
  using namespace flint;
  if (!status) return FLINT_ERR_ARGUMENT;
  void* scratch = head_noalloc_scratch();
  if (scratch == nullptr) return FLINT_ERR_DEVICE;
  uint8_t* word = static_cast<uint8_t*>(scratch) + offsetof(HeadWorkspace, status);
  // a blocking copy: it waits for the head launches already issued on this device
  if (cudaMemcpy(status, word, sizeof(uint32_t), cudaMemcpyDeviceToHost) != cudaSuccess) return FLINT_ERR_LAUNCH;
  if (clear && cudaMemset(word, 0, sizeof(uint32_t)) != cudaSuccess) return FLINT_ERR_LAUNCH;
  return FLINT_OK;
}
