/*
 * flint_b200.h -- C ABI of the B200 (sm_100a) NVFP4 batch-1 decode kernels.
 *
 * Every compute entry point takes plain device pointers, sizes and a cudaStream_t passed as void*, launches
 * asynchronously on that stream and returns FLINT_OK or one of the FLINT_ERR_* codes below; none of them
 * aborts, allocates device memory or synchronises the stream.  The exceptions are marked where declared:
 * the peer-buffer management (flint_peer_alloc / open / close / free / status) and flint_workspace_status.
 * The header is plain C99.
 *
 * NVFP4 tensors use the ModelOpt layout the reference loads (patches/flint-vllm-pr62938.patch,
 * gguf_nvfp4.py, patch:269-319): codes uint8 [N, K/2] with the even k in the low nibble, block scales
 * E4M3 [N, K/16], one fp32 global scale per tensor (per expert for stacked experts).
 *
 * "workspace" arguments are caller-owned device buffers of the size the matching *_workspace_bytes()
 * function returns.  They must be zero-filled once before first use; every kernel leaves them zeroed
 * again (arrival counters reset themselves), so one workspace serves any number of launches that are
 * ordered on one stream.  Launches that share a workspace must not overlap on the GPU.
 *
 * "pdl" != 0 launches with programmatic dependent launch: the kernel prefetches its weights before
 * waiting on the previous kernel in the stream.
 */
#ifndef FLINT_B200_H_
#define FLINT_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  FLINT_OK = 0,
  FLINT_ERR_SHAPE = 1,        /* unsupported or inconsistent sizes */
  FLINT_ERR_ALIGN = 2,        /* pointer or stride not aligned as required (16 B for weight rows) */
  FLINT_ERR_DEVICE = 3,       /* no CUDA device / not sm_100 */
  FLINT_ERR_LAUNCH = 4,       /* cudaLaunchKernelEx failed (the CUDA error is left for cudaGetLastError) */
  FLINT_ERR_WORKSPACE = 5,    /* workspace missing or too small */
  FLINT_ERR_ARGUMENT = 6,     /* null pointer or out-of-range scalar argument */
  FLINT_ERR_SCRATCH = 7       /* request larger than the fixed scratch of an allocation-free entry point */
};

/* L2 prefetch hint: up to 8 device byte ranges (16-byte aligned; a tail below 16 bytes is skipped) that a kernel
 * taking one prefetches into L2 for the op that follows it -- in a decode step, the next layer's weights, whose
 * loads otherwise start only when the next kernel's blocks become resident -- plus, when kv is not NULL, the pages
 * of a paged KV cache that the next attention will read: blocks block_tables[b * bt_stride + p] for
 * p < min(ceil(seq_lens[b] / block_tokens), bt_cols), b < streams, each block_bytes long at kv + block * block_bytes
 * (blocks outside [0, kv_blocks) are skipped), at most max_blocks blocks in all.  Pure hint: no effect on results. */
typedef struct flint_l2_prefetch {
  const void* ptr[8];
  int64_t bytes[8];
  int32_t n;
  const void* kv;
  int64_t block_bytes;
  int64_t kv_blocks;
  const int32_t* block_tables;
  int64_t bt_stride;
  int64_t bt_cols;
  const int32_t* seq_lens;
  int32_t streams;
  int32_t block_tokens;
  int32_t max_blocks;
} flint_l2_prefetch;

/* Library version (major*10000 + minor*100 + patch). */
int flint_version(void);
/* Human-readable name of an error code. */
const char* flint_error_string(int code);
/* "cudaErrorName: description" of the last CUDA runtime call of this library that failed on the calling host thread
 * (the detail behind FLINT_ERR_LAUNCH / FLINT_ERR_DEVICE), or "" if none has. */
const char* flint_last_cuda_error(void);

/* Device-side health.  Every kernel that waits (on an mbarrier, a grid barrier, another CTA's published words) waits
 * for a bounded time and never traps; what went wrong is OR-ed into a sticky status word in its workspace, and the
 * launch returns.  The host reads it between steps.  Workspace kinds (the workspace passed to the entry points of
 * that family) and status bits: */
enum {
  FLINT_WS_LM_HEAD = 0,           /* flint_lm_head_* (plain and sampling workspaces) */
  FLINT_WS_MOE = 1,               /* flint_moe_route / up / down (+ _ep) */
  FLINT_WS_MOE_FUSED = 2,         /* flint_moe_fused */
  FLINT_WS_MOE_BLOCK = 3,         /* flint_moe_block (+ _ep, _peer) */
  FLINT_WS_ATTN_PROJ = 4,         /* flint_attn_qkv, flint_attn_o */
  FLINT_WS_ATTN_BLOCK = 5,        /* flint_attn_block */
  FLINT_WS_DECODE_ATTENTION = 6   /* flint_decode_attention */
};
enum {
  FLINT_STATUS_WAIT_TIMEOUT = 1,  /* a bounded wait gave up: that launch's outputs are invalid */
  FLINT_STATUS_BAD_EXPERT = 2,    /* a routed expert id outside 0..E-1 (clamped) */
  FLINT_STATUS_BAD_SEQUENCE = 4   /* a sequence longer than its block table (clamped to the table) */
};
/* Byte offset of the status word inside a workspace of `kind`, or -1 for an unknown kind (no GPU needed). */
int64_t flint_workspace_status_offset(int kind);
/* Reads the status word of `workspace` (synchronous device-to-host copy); clear != 0 also zeroes a non-zero word. */
int flint_workspace_status(const void* workspace, int kind, uint32_t* status, int clear);

/* ------------------------------------------------------------------------------------------------
 * (4) NVFP4 LM head.
 * Replaces fast/fast_head.py: FastHead.__call__ (lines 200-207) -> nv4_logits_fma (118-121) /
 * nv4_logits (124-129) -> Triton _nv4_fma / _nv4_head (95-115 / 68-90), plus the greedy pick of the
 * external vLLM sampler.
 *
 *   logits[m, v] = gs * sum_k x[m, k] * e2m1(P[v, k]) * e4m3(S[v, k/16])      (fp32)
 *   token_ids[m] = argmax_v logits[m, v]   (lowest v on ties)
 *
 * x bf16 [M, K] row stride ldx elements (M in 1..8); P u8 [V, K/2]; S E4M3 [V, K/16]; K % 128 == 0.
 * logits: fp32 [M, V] row stride ld_logits, or NULL to skip writing them.
 * token_ids: int32 [M] or NULL to skip the argmax.  workspace: flint_lm_head_workspace_bytes().
 * ------------------------------------------------------------------------------------------------ */
int64_t flint_lm_head_workspace_bytes(void);
int flint_lm_head_nv4(const void* x, int64_t ldx, int64_t M, const void* P, const void* S, float gs, int64_t V,
                      int64_t K, float* logits, int64_t ld_logits, int32_t* token_ids, void* workspace, int pdl,
                      void* stream);
/* Same, with the model's final (residual add +) RMSNorm fused in front: x <- bf16((x + res) *
 * rsqrt(mean((x + res)^2) + eps) * norm_w) (res may be NULL; norm_w NULL = flint_lm_head_nv4).  The
 * reference applies model.norm before compute_logits (fast/model.py:831,924-929). */
int flint_lm_head_nv4_fused(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps, int64_t M,
                            const void* P, const void* S, float gs, int64_t V, int64_t K, float* logits,
                            int64_t ld_logits, int32_t* token_ids, void* workspace, int pdl, void* stream);
/* Sampled decoding in the same pass (replaces vLLM's temperature -> top-k -> top-p -> draw that follows the
 * reference's compute_logits, fast/fast_head.py:360-381; the reference's draw is not reproducible, so the rule is
 * this library's own and seeded):
 *   candidates c_0 >= ... >= c_{k-1}: the top_k logits (ties -> lowest id), 1 <= top_k <= 32;
 *   w_i = expf((c_i - c_0) / temperature);  S_j = w_{k-1} + ... + w_j;  candidate j >= 1 survives top-p iff
 *   S_j > (1 - top_p) * S_0 (vLLM's rule: drop while the ascending cumulative probability is <= 1 - top_p);
 *   u = Philox4x32-10(counter {*step, m, 0, 0}, key seeds[m]).x >> 8, times 2^-24;
 *   token_ids[m] = id of the first kept i with w_0 + ... + w_i > u * (sum of the kept w).
 * temperature > 0 (greedy callers use flint_lm_head_nv4_fused); 0 < top_p <= 1.  seeds: uint64 [M] (device);
 * step: int32 device counter read at launch (NULL = 0), so a captured graph draws afresh after the counter moves.
 * logits: fp32 [M, V] output or NULL (then kept in the workspace).  cand_ids / cand_logits: optional [M, top_k]
 * outputs of the sorted candidates; kept: optional [M] count after top-p.
 * workspace: flint_lm_head_sample_workspace_bytes(M, V), 256-byte aligned, zeroed once. */
int64_t flint_lm_head_sample_workspace_bytes(int64_t M, int64_t V);
int flint_lm_head_nv4_sample(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps, int64_t M,
                             const void* P, const void* S, float gs, int64_t V, int64_t K, float* logits,
                             int64_t ld_logits, float temperature, int64_t top_k, float top_p, const uint64_t* seeds,
                             const int32_t* step, int32_t* token_ids, int32_t* cand_ids, float* cand_logits,
                             int32_t* kept, void* workspace, int pdl, void* stream);
/* One vocabulary shard of the head, for a head split over ranks: P / S hold rows index_base .. index_base + V - 1
 * of the full vocabulary; keys_out int64 [M] receives each row's best (value, lowest global id) argmax key
 * ((order-preserving fp32 image << 32 | (0xFFFFFFFF - id)) with the top bit flipped, so signed comparison orders it).
 * The maximum over all shards (a signed int64 MAX all-reduce) is the full-vocabulary key; flint_argmax_keys_to_tokens turns keys into token ids.  Optional fused final norm as
 * flint_lm_head_nv4_fused.  workspace: flint_lm_head_workspace_bytes(). */
int flint_lm_head_nv4_shard(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps, int64_t M,
                            const void* P, const void* S, float gs, int64_t V, int64_t K, int64_t index_base,
                            uint64_t* keys_out, void* workspace, int pdl, void* stream);
/* tokens[m] = the id carried by argmax key keys[m] (M <= 1024). */
int flint_argmax_keys_to_tokens(const uint64_t* keys, int64_t M, int32_t* tokens, int pdl, void* stream);
/* Sampled decoding over a head split over R ranks (vocabulary shards).  Each rank:
 * flint_lm_head_nv4_sample_shard -> its shard's top_k candidates, sorted by (logit desc, id asc), global ids
 * (index_base + row) in cand_ids int32 [M, top_k] and logits in cand_logits fp32 [M, top_k]; scratch_tokens int32 [M]
 * receives a discarded draw; workspace as flint_lm_head_sample_workspace_bytes(M, V).  After gathering every rank's
 * candidates into [R][M][top_k], flint_sample_merge re-selects the top_k of their union and draws with the rule and
 * uniform of flint_lm_head_nv4_sample: the same token as one GPU over the whole vocabulary.  R <= 8, M <= 8. */
int flint_lm_head_nv4_sample_shard(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps, int64_t M,
                                   const void* P, const void* S, float gs, int64_t V, int64_t K, int64_t index_base,
                                   int64_t top_k, int32_t* cand_ids, float* cand_logits, int32_t* scratch_tokens,
                                   void* workspace, int pdl, void* stream);
int flint_sample_merge(const int32_t* cand_ids, const float* cand_logits, int64_t R, int64_t M, int64_t top_k,
                       float temperature, float top_p, const uint64_t* seeds, const int32_t* step, int32_t* token_ids,
                       int32_t* kept, int pdl, void* stream);
/* Allocation-free flint_lm_head_nv4 (no counterpart in the reference: the recipe always runs inside vLLM, which
 * allocates).  For callers that cannot allocate device memory at call time -- an engine that has already given all
 * free HBM to its KV-cache pool, a host runtime that only reaches the library through a C FFI and has no CUDA
 * allocator -- the argmax scratch is a fixed 256-byte array inside the library, one per device, kept until the
 * process exits; no workspace argument.  At most 8 rows (M <= 8); larger requests return FLINT_ERR_SCRATCH, and
 * every other refused call returns its error code before anything is enqueued.  Each call clears the argmax slots
 * first but keeps the scratch's status word, read (and cleared) by flint_lm_head_noalloc_status; calls that overlap
 * on one GPU race on the scratch (use one stream per device).  The first call on a device resolves the scratch
 * address (cudaGetSymbolAddress), so make it before any stream capture. */
int flint_lm_head_nv4_noalloc(const void* x, int64_t ldx, int64_t M, const void* P, const void* S, float gs, int64_t V,
                              int64_t K, float* logits, int64_t ld_logits, int32_t* token_ids, int pdl, void* stream);
/* Status word of the current device's allocation-free head scratch (FLINT_STATUS_* bits, e.g. a bounded wait that
 * gave up), after the launches already issued on that device (a blocking read); clear != 0 resets it. */
int flint_lm_head_noalloc_status(uint32_t* status, int clear);

/* ------------------------------------------------------------------------------------------------
 * (1) MoE decode, 1..8 tokens.  Replaces fast/fp4moe_mar.cu (route_kernel 243-303, route_norm_kernel
 * 311-417, up_mar 67-152, down_mar 157-233) behind fast/fp4moe_decode.py route / route_norm / moe_up /
 * moe_down (lines 61-95), for any expert count / top-k / sizes (the reference hard-codes E=256, k=6).
 * One workspace of flint_moe_workspace_bytes(H) serves all three kernels of a layer (and every layer,
 * launches being stream ordered).
 * ------------------------------------------------------------------------------------------------ */
int64_t flint_moe_workspace_bytes(int64_t H);

/* Router with the (residual add +) RMSNorm fused in (fp4moe_mar.cu:311-417 / fp4moe_decode.py:61-79):
 *   s = x + res (res may be NULL), res_out = bf16(s) (NULL to skip), xn = bf16(s * rsqrt(mean(s^2)+eps) * w)
 *   (norm_w NULL: xn = bf16(s), no norm), logits[m, e] = bf16(xn[m] . gate_w[e]) stored as fp32,
 *   top-k on the logits (score_fn 0 = softmax) or sigmoid scores (score_fn 1), ties -> lowest expert,
 *   weights renormalised over the chosen experts.
 * x, res, xn_out, res_out bf16 [M, H] (row stride ldx for x/res, H for outputs); gate_w bf16 [E, H];
 * logits fp32 [M, E]; topk_ids int32 [M, topk]; topk_weights fp32 [M, topk].  H in {2048, 4096},
 * E % 32 == 0, E <= 512, M <= 8, M * topk <= 64. */
int flint_moe_route(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps, const void* gate_w,
                    int64_t M, int64_t H, int64_t E, int64_t topk, int score_fn, float* logits, int32_t* topk_ids,
                    float* topk_weights, void* xn_out, void* res_out, void* workspace, int pdl, void* stream);

/* Expert gate/up GEMV + SwiGLU (fp4moe_mar.cu:67-152):  act[m*topk+s, :] = bf16(silu(g) * u) with
 * g, u = xn[m] . W13[e, 0:I] * gs13[e], xn[m] . W13[e, I:2I] * gs13[e], e = topk_ids[m, s].
 * xn bf16 [M, H] (stride ldx); w13 u8 [E, 2I, H/2]; s13 E4M3 [E, 2I, H/16]; g13 fp32 [E]; act bf16 [M*topk, I]. */
int flint_moe_up(const void* xn, int64_t ldx, int64_t M, const int32_t* topk_ids, int64_t topk, const void* w13,
                 const void* s13, const float* g13, int64_t E, int64_t I, int64_t H, void* act, void* workspace, int pdl,
                 void* stream);

/* Expert down GEMV + weighted sum (fp4moe_mar.cu:157-233):  y = bf16(act[r] . W2[e] * gs2[e]) per route,
 * out[m] = bf16(sum_s topk_weights[m, s] * y[m*topk+s]) (slot order, fp32).
 * act bf16 [M*topk, I]; w2 u8 [E, H, I/2]; s2 E4M3 [E, H, I/16]; g2 fp32 [E]; out bf16 [M, H]. */
int flint_moe_down(const void* act, int64_t M, const int32_t* topk_ids, const float* topk_weights, int64_t topk,
                   const void* w2, const void* s2, const float* g2, int64_t E, int64_t I, int64_t H, void* out,
                   void* workspace, int pdl, void* stream);

/* The whole decode MoE block in ONE persistent launch (one CTA per SM, three grid barriers): router
 * (+ residual add + RMSNorm) -> top-k -> gate/up GEMV + SwiGLU -> down GEMV -> weighted sum, the three-kernel
 * chain route_norm / moe_up / moe_down (fast/fp4moe_decode.py:70-95, fast/model.py:302-310) fused, with the same
 * numerics and routing as flint_moe_route / flint_moe_up / flint_moe_down above.  out bf16 [M, H]; res_out,
 * xn_out, logits_out, topk_ids_out, topk_weights_out optional (NULL).  H in {2048, 4096}, E % 32 == 0,
 * E <= 2 * SMs, I % 256 == 0, M <= 8.  workspace: flint_moe_fused_workspace_bytes(E, H, I), zeroed once. */
int64_t flint_moe_fused_workspace_bytes(int64_t E, int64_t H, int64_t I);
int flint_moe_fused(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps, const void* gate_w,
                    int64_t M, int64_t H, int64_t E, int64_t topk, int score_fn, const void* w13, const void* s13,
                    const float* g13, const void* w2, const void* s2, const float* g2, int64_t I, void* out,
                    void* res_out, void* xn_out, float* logits_out, int32_t* topk_ids_out, float* topk_weights_out,
                    void* workspace, int pdl, void* stream);

/* Expert-parallel flint_moe_fused (1..8 tokens in one launch): the weights hold experts expert_lo .. expert_lo +
 * n_local - 1 (indexed by local expert); the router and top-k run in full (identical on every rank) and only routes
 * whose expert is local get tiles.  Writes y_out bf16 [M * topk, H] (row m * topk + s = y of route (m, s) when its
 * expert is local, zeros otherwise; the rows of flint_moe_down_ep), res_out, logits / ids / weights as
 * flint_moe_fused.  A sum of y_out over the ranks (one non-zero term per element) and flint_moe_combine give the
 * one-GPU output bit for bit.  Workspace: flint_moe_fused_workspace_bytes(E, H, I). */
int flint_moe_fused_ep(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps, const void* gate_w,
                       int64_t M, int64_t H, int64_t E, int64_t topk, int score_fn, const void* w13, const void* s13,
                       const float* g13, const void* w2, const void* s2, const float* g2, int64_t I, int64_t expert_lo,
                       int64_t n_local, void* y_out, void* res_out, float* logits_out, int32_t* topk_ids_out,
                       float* topk_weights_out, void* workspace, int pdl, void* stream);

/* The decode MoE block for ONE token in one cooperative launch (router + top-k -> gate/up + SwiGLU -> down ->
 * weighted sum, two grid barriers): each CTA loads its share of the gate/up rows and its 16 output rows of every
 * routed expert's down matrix as soon as the routing is known, so the down weights stream in under the gate/up
 * work and the weighted sum needs no cross-CTA reduction.  Same arguments and outputs as flint_moe_fused at M = 1;
 * routing, xn, res_out and the down step have the bits of flint_moe_route / flint_moe_down, act matches
 * flint_moe_up to fp32 rounding.  H = 2048, E % 32 == 0, E <= 2 * SMs, topk <= 8, I % 256 == 0,
 * topk * I / 16 <= 3 * SMs.  workspace: flint_moe_block_workspace_bytes(E, I), zero-filled once, 256-byte aligned.
 * next: optional L2 prefetch (NULL: none), issued once the expert weights are requested (HBM is idle after that). */
int64_t flint_moe_block_workspace_bytes(int64_t E, int64_t I);
int flint_moe_block(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps, const void* gate_w,
                    int64_t H, int64_t E, int64_t topk, int score_fn, const void* w13, const void* s13, const float* g13,
                    const void* w2, const void* s2, const float* g2, int64_t I, void* out, void* res_out, void* xn_out,
                    float* logits_out, int32_t* topk_ids_out, float* topk_weights_out, void* workspace,
                    const flint_l2_prefetch* next, int pdl, void* stream);

/* flint_moe_block with Flint's ungated shared expert in the same launch (replaces the shared groups of the
 * reference's up_mar / down_mar, fast/fp4moe_mar.cu:67-152, 224-231): shared gate/up sh_w13 u8 [2 SI, H/2] (gate rows
 * first) + sh_s13 [2 SI, H/16] + sh_g13 fp32 [1], down sh_w2 u8 [H, SI/2] + sh_s2 [H, SI/16] + sh_g2 fp32 [1];
 * out = bf16(bf16(sum_s tw_s y_s) + bf16(act_sh . W2sh * gs2sh)).  SI % 256 == 0, SI <= 1024, topk < 8; same
 * workspace as flint_moe_block. */
int flint_moe_block_shared(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps, const void* gate_w,
                           int64_t H, int64_t E, int64_t topk, int score_fn, const void* w13, const void* s13,
                           const float* g13, const void* w2, const void* s2, const float* g2, int64_t I,
                           const void* sh_w13, const void* sh_s13, const float* sh_g13, const void* sh_w2,
                           const void* sh_s2, const float* sh_g2, int64_t SI, void* out, void* res_out, void* xn_out,
                           float* logits_out, int32_t* topk_ids_out, float* topk_weights_out, void* workspace,
                           const flint_l2_prefetch* next, int pdl, void* stream);

/* Expert-parallel form of flint_moe_block (the MoE of a model whose experts are split over ranks): this rank's
 * weights hold experts expert_lo .. expert_lo + n_local - 1 (w13 / s13 / g13 / w2 / s2 / g2 indexed by local
 * expert); the router and top-k run in full.  Writes y_out bf16 [topk, H] (row s = y of routed slot s when its
 * expert is local, zeros otherwise) and topk_weights_out fp32 [topk]; res_out as flint_moe_block.  Summing y_out over
 * all ranks (each element has one non-zero term, so the sum is exact) and calling flint_moe_combine gives the
 * single-GPU output of flint_moe_block bit for bit. */
int flint_moe_block_ep(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps, const void* gate_w,
                       int64_t H, int64_t E, int64_t topk, int score_fn, const void* w13, const void* s13, const float* g13,
                       const void* w2, const void* s2, const float* g2, int64_t I, int64_t expert_lo, int64_t n_local,
                       void* y_out, float* topk_weights_out, void* res_out, void* workspace,
                       const flint_l2_prefetch* next, int pdl, void* stream);
/* out bf16 [M, H] = bf16(sum_s topk_weights[m, s] * y[m * topk + s, :]) in slot order (fp32 FMA): the weighted
 * expert sum of the expert-parallel MoE (y summed over ranks first), M <= 8. */
int flint_moe_combine(const void* y, const float* topk_weights, int64_t M, int64_t topk, int64_t H, void* out, int pdl,
                      void* stream);

/* Expert-parallel forms of flint_moe_up / flint_moe_down for 1..8 tokens: the routing (topk_ids over all E experts)
 * is the full one, the weights hold experts expert_lo .. expert_lo + n_local - 1 only.  Up computes the act rows of
 * the routes whose expert is local; down writes y_out bf16 [M * topk, H]: row r = y of route r (m * topk + slot)
 * when its expert is local, zeros otherwise.  Summing y_out over ranks (one non-zero term per element, exact) and
 * flint_moe_combine give flint_moe_down's output bit for bit.  Same workspace as flint_moe_up / flint_moe_down. */
int flint_moe_up_ep(const void* xn, int64_t ldx, int64_t M, const int32_t* topk_ids, int64_t topk, const void* w13,
                    const void* s13, const float* g13, int64_t E, int64_t I, int64_t H, int64_t expert_lo, int64_t n_local,
                    void* act, void* workspace, int pdl, void* stream);
int flint_moe_down_ep(const void* act, int64_t M, const int32_t* topk_ids, int64_t topk, const void* w2, const void* s2,
                      const float* g2, int64_t E, int64_t I, int64_t H, int64_t expert_lo, int64_t n_local, void* y_out,
                      void* workspace, int pdl, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Peer exchange of the multi-GPU decode (one process per GPU; new in this build: the reference decodes on one GPU
 * and has no collective on this path).  Each rank allocates one exchange buffer (flint_peer_alloc: cudaMalloc +
 * zero fill + CUDA IPC handle, 64 bytes), shares the handle with the other ranks (any host channel) and maps theirs
 * (flint_peer_open).  `peers` is then a host array of world pointers, peers[r] = rank r's buffer as mapped in this
 * process (peers[rank] = its own).  Kernels store into peers' buffers over NVLink and raise per-source flags there;
 * every wait is bounded (10 s), after which the kernel records status bit 4 in this rank's buffer
 * (flint_peer_status) and later launches on this rank stop waiting.  All ranks must issue the same sequence of
 * exchange launches.  Kernels that wait on one another must run on different GPUs (one rank per GPU).
 * ------------------------------------------------------------------------------------------------ */
int64_t flint_peer_buffer_bytes(int64_t H);
int flint_peer_alloc(int64_t bytes, void** ptr, void* ipc_handle);
int flint_peer_open(const void* ipc_handle, void** ptr);
int flint_peer_close(void* ptr);                       /* a mapping made by flint_peer_open */
int flint_peer_free(void* ptr);                        /* this rank's own buffer */
int flint_peer_status(const void* own, uint32_t* status);

/* Expert-parallel flint_moe_block with the exchange fused in: weights as flint_moe_block_ep; each down block pushes
 * its rows of the local slots to every rank, waits for every rank's rows of the same block and writes
 * out bf16 [H] = bf16(sum_s tw_s * y_s) in slot order -- the single-GPU flint_moe_block output bit for bit, on every
 * rank.  H = 2048, topk <= 8, 2 <= world <= 8. */
int flint_moe_block_peer(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps, const void* gate_w,
                         int64_t H, int64_t E, int64_t topk, int score_fn, const void* w13, const void* s13,
                         const float* g13, const void* w2, const void* s2, const float* g2, int64_t I, int64_t expert_lo,
                         int64_t n_local, const void* const* peers, int rank, int world, void* out, void* res_out,
                         void* workspace, const flint_l2_prefetch* next, int pdl, void* stream);
/* Data-parallel decode (one stream per rank, experts split in equal contiguous ranges), exchanges fused over NVLink
 * peer memory (no collective library call; bounded waits, the peer-buffer status word records a time-out).
 * flint_dp_gather_peer: this rank's two rows send bf16 [2][H] (attention output, residual) to every rank; out
 * bf16 [world][2][H] = every rank's rows in rank order.
 * flint_dp_combine_peer: y bf16 [world * topk][H] = the per-route rows of every rank's token (flint_moe_fused_ep: this
 * rank's experts' routes, zeros elsewhere); each route's row goes to its token's rank, and out bf16 [H] =
 * bf16(sum_s topk_weights[rank * topk + s] * row_s) in slot order for this rank's token (topk_ids / topk_weights
 * [world][topk], identical on every rank).  E % world == 0, topk <= 8.  y may be NULL when
 * flint_moe_fused_dp_peer has pushed the rows itself: the launch then only waits for every rank's rows and sums.
 * No counterpart in the reference (one GPU). */
int flint_dp_gather_peer(const void* send, int64_t H, const void* const* peers, int rank, int world, void* out, int pdl,
                         void* stream);
int flint_dp_combine_peer(const void* y, const int32_t* topk_ids, const float* topk_weights, int64_t topk, int64_t E,
                          int64_t H, const void* const* peers, int rank, int world, void* out, int pdl, void* stream);
/* Data-parallel MoE layer with both exchanges inside the launch (no counterpart in the reference, which decodes on
 * one GPU): flint_moe_fused_ep on the M = world tokens, where CTA 0 first stores this rank's two rows send bf16
 * [2][H] (attention output, residual) into every rank's token table over NVLink and every CTA waits for all ranks'
 * rows, and where each local route's output rows go straight into its token owner's row table (this rank's flag
 * raised there by the last CTA).  Then flint_dp_combine_peer(NULL, ...) on every rank gives that rank's token's
 * output.  res_out bf16 [world][H], topk_ids_out / topk_weights_out [world][topk] (required), logits_out optional.
 * H = 2048 or 4096, topk <= 8, experts split in equal contiguous ranges; workspace as flint_moe_fused. */
int flint_moe_fused_dp_peer(const void* send, const void* norm_w, float eps, const void* gate_w, int64_t H, int64_t E,
                            int64_t topk, int score_fn, const void* w13, const void* s13, const float* g13,
                            const void* w2, const void* s2, const float* g2, int64_t I, int64_t expert_lo,
                            int64_t n_local, const void* const* peers, int rank, int world, void* res_out,
                            float* logits_out, int32_t* topk_ids_out, float* topk_weights_out, void* workspace, int pdl,
                            void* stream);
/* Vocabulary-shard argmax exchange: keys = this rank's M (<= 8) keys from flint_lm_head_nv4_shard; tokens int32 [M]
 * = the argmax over all ranks' shards (lowest id among the largest logits), -1 if a peer wait timed out. */
int flint_argmax_keys_allmax_peer(const uint64_t* keys, int64_t M, const void* const* peers, int rank, int world,
                                  int32_t* tokens, int pdl, void* stream);

/* ------------------------------------------------------------------------------------------------
 * (2) Deterministic moe_align_block_size.  Replaces fast/patch_align.py:11-30 (_deterministic_align), the
 * vLLM call-site contract of moe_align_block_size (same buffers, same outputs): routes of each expert in
 * ascending route order, each expert padded to block_size, unused slots = numel, expert_ids[blk] = expert
 * of block blk or -1 past the last, num_tokens_post_pad = padded total.  Buffers must be at least as long
 * as vLLM allocates (numel + E*(B-1), or min(numel*B, that) when numel < E).  status: int32 device word,
 * OR-ed with 1 when an id is outside [0, E) (that route is skipped).
 * ------------------------------------------------------------------------------------------------ */
int flint_moe_align(const int32_t* topk_ids, int64_t numel, int64_t num_experts, int64_t block_size, int32_t* sorted_ids,
                    int64_t n_sorted, int32_t* expert_ids, int64_t n_blocks, int32_t* num_tokens_post_pad,
                    int32_t* status, int pdl, void* stream);

/* ------------------------------------------------------------------------------------------------
 * (3) Decode attention block: QKV projection (+ q/k norm, RoPE, paged KV write), paged split-K GQA decode
 * attention, O projection.  Replaces fast/attn_gemv2.cu (qkv_gemv_kernel 101-150, qkv_head_kernel
 * 170-265, o_gemv_kernel 268-289) behind fast/attn_gemv.py qkv_gemv / qkv_head / o_gemv (lines 24-58),
 * and the Flint PR's flint_decode_attention (patch:2539-2605).  1..8 tokens.
 * ------------------------------------------------------------------------------------------------ */
int64_t flint_attn_proj_workspace_bytes(void);

/* s = x + res (res may be NULL), res_out = bf16(s) (may be NULL), xn = bf16(s*rsqrt(mean(s^2)+eps)*norm_w),
 * qkv_out[m] = bf16(gs * xn[m] . dequant(W, S)^T)  (W u8 [N, H/2], S E4M3 [N, H/16], gs fp32 device scalar,
 * N = (num_q_heads + 2*num_kv_heads) * 128).
 * head_mode 1 (qkv_head): per q/k head n = bf16(y * rsqrt(mean(y^2)+eps_head) * q_norm_w|k_norm_w), NeoX RoPE
 * from cos_sin fp32 [max_pos, 128] (cos | sin; NULL = no RoPE) at positions[m] (int64), q heads to q_out bf16
 * [M, num_q_heads*128], k heads back into qkv_out and to k_cache, v heads (unnormalised) to v_cache, at
 * element offset (slot/block_size)*stride_block + (slot%block_size)*stride_slot + kv_head*stride_head of
 * slots[m] (int64; < 0 skips the write).  H % 512 == 0.
 * tokens: NULL, or int32 [M] device token ids: row m of x is then x + tokens[m] * ldx (the embedding lookup of
 * the first layer fused into the load; res must be NULL). */
int flint_attn_qkv(const void* x, int64_t ldx, const int32_t* tokens, const void* res, const void* norm_w, float eps, const void* W, const void* S,
                   const float* gs, int64_t M, int64_t H, int64_t N, int64_t num_q_heads, int64_t num_kv_heads,
                   int head_mode, const void* q_norm_w, const void* k_norm_w, float eps_head, const int64_t* positions,
                   const float* cos_sin, int64_t cos_sin_stride, void* k_cache, void* v_cache, int64_t stride_block,
                   int64_t stride_slot, int64_t stride_head, int64_t block_size, const int64_t* slots, void* q_out,
                   void* qkv_out, void* res_out, void* workspace, int pdl, void* stream);

/* y[m] = bf16(gs * a[m] . dequant(W, S)^T);  a bf16 [M, K] (stride lda), W u8 [N, K/2], S E4M3 [N, K/16].
 * K % 1024 == 0, N % 64 == 0. */
int flint_attn_o(const void* a, int64_t lda, int64_t M, const void* W, const void* S, const float* gs, int64_t N, int64_t K,
                 void* y, void* workspace, int pdl, void* stream);

/* The whole decode attention block in ONE cooperative launch (fuses flint_attn_qkv in head mode, the paged decode
 * attention and flint_attn_o; replaces fast/attn_gemv2.cu qkv_head_kernel 170-265 + o_gemv_kernel 268-289 and the PR
 * decode attention patch:1741-2415 with the same rounding points):
 *   s = x + res (res NULL: s = x; tokens non-NULL: row m of x is x[tokens[m]], an embedding gather), res_out = bf16(s),
 *   y = bf16(gs_qkv * rmsnorm(s) . Wqkv^T), q / k heads RMSNorm'd (q_norm_w / k_norm_w, eps_head) and NeoX-roped
 *   (cos_sin [max_pos, 128] at positions; NULL: no RoPE), the new k / v written to kv_cache at slots[m] (< 0: skip),
 *   paged GQA attention over seq_lens[m] tokens (block_tables, sinks, sliding window, scale), then
 *   out = bf16(gs_o * attn . Wo^T).
 * kv_cache: HND bf16 [num_blocks, num_kv_heads, 16, 256] (K | V), strides in elements; head dim 128; the page of the
 * current token is patched in shared memory, so attention sees the new k / v exactly as if read back from the cache.
 * res / res_out / out rows are ldr elements apart.  q_out bf16 [M, nq*128] and attn_out bf16 [M, nq*128] are optional
 * outputs.  M <= 8, num_q_heads / num_kv_heads <= 8, H % 256 == 0, n_o % 16 == 0.  workspace:
 * flint_attn_block_workspace_bytes(n_qkv, nq*128), zero-filled once, 256-byte aligned (self-resetting). */
int64_t flint_attn_block_workspace_bytes(int64_t n_qkv, int64_t k_o);
int flint_attn_block(const void* x, int64_t ldx, const int32_t* tokens, const void* res, int64_t ldr, const void* norm_w,
                     float eps, int64_t M, int64_t H, const void* Wqkv, const void* Sqkv, const float* gs_qkv,
                     int64_t num_q_heads, int64_t num_kv_heads, const void* q_norm_w, const void* k_norm_w, float eps_head,
                     const int64_t* positions, const float* cos_sin, int64_t cs_stride, void* kv_cache, int64_t num_blocks,
                     int64_t stride_block, int64_t stride_head, const int32_t* block_tables, int64_t bt_stride,
                     int64_t max_blocks, const int32_t* seq_lens, const int64_t* slots, const float* sinks, int64_t window,
                     float scale, const void* Wo, const void* So, const float* gs_o, int64_t n_o, void* out, void* res_out,
                     void* q_out, void* attn_out, void* workspace, int pdl, void* stream);

/* Paged decode attention with optional sinks and sliding window, one query token per request:
 * q bf16 [batch, num_q_heads, 128] (request stride q_stride_b elements); kv_cache bf16 HND
 * [num_blocks, num_kv_heads, 16, 256] (K in [..., :128], V in [..., 128:], element strides stride_block /
 * stride_head, 256-element token rows); block_tables int32 [batch, max_blocks] (row stride bt_stride);
 * seq_lens int32 [batch] (KV length including the current token; 0 writes zeros); sinks fp32 [num_q_heads]
 * or NULL; window 0 = full attention, else the last `window` positions; out bf16 [batch, num_q_heads, 128].
 * num_q_heads / num_kv_heads <= 8.  splits: flint_decode_attention_splits(batch, kv_heads) (any value in
 * 1..256 works; the workspace must match).  block_tables / seq_lens are read before the PDL wait: they must
 * not be written by the kernel launched just before this one. */
int64_t flint_decode_attention_splits(int64_t batch, int64_t num_kv_heads);
int64_t flint_decode_attention_workspace_bytes(int64_t batch, int64_t num_kv_heads, int64_t splits);
int flint_decode_attention(const void* q, int64_t q_stride_b, const void* kv_cache, int64_t num_blocks,
                           int64_t num_kv_heads, int64_t stride_block, int64_t stride_head, const int32_t* block_tables,
                           int64_t bt_stride, int64_t max_blocks, const int32_t* seq_lens, const float* sinks,
                           int64_t window, float scale, int64_t batch, int64_t num_q_heads, void* out, int64_t out_stride_b,
                           int64_t splits, void* workspace, int pdl, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Decode-step bookkeeping on the device (vLLM's GPUModelRunner prepares these on the host each step):
 * history[m, *step] = tokens[m] (if history and *step < max_steps), next_tokens[m] = tokens[m] (optional),
 * positions[m] += 1, seq_lens[m] = positions[m] + 1,
 * slots[m] = block_tables[m, pos / block_size] * block_size + pos % block_size (-1 past max_blocks), *step += 1.
 * ------------------------------------------------------------------------------------------------ */
int flint_decode_advance(const int32_t* tokens, int64_t M, int64_t* positions, int32_t* seq_lens, int64_t* slots,
                         const int32_t* block_tables, int64_t bt_stride, int64_t max_blocks, int64_t block_size,
                         int32_t* history, int64_t hist_stride, int32_t* step, int64_t max_steps, int32_t* next_tokens,
                         int pdl, void* stream);

/* ------------------------------------------------------------------------------------------------
 * Checkpoint format: GGUF NVFP4 (ggml type 40) -> the ModelOpt NVFP4 layout of every kernel above.
 * ------------------------------------------------------------------------------------------------ */

/* Replaces gguf_nvfp4._repack_nvfp4 (patch:269-288).  blocks: rows x (n_cols/64) GGUF super-blocks of 36 bytes
 * (4 UE4M3 scale bytes, then 4 x 8 code bytes: low nibbles = values 0..7 of the sub-block, high nibbles = 8..15),
 * 16-byte aligned.  Writes packed u8 [rows, n_cols/2] (16-byte aligned; even value in the low nibble) and scales
 * E4M3 bits u8 [rows, n_cols/16] (4-byte aligned): 0x7F -> 0, other bytes with the sign bit cleared.  A scale byte
 * 0xFF is not representable: every warp that met one adds 1 to *bad_blocks (device int32, zeroed by the caller);
 * its outputs are then meaningless (the reference raises ValueError).  n_cols % 64 == 0. */
int flint_gguf_nvfp4_repack(const void* blocks, int64_t rows, int64_t n_cols, void* packed, void* scales,
                            int32_t* bad_blocks, int pdl, void* stream);

/* Replaces gguf_nvfp4.dequantize_nvfp4 (patch:295-319).  out[r, k] = e2m1(P) * e4m3(S) (exact), times
 * *global_scale (device fp32, optional; one fp32 multiply, round to nearest), stored as fp32 (out_f32 = 1) or
 * rounded once to bf16.  P u8 [rows, n_cols/2] (8-byte aligned), S u8 [rows, n_cols/16], out 16-byte aligned.
 * n_cols % 16 == 0. */
int flint_nvfp4_dequant(const void* P, const void* S, int64_t rows, int64_t n_cols, const float* global_scale,
                        int out_f32, void* out, int pdl, void* stream);

/* Marlin-processed NVFP4 (the tensors vLLM holds after its Marlin repack and that fast/model.py:271-282 hands to
 * fp4moe_decode.MarlinDecodeWeights; layout fast/fp4moe_mar.cu:1-7) -> the ModelOpt layout of every kernel above.
 * weight int32 [E][K/16][N/64][128 words] (4-byte aligned), weight_scale u8 [E][K/16][N] (processed S0E5M3 bytes,
 * permuted inside each 64-column group), global_scale fp32 [E] (processed).  Writes packed u8 [E][N][K/2] (8-byte
 * aligned), scales E4M3 bits u8 [E][N][K/16] (scale byte h -> h - 0x78, 0 stays 0) and global_out fp32 [E]
 * (= global_scale * 2^-119), so e2m1 * e4m3 * gs equals the reference's e2m1 * fp16(h << 7) * g * 2^-126 exactly.
 * A non-zero scale byte outside 0x80..0xF6 is not a processed scale: the CTAs that met one add 1 to *bad (device
 * int32, zeroed by the caller) and write 0 for it.  N % 64 == 0, K % 16 == 0. */
int flint_marlin_nvfp4_unpack(const void* weight, const void* weight_scale, const float* global_scale, int64_t E,
                              int64_t N, int64_t K, void* packed, void* scales, float* global_out, int32_t* bad, int pdl,
                              void* stream);

/* FlashInfer W4A16 NVFP4 expert tensors (what the Flint PR's prepare_weights makes for its grouped MoE,
 * vllm/models/flint/ops/moe_cute.py, patch:4061-4091) -> the ModelOpt layout of every kernel above.
 * w1 u8 [E][2I][H/2] (gate/up rows interleaved: per 128-row block, 64 up rows then 64 gate rows), w1_sf the stored
 * (contiguous) block scales of those rows [E][2I/128][H/64][32][4][4], w2 u8 [E][H][I/2], w2_sf [E][H/128][I/64][32]
 * [4][4] (the PR returns the scales as permuted views of these arrays).  Writes w13_out [E][2I][H/2] ([gate; up]),
 * s13_out [E][2I][H/16], w2_out [E][H][I/2], s2_out [E][H][I/16]: byte moves only, bit-exact.  H % 128 == 0,
 * I % 64 == 0; code arrays 16-byte aligned. */
int flint_flashinfer_nvfp4_unpack(const void* w1, const void* w1_sf, const void* w2, const void* w2_sf, int64_t E,
                                  int64_t H, int64_t I, void* w13_out, void* s13_out, void* w2_out, void* s2_out,
                                  int pdl, void* stream);

/* Prefill-side grouped MoE (the Flint PR runs prompts through FlashInfer's grouped GEMMs, grouped_moe at
 * patch:4093-4212; here with this library's NVFP4 tiles).  With the deterministic align of the prompt's routes
 * (flint_moe_align, block size 64: sorted_ids [max_blocks * 64], expert_ids [max_blocks], num_tokens_post_pad [1]):
 *   flint_rows_to_f16: rows bf16 [rows][ld >= K] -> dst f16 [rows][K] = x * 2^shift[row] (the per-row power of two of
 *     the decode kernels, exact);
 *   flint_moe_grouped_up: xh = the tokens' f16 rows [T][H] (and their shifts) -> act bf16 [numel][I] per route
 *     (route = token * topk + slot): bf16(silu(g) * u) of the route's expert, g / u in fp32 (as flint_moe_up);
 *   flint_moe_grouped_down: ah = the routes' f16 act rows [numel][I] -> y bf16 [numel][H] per route (as
 *     flint_moe_down's per-route rows);
 * then flint_moe_combine(y, topk_weights, T, topk, H, out) for the slot-order weighted sum.  Weights in the ModelOpt
 * layout of the other MoE entry points; H and I multiples of 256; workspace: one status word (4 bytes, zeroed).
 * tensor_cores: 1 = tcgen05.mma with the accumulator in tensor memory, 0 = mma.sync (same tiles and rounding points;
 * the fp32 sums differ in order). */
int flint_rows_to_f16(const void* src, int64_t ld, int64_t rows, int64_t K, void* dst, int32_t* shift, int pdl,
                      void* stream);
int flint_moe_grouped_up(const void* xh, const int32_t* shift, const int32_t* sorted_ids, const int32_t* expert_ids,
                         const int32_t* num_tokens_post_pad, int64_t numel, int64_t topk, int64_t E, const void* w13,
                         const void* s13, const float* g13, int64_t H, int64_t I, int64_t max_blocks, void* act,
                         void* workspace, int tensor_cores, int pdl, void* stream);
int flint_moe_grouped_down(const void* ah, const int32_t* shift, const int32_t* sorted_ids, const int32_t* expert_ids,
                           const int32_t* num_tokens_post_pad, int64_t numel, int64_t topk, int64_t E, const void* w2,
                           const void* s2, const float* g2, int64_t H, int64_t I, int64_t max_blocks, void* y,
                           void* workspace, int tensor_cores, int pdl, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FLINT_B200_H_ */
