/*
 * flint_b200.h -- C ABI of the B200 (sm_100a) NVFP4 batch-1 decode kernels.
 *
 * Every entry point takes plain device pointers, sizes and a cudaStream_t passed as void*, launches
 * asynchronously on that stream and returns FLINT_OK or one of the FLINT_ERR_* codes below.  Nothing
 * here aborts, allocates device memory or synchronises the stream.
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
  FLINT_ERR_ARGUMENT = 6      /* null pointer or out-of-range scalar argument */
};

/* Library version (major*10000 + minor*100 + patch). */
int flint_version(void);
/* Human-readable name of an error code. */
const char* flint_error_string(int code);

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

#ifdef __cplusplus
}
#endif

#endif /* FLINT_B200_H_ */
