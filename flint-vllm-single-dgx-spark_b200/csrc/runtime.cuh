// Host-side launch helpers shared by the entry points.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/flint_b200.h"

namespace flint {

// SM count of the current device (cached), or -1 if there is none / it is not sm_10x.
int num_sms(int* dev_out = nullptr);

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Records the CUDA error of a failed runtime call made by this library (per host thread; flint_last_cuda_error) and
// returns the library status for it: FLINT_OK for cudaSuccess, else `code`.
int record_cuda(cudaError_t e, int code);
// Records a library diagnostic in the same slot (flint_last_cuda_error).
void record_message(const char* msg);

// Byte offset of the sticky status word inside each kernel family's workspace (flint_workspace_status_offset);
// each is defined beside its workspace struct.
int64_t status_offset_lm_head();
int64_t status_offset_moe();
int64_t status_offset_moe_fused();
int64_t status_offset_moe_block();
int64_t status_offset_attn_proj();
int64_t status_offset_attn_block();
int64_t status_offset_decode_attention();

// Every kernel runs with the maximum shared-memory carveout, so consecutive kernels of a decode step never make an
// SM re-partition L1 / shared memory between them.  Set once per (kernel, device).
bool carveout_pending(const void* kern);

template <typename... KArgs>
inline void set_max_carveout(void (*kern)(KArgs...)) {
  if (!carveout_pending(reinterpret_cast<const void*>(kern))) return;
  cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, (int)cudaSharedmemCarveoutMaxShared);
}

// Launch with optional programmatic dependent launch (PDL); returns FLINT_OK / FLINT_ERR_LAUNCH.
template <typename... KArgs, typename... Args>
int launch(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, void* stream, int pdl, Args... args) {
  set_max_carveout(kern);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 1 : 0;
  return record_cuda(cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...), FLINT_ERR_LAUNCH);
}

// Launch with a thread-block cluster of `cluster` CTAs along x (grid.x must be a multiple), optional PDL.
template <typename... KArgs, typename... Args>
int launch_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, void* stream, int pdl, int cluster,
                   Args... args) {
  set_max_carveout(kern);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeClusterDimension;
  at[0].val.clusterDim.x = cluster;
  at[0].val.clusterDim.y = 1;
  at[0].val.clusterDim.z = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 2 : 1;
  return record_cuda(cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...), FLINT_ERR_LAUNCH);
}

}  // namespace flint
