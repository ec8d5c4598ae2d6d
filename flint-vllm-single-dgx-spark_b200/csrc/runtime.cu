// Library-wide host helpers: version, error strings, per-device properties.
#include "runtime.cuh"

#include <stdio.h>

#include <mutex>
#include "tma.cuh"

#include <cudaTypedefs.h>

namespace flint {

int num_sms(int* dev_out) {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  if (dev_out) *dev_out = dev;
  if (dev < 0 || dev >= 64) return -1;
  if (cache[dev] == 0) {
    int n = 0, major = 0;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return -1;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return -1;
    if (major != 10) return -1;
    cache[dev] = n;
  }
  return cache[dev];
}

static PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

int encode_u8_2d(CUtensorMap* map, const void* base, uint64_t cols_bytes, uint64_t rows, uint64_t row_stride_bytes,
                 uint32_t box_cols, uint32_t box_rows, bool swizzle128) {
  auto fn = get_encode_fn();
  if (!fn) return FLINT_ERR_DEVICE;
  if (!aligned(base, 16) || row_stride_bytes % 16 != 0) return FLINT_ERR_ALIGN;
  cuuint64_t dims[2] = {cols_bytes, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_cols, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE,
                        swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FLINT_OK : FLINT_ERR_ALIGN;
}

int encode_u8_2d_swz(CUtensorMap* map, const void* base, uint64_t cols_bytes, uint64_t rows, uint64_t row_stride_bytes,
                     uint32_t box_rows, int swizzle_bytes) {
  auto fn = get_encode_fn();
  if (!fn) return FLINT_ERR_DEVICE;
  if (!aligned(base, 16) || row_stride_bytes % 16 != 0) return FLINT_ERR_ALIGN;
  const CUtensorMapSwizzle swz = swizzle_bytes == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                 : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                 : swizzle_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B
                                                        : CU_TENSOR_MAP_SWIZZLE_NONE;
  if (swz == CU_TENSOR_MAP_SWIZZLE_NONE) return FLINT_ERR_ARGUMENT;
  cuuint64_t dims[2] = {cols_bytes, rows};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {(cuuint32_t)swizzle_bytes, box_rows};
  cuuint32_t estr[2] = {1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FLINT_OK : FLINT_ERR_ALIGN;
}

int encode_u8_3d(CUtensorMap* map, const void* base, const uint64_t dims[3], const uint64_t strides_bytes[2],
                 const uint32_t box[3], bool swizzle128) {
  auto fn = get_encode_fn();
  if (!fn) return FLINT_ERR_DEVICE;
  if (!aligned(base, 16) || strides_bytes[0] % 16 != 0 || strides_bytes[1] % 16 != 0) return FLINT_ERR_ALIGN;
  cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t st[2] = {strides_bytes[0], strides_bytes[1]};
  cuuint32_t b[3] = {box[0], box[1], box[2]};
  cuuint32_t e[3] = {1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), d, st, b, e,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FLINT_OK : FLINT_ERR_ALIGN;
}

int encode_bf16_5d(CUtensorMap* map, const void* base, const uint64_t dims[5], const uint64_t strides_bytes[4],
                   const uint32_t box[5]) {
  auto fn = get_encode_fn();
  if (!fn) return FLINT_ERR_DEVICE;
  if (!aligned(base, 16)) return FLINT_ERR_ALIGN;
  for (int i = 0; i < 4; ++i)
    if (strides_bytes[i] % 16 != 0) return FLINT_ERR_ALIGN;
  cuuint64_t d[5] = {dims[0], dims[1], dims[2], dims[3], dims[4]};
  cuuint64_t st[4] = {strides_bytes[0], strides_bytes[1], strides_bytes[2], strides_bytes[3]};
  cuuint32_t b[5] = {box[0], box[1], box[2], box[3], box[4]};
  cuuint32_t e[5] = {1, 1, 1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 5, const_cast<void*>(base), d, st, b, e,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FLINT_OK : FLINT_ERR_ALIGN;
}

int encode_bf16_4d(CUtensorMap* map, const void* base, const uint64_t dims[4], const uint64_t strides_bytes[3],
                   const uint32_t box[4]) {
  auto fn = get_encode_fn();
  if (!fn) return FLINT_ERR_DEVICE;
  if (!aligned(base, 16)) return FLINT_ERR_ALIGN;
  for (int i = 0; i < 3; ++i)
    if (strides_bytes[i] % 16 != 0) return FLINT_ERR_ALIGN;
  cuuint64_t d[4] = {dims[0], dims[1], dims[2], dims[3]};
  cuuint64_t s[3] = {strides_bytes[0], strides_bytes[1], strides_bytes[2]};
  cuuint32_t b[4] = {box[0], box[1], box[2], box[3]};
  cuuint32_t e[4] = {1, 1, 1, 1};
  const CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), d, s, b, e,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FLINT_OK : FLINT_ERR_ALIGN;
}

}  // namespace flint

namespace flint {

static thread_local char g_last_cuda_error[256] = "";

int record_cuda(cudaError_t e, int code) {
  if (e == cudaSuccess) return FLINT_OK;
  snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s: %s", cudaGetErrorName(e), cudaGetErrorString(e));
  return code;
}

bool carveout_pending(const void* kern) {
  static std::mutex mu;
  static const void* done_kern[256];
  static int done_dev[256];
  static int n_done = 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return false;
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < n_done; ++i)
    if (done_kern[i] == kern && done_dev[i] == dev) return false;
  if (n_done < 256) {
    done_kern[n_done] = kern;
    done_dev[n_done] = dev;
    ++n_done;
  }
  return true;
}

void record_message(const char* msg) { snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s", msg); }

}  // namespace flint

extern "C" const char* flint_last_cuda_error(void) { return flint::g_last_cuda_error; }

extern "C" int flint_version(void) { return 100; }

extern "C" int64_t flint_workspace_status_offset(int kind) {
  using namespace flint;
  switch (kind) {
    case FLINT_WS_LM_HEAD: return status_offset_lm_head();
    case FLINT_WS_MOE: return status_offset_moe();
    case FLINT_WS_MOE_FUSED: return status_offset_moe_fused();
    case FLINT_WS_MOE_BLOCK: return status_offset_moe_block();
    case FLINT_WS_ATTN_PROJ: return status_offset_attn_proj();
    case FLINT_WS_ATTN_BLOCK: return status_offset_attn_block();
    case FLINT_WS_DECODE_ATTENTION: return status_offset_decode_attention();
    default: return -1;
  }
}

extern "C" int flint_workspace_status(const void* workspace, int kind, uint32_t* status, int clear) {
  const int64_t off = flint_workspace_status_offset(kind);
  if (!workspace || !status) return FLINT_ERR_ARGUMENT;
  if (off < 0) return FLINT_ERR_ARGUMENT;
  uint8_t* word = (uint8_t*)workspace + off;
  int rc = flint::record_cuda(cudaMemcpy(status, word, 4, cudaMemcpyDeviceToHost), FLINT_ERR_DEVICE);
  if (rc == FLINT_OK && clear && *status) rc = flint::record_cuda(cudaMemset(word, 0, 4), FLINT_ERR_DEVICE);
  return rc;
}

extern "C" const char* flint_error_string(int code) {
  switch (code) {
    case FLINT_OK: return "ok";
    case FLINT_ERR_SHAPE: return "unsupported or inconsistent shape";
    case FLINT_ERR_ALIGN: return "misaligned pointer or stride";
    case FLINT_ERR_DEVICE: return "no sm_100 CUDA device";
    case FLINT_ERR_LAUNCH: return "kernel launch failed";
    case FLINT_ERR_WORKSPACE: return "workspace missing or too small";
    case FLINT_ERR_ARGUMENT: return "invalid argument";
    case FLINT_ERR_SCRATCH: return "request exceeds the fixed scratch of the allocation-free entry point";
    default: return "unknown error";
  }
}
