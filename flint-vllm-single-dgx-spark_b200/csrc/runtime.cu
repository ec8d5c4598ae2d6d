// Library-wide host helpers: version, error strings, per-device properties.
#include "runtime.cuh"

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

}  // namespace flint

extern "C" int flint_version(void) { return 100; }

extern "C" const char* flint_error_string(int code) {
  switch (code) {
    case FLINT_OK: return "ok";
    case FLINT_ERR_SHAPE: return "unsupported or inconsistent shape";
    case FLINT_ERR_ALIGN: return "misaligned pointer or stride";
    case FLINT_ERR_DEVICE: return "no sm_100 CUDA device";
    case FLINT_ERR_LAUNCH: return "kernel launch failed";
    case FLINT_ERR_WORKSPACE: return "workspace missing or too small";
    case FLINT_ERR_ARGUMENT: return "invalid argument";
    default: return "unknown error";
  }
}
