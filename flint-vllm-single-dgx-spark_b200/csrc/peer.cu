// Peer exchange buffers (CUDA IPC) and the vocabulary-shard argmax exchange of the multi-GPU decode.
//
// The reference decodes on one GPU and has no collective on this path; these entry points are new in this build
// (expert-parallel MoE + vocabulary-sharded head, one process per GPU).  Buffer layout and protocol: peer.cuh.
#include "common.cuh"
#include "peer.cuh"
#include "runtime.cuh"

#include <string.h>

namespace flint {

// One warp.  Stores this rank's M flipped-top-bit argmax keys into every rank's key table, raises its flag on every
// rank, waits for every rank's keys, then token[m] = the id of the signed maximum over ranks (the lowest id among
// the largest logits of the whole vocabulary).
__global__ void keys_allmax_peer_kernel(const unsigned long long* __restrict__ keys, int M, const PeerSet ps,
                                        int* __restrict__ tokens) {
  pdl_wait();
  const int lane = threadIdx.x, W = ps.world, r = ps.rank;
  PeerHeader* own = peer_header(ps.base[r]);
  const unsigned ep = ld_relaxed_sys_u32(&own->head_epoch) + 1u, par = ep & 1u;
  for (int i = lane; i < M * W; i += 32) {
    const int p = i % W, m = i / W;
    peer_head_keys(ps.base[p], par)[r * kPeerRowsMax + m] = keys[m];
  }
  __threadfence_system();
  __syncwarp();
  if (lane < W) st_release_sys_u32(peer_head_flags(ps.base[lane]) + r, ep);
  bool ok = true;
  if (lane < W) ok = peer_wait(peer_head_flags(ps.base[r]) + lane, ep, own);
  ok = __all_sync(0xffffffffu, ok);
  __syncwarp();   // orders every lane's reads after the acquiring lanes' loads
  if (lane < M) {
    const unsigned long long* kb = peer_head_keys(ps.base[r], par);
    long long best = (long long)__ldcg(kb + lane);
    for (int s = 1; s < W; ++s) best = max(best, (long long)__ldcg(kb + s * kPeerRowsMax + lane));
    tokens[lane] = ok ? (int)argmax_key_index((unsigned long long)best) : -1;
  }
  __syncwarp();
  if (lane == 0) own->head_epoch = ep;
  pdl_trigger();
}

int peer_set(const void* const* peers, int rank, int world, PeerSet* ps) {
  if (!peers) return FLINT_ERR_ARGUMENT;
  if (world < 2 || world > kPeerMax || rank < 0 || rank >= world) return FLINT_ERR_SHAPE;
  memset(ps, 0, sizeof(*ps));
  for (int i = 0; i < world; ++i) {
    if (!peers[i]) return FLINT_ERR_ARGUMENT;
    if (!aligned(peers[i], 256)) return FLINT_ERR_ALIGN;
    ps->base[i] = (uint8_t*)peers[i];
  }
  ps->rank = rank;
  ps->world = world;
  return FLINT_OK;
}

}  // namespace flint

using namespace flint;

extern "C" int64_t flint_peer_buffer_bytes(int64_t H) {
  if (H < 16 || H > 65536) return -1;
  return (int64_t)peer_buffer_bytes((int)H);
}

extern "C" int flint_peer_alloc(int64_t bytes, void** ptr, void* ipc_handle) {
  if (!ptr || !ipc_handle || bytes < (int64_t)kPeerMoeRowsOff) return FLINT_ERR_ARGUMENT;
  void* p = nullptr;
  if (cudaMalloc(&p, (size_t)bytes) != cudaSuccess) return record_cuda(cudaGetLastError(), FLINT_ERR_DEVICE);
  cudaIpcMemHandle_t h;
  if (cudaMemset(p, 0, (size_t)bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess ||
      cudaIpcGetMemHandle(&h, p) != cudaSuccess) {
    const int rc = record_cuda(cudaGetLastError(), FLINT_ERR_DEVICE);
    cudaFree(p);
    return rc;
  }
  static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
  memcpy(ipc_handle, &h, sizeof(h));
  *ptr = p;
  return FLINT_OK;
}

extern "C" int flint_peer_open(const void* ipc_handle, void** ptr) {
  if (!ipc_handle || !ptr) return FLINT_ERR_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  void* p = nullptr;
  if (cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
    return record_cuda(cudaGetLastError(), FLINT_ERR_DEVICE);
  *ptr = p;
  return FLINT_OK;
}

extern "C" int flint_peer_close(void* ptr) {
  if (!ptr) return FLINT_ERR_ARGUMENT;
  return record_cuda(cudaIpcCloseMemHandle(ptr), FLINT_ERR_DEVICE);
}

extern "C" int flint_peer_free(void* ptr) {
  if (!ptr) return FLINT_ERR_ARGUMENT;
  return record_cuda(cudaFree(ptr), FLINT_ERR_DEVICE);
}

extern "C" int flint_peer_status(const void* own, uint32_t* status) {
  if (!own || !status) return FLINT_ERR_ARGUMENT;
  return record_cuda(cudaMemcpy(status, (const uint8_t*)own + offsetof(PeerHeader, status), 4, cudaMemcpyDeviceToHost),
                     FLINT_ERR_DEVICE);
}

extern "C" int flint_argmax_keys_allmax_peer(const uint64_t* keys, int64_t M, const void* const* peers, int rank,
                                             int world, int32_t* tokens, int pdl, void* stream) {
  if (!keys || !tokens) return FLINT_ERR_ARGUMENT;
  if (M < 1 || M > kPeerRowsMax) return FLINT_ERR_SHAPE;
  PeerSet ps;
  const int rc = peer_set(peers, rank, world, &ps);
  if (rc) return rc;
  return launch(keys_allmax_peer_kernel, dim3(1), dim3(32), 0, stream, pdl,
                reinterpret_cast<const unsigned long long*>(keys), (int)M, ps, (int*)tokens);
}
