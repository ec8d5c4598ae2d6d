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

// ---- data-parallel decode (one stream per rank, experts split over the ranks) ----
//
// Token gather, one CTA: this rank's two rows (attention output, residual: bf16 [2][H]) go into every rank's token
// table at [parity][rank] with 16-byte stores, then its flag on every rank; once every rank's flag shows this
// launch, the table is copied to `out` [world][2][H] (a fixed buffer, so captured graphs keep their pointers).
__global__ void dp_gather_peer_kernel(const bf16* __restrict__ send, int H, const PeerSet ps, bf16* __restrict__ out) {
  __shared__ int s_ok;
  pdl_wait();
  const int tid = threadIdx.x, W = ps.world, r = ps.rank;
  PeerHeader* own = peer_header(ps.base[r]);
  const unsigned ep = ld_relaxed_sys_u32(&own->dp_tok_epoch) + 1u, par = ep & 1u;
  const int n16 = 2 * H / 8;                                       // 16-byte units of the two rows
  const uint4* src = reinterpret_cast<const uint4*>(send);
  for (int i = tid; i < n16 * W; i += blockDim.x) {
    const int p = i / n16, u = i - p * n16;
    reinterpret_cast<uint4*>(peer_dp_tokens(ps.base[p], par, H) + (size_t)r * 2 * H)[u] = src[u];
  }
  __threadfence_system();
  __syncthreads();
  if (tid < W) st_release_sys_u32(reinterpret_cast<unsigned*>(ps.base[tid] + kPeerDpTokFlagsOff) + r, ep);
  if (tid == 0) s_ok = 1;
  __syncthreads();
  if (tid < W && !peer_wait(reinterpret_cast<unsigned*>(ps.base[r] + kPeerDpTokFlagsOff) + tid, ep, own)) s_ok = 0;
  __syncthreads();                                                 // orders the copy after the acquiring loads
  const uint4* tab = reinterpret_cast<const uint4*>(peer_dp_tokens(ps.base[r], par, H));
  for (int i = tid; i < n16 * W; i += blockDim.x) reinterpret_cast<uint4*>(out)[i] = s_ok ? __ldcg(tab + i) : make_uint4(0, 0, 0, 0);
  __syncthreads();
  if (tid == 0) own->dp_tok_epoch = ep;
  pdl_trigger();
}

// Row scatter + combine, one CTA: y [world * topk][H] holds the rows of every token's routes whose expert is local
// (zeros elsewhere); the rows of token m's local routes go to rank m's row table at [parity][this rank][slot], then
// this rank's flag on every rank.  Once every flag shows this launch, out[h] = bf16(sum_s tw[s] * row_s[h]) in slot
// order (fp32 FMA), row_s read from the rank that owns expert ids[rank * topk + s] (experts split in equal
// contiguous ranges): the one-GPU weighted sum bit for bit.  y NULL: flint_moe_fused_dp_peer has already pushed the
// rows and raised the flags, and this launch only waits and sums.
__global__ void dp_combine_peer_kernel(const bf16* __restrict__ y, const int* __restrict__ ids,
                                       const float* __restrict__ tw, int topk, int E, int H, const PeerSet ps,
                                       bf16* __restrict__ out) {
  __shared__ int s_ok, s_src[kPeerSlots];
  pdl_wait();
  const int tid = threadIdx.x, W = ps.world, r = ps.rank, per = E / W;
  PeerHeader* own = peer_header(ps.base[r]);
  // (y NULL: flint_moe_fused_dp_peer pushed the rows, raised the flags and advanced the epoch itself)
  const unsigned ep = ld_relaxed_sys_u32(&own->dp_row_epoch) + (y ? 1u : 0u), par = ep & 1u;
  const int n16 = H / 8;
  for (int i = tid; y && i < W * topk * n16; i += blockDim.x) {   // push this rank's local routes of every token
    const int route = i / n16, u = i - route * n16, m = route / topk, s = route - m * topk;
    const int e = ids[route];
    if (e < r * per || e >= (r + 1) * per) continue;
    reinterpret_cast<uint4*>(peer_dp_rows(ps.base[m], par, H) + ((size_t)r * kPeerSlots + s) * H)[u] =
        reinterpret_cast<const uint4*>(y + (size_t)route * H)[u];
  }
  if (tid < topk) {
    const int e = ids[r * topk + tid];
    s_src[tid] = min(max(e / per, 0), W - 1);
  }
  __threadfence_system();
  __syncthreads();
  if (y && tid < W) st_release_sys_u32(reinterpret_cast<unsigned*>(ps.base[tid] + kPeerDpRowFlagsOff) + r, ep);
  if (tid == 0) s_ok = 1;
  __syncthreads();
  if (tid < W && !peer_wait(reinterpret_cast<unsigned*>(ps.base[r] + kPeerDpRowFlagsOff) + tid, ep, own)) s_ok = 0;
  __syncthreads();
  const bf16* rows = peer_dp_rows(ps.base[r], par, H);
  for (int h = tid; h < H; h += blockDim.x) {
    float acc = 0.f;
    for (int s = 0; s < topk; ++s) acc = fmaf(tw[r * topk + s], peer_ldcg_bf16(rows + ((size_t)s_src[s] * kPeerSlots + s) * H + h), acc);
    out[h] = __float2bfloat16_rn(s_ok ? acc : 0.f);
  }
  __syncthreads();
  if (tid == 0 && y) own->dp_row_epoch = ep;
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

extern "C" int flint_dp_gather_peer(const void* send, int64_t H, const void* const* peers, int rank, int world, void* out,
                                    int pdl, void* stream) {
  if (!send || !out) return FLINT_ERR_ARGUMENT;
  if (H < 8 || H % 8 != 0 || H > 65536) return FLINT_ERR_SHAPE;
  if (!aligned(send, 16) || !aligned(out, 16)) return FLINT_ERR_ALIGN;
  PeerSet ps;
  const int rc = peer_set(peers, rank, world, &ps);
  if (rc) return rc;
  return launch(dp_gather_peer_kernel, dim3(1), dim3(512), 0, stream, pdl, (const bf16*)send, (int)H, ps, (bf16*)out);
}

extern "C" int flint_dp_combine_peer(const void* y, const int32_t* topk_ids, const float* topk_weights, int64_t topk,
                                     int64_t E, int64_t H, const void* const* peers, int rank, int world, void* out,
                                     int pdl, void* stream) {
  if (!topk_ids || !topk_weights || !out) return FLINT_ERR_ARGUMENT;
  if (topk < 1 || topk > kPeerSlots || H < 8 || H % 8 != 0 || H > 65536 || E < world || E % world != 0)
    return FLINT_ERR_SHAPE;
  if (y && !aligned(y, 16)) return FLINT_ERR_ALIGN;
  PeerSet ps;
  const int rc = peer_set(peers, rank, world, &ps);
  if (rc) return rc;
  return launch(dp_combine_peer_kernel, dim3(1), dim3(512), 0, stream, pdl, (const bf16*)y, (const int*)topk_ids,
                topk_weights, (int)topk, (int)E, (int)H, ps, (bf16*)out);
}
