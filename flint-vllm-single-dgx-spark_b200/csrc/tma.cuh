// TMA (cp.async.bulk.tensor) + mbarrier helpers for the weight-streaming kernels.
//
// Weights are fetched as 2-D tiles of their row-major byte image: codes [rows, K/2] u8 in boxes of 128 B x 128 rows
// with the 128-byte swizzle (16-byte unit u of row r lands at unit u ^ (r & 7)), and block scales [rows, K/16] u8
// in boxes of 16 B x 128 rows without swizzle.  No multicast is used anywhere.
// Every wait is bounded: after FLINT_WAIT_LIMIT polls the waiter records an error and stops waiting.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/flint_b200.h"

#ifndef FLINT_WAIT_LIMIT
#define FLINT_WAIT_LIMIT (1u << 22)
#endif

namespace flint {

// status word bits written by kernels into their workspace (0 = healthy)
enum : unsigned { STATUS_WAIT_TIMEOUT = 1u };

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase of the given parity; returns false (and sets *status) on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, unsigned parity, unsigned* status) {
#pragma unroll 1
  for (unsigned i = 0; i < FLINT_WAIT_LIMIT; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (status) atomicOr(status, STATUS_WAIT_TIMEOUT);
  return false;
}

// L2 policy for read-once streams (weights, KV pages): evict first, so the gigabytes streamed per decode step do not
// push the kernels' code, activations and workspaces out of L2.
__device__ __forceinline__ uint64_t l2_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 2-D tensor tile load into shared memory, completion counted on `bar` (transaction bytes), streaming L2 policy.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar)),
        "l"(l2_evict_first())
      : "memory");
}
// 4-D tensor tile load (x, y, z, w) into shared memory, streaming L2 policy.
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, int x, int y, int z, int w, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar)),
        "l"(l2_evict_first())
      : "memory");
}
// 3-D tensor tile load (x, y, z), streaming L2 policy.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4}], [%5], %6;"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)),
        "l"(l2_evict_first())
      : "memory");
}
// 5-D tensor tile load, streaming L2 policy.
__device__ __forceinline__ void tma_load_5d(void* smem_dst, const CUtensorMap* map, int x, int y, int z, int w, int v,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;"
      ::"r"(smem_u32(smem_dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(v),
        "r"(smem_u32(bar)), "l"(l2_evict_first())
      : "memory");
}
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- L2 prefetch of the next op's bytes (flint_l2_prefetch) ----
struct L2Prefetch {
  const uint8_t* ptr[8];
  unsigned long long n16[8];           // 16-byte units of each range
  int n;
  // paged KV pages (kv != nullptr): see flint_l2_prefetch
  const uint8_t* kv;
  unsigned long long block_bytes, kv_blocks;
  const int* bt;
  long long bt_stride;
  int bt_cols, streams, block_tokens, max_blocks;
  const int* seq_lens;
};

// Host: validates and converts the ABI struct (NULL or n = 0: nothing); false on a bad range.
inline bool l2_prefetch_pack(const flint_l2_prefetch* in, L2Prefetch* out) {
  *out = L2Prefetch{};
  if (!in || in->n == 0) return true;
  if (in->n < 0 || in->n > 8) return false;
  for (int r = 0; r < in->n; ++r) {
    if (!in->ptr[r] || in->bytes[r] < 0 || (reinterpret_cast<uintptr_t>(in->ptr[r]) & 15)) return false;
    out->ptr[r] = static_cast<const uint8_t*>(in->ptr[r]);
    out->n16[r] = (unsigned long long)in->bytes[r] >> 4;
  }
  out->n = in->n;
  if (in->kv) {
    if (!in->block_tables || !in->seq_lens || in->streams < 1 || in->streams > 8 || in->block_tokens < 1 ||
        in->block_bytes < 16 || (in->block_bytes & 15) || in->kv_blocks < 1 || in->bt_cols < 1 ||
        in->bt_stride < in->bt_cols || in->max_blocks < 0 || (reinterpret_cast<uintptr_t>(in->kv) & 15))
      return false;
    out->kv = static_cast<const uint8_t*>(in->kv);
    out->block_bytes = (unsigned long long)in->block_bytes;
    out->kv_blocks = (unsigned long long)in->kv_blocks;
    out->bt = in->block_tables;
    out->bt_stride = in->bt_stride;
    out->bt_cols = (int)(in->bt_cols < (1 << 30) ? in->bt_cols : (1 << 30));
    out->seq_lens = in->seq_lens;
    out->streams = in->streams;
    out->block_tokens = in->block_tokens;
    out->max_blocks = in->max_blocks;
  }
  return true;
}

__device__ __forceinline__ void l2_prefetch_bulk(const uint8_t* p, unsigned long long bytes) {
  for (unsigned long long u = 0; u < bytes; u += 32768) {
    const unsigned long long k = bytes - u < 32768 ? bytes - u : 32768;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p + u), "r"((uint32_t)k) : "memory");
  }
}

// One thread: this CTA's 1/nb share of every range, as bulk L2 prefetches of at most 32 KB, then its share of the
// KV pages.  The page list reads seq_lens / block tables: the caller issues this only where they are final.
__device__ __forceinline__ void l2_prefetch_share(const L2Prefetch& pf, int cta, int nb) {
  for (int r = 0; r < pf.n; ++r) {
    const unsigned long long lo = pf.n16[r] * cta / nb, hi = pf.n16[r] * (cta + 1) / nb;
    if (hi > lo) l2_prefetch_bulk(pf.ptr[r] + lo * 16, (hi - lo) * 16);
  }
  if (pf.kv == nullptr) return;
  int npg[8], total = 0;
  for (int b = 0; b < pf.streams; ++b) {
    const int seq = pf.seq_lens[b];
    int n = seq > 0 ? (seq + pf.block_tokens - 1) / pf.block_tokens : 0;
    if (n > pf.bt_cols) n = pf.bt_cols;
    npg[b] = n;
    total += n;
  }
  if (total > pf.max_blocks) total = pf.max_blocks;
  const int lo = (int)((long long)total * cta / nb), hi = (int)((long long)total * (cta + 1) / nb);
  int b = 0, base = 0;
  for (int i = lo; i < hi; ++i) {
    while (b < pf.streams && i >= base + npg[b]) base += npg[b++];
    if (b >= pf.streams) break;
    const int blk = pf.bt[(long long)b * pf.bt_stride + (i - base)];
    if (blk >= 0 && (unsigned long long)blk < pf.kv_blocks) l2_prefetch_bulk(pf.kv + (unsigned long long)blk * pf.block_bytes, pf.block_bytes);
  }
}

// ---- host: tensor-map encoding through the driver entry point (no libcuda link needed) ----
int encode_u8_2d(CUtensorMap* map, const void* base, uint64_t cols_bytes, uint64_t rows, uint64_t row_stride_bytes,
                 uint32_t box_cols, uint32_t box_rows, bool swizzle128);
// u8 2-D map, box rows of `swizzle_bytes` (32, 64 or 128) with that swizzle: 16-byte unit u of a row at byte
// address A lands at unit u ^ ((A >> 7) & (swizzle_bytes / 16 - 1)).
int encode_u8_2d_swz(CUtensorMap* map, const void* base, uint64_t cols_bytes, uint64_t rows, uint64_t row_stride_bytes,
                     uint32_t box_rows, int swizzle_bytes);
// bf16 4-D map (dims innermost first, strides in bytes for dims 1..3), 128-byte swizzle.
int encode_bf16_4d(CUtensorMap* map, const void* base, const uint64_t dims[4], const uint64_t strides_bytes[3],
                   const uint32_t box[4]);
// u8 3-D map (dims innermost first, strides in bytes for dims 1..2), optional 128-byte swizzle.
int encode_u8_3d(CUtensorMap* map, const void* base, const uint64_t dims[3], const uint64_t strides_bytes[2],
                 const uint32_t box[3], bool swizzle128);
// bf16 5-D map (dims innermost first, strides in bytes for dims 1..4), 128-byte swizzle.
int encode_bf16_5d(CUtensorMap* map, const void* base, const uint64_t dims[5], const uint64_t strides_bytes[4],
                   const uint32_t box[5]);

}  // namespace flint
