// Peer exchange buffers of the multi-GPU decode (one process per GPU).
//
// Every rank owns one buffer (cudaMalloc'd, zero-filled) and maps every other rank's buffer into its address space
// through CUDA IPC, so a kernel can store into a peer's buffer over NVLink and raise a flag there.  Layout (bytes):
//
//   [0, 256)            PeerHeader: launch epochs of the two exchanges, sticky status
//   [256, 4352)         MoE flags u32 [128 down blocks][8 source ranks]: epoch of the last rows received
//   [4352, 4384)        head flags u32 [8 source ranks]
//   [4608, 5632)        head keys u64 [2 parities][8 source ranks][8 rows]
//   [8192, 8192+32H)    MoE rows bf16 [2 parities][8 slots][H]
//   [4384, 4416)        data-parallel token flags u32 [8 source ranks]
//   [4416, 4448)        data-parallel row flags u32 [8 source ranks]
//   [8192+32H, +64H)    data-parallel tokens bf16 [2 parities][8 source ranks][2 rows: attention output, residual][H]
//   [8192+96H, +256H)   data-parallel rows bf16 [2 parities][8 source ranks][8 slots][H] (the routes of this rank's
//                       token that the source rank computed)
//
// Protocol (both exchanges): the writer stores its data into every rank's buffer (its own included), fences at
// system scope, then stores the launch epoch into its flag slot on every rank with a release store; the reader
// polls its own flags with acquire loads until every source shows the epoch.  Every rank signals and waits on every
// rank at every launch, so no rank gets more than one launch ahead of another; the data regions alternate between
// two parities by epoch, so a rank one launch ahead never overwrites rows a slower rank is still reading.  Epochs
// are counted on the device (each launch reads the header's epoch and its last block advances it by one), so
// captured CUDA graphs replay the protocol unchanged.  Waits are bounded in time; a wait that runs out records
// STATUS_PEER_TIMEOUT in the header, and later launches on that rank skip their waits (their outputs are then
// garbage and the host must read the status).
#pragma once
#include "common.cuh"

namespace flint {

constexpr int kPeerMax = 8;
constexpr int kPeerMoeBlocks = 128;               // MoE down blocks (H / 16 at H = 2048)
constexpr size_t kPeerMoeFlagsOff = 256;
constexpr size_t kPeerHeadFlagsOff = kPeerMoeFlagsOff + (size_t)kPeerMoeBlocks * kPeerMax * 4;
constexpr size_t kPeerHeadKeysOff = 4608;
constexpr size_t kPeerMoeRowsOff = 8192;
constexpr int kPeerSlots = 8;
constexpr size_t kPeerDpTokFlagsOff = 4384;
constexpr size_t kPeerDpRowFlagsOff = 4416;
constexpr int kPeerRowsMax = 8;                   // head rows (tokens) per exchange
constexpr unsigned long long kPeerWaitNs = 10ull * 1000 * 1000 * 1000;   // 10 s
enum : unsigned { STATUS_PEER_TIMEOUT = 4u };

static_assert(kPeerHeadFlagsOff + kPeerMax * 4 <= kPeerHeadKeysOff, "peer layout");
static_assert(kPeerHeadKeysOff + 2 * kPeerMax * kPeerRowsMax * 8 <= kPeerMoeRowsOff, "peer layout");
static_assert(kPeerHeadFlagsOff + kPeerMax * 4 <= kPeerDpTokFlagsOff && kPeerDpRowFlagsOff + kPeerMax * 4 <= kPeerHeadKeysOff,
              "peer layout");

struct PeerHeader {
  unsigned moe_epoch;
  unsigned head_epoch;
  unsigned status;
  unsigned dp_tok_epoch;                          // data-parallel token gather launches
  unsigned dp_row_epoch;                          // data-parallel row scatter launches
  unsigned pad[59];
};

struct PeerSet {
  uint8_t* base[kPeerMax];                        // base[r]: rank r's buffer as mapped in this process
  int rank, world;
};

// Host: validates and packs the per-rank buffer pointers of one exchange (FLINT_OK or an error code).
int peer_set(const void* const* peers, int rank, int world, PeerSet* ps);

__host__ __device__ constexpr size_t peer_dp_tok_off(int H) { return kPeerMoeRowsOff + (size_t)2 * kPeerSlots * H * 2; }
__host__ __device__ constexpr size_t peer_dp_row_off(int H) { return peer_dp_tok_off(H) + (size_t)2 * kPeerMax * 2 * H * 2; }
__host__ __device__ constexpr size_t peer_buffer_bytes(int H) {
  return peer_dp_row_off(H) + (size_t)2 * kPeerMax * kPeerSlots * H * 2;
}

__device__ __forceinline__ PeerHeader* peer_header(uint8_t* b) { return reinterpret_cast<PeerHeader*>(b); }
__device__ __forceinline__ unsigned* peer_moe_flags(uint8_t* b) { return reinterpret_cast<unsigned*>(b + kPeerMoeFlagsOff); }
__device__ __forceinline__ unsigned* peer_head_flags(uint8_t* b) { return reinterpret_cast<unsigned*>(b + kPeerHeadFlagsOff); }
__device__ __forceinline__ unsigned long long* peer_head_keys(uint8_t* b, unsigned parity) {
  return reinterpret_cast<unsigned long long*>(b + kPeerHeadKeysOff) + (size_t)parity * kPeerMax * kPeerRowsMax;
}
__device__ __forceinline__ bf16* peer_moe_rows(uint8_t* b, unsigned parity, int H) {
  return reinterpret_cast<bf16*>(b + kPeerMoeRowsOff) + (size_t)parity * kPeerSlots * H;
}
__device__ __forceinline__ bf16* peer_dp_tokens(uint8_t* b, unsigned parity, int H) {   // [8 src][2][H]
  return reinterpret_cast<bf16*>(b + peer_dp_tok_off(H)) + (size_t)parity * kPeerMax * 2 * H;
}
__device__ __forceinline__ bf16* peer_dp_rows(uint8_t* b, unsigned parity, int H) {     // [8 src][8 slots][H]
  return reinterpret_cast<bf16*>(b + peer_dp_row_off(H)) + (size_t)parity * kPeerMax * kPeerSlots * H;
}

__device__ __forceinline__ void st_release_sys_u32(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned ld_relaxed_sys_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned peer_pack_bf16x2(float lo, float hi) {
  return (unsigned)__bfloat16_as_ushort(__float2bfloat16_rn(lo)) |
         ((unsigned)__bfloat16_as_ushort(__float2bfloat16_rn(hi)) << 16);
}
// Received rows are read around L1 (peers wrote them into this GPU's L2).
__device__ __forceinline__ float peer_ldcg_bf16(const bf16* p) {
  return __bfloat162float(__ushort_as_bfloat16(__ldcg(reinterpret_cast<const unsigned short*>(p))));
}

// Poll *flag until it reaches `epoch` (wrap-safe), at most kPeerWaitNs; false (and the sticky status) on time-out.
__device__ __forceinline__ bool peer_wait(const unsigned* flag, unsigned epoch, PeerHeader* own) {
  if (ld_relaxed_sys_u32(&own->status) & STATUS_PEER_TIMEOUT) return false;
  const unsigned long long t0 = global_ns();
  unsigned i = 0;
#pragma unroll 1
  while ((int)(ld_acquire_sys_u32(flag) - epoch) < 0) {
    if ((++i & 255u) == 0 && (global_ns() - t0 > kPeerWaitNs || i > (1u << 30))) {
      atomicOr(&own->status, STATUS_PEER_TIMEOUT);
      return false;
    }
  }
  return true;
}

}  // namespace flint
