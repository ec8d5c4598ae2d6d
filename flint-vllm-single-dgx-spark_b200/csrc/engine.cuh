// Tile-streaming engine shared by the NVFP4 GEMV kernels (MoE gate/up and down, attention QKV and O projections).
//
// A CTA has NW consumer warps and one TMA producer warp (warp NW).  It processes a list of tiles; a tile is
// (NW*16 weight rows) x (nks 256-k slices), fetched as one stage per slice.  A stage is NBOX boxes of BOXROWS rows
// (NBOX*BOXROWS = NW*16), so a tile may pair rows from two places of a matrix (gate rows with the matching up rows).
// Stages flow through an NS-deep shared-memory ring guarded by full/empty mbarriers; the producer runs ahead by up to
// NS stages across tile boundaries.  After the last slice of a tile every consumer warp writes its fp32 16 x 8
// accumulator fragment to a shared tile buffer, the consumer warps synchronise on a named barrier and the plan's
// epilogue runs on the completed tile (all consumer threads), followed by a second named barrier.
//
// Plan interface (device):
//   int  ntiles() const;                                  tiles of this CTA
//   int  nks() const;                                     slices per tile
//   void box(int tile, int b, int& y) const;              first matrix row of box b of the tile
//   const CUtensorMap* map_codes() / map_scales() const;
//   const __half* xrow(int tile, int n, bool& active) const;   staged activation row of mma column n
//   int  kslice0(int tile) const;                         first slice index (for split-K plans; usually 0)
//   void epilogue(int tile, const float* dt, int tid, int nthreads);   dt[row * 8 + n], row in [0, NW*16)
#pragma once
#include "nvfp4_tile.cuh"

namespace flint {

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

template <int NW, int NS, int BOXROWS>
struct EngineSmem {
  static constexpr int ROWS = NW * 16;
  static constexpr int NBOX = ROWS / BOXROWS;
  static constexpr int code_bytes = ROWS * 128;
  static constexpr int scale_bytes = ROWS * 16;
  static constexpr int ring_bytes = NS * (code_bytes + scale_bytes);
  static constexpr int dtile_bytes = ROWS * 8 * 4;
  static_assert(NBOX * BOXROWS == ROWS, "boxes must tile the stage");
  static_assert((BOXROWS * 128) % 1024 == 0, "128B-swizzled boxes need 1024-byte aligned destinations");
};

// Producer half: warp NW, lane 0 issues every stage of the plan (may run before the PDL wait when the weights do not
// depend on the previous kernel).
template <int NW, int NS, int BOXROWS, class Plan>
__device__ __forceinline__ void engine_produce(const Plan& plan, uint8_t* smem, uint64_t* bars, unsigned* status) {
  using L = EngineSmem<NW, NS, BOXROWS>;
  uint64_t* full = bars;
  uint64_t* empty = bars + NS;
  const int total = plan.ntiles() * plan.nks();
  if ((threadIdx.x & 31) != 0 || total == 0) return;
  tma_prefetch_desc(plan.map_codes());
  tma_prefetch_desc(plan.map_scales());
  const int nks = plan.nks();
  int tile = 0, ks = 0, slot = 0;
  unsigned phase = 0;
  for (int s = 0; s < total; ++s) {
    if (s >= NS && !mbar_wait(&empty[slot], phase ^ 1u, status)) break;
    mbar_arrive_expect_tx(&full[slot], L::code_bytes + L::scale_bytes);
    const int kx = plan.kslice0(tile) + ks;
#pragma unroll
    for (int b = 0; b < L::NBOX; ++b) {
      int y;
      plan.box(tile, b, y);
      tma_load_2d(smem + slot * L::code_bytes + b * BOXROWS * 128, plan.map_codes(), kx * 128, y, &full[slot]);
      tma_load_2d(smem + NS * L::code_bytes + slot * L::scale_bytes + b * BOXROWS * 16, plan.map_scales(), kx * 16, y,
                  &full[slot]);
    }
    if (++ks == nks) { ks = 0; ++tile; }
    if (++slot == NS) { slot = 0; phase ^= 1u; }
  }
}

// Consumer half: warps 0..NW-1.  dtile: shared fp32 buffer of ROWS*8 floats.  Uses named barrier 1.
template <int NW, int NS, int BOXROWS, class Plan>
__device__ __forceinline__ void engine_consume(Plan& plan, uint8_t* smem, float* dtile, uint64_t* bars, unsigned* status) {
  using L = EngineSmem<NW, NS, BOXROWS>;
  uint64_t* full = bars;
  uint64_t* empty = bars + NS;
  uint8_t* ring_codes = smem;
  uint8_t* ring_scales = smem + NS * L::code_bytes;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int ntiles = plan.ntiles(), nks = plan.nks();
  const int g = lane >> 2, t = lane & 3;
  const int prow = 16 * warp + tile_phi(g);
  int slot = 0;
  unsigned phase = 0;
  bool ok = true;
  for (int tile = 0; tile < ntiles; ++tile) {
    bool active;
    const __half* xrow = plan.xrow(tile, g, active);
    float acc[4][4];
    zero_acc(acc);
    const int ks0 = plan.kslice0(tile);
    for (int ks = 0; ks < nks; ++ks) {
      if (ok && !mbar_wait(&full[slot], phase, status)) ok = false;
      if (ok)
        consume_stage(ring_codes + slot * L::code_bytes, ring_scales + slot * L::scale_bytes, warp, g, t, ks0 + ks, xrow,
                      active, acc);
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
      if (++slot == NS) { slot = 0; phase ^= 1u; }
    }
    float d[4];
    sum_acc(acc, d);
    dtile[prow * 8 + 2 * t] = d[0];
    dtile[prow * 8 + 2 * t + 1] = d[1];
    dtile[(prow + 8) * 8 + 2 * t] = d[2];
    dtile[(prow + 8) * 8 + 2 * t + 1] = d[3];
    named_bar_sync(1, NW * 32);
    plan.epilogue(tile, dtile, threadIdx.x, NW * 32);
    named_bar_sync(1, NW * 32);
  }
}

// ---- thread-block cluster split-K ----------------------------------------------------------------------------
// CL CTAs of a cluster stream disjoint K ranges of the same tile.  Ranks 1..CL-1 push their fp32 partial tile into
// rank 0's shared memory (pslot[rank-1], distributed shared memory stores) and arrive on rank 0's cluster mbarrier;
// rank 0 adds the partials to its own in rank order (deterministic) and runs the epilogue.  One tile per cluster.
__device__ __forceinline__ unsigned cluster_rank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t mapa_shared(const void* p, unsigned rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_f32x2(uint32_t addr, float a, float b) {
  asm volatile("st.shared::cluster.v2.f32 [%0], {%1, %2};" ::"r"(addr), "f"(a), "f"(b) : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, unsigned parity) {
  uint32_t ok;
  asm volatile(
      "{\n.reg .pred p;\n"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n"
      "selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Consumer half for a cluster split-K plan with at most one tile per CTA.  pslot: rank 0's buffer of (CL-1)*ROWS*8
// floats; clbar: rank 0's mbarrier (initialised with count CL-1 before the kernel's opening cluster barrier).
template <int NW, int NS, int BOXROWS, int CL, class Plan>
__device__ __forceinline__ void engine_consume_cluster(Plan& plan, uint8_t* smem, float* dtile, float* pslot, uint64_t* clbar,
                                                       uint64_t* bars, unsigned* status) {
  using L = EngineSmem<NW, NS, BOXROWS>;
  uint64_t* full = bars;
  uint64_t* empty = bars + NS;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int prow = 16 * warp + tile_phi(g);
  const unsigned rank = cluster_rank();
  if (plan.ntiles() == 0) return;
  bool active;
  const __half* xrow = plan.xrow(0, g, active);
  float acc[4][4];
  zero_acc(acc);
  const int ks0 = plan.kslice0(0), nks = plan.nks();
  int slot = 0;
  unsigned phase = 0;
  bool ok = true;
  for (int ks = 0; ks < nks; ++ks) {
    if (ok && !mbar_wait(&full[slot], phase, status)) ok = false;
    if (ok)
      consume_stage(smem + slot * L::code_bytes, smem + NS * L::code_bytes + slot * L::scale_bytes, warp, g, t, ks0 + ks,
                    xrow, active, acc);
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[slot]);
    if (++slot == NS) { slot = 0; phase ^= 1u; }
  }
  float d[4];
  sum_acc(acc, d);
  if (rank != 0) {
    float* base = pslot + (rank - 1) * L::ROWS * 8;
    st_cluster_f32x2(mapa_shared(base + prow * 8 + 2 * t, 0), d[0], d[1]);
    st_cluster_f32x2(mapa_shared(base + (prow + 8) * 8 + 2 * t, 0), d[2], d[3]);
    asm volatile("fence.acq_rel.cluster;" ::: "memory");
    named_bar_sync(1, NW * 32);
    if (threadIdx.x == 0) mbar_arrive_remote(mapa_shared(clbar, 0));
    return;
  }
  bool got = true;
  if (CL > 1) {
    got = false;
    for (unsigned i = 0; i < FLINT_WAIT_LIMIT && !got; ++i) got = mbar_try_wait_cluster(clbar, 0);
    if (!got && threadIdx.x == 0) atomicOr(status, STATUS_WAIT_TIMEOUT);
  }
#pragma unroll
  for (int r = 1; r < CL; ++r) {
    const float* base = pslot + (r - 1) * L::ROWS * 8;
    if (got) {
      d[0] += base[prow * 8 + 2 * t];
      d[1] += base[prow * 8 + 2 * t + 1];
      d[2] += base[(prow + 8) * 8 + 2 * t];
      d[3] += base[(prow + 8) * 8 + 2 * t + 1];
    }
  }
  dtile[prow * 8 + 2 * t] = d[0];
  dtile[prow * 8 + 2 * t + 1] = d[1];
  dtile[(prow + 8) * 8 + 2 * t] = d[2];
  dtile[(prow + 8) * 8 + 2 * t + 1] = d[3];
  named_bar_sync(1, NW * 32);
  plan.epilogue(0, dtile, threadIdx.x, NW * 32);
}

// mbarrier initialisation for the engine (thread 0), followed by a CTA barrier.
template <int NW, int NS>
__device__ __forceinline__ void engine_init_bars(uint64_t* bars) {
  if (threadIdx.x == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&bars[i], 1);
      mbar_init(&bars[NS + i], NW);
    }
    fence_mbar_init();
  }
  __syncthreads();
}

}  // namespace flint
