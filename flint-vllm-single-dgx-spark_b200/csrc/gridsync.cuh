// Grid-wide barrier for persistent (cooperatively launched) kernels.
//
// A monotonic arrival counter: barrier k of a launch completes when the counter reaches (k + 1) * nblocks.  Each
// CTA's thread 0 adds 1 with a release reduction (no return value) and polls the counter with acquire loads; the
// CTA's other participating threads wait on a named barrier on both sides, which orders their memory operations
// with thread 0's release / acquire (both are cumulative), so no separate fences are needed.  Polls are bounded: after FLINT_WAIT_LIMIT polls the
// CTA records STATUS_WAIT_TIMEOUT and stops waiting.  At the end of a launch every CTA calls grid_sync_retire; the
// last one to do so zeroes the counter for the next launch (all CTAs have finished polling by then).
#pragma once
#include "tma.cuh"

namespace flint {

struct GridSync {
  unsigned count;
  unsigned retired;
  unsigned pad[30];
};

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Called by threads [0, nthreads) of every CTA (thread 0 among them); k = barrier index within the launch.
// Returns false (on every participating thread) if this CTA timed out.
__device__ __forceinline__ bool grid_sync(GridSync* gs, unsigned nblocks, unsigned k, int nthreads, int bar, int* s_ok,
                                          unsigned* status) {
  asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthreads) : "memory");
  if (threadIdx.x == 0) {
    int ok = 1;
    asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(&gs->count) : "memory");
    const unsigned target = (k + 1) * nblocks;
    unsigned i = 0;
#pragma unroll 1
    while ((int)(ld_acquire_u32(&gs->count) - target) < 0) {
      if (++i > FLINT_WAIT_LIMIT) {
        atomicOr(status, STATUS_WAIT_TIMEOUT);
        ok = 0;
        break;
      }
    }
    *s_ok = ok;
  }
  asm volatile("bar.sync %0, %1;" ::"r"(bar), "r"(nthreads) : "memory");
  return *s_ok != 0;
}

// Thread 0 of every CTA, after its last grid_sync of the launch.  `bump`, `bump2` (optional): launch counters the
// last CTA increments (every CTA has read them by then).
__device__ __forceinline__ void grid_sync_retire(GridSync* gs, unsigned nblocks, unsigned* bump = nullptr,
                                                 unsigned* bump2 = nullptr) {
  if (threadIdx.x != 0) return;
  if (atomicAdd(&gs->retired, 1u) == nblocks - 1) {
    atomicExch(&gs->count, 0u);
    atomicExch(&gs->retired, 0u);
    if (bump) atomicAdd(bump, 1u);
    if (bump2) atomicAdd(bump2, 1u);
  }
}

}  // namespace flint
