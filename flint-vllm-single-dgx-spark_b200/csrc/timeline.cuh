// Development instrumentation, compiled out unless asked for:
//  * -DFLINT_TIMELINE: per-CTA %globaltimer stamps at named points of the block kernels, kept in a file-scope device
//    array of the kernel's .cu file and read back through that file's flint_timeline_<kernel> entry point (declared
//    only in such builds).  A stamp is one 64-bit store by one thread; it adds no barrier and skips no work.
//  * -DFLINT_POLL_SLEEP_NS=n: a __nanosleep(n) after every unsuccessful poll of a tagged word or counter, to trade a
//    little wake-up latency for less L2 polling traffic (0, the default: spin).
#pragma once

#ifndef FLINT_POLL_SLEEP_NS
#define FLINT_POLL_SLEEP_NS 0
#endif

namespace flint {

__device__ __forceinline__ void poll_pause() {
#if FLINT_POLL_SLEEP_NS > 0
  __nanosleep(FLINT_POLL_SLEEP_NS);
#endif
}

constexpr int kTlSlots = 32;         // stamps per CTA
constexpr int kTlCtas = 160;         // CTAs recorded (>= the SM count of a B200)

}  // namespace flint

#ifdef FLINT_TIMELINE
#define FLINT_TL_BUFFER static __device__ unsigned long long g_flint_tl[flint::kTlCtas * flint::kTlSlots];
#define FLINT_TL(i)                                                                           \
  do {                                                                                        \
    unsigned long long t_;                                                                    \
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t_));                                    \
    if (blockIdx.x < flint::kTlCtas) g_flint_tl[blockIdx.x * flint::kTlSlots + (i)] = t_;     \
  } while (0)
#define FLINT_TL_READER(name)                                                                 \
  extern "C" int name(unsigned long long* out) {                                              \
    return cudaMemcpyFromSymbol(out, g_flint_tl, sizeof(g_flint_tl)) == cudaSuccess ? 0 : 4;  \
  }
#else
#define FLINT_TL_BUFFER
#define FLINT_TL(i) \
  do {              \
  } while (0)
#define FLINT_TL_READER(name)
#endif
