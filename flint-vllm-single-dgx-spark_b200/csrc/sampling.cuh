// Seeded top-k -> top-p -> draw for the LM head (one warp per token row).
//
// Contract (the reference hands its fp32 logits to vLLM's sampler, fast/fast_head.py:360-381, whose draw is not
// reproducible outside vLLM; this library defines its own seeded rule and the CPU checker restates it):
//   1. candidates: the top_k logits by (value desc, index asc), 1 <= top_k <= 32;  c_0 >= c_1 >= ...
//   2. w_i = expf((c_i - c_0) / T) in fp32;
//   3. top-p as vLLM applies it (ascending cumulative probability <= 1 - p is dropped, the best is always kept):
//      S_j = w_{k-1} + ... + w_j summed from the smallest up; candidate j >= 1 is kept iff S_j > (1 - p) * S_0;
//      the kept set is the prefix 0..J-1;
//   4. u = (philox4x32_10(counter = {step, row, 0, 0}, key = {seed lo, seed hi}).x >> 8) * 2^-24, in [0, 1);
//      C_i = w_0 + ... + w_i summed upward; the token is the first i < J with C_i > u * C_{J-1} (J-1 if none).
//
// Selection is exact (ties -> lowest index) in two levels.  Each CTA writes the logits of its rows, then selects
// its own top_k: the top_k-th largest of the 32 lane maxima bounds the CTA's top_k-th value from below, so only
// keys at or above it are compacted into shared memory and ranked.  The last CTA bounds the global top_k-th value
// the same way from the CTA maxima (each CTA list is sorted, its first entry is the CTA maximum), compacts the
// candidates at or above that bound and ranks them.
#pragma once
#include "common.cuh"

namespace flint {

constexpr int kSampleMaxK = 32;
constexpr int kSampleMaxCtas = 160;
constexpr int kSampleSurvivors = 1024;      // shared-memory candidate buffer per token row (keys)

// Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random numbers: as easy as 1, 2, 3", SC'11): ten rounds
// of two 32x32->64 multiplies, the key bumped by the Weyl constants between rounds.
__device__ __forceinline__ void philox4x32_10(uint32_t c[4], uint32_t k0, uint32_t k1) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r) {
      k0 += 0x9E3779B9u;
      k1 += 0xBB67AE85u;
    }
    const uint32_t lo0 = 0xD2511F53u * c[0], hi0 = __umulhi(0xD2511F53u, c[0]);
    const uint32_t lo1 = 0xCD9E8D57u * c[2], hi1 = __umulhi(0xCD9E8D57u, c[2]);
    const uint32_t n0 = hi1 ^ c[1] ^ k0, n2 = hi0 ^ c[3] ^ k1;
    c[0] = n0;
    c[1] = lo1;
    c[2] = n2;
    c[3] = lo0;
  }
}

__device__ __forceinline__ float sample_uniform(unsigned long long seed, uint32_t step, uint32_t row) {
  uint32_t c[4] = {step, row, 0u, 0u};
  philox4x32_10(c, (uint32_t)seed, (uint32_t)(seed >> 32));
  return (float)(c[0] >> 8) * 0x1p-24f;
}

__device__ __forceinline__ unsigned long long shfl_u64(unsigned long long v, int src) {
  const uint32_t lo = __shfl_sync(0xffffffffu, (uint32_t)v, src);
  const uint32_t hi = __shfl_sync(0xffffffffu, (uint32_t)(v >> 32), src);
  return ((unsigned long long)hi << 32) | lo;
}

__device__ __forceinline__ unsigned long long warp_max_u64(unsigned long long v) {
  const uint32_t hi = __reduce_max_sync(0xffffffffu, (uint32_t)(v >> 32));
  const uint32_t lo = __reduce_max_sync(0xffffffffu, (uint32_t)(v >> 32) == hi ? (uint32_t)v : 0u);
  return ((unsigned long long)hi << 32) | lo;
}

// K-th largest (1 <= K <= 32) of the 32 lane values; every lane gets it.  Non-zero keys are distinct.
__device__ __forceinline__ unsigned long long warp_kth_largest(unsigned long long v, int K) {
  int gt = 0, ge = 0;
#pragma unroll 8
  for (int j = 0; j < 32; ++j) {
    const unsigned long long o = shfl_u64(v, j);
    gt += o > v;
    ge += o >= v;
  }
  return warp_max_u64((gt < K && ge >= K) ? v : 0ull);
}

// Top K (sorted, descending; zero-padded) of n distinct non-zero keys held in shared memory; one warp.
__device__ __forceinline__ void warp_select_sorted(const unsigned long long* buf, int n, int K, unsigned long long* out,
                                                   int lane) {
  if (n <= 64) {           // rank each candidate against all others
    for (int i = lane; i < K; i += 32)
      if (i >= n) out[i] = 0ull;
    for (int i = lane; i < n; i += 32) {
      const unsigned long long v = buf[i];
      int rank = 0;
      for (int j = 0; j < n; ++j) rank += buf[j] > v;
      if (rank < K) out[rank] = v;
    }
  } else {                 // K rounds of "largest below the previous pick"
    unsigned long long ceil = ~0ull;
    for (int r = 0; r < K; ++r) {
      unsigned long long best = 0ull;
      for (int i = lane; i < n; i += 32) {
        const unsigned long long v = buf[i];
        if (v < ceil && v > best) best = v;
      }
      best = warp_max_u64(best);
      if (lane == 0) out[r] = best;
      ceil = best;
    }
  }
  __syncwarp();
}

// Compact the keys >= T (and non-zero) of one lane-strided pass into buf; returns the count (may exceed cap, in
// which case only the first cap were stored).
__device__ __forceinline__ int warp_compact_ge(unsigned long long key, unsigned long long T, unsigned long long* buf,
                                               int base, int cap, int lane) {
  const bool pred = key != 0ull && key >= T;
  const unsigned b = __ballot_sync(0xffffffffu, pred);
  if (pred) {
    const int pos = base + __popc(b & ((1u << lane) - 1u));
    if (pos < cap) buf[pos] = key;
  }
  return base + __popc(b);
}

// The sampling rule (steps 2-4 of the contract) on the sorted candidates top[0..K) of one row; lane 0 returns the
// chosen position and the kept count; w is K floats of shared scratch.
__device__ __forceinline__ int sample_sorted(const unsigned long long* top, int K, float temperature, float top_p,
                                             float u, float* w, int lane, int* kept) {
  int Kv = 0;
  for (int i = 0; i < K; ++i) Kv += top[i] != 0ull;
  const float c0 = argmax_key_value(top[0]);
  if (lane < Kv) w[lane] = expf((argmax_key_value(top[lane]) - c0) / temperature);
  __syncwarp();
  int pick = 0, J = 1;
  if (lane == 0 && Kv > 0) {
    float S[kSampleMaxK];
    float s = 0.f;
    for (int j = Kv - 1; j >= 0; --j) {
      s += w[j];
      S[j] = s;
    }
    const float thr = (1.0f - top_p) * S[0];
    while (J < Kv && S[J] > thr) ++J;
    float P = 0.f;
    for (int i = 0; i < J; ++i) P += w[i];
    const float target = u * P;
    float C = 0.f;
    pick = J - 1;
    for (int i = 0; i < J; ++i) {
      C += w[i];
      if (C > target) {
        pick = i;
        break;
      }
    }
  }
  *kept = J;
  return pick;
}

}  // namespace flint
