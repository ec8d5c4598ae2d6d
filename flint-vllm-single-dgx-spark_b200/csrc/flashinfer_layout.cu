// FlashInfer W4A16 NVFP4 expert tensors -> the ModelOpt NVFP4 layout the decode kernels read.
//
// The Flint PR prepares its grouped (prefill) MoE weights for FlashInfer's SM100 NVFP4-weight GEMMs with
// prepare_weights (vllm/models/flint/ops/moe_cute.py, patch:4061-4091):
//   gate/up rows  ModelOpt [gate; up] (2I rows) -> per 128-row block b: up rows 64 b .. 64 b + 63, then gate rows
//                 64 b .. 64 b + 63 (codes and block scales alike);
//   block scales  bytes [E][rows][groups] (groups = K/16, after that row order) stored as
//                 [E][rows/128][groups/4][32][4][4]: byte (r, g) at [r/128][g/4][r%32][(r%128)/32][g%4];
//   down          codes unchanged, scales in the same 6-D order.
// This file inverts that: ModelOpt row r of gate/up comes from interleaved row ((r mod I) / 64) 128 + (r < I ? 64 :
// 0) + r mod 64, and every scale byte from its 6-D place.  Pure byte moves (bit-exact); one-time weight preparation,
// (K/2 + K/16) B read and written per row.  Codes: one thread per 16-byte unit of a row; scales: one per byte.
#include "common.cuh"
#include "runtime.cuh"

namespace flint {

constexpr int kFlThreads = 256;

// ModelOpt gate/up row r (of 2I) -> the interleaved row holding it
__device__ __forceinline__ int fl_gateup_row(int r, int I) {
  const int gate = r < I, v = gate ? r : r - I;
  return (v >> 6) * 128 + (gate ? 64 : 0) + (v & 63);
}

// codes: out[e][r][:] = in[e][interleave ? fl_gateup_row(r) : r][:], rows of `units` 16-byte units
__global__ void __launch_bounds__(kFlThreads)
fl_codes_kernel(const uint4* __restrict__ in, uint4* __restrict__ out, long long total, int rows, int units, int I,
                int interleave) {
  pdl_wait();
  for (long long i = (long long)blockIdx.x * kFlThreads + threadIdx.x; i < total; i += (long long)gridDim.x * kFlThreads) {
    const long long row = i / units;                               // e * rows + r
    const int u = (int)(i - row * units), r = (int)(row % rows);
    const long long e = row / rows;
    const int src = interleave ? fl_gateup_row(r, I) : r;
    out[i] = in[(e * rows + src) * units + u];
  }
  pdl_trigger();
}

// scales: out[e][r][g] = phys[e][sr/128][g/4][sr%32][(sr%128)/32][g%4], sr the source row
__global__ void __launch_bounds__(kFlThreads)
fl_scales_kernel(const uint8_t* __restrict__ phys, uint8_t* __restrict__ out, long long total, int rows, int groups,
                 int I, int interleave) {
  pdl_wait();
  const int mt = rows / 128, kt = groups / 4;
  for (long long i = (long long)blockIdx.x * kFlThreads + threadIdx.x; i < total; i += (long long)gridDim.x * kFlThreads) {
    const long long row = i / groups;
    const int g = (int)(i - row * groups), r = (int)(row % rows);
    const long long e = row / rows;
    const int sr = interleave ? fl_gateup_row(r, I) : r;
    const long long src = ((((e * mt + sr / 128) * kt + g / 4) * 32 + (sr & 31)) * 4 + ((sr & 127) >> 5)) * 4 + (g & 3);
    out[i] = phys[src];
  }
  pdl_trigger();
}

static unsigned fl_grid(long long total) {
  const long long per = (long long)num_sms() * 8;                 // a few waves of 256 threads per SM
  const long long need = (total + kFlThreads - 1) / kFlThreads;
  return (unsigned)(need < per ? (need > 0 ? need : 1) : per);
}

}  // namespace flint

extern "C" int flint_flashinfer_nvfp4_unpack(const void* w1, const void* w1_sf, const void* w2, const void* w2_sf,
                                             int64_t E, int64_t H, int64_t I, void* w13_out, void* s13_out,
                                             void* w2_out, void* s2_out, int pdl, void* stream) {
  using namespace flint;
  if (!w1 || !w1_sf || !w2 || !w2_sf || !w13_out || !s13_out || !w2_out || !s2_out) return FLINT_ERR_ARGUMENT;
  if (E < 1 || E > 65535 || H < 128 || H % 128 != 0 || I < 64 || I % 64 != 0 || H > (1 << 16) || I > (1 << 16))
    return FLINT_ERR_SHAPE;                                       // 2I and H rows in 128-row blocks, K/16 in 4s
  if (!aligned(w1, 16) || !aligned(w2, 16) || !aligned(w13_out, 16) || !aligned(w2_out, 16)) return FLINT_ERR_ALIGN;
  if (num_sms() <= 0) return FLINT_ERR_DEVICE;
  const int r13 = (int)(2 * I), r2 = (int)H, u13 = (int)(H / 32), u2 = (int)(I / 32), g13 = (int)(H / 16),
            g2 = (int)(I / 16);
  const long long c13 = E * r13 * (long long)u13, c2 = E * r2 * (long long)u2;
  const long long s13 = E * r13 * (long long)g13, s2 = E * r2 * (long long)g2;
  int rc = launch(fl_codes_kernel, dim3(fl_grid(c13)), dim3(kFlThreads), 0, stream, pdl, (const uint4*)w1,
                  (uint4*)w13_out, c13, r13, u13, (int)I, 1);
  if (!rc) rc = launch(fl_scales_kernel, dim3(fl_grid(s13)), dim3(kFlThreads), 0, stream, pdl, (const uint8_t*)w1_sf,
                       (uint8_t*)s13_out, s13, r13, g13, (int)I, 1);
  if (!rc) rc = launch(fl_codes_kernel, dim3(fl_grid(c2)), dim3(kFlThreads), 0, stream, pdl, (const uint4*)w2,
                       (uint4*)w2_out, c2, r2, u2, (int)I, 0);
  if (!rc) rc = launch(fl_scales_kernel, dim3(fl_grid(s2)), dim3(kFlThreads), 0, stream, pdl, (const uint8_t*)w2_sf,
                       (uint8_t*)s2_out, s2, r2, g2, (int)I, 0);
  return rc;
}
