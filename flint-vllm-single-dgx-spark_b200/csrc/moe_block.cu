// (1) MoE decode block for one token: router + top-k, NVFP4 gate/up GEMV + SwiGLU, NVFP4 down GEMV and the
// weighted expert sum in ONE cooperative launch (one CTA per SM, no grid barrier: the router logits and the
// activations cross between CTAs as epoch-tagged words, tagged.cuh).  Replaces the reference's
// route_norm_kernel -> up_mar -> down_mar chain (fast/fp4moe_mar.cu:311-417, 67-152, 157-233; driven by
// fast/model.py:302-310) at batch 1, where every routed expert is distinct (topk <= 8).
//
//  R  every CTA: s = x + res, xn = bf16(RMSNorm(s)) in one register pass (CTA 0 publishes res_out / xn); CTAs own
//     router rows e = cta, cta + grid (prefetched into registers before the PDL wait) and publish bf16 logits.
//  U  every CTA: top-k from the logits once all carry this launch's tag (redundant, identical everywhere).  The TMA producer then loads, in one go,
//     the CTA's share of the up work (units of 16 gate + 16 up rows x H, balanced over the CTAs) and its down block
//     (16 output rows of every routed expert) into shared memory; the down weights land while the up units run.
//     Per unit the 8 warps split K, the partial tiles are summed in warp order and act = bf16(silu(g) * u) is
//     published to the workspace.
//  D  CTA c < H/16, once the act rows of the routed slots carry this launch's tag: warp s computes y_s = bf16(act_s . W2[e_s] * gs2[e_s]) for the block's 16 rows (one 16-row
//     tile over all of I, the accumulation order of moe_down), then out = bf16(sum_s tw_s * y_s) in slot order.
//
// Routing, xn, res_out and the down step have the bits of flint_moe_route / flint_moe_down; the gate/up sums split
// K across warps, so act (and hence out) agrees with the chain to fp32 rounding, not bit for bit.
//
// Shared expert (Flint's ungated shared MLP, SI = its intermediate size, flint_moe_block_shared): its gate/up rows are
// extra up units after the routed ones (same 16 + 16-row units over all of H, so the work stays balanced over the
// CTAs), its activation row is published beside the routed ones, and in phase D a spare warp (topk < 8) computes the
// block's 16 shared output rows from its down block, loaded with the routed down blocks.  out = bf16(bf16(sum_s tw_s
// y_s) + y_shared) with y_shared = bf16(act_sh . W2sh * gs2sh): the PR's combine rule (patch:3391-3397) and the
// rounding of the chain (routed down, shared down, one bf16 add), replacing the GB10 kernels' shared groups inside
// up_mar / down_mar (fast/fp4moe_mar.cu:67-152, 224-231) -- one launch instead of three.
//
// Expert-parallel mode (y_out given): this rank holds experts [e_lo, e_hi) only; the router and top-k run in full
// (identical on every rank), only routed slots whose expert is local get up units and down rows, and instead of
// the weighted sum the kernel writes y[slot][H] (bf16 y_s for local slots, zero rows otherwise) and the routing
// weights; a sum over ranks (exact: one non-zero term per element) followed by flint_moe_combine gives the
// single-GPU output bit for bit.
//
// Peer mode (peers given): expert parallel with the exchange fused in.  After phase D, block c stores the 16 rows of
// each local slot straight into every rank's exchange buffer over NVLink (its own included), raises its flag (c, rank)
// on every rank, waits until all ranks' flags for block c show this launch, and computes out rows 16c..16c+15 =
// bf16(sum_s tw_s * y_s) in slot order from the received rows (exactly one rank owns each slot).  No collective
// library call, no zero rows, no extra launch; the output equals the single-GPU block bit for bit (peer.cuh has the
// protocol).
#include "gridsync.cuh"
#include "moe_common.cuh"
#include "peer.cuh"
#include "tagged.cuh"
#include "runtime.cuh"
#include "timeline.cuh"

#include <algorithm>

// phase stamps of development builds (-DFLINT_TIMELINE): 0 entry, 1 PDL wait done, 2 norm + router rows published,
// 3 top-k known, 4 up units done, 5 down rows done, 6 output written, 7 logits seen, 8 top-k computed (warp 0),
// 9 first up unit landed; producer: 10 plan received, 11 loads issued
FLINT_TL_BUFFER

namespace flint {

constexpr int kXW = 8;                  // consumer warps
constexpr int kXT = kXW * 32;
constexpr int kXMaxUnits = 3;           // up units (16 gate + 16 up rows) per CTA
constexpr int kXMaxSlots = 8;           // routed experts
constexpr int kXMaxShared = 1024;       // shared expert intermediate size (its act row is staged by one warp)

struct MoeBlockWs {
  GridSync sync;
  unsigned status;
  unsigned epoch;                       // launches so far: the tag of this launch's published words is epoch + 1
  unsigned pad[30];
  // followed by: logits as tagged words [E] (data = fp32 bits), act as tagged words [8][I / 2] (data = bf16 pair),
  // the shared expert's act as tagged words [kXMaxShared / 2]
};

struct MoeBlockArgs {
  const bf16* x;
  int64_t ldx;
  const bf16* res;
  const bf16* nw;
  float eps;
  const bf16* gate_w;
  int E, topk, score_fn, H, I;
  const float* g13;
  const float* g2;
  bf16* out;
  bf16* res_out;
  bf16* xn_out;
  float* logits_out;
  int* ids_out;
  float* tw_out;
  uint32_t unit_bytes, dslot_bytes, off_dn, off_xn, off_xs, off_xa, off_red;
  int e_lo, e_hi;                    // local experts (weights hold rows of experts e_lo .. e_hi-1 only)
  bf16* y_out;                       // expert-parallel mode: per-slot outputs [topk][H] (NULL: weighted sum to out)
  MoeBlockWs* ws;
  int peer_mode;                     // expert parallel with the fused peer exchange
  PeerSet peers;
  L2Prefetch pf;                     // the next op's bytes, pulled into L2 during phase D
  int SI;                            // shared expert intermediate size (0: none)
  const float* g13_sh;
  const float* g2_sh;
  uint32_t off_dn_sh, off_xa_sh;     // its down block and its staged act row in shared memory
};

static size_t moe_block_ws_bytes(int E, int I) {
  return sizeof(MoeBlockWs) + (size_t)E * 8 + (size_t)kXMaxSlots * (I / 2) * 8 + (size_t)(kXMaxShared / 2) * 8 + 256;
}

__device__ __forceinline__ void xsync() { asm volatile("bar.sync 1, %0;" ::"r"(kXT) : "memory"); }
__device__ __forceinline__ bool xsync_and(bool pred) {
  int r;
  asm volatile("{\n.reg .pred p, q;\nsetp.ne.s32 p, %1, 0;\nbar.red.and.pred q, 1, %2, p;\nselp.s32 %0, 1, 0, q;\n}"
               : "=r"(r) : "r"((int)pred), "r"(kXT) : "memory");
  return r != 0;
}

template <int NV>   // H / 256
__global__ void __launch_bounds__((kXW + 1) * 32, 1)
moe_block_kernel(const __grid_constant__ CUtensorMap up_c, const __grid_constant__ CUtensorMap up_s,
                 const __grid_constant__ CUtensorMap dn_c, const __grid_constant__ CUtensorMap dn_s,
                 const __grid_constant__ CUtensorMap sh_up_c, const __grid_constant__ CUtensorMap sh_up_s,
                 const __grid_constant__ CUtensorMap sh_dn_c, const __grid_constant__ CUtensorMap sh_dn_s,
                 const MoeBlockArgs a) {
  constexpr int H = NV * 256;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar_up[kXMaxUnits], bar_dn, bar_plan;
  __shared__ int s_ids[kXMaxSlots];
  __shared__ float s_tw[kXMaxSlots];
  __shared__ int shift_x[kMaxTokens], shift_a[kXMaxSlots];
  __shared__ float red_n[kXW * 8 + 8];
  __shared__ float ybuf[kXMaxSlots][16];
  __shared__ int s_local[kXMaxSlots], s_nlocal;
  __shared__ float ysh[16];
  __shared__ int shift_sh;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nb = gridDim.x, cta = blockIdx.x;
  const int E = a.E, I = a.I, topk = a.topk, SI = a.SI;
  if (tid == 0) FLINT_TL(0);
  const int nks_u = H / kSliceK, nks_d = I / kSliceK, jpe = I / 16, nks_sh = SI / kSliceK;
  const bool has_dn = cta < H / 16;
  // up units follow the local routed slots (known after top-k): unit u -> slot s_local[u / jpe], rows 16 (u % jpe);
  // then the shared expert's SI / 16 units
  auto unit_range = [&](int& u0, int& nu) {        // 32-bit: U <= 8 slots x I / 16 + SI / 16 units, cta < 2^16
    const unsigned U = (unsigned)(s_nlocal * jpe + SI / 16);
    u0 = (int)((unsigned)cta * U / (unsigned)nb);
    nu = (int)((unsigned)(cta + 1) * U / (unsigned)nb) - u0;
  };
  MoeBlockWs* ws = a.ws;
  unsigned* status = &ws->status;
  unsigned long long* lg = reinterpret_cast<unsigned long long*>(ws + 1);    // tagged logits
  unsigned long long* act_g = lg + E;                                         // tagged act pairs
  unsigned long long* act_sh = act_g + kXMaxSlots * (I / 2);                  // the shared expert's
  uint8_t* up_base = smem;                              // [unit][gate codes | up codes | gate scales | up scales]
  uint8_t* dn_base = smem + a.off_dn;                   // [slot][codes | scales]
  bf16* xnb = reinterpret_cast<bf16*>(smem + a.off_xn);
  __half* xs = reinterpret_cast<__half*>(smem + a.off_xs);
  __half* xa = reinterpret_cast<__half*>(smem + a.off_xa);
  float* red = reinterpret_cast<float*>(smem + a.off_red);   // [2][8 warps][16 rows][8 cols]

  if (tid == 0) {
    for (int i = 0; i < kXMaxUnits; ++i) mbar_init(&bar_up[i], 1);
    mbar_init(&bar_dn, 1);
    mbar_init(&bar_plan, 1);
    fence_mbar_init();
  }
  __syncthreads();

  // router rows of this CTA: e = cta (+ nb), one warp each, prefetched before the wait
  const int my_row = cta + warp * nb;
  const bool has_row = warp < 2 && my_row < E;
  uint4 wv[NV];
  if (has_row) {
    const uint4* wp = reinterpret_cast<const uint4*>(a.gate_w + (int64_t)my_row * H);
#pragma unroll
    for (int i = 0; i < NV; ++i) wv[i] = ldg_stream_v4(wp + lane + 32 * i);
  }
  // the next op's bytes (its weights, the KV pages it reads) into L2 while this kernel's routing runs: HBM is idle
  // until the expert weights are requested.  Only bytes no pending kernel writes are named here (the next layer's
  // weights and KV pages, block tables and sequence lengths are final before this step's first kernel).
  if (warp == kXW && lane == 0) l2_prefetch_share(a.pf, cta, nb);
  // the norm weights (this thread's 8) do not depend on the previous kernel either
  const uint4 nwc = tid < H / 8 ? reinterpret_cast<const uint4*>(a.nw)[tid] : make_uint4(0u, 0u, 0u, 0u);
  pdl_wait();
  if (tid == 0) FLINT_TL(1);

  if (warp == kXW) {
    // ---- producer: once the routing is known, this CTA's up units and down block ----
    if (lane == 0) {
      tma_prefetch_desc(&up_c);
      tma_prefetch_desc(&up_s);
      tma_prefetch_desc(&dn_c);
      tma_prefetch_desc(&dn_s);
      if (SI > 0) {
        tma_prefetch_desc(&sh_up_c);
        tma_prefetch_desc(&sh_up_s);
        tma_prefetch_desc(&sh_dn_c);
        tma_prefetch_desc(&sh_dn_s);
      }
      if (!mbar_wait(&bar_plan, 0, status)) return;
      FLINT_TL(10);
      int u0, nu;
      unit_range(u0, nu);
      const int routed_units = s_nlocal * jpe;
      for (int u = 0; u < nu; ++u) {
        const int unit = u0 + u;
        const bool shared = unit >= routed_units;
        int rows_g, rows_u;
        if (shared) {                                   // shared expert: gate rows [0, SI), up rows [SI, 2 SI)
          rows_g = (unit - routed_units) * 16;
          rows_u = rows_g + SI;
        } else {
          const int s = s_local[unit / jpe], j = unit - (unit / jpe) * jpe;
          rows_g = (s_ids[s] - a.e_lo) * 2 * I + j * 16;
          rows_u = rows_g + I;
        }
        const CUtensorMap* mc = shared ? &sh_up_c : &up_c;
        const CUtensorMap* ms = shared ? &sh_up_s : &up_s;
        uint8_t* b = up_base + u * a.unit_bytes;
        mbar_arrive_expect_tx(&bar_up[u], 2 * nks_u * (2048 + 256));
        tma_load_3d(b, mc, 0, rows_g, 0, &bar_up[u]);
        tma_load_3d(b + nks_u * 2048, mc, 0, rows_u, 0, &bar_up[u]);
        tma_load_3d(b + 2 * nks_u * 2048, ms, 0, rows_g, 0, &bar_up[u]);
        tma_load_3d(b + 2 * nks_u * 2048 + nks_u * 256, ms, 0, rows_u, 0, &bar_up[u]);
      }
      if (has_dn && (s_nlocal > 0 || SI > 0)) {
        mbar_arrive_expect_tx(&bar_dn, (s_nlocal * nks_d + nks_sh) * (2048 + 256));
        for (int s = 0; s < topk; ++s) {
          if (s_ids[s] < a.e_lo || s_ids[s] >= a.e_hi) continue;
          const int rows = (s_ids[s] - a.e_lo) * H + cta * 16;
          uint8_t* b = dn_base + s * a.dslot_bytes;
          tma_load_3d(b, &dn_c, 0, rows, 0, &bar_dn);
          tma_load_3d(b + nks_d * 2048, &dn_s, 0, rows, 0, &bar_dn);
        }
        if (SI > 0) {                                   // the shared expert's 16 down rows of this block
          uint8_t* b = smem + a.off_dn_sh;
          tma_load_3d(b, &sh_dn_c, 0, cta * 16, 0, &bar_dn);
          tma_load_3d(b + nks_sh * 2048, &sh_dn_s, 0, cta * 16, 0, &bar_dn);
        }
      }
      FLINT_TL(11);
    }
    return;
  }

  // ================= consumers =================
  // this launch's tag for the words it publishes (the last CTA to retire advances ws->epoch)
  unsigned ep;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(ep) : "l"(&ws->epoch) : "memory");
  ep += 1u;
  // ---- R: norm, router rows ----
  add_rmsnorm_1pass_w(a.x, a.ldx, a.res, nwc, a.eps, 1, H, xnb, cta == 0 ? a.res_out : nullptr,
                      cta == 0 ? a.xn_out : nullptr, red_n, kXT, 1);
  if (has_row) {
    const uint4* xp = reinterpret_cast<const uint4*>(xnb);
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      float xf[8], wf[8];
      bf16x8_to_f32(xp[lane + 32 * i], xf);
      bf16x8_to_f32(wv[i], wf);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc = fmaf(wf[j], xf[j], acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) st_tagged(lg + my_row, ep, __float_as_uint(bf16r(acc)));
  }
  stage_rows_f16(xnb, H, 1, H, xs, shift_x, red_n, kXT, 1);
  if (tid == 0) FLINT_TL(2);

  // ---- U: top-k once every CTA's router rows carry this launch's tag (no grid barrier), then the up units ----
  if (warp == 0) {
    constexpr int PER = 8;                              // E <= 256
    const int per = E / 32;
    float lv[PER];
    unsigned need = 0, got = 0;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      lv[j] = 0.f;
      if (j < per) need |= 1u << j;
    }
#pragma unroll 1
    for (unsigned it = 0; __any_sync(0xffffffffu, got != need); ++it) {
      if (it == FLINT_WAIT_LIMIT) {
        atomicOr(status, STATUS_WAIT_TIMEOUT);
        break;
      }
      if (it > 0) poll_pause();
#pragma unroll
      for (int j = 0; j < PER; ++j)
        if ((need & ~got) & (1u << j)) {
          const unsigned long long w = ld_tagged(lg + lane + 32 * j);
          if (tag_is(w, ep)) {
            lv[j] = __uint_as_float((uint32_t)w);
            got |= 1u << j;
          }
        }
    }
    if (lane == 0) FLINT_TL(7);
    int my_e;
    float my_w;
    warp_topk_regs<PER>(lv, per, topk, a.score_fn, lane, my_e, my_w);
    if (lane == 0) FLINT_TL(8);
    if (lane < topk) {
      s_ids[lane] = my_e;
      s_tw[lane] = my_w;
      if (cta == 0) {
        if (a.ids_out) a.ids_out[lane] = my_e;
        if (a.tw_out) a.tw_out[lane] = my_w;
      }
    }
    const bool loc = lane < topk && my_e >= a.e_lo && my_e < a.e_hi;
    const unsigned lm = __ballot_sync(0xffffffffu, loc);
    if (loc) s_local[__popc(lm & ((1u << lane) - 1u))] = lane;
    if (lane == 0) s_nlocal = __popc(lm);
  }
  xsync();
  if (cta == 0 && a.logits_out)                         // every tag was seen by warp 0 before the xsync
    for (int i = tid; i < E; i += kXT) a.logits_out[i] = __uint_as_float((uint32_t)ld_tagged(lg + i));
  if (tid == 0) mbar_arrive(&bar_plan);                 // release the producer
  if (tid == 0) FLINT_TL(3);

  const int g = lane >> 2, t = lane & 3;
  const __half* xrow = xs;                              // token 0 (lanes g > 0 feed zero columns)
  const bool active = g == 0;
  int u0, nu;
  unit_range(u0, nu);
  const int routed_units = s_nlocal * jpe;
  #pragma unroll 1
  for (int u = 0; u < nu; ++u) {
    if (!xsync_and(mbar_wait(&bar_up[u], 0, status))) break;
    if (tid == 0 && u == 0) FLINT_TL(9);
    const int unit = u0 + u;
    const bool shared = unit >= routed_units;
    const int s = shared ? 0 : s_local[unit / jpe];
    const int j = shared ? unit - routed_units : unit - (unit / jpe) * jpe;
    const float g13u = shared ? a.g13_sh[0] : a.g13[s_ids[s] - a.e_lo];
    unsigned long long* act_dst = shared ? act_sh : act_g + (int64_t)s * (I / 2);
    const uint8_t* b = up_base + u * a.unit_bytes;
    float acc_g[4][4], acc_u[4][4];
    zero_acc(acc_g);
    zero_acc(acc_u);
    #pragma unroll 1
    for (int ks = warp; ks < nks_u; ks += kXW) {
      consume_stage(b + ks * 2048, b + 2 * nks_u * 2048 + ks * 256, 0, g, t, ks, xrow, active, acc_g);
      consume_stage(b + (nks_u + ks) * 2048, b + 2 * nks_u * 2048 + (nks_u + ks) * 256, 0, g, t, ks, xrow, active, acc_u);
    }
    float dg[4], du[4];
    sum_acc(acc_g, dg);
    sum_acc(acc_u, du);
    if (t == 0) {                                       // column 0 = the token
      const int r0 = tile_phi(g);
      red[(0 * kXW + warp) * 16 + r0] = dg[0];
      red[(0 * kXW + warp) * 16 + r0 + 8] = dg[2];
      red[(1 * kXW + warp) * 16 + r0] = du[0];
      red[(1 * kXW + warp) * 16 + r0 + 8] = du[2];
    }
    xsync();
    if (tid < 16) {
      float gs = 0.f, us = 0.f;
#pragma unroll
      for (int w = 0; w < kXW; ++w) {
        gs += red[(0 * kXW + w) * 16 + tid];
        us += red[(1 * kXW + w) * 16 + tid];
      }
      const float sc = ldexpf(g13u, -shift_x[0]);
      const float gv = gs * sc, uv = us * sc;
      const float silu = gv / (1.0f + expf(-gv));
      const unsigned vb = __bfloat16_as_ushort(__float2bfloat16_rn(silu * uv));
      const unsigned hi = __shfl_down_sync(0x0000ffffu, vb, 1);   // act pair (2i, 2i+1) -> one tagged word
      if ((tid & 1) == 0) st_tagged(act_dst + (j * 16 + tid) / 2, ep, vb | (hi << 16));
    }
    xsync();
  }
  if (tid == 0) FLINT_TL(4);
  pdl_trigger();

  // ---- D: this CTA's 16 output rows over every routed expert, then the slot-order sum ----
  if (has_dn) {
    {
      if (warp < topk && (s_ids[warp] < a.e_lo || s_ids[warp] >= a.e_hi)) {
        if (lane < 16) ybuf[warp][lane] = 0.f;           // expert of another rank
      } else if (warp < topk) {
        // warp s: slot s's act row once its words carry this launch's tag (each warp on its own row, no block-wide
        // staging), then the 16 down rows of this block for that slot
        const int s = warp, e = s_ids[s] - a.e_lo;
        __half* arow = xa + s * xs_stride(I);
        stage_row_f16_tagged_warp(act_g + (int64_t)s * (I / 2), I, ep, arow, &shift_a[s], lane, status);
        const uint8_t* b = dn_base + s * a.dslot_bytes;
        const bool act_col = g == 0;
        float acc[4][4];
        zero_acc(acc);
        if (__all_sync(0xffffffffu, mbar_wait(&bar_dn, 0, status))) {
          #pragma unroll 1
          for (int ks = 0; ks < nks_d; ++ks) consume_stage(b + ks * 2048, b + nks_d * 2048 + ks * 256, 0, g, t, ks, arow, act_col, acc);
        }
        float d[4];
        sum_acc(acc, d);
        if (t == 0) {
          const int r0 = tile_phi(g);
          const float sc = ldexpf(a.g2[e], -shift_a[s]);
          ybuf[s][r0] = bf16r(d[0] * sc);
          ybuf[s][r0 + 8] = bf16r(d[2] * sc);
        }
      } else if (SI > 0 && warp == topk) {
        // the shared expert's 16 down rows of this block, from its act row (same accumulation as a routed slot)
        __half* arow = reinterpret_cast<__half*>(smem + a.off_xa_sh);
        stage_row_f16_tagged_warp(act_sh, SI, ep, arow, &shift_sh, lane, status);
        const uint8_t* b = smem + a.off_dn_sh;
        float acc[4][4];
        zero_acc(acc);
        if (__all_sync(0xffffffffu, mbar_wait(&bar_dn, 0, status))) {
          #pragma unroll 1
          for (int ks = 0; ks < nks_sh; ++ks) consume_stage(b + ks * 2048, b + nks_sh * 2048 + ks * 256, 0, g, t, ks, arow, g == 0, acc);
        }
        float d[4];
        sum_acc(acc, d);
        if (t == 0) {
          const int r0 = tile_phi(g);
          const float sc = ldexpf(a.g2_sh[0], -shift_sh);
          ysh[r0] = bf16r(d[0] * sc);
          ysh[r0 + 8] = bf16r(d[2] * sc);
        }
      }
      xsync();
      if (tid == 0) FLINT_TL(5);
      if (a.y_out) {
        for (int i = tid; i < topk * 16; i += kXT)
          a.y_out[(int64_t)(i >> 4) * H + cta * 16 + (i & 15)] = __float2bfloat16_rn(ybuf[i >> 4][i & 15]);
      } else if (a.peer_mode) {
        if (warp == 0) {
          // push the local slots' rows of this block to every rank, flag, wait for every rank, combine
          uint8_t* const mine = a.peers.base[a.peers.rank];
          PeerHeader* own = peer_header(mine);
          const unsigned ep = ld_relaxed_sys_u32(&own->moe_epoch) + 1u, par = ep & 1u;
          const int W = a.peers.world, nl = s_nlocal;
          for (int i = lane; i < nl * W * 2; i += 32) {
            const int j = i / (2 * W), p = (i >> 1) - j * W, half = i & 1, s = s_local[j];
            const float* yv = &ybuf[s][half * 8];
            uint4 v;
            v.x = peer_pack_bf16x2(yv[0], yv[1]);
            v.y = peer_pack_bf16x2(yv[2], yv[3]);
            v.z = peer_pack_bf16x2(yv[4], yv[5]);
            v.w = peer_pack_bf16x2(yv[6], yv[7]);
            *reinterpret_cast<uint4*>(peer_moe_rows(a.peers.base[p], par, H) + (int64_t)s * H + cta * 16 + half * 8) = v;
          }
          __threadfence_system();
          __syncwarp();
          if (lane < W) st_release_sys_u32(peer_moe_flags(a.peers.base[lane]) + cta * kPeerMax + a.peers.rank, ep);
          bool ok = true;
          if (lane < W) ok = peer_wait(peer_moe_flags(mine) + cta * kPeerMax + lane, ep, own);
          ok = __all_sync(0xffffffffu, ok);
          __syncwarp();   // orders every lane's reads after the acquiring lanes' loads
          if (ok && lane < 16) {
            const bf16* rows = peer_moe_rows(mine, par, H) + cta * 16 + lane;
            float acc = 0.f;
            for (int s = 0; s < topk; ++s) acc = fmaf(s_tw[s], peer_ldcg_bf16(rows + (int64_t)s * H), acc);
            a.out[cta * 16 + lane] = __float2bfloat16_rn(acc);
          }
        }
      } else if (tid < 16) {
        float acc = 0.f;
        for (int s = 0; s < topk; ++s) acc = fmaf(s_tw[s], ybuf[s][tid], acc);
        // with a shared expert: bf16(bf16(routed) + shared), as the chain's routed down + shared down + bf16 add
        const float o = SI > 0 ? bf16r(acc) + ysh[tid] : acc;
        a.out[cta * 16 + tid] = __float2bfloat16_rn(o);
      }
    }
  }
  if (tid == 0) FLINT_TL(6);
  grid_sync_retire(&ws->sync, nb, &ws->epoch, a.peer_mode ? &peer_header(a.peers.base[a.peers.rank])->moe_epoch : nullptr);
}

// out[m][r] = bf16(sum_s tw[m][s] * y[m topk + s][r]) in slot order (the weighted sum of flint_moe_block /
// flint_moe_down after an expert-parallel sum of the per-route rows over ranks).
__global__ void moe_combine_kernel(const bf16* __restrict__ y, const float* __restrict__ tw, int topk, int H,
                                   bf16* __restrict__ out) {
  pdl_wait();
  const int r = blockIdx.x * blockDim.x + threadIdx.x, m = blockIdx.y;
  if (r < H) {
    float acc = 0.f;
    for (int s = 0; s < topk; ++s)
      acc = fmaf(tw[m * topk + s], __bfloat162float(y[(int64_t)(m * topk + s) * H + r]), acc);
    out[(int64_t)m * H + r] = __float2bfloat16_rn(acc);
  }
  pdl_trigger();
}

}  // namespace flint

using namespace flint;

int64_t flint::status_offset_moe_block() { return (int64_t)offsetof(MoeBlockWs, status); }

extern "C" int64_t flint_moe_block_workspace_bytes(int64_t E, int64_t I) { return (int64_t)moe_block_ws_bytes((int)E, (int)I); }

static int moe_block_launch(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps,
                            const void* gate_w, int64_t H, int64_t E, int64_t topk, int score_fn, const void* w13,
                            const void* s13, const float* g13, const void* w2, const void* s2, const float* g2, int64_t I,
                            int64_t e_lo, int64_t n_local, void* out, void* y_out, void* res_out, void* xn_out,
                            float* logits_out, int32_t* topk_ids_out, float* topk_weights_out, void* workspace,
                            const flint_l2_prefetch* next, int pdl, void* stream, const PeerSet* peers = nullptr,
                            const void* sh_w13 = nullptr, const void* sh_s13 = nullptr, const float* sh_g13 = nullptr,
                            const void* sh_w2 = nullptr, const void* sh_s2 = nullptr, const float* sh_g2 = nullptr,
                            int64_t SI = 0) {
  if (!x || !norm_w || !gate_w || !w13 || !s13 || !g13 || !w2 || !s2 || !g2 || (!out && !y_out) || !workspace)
    return FLINT_ERR_ARGUMENT;
  if (SI != 0) {                           // the shared expert: one-GPU weighted-sum mode only
    if (!sh_w13 || !sh_s13 || !sh_g13 || !sh_w2 || !sh_s2 || !sh_g2 || !out || y_out || peers) return FLINT_ERR_ARGUMENT;
    if (SI < kSliceK || SI % kSliceK != 0 || SI > kXMaxShared || topk >= kXW) return FLINT_ERR_SHAPE;
    if (!aligned(sh_w13, 16) || !aligned(sh_s13, 16) || !aligned(sh_w2, 16) || !aligned(sh_s2, 16)) return FLINT_ERR_ALIGN;
  }
  if (peers && (!out || y_out)) return FLINT_ERR_ARGUMENT;
  if (peers && (H / 16 != kPeerMoeBlocks || topk > kPeerSlots)) return FLINT_ERR_SHAPE;
  if (e_lo < 0 || n_local < 1 || e_lo + n_local > E || (y_out && !topk_weights_out)) return FLINT_ERR_ARGUMENT;
  const int sms = num_sms();
  if (sms <= 0) return FLINT_ERR_DEVICE;
  if (H != 2048 || E < 32 || E % 32 != 0 || E > 256 || E > 2 * sms || topk < 1 || I > 1024 ||
      topk > kXMaxSlots || topk > E || I < kSliceK || I % kSliceK != 0 || ldx < H || score_fn < 0 || score_fn > 1 ||
      H / 16 > sms)
    return FLINT_ERR_SHAPE;
  const int U = (int)(topk * (I / 16) + SI / 16);
  if ((U + sms - 1) / sms > kXMaxUnits) return FLINT_ERR_SHAPE;
  if (!aligned(x, 16) || ldx % 8 != 0 || (res && !aligned(res, 16)) || !aligned(norm_w, 16) || !aligned(gate_w, 16) ||
      !aligned(w13, 16) || !aligned(s13, 16) || !aligned(w2, 16) || !aligned(s2, 16) || (out && !aligned(out, 16)) ||
      (y_out && !aligned(y_out, 16)) ||
      (res_out && !aligned(res_out, 16)) || (xn_out && !aligned(xn_out, 16)) || !aligned(workspace, 256))
    return FLINT_ERR_ALIGN;
  auto up = [](size_t v, size_t al) { return (v + al - 1) / al * al; };
  const int nks_u = (int)(H / kSliceK), nks_d = (int)(I / kSliceK);
  MoeBlockArgs a{};
  a.unit_bytes = (uint32_t)up((size_t)2 * nks_u * (2048 + 256), 1024);
  a.dslot_bytes = (uint32_t)up((size_t)nks_d * (2048 + 256), 1024);
  a.off_dn = kXMaxUnits * a.unit_bytes;
  a.off_xn = a.off_dn + kXMaxSlots * a.dslot_bytes;
  a.off_xs = a.off_xn + (uint32_t)up((size_t)H * 2, 1024);
  a.off_xa = a.off_xs + (uint32_t)up((size_t)xs_stride((int)H) * 2, 1024);
  a.off_dn_sh = a.off_xa + (uint32_t)up((size_t)kXMaxSlots * xs_stride((int)I) * 2, 1024);
  a.off_xa_sh = a.off_dn_sh + (uint32_t)up((size_t)(SI / kSliceK) * (2048 + 256), 1024);
  a.off_red = a.off_xa_sh + (uint32_t)up(SI > 0 ? (size_t)xs_stride((int)SI) * 2 : 0, 1024);
  const size_t smem = 1024 + a.off_red + 2 * kXW * 16 * 4;
  if (smem > 227 * 1024 - 2048) return FLINT_ERR_SHAPE;

  // weights as 3-D views [slice][row][bytes of the slice]: one box per 16-row block over all of K
  auto enc3 = [](CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t row_bytes, uint64_t nks,
                 bool swz) {
    const uint64_t d[3] = {inner, rows, nks};
    const uint64_t st[2] = {row_bytes, inner};
    const uint32_t bx[3] = {(uint32_t)inner, 16u, (uint32_t)nks};
    return encode_u8_3d(m, base, d, st, bx, swz);
  };
  CUtensorMap uc, us, dc, ds;
  int rc = enc3(&uc, w13, 128, (uint64_t)n_local * 2 * I, H / 2, nks_u, true);
  if (!rc) rc = enc3(&us, s13, 16, (uint64_t)n_local * 2 * I, H / 16, nks_u, false);
  if (!rc) rc = enc3(&dc, w2, 128, (uint64_t)n_local * H, I / 2, nks_d, true);
  if (!rc) rc = enc3(&ds, s2, 16, (uint64_t)n_local * H, I / 16, nks_d, false);
  if (rc) return rc;
  CUtensorMap suc = uc, sus = us, sdc = dc, sds = ds;   // unused copies without a shared expert
  if (SI > 0) {
    const int nks_sh = (int)(SI / kSliceK);
    rc = enc3(&suc, sh_w13, 128, (uint64_t)2 * SI, H / 2, nks_u, true);
    if (!rc) rc = enc3(&sus, sh_s13, 16, (uint64_t)2 * SI, H / 16, nks_u, false);
    if (!rc) rc = enc3(&sdc, sh_w2, 128, (uint64_t)H, SI / 2, nks_sh, true);
    if (!rc) rc = enc3(&sds, sh_s2, 16, (uint64_t)H, SI / 16, nks_sh, false);
    if (rc) return rc;
  }
  a.SI = (int)SI;
  a.g13_sh = sh_g13;
  a.g2_sh = sh_g2;

  a.x = (const bf16*)x; a.ldx = ldx; a.res = (const bf16*)res; a.nw = (const bf16*)norm_w; a.eps = eps;
  a.gate_w = (const bf16*)gate_w; a.E = (int)E; a.topk = (int)topk; a.score_fn = score_fn; a.H = (int)H; a.I = (int)I;
  a.g13 = g13; a.g2 = g2; a.out = (bf16*)out; a.res_out = (bf16*)res_out; a.xn_out = (bf16*)xn_out;
  a.logits_out = logits_out; a.ids_out = topk_ids_out; a.tw_out = topk_weights_out;
  a.e_lo = (int)e_lo; a.e_hi = (int)(e_lo + n_local); a.y_out = (bf16*)y_out;
  a.ws = static_cast<MoeBlockWs*>(workspace);
  if (peers) {
    a.peer_mode = 1;
    a.peers = *peers;
  }
  if (!l2_prefetch_pack(next, &a.pf)) return FLINT_ERR_ARGUMENT;

  // H = 2048: the single-pass norm keeps one 8-wide chunk per consumer thread
  void (*kern)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap,
               MoeBlockArgs) = moe_block_kernel<8>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return record_cuda(cudaGetLastError(), FLINT_ERR_LAUNCH);
  set_max_carveout(kern);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3((kXW + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 2 : 1;
  return record_cuda(cudaLaunchKernelEx(&cfg, kern, uc, us, dc, ds, suc, sus, sdc, sds, a), FLINT_ERR_LAUNCH);
}

extern "C" int flint_moe_block(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps, const void* gate_w,
                               int64_t H, int64_t E, int64_t topk, int score_fn, const void* w13, const void* s13,
                               const float* g13, const void* w2, const void* s2, const float* g2, int64_t I, void* out,
                               void* res_out, void* xn_out, float* logits_out, int32_t* topk_ids_out,
                               float* topk_weights_out, void* workspace, const flint_l2_prefetch* next, int pdl,
                               void* stream) {
  return moe_block_launch(x, ldx, res, norm_w, eps, gate_w, H, E, topk, score_fn, w13, s13, g13, w2, s2, g2, I, 0, E, out,
                          nullptr, res_out, xn_out, logits_out, topk_ids_out, topk_weights_out, workspace, next, pdl,
                          stream);
}

extern "C" int flint_moe_block_shared(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps,
                                      const void* gate_w, int64_t H, int64_t E, int64_t topk, int score_fn,
                                      const void* w13, const void* s13, const float* g13, const void* w2, const void* s2,
                                      const float* g2, int64_t I, const void* sh_w13, const void* sh_s13,
                                      const float* sh_g13, const void* sh_w2, const void* sh_s2, const float* sh_g2,
                                      int64_t SI, void* out, void* res_out, void* xn_out, float* logits_out,
                                      int32_t* topk_ids_out, float* topk_weights_out, void* workspace,
                                      const flint_l2_prefetch* next, int pdl, void* stream) {
  if (SI < 1) return FLINT_ERR_SHAPE;
  return moe_block_launch(x, ldx, res, norm_w, eps, gate_w, H, E, topk, score_fn, w13, s13, g13, w2, s2, g2, I, 0, E, out,
                          nullptr, res_out, xn_out, logits_out, topk_ids_out, topk_weights_out, workspace, next, pdl,
                          stream, nullptr, sh_w13, sh_s13, sh_g13, sh_w2, sh_s2, sh_g2, SI);
}

extern "C" int flint_moe_block_ep(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps,
                                  const void* gate_w, int64_t H, int64_t E, int64_t topk, int score_fn, const void* w13,
                                  const void* s13, const float* g13, const void* w2, const void* s2, const float* g2,
                                  int64_t I, int64_t expert_lo, int64_t n_local, void* y_out, float* topk_weights_out,
                                  void* res_out, void* workspace, const flint_l2_prefetch* next, int pdl,
                                  void* stream) {
  return moe_block_launch(x, ldx, res, norm_w, eps, gate_w, H, E, topk, score_fn, w13, s13, g13, w2, s2, g2, I, expert_lo,
                          n_local, nullptr, y_out, res_out, nullptr, nullptr, nullptr, topk_weights_out, workspace, next,
                          pdl, stream);
}

extern "C" int flint_moe_combine(const void* y, const float* topk_weights, int64_t M, int64_t topk, int64_t H, void* out,
                                 int pdl, void* stream) {
  if (!y || !topk_weights || !out) return FLINT_ERR_ARGUMENT;
  if (M < 1 || M > 65535 || topk < 1 || topk > kXMaxSlots || H < 1 || H > (1 << 20)) return FLINT_ERR_SHAPE;
  return launch(moe_combine_kernel, dim3((unsigned)((H + 255) / 256), (unsigned)M), dim3(256), 0, stream, pdl,
                (const bf16*)y, topk_weights, (int)topk, (int)H, (bf16*)out);
}

extern "C" int flint_moe_block_peer(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps,
                                    const void* gate_w, int64_t H, int64_t E, int64_t topk, int score_fn, const void* w13,
                                    const void* s13, const float* g13, const void* w2, const void* s2, const float* g2,
                                    int64_t I, int64_t expert_lo, int64_t n_local, const void* const* peers, int rank,
                                    int world, void* out, void* res_out, void* workspace, const flint_l2_prefetch* next,
                                    int pdl, void* stream) {
  PeerSet ps;
  const int rc = peer_set(peers, rank, world, &ps);
  if (rc) return rc;
  return moe_block_launch(x, ldx, res, norm_w, eps, gate_w, H, E, topk, score_fn, w13, s13, g13, w2, s2, g2, I, expert_lo,
                          n_local, out, nullptr, res_out, nullptr, nullptr, nullptr, nullptr, workspace, next, pdl, stream,
                          &ps);
}

FLINT_TL_READER(flint_timeline_moe_block)
