// (1) Fused MoE decode block: one persistent kernel per MoE layer for 1..8 tokens.
// Replaces the reference's three-kernel chain route_norm_kernel -> up_mar -> down_mar (fast/fp4moe_mar.cu:311-417,
// 67-152, 157-233; driven by fast/model.py:302-310) with one launch of one CTA per SM and three grid barriers:
//
//   R  every CTA: s = x + res, xn = bf16(RMSNorm(s)) (same fixed order everywhere); CTA 0 publishes res_out / xn;
//      CTAs own router rows e = cta, cta + grid (weights prefetched into registers before the PDL wait) and write
//      bf16 logits                                                                          -> grid barrier 0
//   U  every CTA: top-k of each token from the logits (redundant, identical), routes grouped by expert;
//      each CTA streams its share of (gate 64 rows + up 64 rows) x H tiles through the TMA ring and writes
//      act = bf16(silu(g) * u); the producer warp keeps streaming the CTA's down tiles behind them
//                                                                                           -> grid barrier 1
//   D  stage all act rows, y = bf16(act . W2[e] * gs2[e]) for the CTA's 128-row down tiles -> grid barrier 2
//   F  out[m, r] = bf16(sum_s tw[m, s] * y[m*k + s, r]) in slot order for the CTA's rows
//
// Numerics are those of the per-op kernels in moe.cu (same reduction orders), so routing is bit identical to them.
// Up tiles are split evenly over all CTAs, and so are down tiles: every CTA works in both phases, its producer
// streaming its down tiles into the ring behind its up tiles (they do not depend on the activations), so the down
// weights are in flight while the grid waits at barrier 1.
//
// Expert-parallel mode (flint_moe_fused_ep, y_out given): the weights hold experts [e_lo, e_hi) only; the router and
// top-k run in full (identical on every rank), only routes whose expert is local get tiles, and phase F writes
// y_out[m * topk + s] = y of each local route (zero rows for the others) instead of the weighted sum: summed over the
// ranks (one non-zero term per element) and combined in slot order they give the one-GPU output bit for bit, and the
// rows equal flint_moe_down_ep's.
//
// Data-parallel mode over NVLink peer memory (flint_moe_fused_dp_peer; one stream per GPU, expert-parallel MoE): the
// launch is also the exchange.  In phase R, CTA 0 stores this rank's two rows (attention output, residual) into every
// rank's token table and raises its flag there; every CTA waits for all ranks' flags and normalises the M = world
// tokens from its own table.  In phase F each local route's rows go straight into the token owner's row table, and
// the last CTA to finish raises this rank's row flag on every rank; flint_dp_combine_peer (rows already pushed) then
// forms each rank's weighted sum.  The tables, flags and epochs are those of flint_dp_gather_peer /
// flint_dp_combine_peer (peer.cuh); every wait is bounded in time.
#include "gridsync.cuh"
#include "moe_common.cuh"
#include "peer.cuh"
#include "runtime.cuh"
#include "timeline.cuh"

#include <string.h>

// Timeline stamps (-DFLINT_TIMELINE builds only): 0 entry, 1 PDL wait done, 2 norm + router rows + staging, 3 barrier 0,
// 4 plan released, 5 first gate/up tile done, 6 gate/up tiles done, 7 barrier 1, 8 act rows staged, 9 down tiles done,
// 10 barrier 2, 11 output written, 12 producer: first stage issued, 13 producer: last gate/up stage issued,
// 14 producer: last stage issued, 15 norm done, 16 router rows written, 17 top-k done.
FLINT_TL_BUFFER

namespace flint {

constexpr int kFW = 8, kFBox = 64;

struct MoeFusedWs {
  GridSync sync;
  unsigned status;
  unsigned pad[31];
  // followed by: logits fp32 [8][E], act bf16 [64][I], y bf16 [64][H]
};

struct MoeFusedArgs {
  const bf16* x;
  int64_t ldx;
  const bf16* res;
  const bf16* nw;
  float eps;
  const bf16* gate_w;
  int E, topk, score_fn;
  const float* g13;
  const float* g2;
  int M, H, I;
  bf16* out;
  bf16* res_out;
  bf16* xn_out;
  float* logits_out;
  int* ids_out;
  float* tw_out;
  MoeFusedWs* ws;
  int e_lo, e_hi;                    // local experts (expert-parallel mode; 0 and kNotLocal otherwise)
  bf16* y_out;                       // expert-parallel mode: per-route rows [M * topk][H]
  int nslot_cap;                     // act rows a CTA can stage (the routes of the groups its down tiles span)
  int peer;                          // data-parallel peer mode (ps, send valid; M = world)
  const bf16* send;                  // peer mode: this rank's rows [2][H] (attention output, residual)
  PeerSet ps;
};

__host__ __device__ inline size_t moe_fused_ws_bytes(int E, int H, int I) {
  return sizeof(MoeFusedWs) + (size_t)kMaxTokens * E * 4 + (size_t)kMaxRoutes * I * 2 + (size_t)kMaxRoutes * H * 2;
}


// KG consumer groups of kFW warps: group g works on the CTA's tiles g, g + KG, ... of each phase, two tiles' stages
// interleaved in the ring, each tile computed exactly as by one group (same warp / row mapping and sums), so KG
// changes the speed only.  KG = 2 needs H = 2048 (its norm gives each thread half the rows of one chunk).
template <int NS, int NV, int KG>
__global__ void __launch_bounds__((KG * kFW + 1) * 32, 1)
moe_fused_kernel(const __grid_constant__ CUtensorMap up_c, const __grid_constant__ CUtensorMap up_s,
                 const __grid_constant__ CUtensorMap dn_c, const __grid_constant__ CUtensorMap dn_s, const MoeFusedArgs a) {
  using L = EngineSmem<kFW, NS, kFBox>;
  constexpr int GT = kFW * 32;              // threads of one consumer group
  constexpr int NT = KG * GT;               // consumer threads
  constexpr int PW = KG * kFW;              // the producer warp
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __half* xs = reinterpret_cast<__half*>(smem + L::ring_bytes + KG * L::dtile_bytes);   // f16 [M][H+8]
  uint8_t* region = reinterpret_cast<uint8_t*>(xs + a.M * xs_stride(a.H));              // phase R: bf16 xn; D: f16 act
  bf16* xnb = reinterpret_cast<bf16*>(region);
  __half* xa = reinterpret_cast<__half*>(region);
  __shared__ uint64_t bars[2 * NS];
  __shared__ uint64_t plan_bar;
  __shared__ Groups G;
  __shared__ int sorted[kMaxRoutes], ids_s[kMaxRoutes], ids_c[kMaxRoutes];
  __shared__ float tw_s[kMaxRoutes];
  __shared__ int shift_x[kMaxTokens], shift_a[kMaxRoutes];
  __shared__ float red[kFW * kMaxRoutes];
  __shared__ int s_ok;
  __shared__ int tiles[4];                   // this CTA's up tiles [tiles[0], tiles[1]), down tiles [tiles[2], tiles[3])

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int M = a.M, H = a.H, I = a.I, E = a.E, topk = a.topk, R = M * topk;
  const unsigned nb = gridDim.x;
  MoeFusedWs* ws = a.ws;
  unsigned* status = &ws->status;
  float* lg = reinterpret_cast<float*>(ws + 1);
  bf16* act_g = reinterpret_cast<bf16*>(lg + kMaxTokens * E);
  bf16* y_g = act_g + (size_t)kMaxRoutes * I;
  const int nks_up = H / kSliceK, nks_dn = I / kSliceK;
  const int tpu = I / kFBox, tpd = H / (2 * kFBox);

  if (tid == 0) {
    for (int i = 0; i < NS; ++i) {
      mbar_init(&bars[i], 1);
      mbar_init(&bars[NS + i], kFW);
    }
    mbar_init(&plan_bar, 1);
    fence_mbar_init();
  }
  __syncthreads();
  if (tid == 0) FLINT_TL(0);

  // router rows of this CTA: e = blockIdx.x (+ gridDim.x), one warp each, prefetched before the wait
  // Router dots: this CTA's rows are blockIdx.x and blockIdx.x + nb (E <= 2 nb); (row, token) pair p is row
  // blockIdx.x + (p / M) nb and token p % M, and consumer warp w takes pairs w, w + kFW, ...  A warp's first row is
  // prefetched into registers before the PDL wait.
  const int npairs = ((int)blockIdx.x < E ? M : 0) + ((int)(blockIdx.x + nb) < E ? M : 0);
  int wv_rk = warp < PW && warp < npairs ? warp / M : -1;    // row (0 or 1) held in wv
  uint4 wv[NV];
  if (wv_rk >= 0) {
    const uint4* wp = reinterpret_cast<const uint4*>(a.gate_w + (int64_t)(blockIdx.x + wv_rk * nb) * H);
#pragma unroll
    for (int i = 0; i < NV; ++i) wv[i] = ldg_stream_v4(wp + lane + 32 * i);
  }
  // the norm weights (this thread's 8) do not depend on the previous kernel either
  const uint4 nwc = tid < NT && (KG > 1 || tid < H / 8) ? reinterpret_cast<const uint4*>(a.nw)[tid % (H / 8)]
                                                        : make_uint4(0u, 0u, 0u, 0u);
  pdl_wait();
  if (tid == 0) FLINT_TL(1);

  if (warp == PW) {
    // ---------------- producer: wait for the routing plan, then stream up tiles followed by down tiles ----------------
    // (per phase, the tiles of consumer groups 0 .. KG-1 go in rounds of KG tiles, their stages interleaved: stage k of
    // round member j is stage number round_base + k * (members) + j of the phase)
    if (lane == 0) {
      bool ok = false;
      for (unsigned i = 0; i < FLINT_WAIT_LIMIT && !ok; ++i) ok = mbar_try_wait(&plan_bar, 0);
      if (!ok) {
        atomicOr(status, STATUS_WAIT_TIMEOUT);
        return;
      }
      tma_prefetch_desc(&up_c);
      tma_prefetch_desc(&dn_c);
      const int u0 = tiles[0], u1 = tiles[1], d0 = tiles[2], d1 = tiles[3];
      int slot = 0, s = 0;
      unsigned phase = 0;
      for (int ph = 0; ph < 2; ++ph) {
        const bool up = ph == 0;
        const int t0 = up ? u0 : d0, n = up ? u1 - u0 : d1 - d0, nks = up ? nks_up : nks_dn;
        const CUtensorMap* mc = up ? &up_c : &dn_c;
        const CUtensorMap* ms = up ? &up_s : &dn_s;
        for (int rb = 0; rb < n; rb += KG) {
          const int members = min(KG, n - rb);
          for (int ks = 0; ks < nks; ++ks) {
            for (int j = 0; j < members; ++j, ++s) {
              const int t = t0 + rb + j;                        // up tile, or down tile (numbered from 0)
              int y0, y1;
              if (up) {
                const int u = t / tpu, jj = t - u * tpu;
                y0 = G.exp[u] * 2 * I + jj * kFBox;
                y1 = y0 + I;
              } else {
                const int u = t / tpd, jj = t - u * tpd;
                y0 = G.exp[u] * H + jj * 2 * kFBox;
                y1 = y0 + kFBox;
              }
              if (s >= NS && !mbar_wait(&bars[NS + slot], phase ^ 1u, status)) return;
              mbar_arrive_expect_tx(&bars[slot], L::code_bytes + L::scale_bytes);
              uint8_t* cdst = smem + slot * L::code_bytes;
              uint8_t* sdst = smem + NS * L::code_bytes + slot * L::scale_bytes;
              tma_load_2d(cdst, mc, ks * 128, y0, &bars[slot]);
              tma_load_2d(sdst, ms, ks * 16, y0, &bars[slot]);
              tma_load_2d(cdst + kFBox * 128, mc, ks * 128, y1, &bars[slot]);
              tma_load_2d(sdst + kFBox * 16, ms, ks * 16, y1, &bars[slot]);
              if (s == 0) FLINT_TL(12);
              if (++slot == NS) { slot = 0; phase ^= 1u; }
            }
          }
        }
        if (up) FLINT_TL(13);
      }
      FLINT_TL(14);
    }
    return;
  }

  // ---------------- phase R: norm, router rows ----------------
  // (one global pass with every token's chunk loaded at once when a thread owns one 8-wide chunk per row; the same
  // per-thread chains, butterfly and warp order as the two-pass form, so xn has the same bits)
  // (H / 8 <= NT: one pass that also stages xn as f16 from registers; the same bits as the two-pass norm followed by
  // stage_rows_f16, which the wider rows use)
  const bf16* xin = a.x;
  const bf16* rin = a.res;
  int64_t ldin = a.ldx;
  unsigned ep_tok = 0, ep_row = 0;
  if (a.peer) {
    // every rank's (attention output, residual) rows into every rank's token table, this rank's flag there; then
    // this CTA waits for every rank's flag and reads the M = world tokens from its own table
    const int W = a.ps.world, rk = a.ps.rank, n16 = 2 * H / 8;
    PeerHeader* own = peer_header(a.ps.base[rk]);
    ep_tok = ld_relaxed_sys_u32(&own->dp_tok_epoch) + 1u;
    ep_row = ld_relaxed_sys_u32(&own->dp_row_epoch) + 1u;
    if (blockIdx.x == 0) {
      const uint4* src = reinterpret_cast<const uint4*>(a.send);
      for (int i = tid; i < n16 * W; i += NT) {
        const int p = i / n16, u = i - p * n16;
        reinterpret_cast<uint4*>(peer_dp_tokens(a.ps.base[p], ep_tok & 1u, H) + (size_t)rk * 2 * H)[u] = src[u];
      }
      __threadfence_system();
      named_bar_sync(2, NT);
      if (tid < W) st_release_sys_u32(reinterpret_cast<unsigned*>(a.ps.base[tid] + kPeerDpTokFlagsOff) + rk, ep_tok);
    }
    if (tid < W && !peer_wait(reinterpret_cast<unsigned*>(a.ps.base[rk] + kPeerDpTokFlagsOff) + tid, ep_tok, own))
      atomicOr(status, STATUS_WAIT_TIMEOUT);
    named_bar_sync(2, NT);                                  // orders the table reads after the acquiring polls
    xin = peer_dp_tokens(a.ps.base[rk], ep_tok & 1u, H);
    rin = xin + H;
    ldin = 2 * H;
  }
  const bool one_pass = KG > 1 || H / 8 <= NT;
  if (KG > 1) {                             // (the weight ring is free until the plan: the rows' copies go there)
    norm_xn_stage_f16_compact(xin, ldin, rin, nwc, a.eps, M, H, xnb, blockIdx.x == 0 ? a.xn_out : nullptr,
                              blockIdx.x == 0 ? a.res_out : nullptr, xs, shift_x, red, NT, 2,
                              reinterpret_cast<bf16*>(smem));
  } else if (one_pass) {
    norm_xn_stage_f16(xin, ldin, rin, nwc, a.eps, M, H, xnb, blockIdx.x == 0 ? a.xn_out : nullptr,
                      blockIdx.x == 0 ? a.res_out : nullptr, xs, shift_x, red, NT, 2, a.peer != 0);
  } else {
    add_rmsnorm_2pass(xin, ldin, rin, a.nw, a.eps, M, H, xnb, red, NT, 2);
  }
  if (tid == 0) FLINT_TL(15);
  if (blockIdx.x == 0 && !one_pass) {
    for (int idx = tid; idx < M * (H / 8); idx += NT) {
      const int m = idx / (H / 8), k8 = idx - m * (H / 8);
      if (a.xn_out) reinterpret_cast<uint4*>(a.xn_out + (int64_t)m * H)[k8] = reinterpret_cast<const uint4*>(xnb + m * H)[k8];
      if (a.res_out) {
        float f[8], g[8];
        bf16x8_to_f32(__ldcg(reinterpret_cast<const uint4*>(xin + m * ldin) + k8), f);
        if (rin) {
          bf16x8_to_f32(__ldcg(reinterpret_cast<const uint4*>(rin + m * ldin) + k8), g);
#pragma unroll
          for (int j = 0; j < 8; ++j) f[j] += g[j];
        }
        uint32_t rk[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          __nv_bfloat162 r2 = __floats2bfloat162_rn(f[2 * j], f[2 * j + 1]);
          rk[j] = *reinterpret_cast<uint32_t*>(&r2);
        }
        reinterpret_cast<uint4*>(a.res_out + (int64_t)m * H)[k8] = make_uint4(rk[0], rk[1], rk[2], rk[3]);
      }
    }
  }
  // one (row, token) dot per warp and pair: per lane the chain over i, then j, then the xor butterfly (the route
  // kernel's order)
  for (int p = warp; p < npairs; p += PW) {
    const int rk = p / M, m = p - rk * M, row = (int)blockIdx.x + rk * (int)nb;
    if (rk != wv_rk) {                                    // a second row (E > nb and pairs beyond the first 8)
      const uint4* wp = reinterpret_cast<const uint4*>(a.gate_w + (int64_t)row * H);
#pragma unroll
      for (int i = 0; i < NV; ++i) wv[i] = ldg_stream_v4(wp + lane + 32 * i);
      wv_rk = rk;
    }
    const uint4* xp = reinterpret_cast<const uint4*>(xnb + m * H);
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
    if (lane == 0) __stcg(lg + m * E + row, bf16r(acc));
  }
  if (tid == 0) FLINT_TL(16);
  if (!one_pass) stage_rows_f16(xnb, H, M, H, xs, shift_x, red, NT, 2);
  if (tid == 0) FLINT_TL(2);
  if (!grid_sync(&ws->sync, nb, 0, NT, 2, &s_ok, status)) return;
  if (tid == 0) FLINT_TL(3);

  // ---------------- phase U: top-k, groups, plan, gate/up tiles ----------------
  if (warp < M) {
    int my_e;
    float my_w;
    if (E <= 256) {                          // the logits in registers, each lane's keys sorted once (same bits)
      constexpr int PER = 8;
      const int per = E / 32;
      float lv[PER];
#pragma unroll
      for (int j = 0; j < PER; ++j) lv[j] = j < per ? __ldcg(lg + warp * E + lane + 32 * j) : 0.f;
      warp_topk_regs<PER>(lv, per, topk, a.score_fn, lane, my_e, my_w);
    } else {
      warp_topk(lg + warp * E, E, topk, a.score_fn, lane, my_e, my_w);
    }
    if (lane < topk) {
      ids_s[warp * topk + lane] = my_e;
      tw_s[warp * topk + lane] = my_w;
      if (blockIdx.x == 0) {
        if (a.ids_out) a.ids_out[warp * topk + lane] = my_e;
        if (a.tw_out) a.tw_out[warp * topk + lane] = my_w;
      }
    }
  }
  if (blockIdx.x == 0 && a.logits_out)
    for (int i = tid; i < M * E; i += NT) a.logits_out[i] = __ldcg(lg + i);
  named_bar_sync(2, NT);
  if (tid == 0) FLINT_TL(17);
  build_groups(ids_s, R, topk, E, G, sorted, ids_c, status, NT, 2, a.e_lo, a.e_hi);
  const int U = G.n * tpu, Dn = G.n * tpd;
  const int u0 = (int)((long)blockIdx.x * U / nb), u1 = (int)((long)(blockIdx.x + 1) * U / nb);
  const int d0 = (int)((long)blockIdx.x * Dn / nb), d1 = (int)((long)(blockIdx.x + 1) * Dn / nb);
  if (tid == 0) {
    tiles[0] = u0;
    tiles[1] = u1;
    tiles[2] = d0;
    tiles[3] = d1;
    mbar_arrive(&plan_bar);                  // release the producer
    FLINT_TL(4);
  }

  // this thread's consumer group (its own dtile and named barrier), its warp and thread within the group
  const int cg = warp / kFW, wg = warp - cg * kFW, gtid = tid - cg * GT, gbar = 1 + 2 * cg;   // barriers 1 and 3
  float* dtile = reinterpret_cast<float*>(smem + L::ring_bytes + cg * L::dtile_bytes);
  const int g = lane >> 2, t = lane & 3;
  const int prow = 16 * wg + tile_phi(g);
  bool ok = true;
  // stage k of the tile at position i of a phase with n tiles of nks stages each, numbered from `base`: rounds of KG
  // tiles, a round's stages interleaved (the producer's order)
  auto run_tile = [&](int nks, int base, int n, int i, const __half* xrow, bool active, float (&d)[4]) {
    const int rb = i - i % KG, members = min(KG, n - rb);
    const int s0 = base + rb * nks + (i - rb);
    float acc[4][4];
    zero_acc(acc);
    for (int ks = 0; ks < nks; ++ks) {
      const int sidx = s0 + ks * members, slot = sidx % NS;
      const unsigned phase = (unsigned)(sidx / NS) & 1u;
      if (ok && !mbar_wait(&bars[slot], phase, status)) ok = false;
      if (ok)
        consume_stage(smem + slot * L::code_bytes, smem + NS * L::code_bytes + slot * L::scale_bytes, wg, g, t, ks, xrow,
                      active, acc);
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars[NS + slot]);
    }
    sum_acc(acc, d);
  };
  auto store_dtile = [&](const float (&d)[4]) {
    dtile[prow * 8 + 2 * t] = d[0];
    dtile[prow * 8 + 2 * t + 1] = d[1];
    dtile[(prow + 8) * 8 + 2 * t] = d[2];
    dtile[(prow + 8) * 8 + 2 * t + 1] = d[3];
    named_bar_sync(gbar, GT);
  };

  const int nup = u1 - u0;
  for (int i = cg; i < nup; i += KG) {
    const int tt = u0 + i, u = tt / tpu, j = tt - u * tpu, cnt = G.cnt[u], e = G.exp[u];
    const bool active = g < cnt;
    float d[4];
    run_tile(nks_up, 0, nup, i, xs + (active ? G.tok[u][g] : 0) * xs_stride(H), active, d);
    store_dtile(d);
    for (int idx = gtid; idx < kFBox * 8; idx += GT) {
      const int n = idx / kFBox, r = idx - n * kFBox;
      if (n >= cnt) continue;
      const float sc = ldexpf(a.g13[e], -shift_x[G.tok[u][n]]);
      const float gv = dtile[r * 8 + n] * sc, uv = dtile[(kFBox + r) * 8 + n] * sc;
      const float silu = gv / (1.0f + expf(-gv));
      __stcg(reinterpret_cast<unsigned short*>(act_g + (int64_t)G.route[u][n] * I + j * kFBox + r),
             __bfloat16_as_ushort(__float2bfloat16_rn(silu * uv)));
    }
    named_bar_sync(gbar, GT);
    if (tid == 0 && i == 0) FLINT_TL(5);
  }
  if (tid == 0) FLINT_TL(6);
  if (!grid_sync(&ws->sync, nb, 1, NT, 2, &s_ok, status)) return;
  if (tid == 0) FLINT_TL(7);

  // ---------------- phase D: down tiles ----------------
  // stage the act rows of this CTA's down tiles only: group u of d0 / tpd .. (d1 - 1) / tpd, route c of the group,
  // goes to slot (u - ua) * 8 + c
  const int ua = d0 / tpd;
  if (d1 > d0) {
    int nslot = ((d1 - 1) / tpd - ua + 1) * 8;
    if (nslot > a.nslot_cap) {                            // cannot happen within the launch's bound; never overrun
      if (tid == 0) atomicOr(status, 2u);
      nslot = a.nslot_cap;
    }
    stage_rows_f16_map(act_g, I, nslot, I, xa, shift_a, red, NT, 2, true, [&](int i) {
      const int u = ua + (i >> 3), c = i & 7;
      return c < G.cnt[u] ? G.route[u][c] : -1;
    });
  }
  if (tid == 0) FLINT_TL(8);
  const int ndn = d1 - d0;
  for (int i = cg; i < ndn; i += KG) {
    const int td = d0 + i, u = td / tpd, j = td - u * tpd, cnt = G.cnt[u], e = G.exp[u], slot0 = (u - ua) * 8;
    const bool active = g < cnt && slot0 + g < a.nslot_cap;
    float d[4];
    run_tile(nks_dn, nup * nks_up, ndn, i, xa + (slot0 + (active ? g : 0)) * xs_stride(I), active, d);
    store_dtile(d);
    for (int idx = gtid; idx < 2 * kFBox * 8; idx += GT) {
      const int n = idx / (2 * kFBox), r = idx - n * (2 * kFBox);
      if (n >= cnt || slot0 + n >= a.nslot_cap) continue;
      const int route = G.route[u][n];
      const float y = dtile[r * 8 + n] * ldexpf(a.g2[e], -shift_a[slot0 + n]);
      __stcg(reinterpret_cast<unsigned short*>(y_g + (int64_t)route * H + j * 2 * kFBox + r),
             __bfloat16_as_ushort(__float2bfloat16_rn(y)));
    }
    named_bar_sync(gbar, GT);
  }
  if (tid == 0) FLINT_TL(9);
  pdl_trigger();
  if (!grid_sync(&ws->sync, nb, 2, NT, 2, &s_ok, status)) return;
  if (tid == 0) FLINT_TL(10);

  // ---------------- phase F: weighted sum in slot order (expert parallel: the local routes' rows) ----------------
  const int rows_per = (H + nb - 1) / nb;
  const int r0 = blockIdx.x * rows_per, r1 = min(H, r0 + rows_per);
  if (a.peer) {
    // each local route's rows into its token owner's row table at [this rank][slot]; the last CTA raises this rank's
    // row flag on every rank (every CTA's stores fenced before it counts itself) and advances both epochs
    const int W = a.ps.world, rk = a.ps.rank;
    for (int idx = tid; idx < (r1 - r0) * R; idx += NT) {
      const int route = idx / (r1 - r0), r = r0 + idx - route * (r1 - r0);
      if (ids_c[route] == kNotLocal) continue;
      const int m = route / topk, s = route - m * topk;
      const unsigned short b = __ldcg(reinterpret_cast<const unsigned short*>(y_g + (int64_t)route * H + r));
      reinterpret_cast<unsigned short*>(peer_dp_rows(a.ps.base[m], ep_row & 1u, H) +
                                        ((size_t)rk * kPeerSlots + s) * H)[r] = b;
    }
    __threadfence_system();
    named_bar_sync(2, NT);
    if (tid == 0) {
      FLINT_TL(11);
      if (atomicAdd(&ws->sync.retired, 1u) == nb - 1) {
        atomicExch(&ws->sync.count, 0u);
        atomicExch(&ws->sync.retired, 0u);
        __threadfence_system();
        for (int w = 0; w < W; ++w)
          st_release_sys_u32(reinterpret_cast<unsigned*>(a.ps.base[w] + kPeerDpRowFlagsOff) + rk, ep_row);
        PeerHeader* own = peer_header(a.ps.base[rk]);
        own->dp_tok_epoch = ep_tok;
        own->dp_row_epoch = ep_row;                       // the receive-and-sum launch waits for this epoch
      }
    }
    return;
  }
  if (a.y_out) {
    for (int idx = tid; idx < (r1 - r0) * R; idx += NT) {
      const int route = idx / (r1 - r0), r = r0 + idx - route * (r1 - r0);
      const unsigned short b = ids_c[route] != kNotLocal
                                   ? __ldcg(reinterpret_cast<const unsigned short*>(y_g + (int64_t)route * H + r))
                                   : (unsigned short)0;
      reinterpret_cast<unsigned short*>(a.y_out)[(int64_t)route * H + r] = b;
    }
    if (tid == 0) FLINT_TL(11);
    grid_sync_retire(&ws->sync, nb);
    return;
  }
  for (int idx = tid; idx < (r1 - r0) * M; idx += NT) {
    const int m = idx / (r1 - r0), r = r0 + idx - m * (r1 - r0);
    float acc = 0.f;
    for (int s = 0; s < topk; ++s) {
      const unsigned short b = __ldcg(reinterpret_cast<const unsigned short*>(y_g + (int64_t)(m * topk + s) * H + r));
      acc = fmaf(tw_s[m * topk + s], bf16_bits_to_f32(b), acc);
    }
    a.out[(int64_t)m * H + r] = __float2bfloat16_rn(acc);
  }
  if (tid == 0) FLINT_TL(11);
  grid_sync_retire(&ws->sync, nb);
}

// dynamic shared memory: alignment slack, ring + dtile, the f16 token rows, and a region that holds the bf16 token rows
// in phase R and the staged act rows in phase D
static size_t moe_fused_smem(size_t ring_and_dtile, const MoeFusedArgs& a) {
  const size_t region = std::max((size_t)a.nslot_cap * xs_stride(a.I) * 2, (size_t)a.M * a.H * 2);
  return 1024 + ring_and_dtile + (size_t)a.M * xs_stride(a.H) * 2 + region;
}

template <int NS, int NV, int KG>
static int launch_fused(int sms, const CUtensorMap& uc, const CUtensorMap& us, const CUtensorMap& dc, const CUtensorMap& ds,
                        const MoeFusedArgs& a, int pdl, void* stream) {
  using L = EngineSmem<kFW, NS, kFBox>;
  const size_t smem = moe_fused_smem(L::ring_bytes + KG * L::dtile_bytes, a);
  auto kern = moe_fused_kernel<NS, NV, KG>;
  cudaFuncAttributes fa{};
  if (cudaFuncGetAttributes(&fa, kern) != cudaSuccess) return FLINT_ERR_LAUNCH;
  if (smem + fa.sharedSizeBytes > 227 * 1024) return FLINT_ERR_SHAPE;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return FLINT_ERR_LAUNCH;
  set_max_carveout(kern);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3((KG * kFW + 1) * 32);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 2 : 1;
  return record_cuda(cudaLaunchKernelEx(&cfg, kern, uc, us, dc, ds, a), FLINT_ERR_LAUNCH);
}

}  // namespace flint

using namespace flint;

int64_t flint::status_offset_moe_fused() { return (int64_t)offsetof(MoeFusedWs, status); }

FLINT_TL_READER(flint_timeline_moe_fused)

extern "C" int64_t flint_moe_fused_workspace_bytes(int64_t E, int64_t H, int64_t I) {
  return (int64_t)moe_fused_ws_bytes((int)E, (int)H, (int)I);
}

static int moe_fused_launch(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps, const void* gate_w,
                            int64_t M, int64_t H, int64_t E, int64_t topk, int score_fn, const void* w13, const void* s13,
                            const float* g13, const void* w2, const void* s2, const float* g2, int64_t I, int64_t e_lo,
                            int64_t n_local, void* out, void* y_out, void* res_out, void* xn_out, float* logits_out,
                            int32_t* topk_ids_out, float* topk_weights_out, void* workspace, int pdl, void* stream,
                            const PeerSet* ps = nullptr) {
  if (!x || !norm_w || !gate_w || !w13 || !s13 || !g13 || !w2 || !s2 || !g2 || (!out && !y_out && !ps) || !workspace)
    return FLINT_ERR_ARGUMENT;
  if (e_lo < 0 || n_local < 1 || e_lo + n_local > E) return FLINT_ERR_ARGUMENT;
  if (y_out && !aligned(y_out, 16)) return FLINT_ERR_ALIGN;
  const int sms = num_sms();
  if (sms <= 0) return FLINT_ERR_DEVICE;
  if (M < 1 || M > kMaxTokens || (H != 2048 && H != 4096) || E < 32 || E % 32 != 0 || E > 2 * sms || topk < 1 ||
      topk > 32 || topk > E || M * topk > kMaxRoutes || I < kSliceK || I % kSliceK != 0 || I > 8192 || ldx < H ||
      ldx % 8 != 0 || (score_fn != 0 && score_fn != 1))
    return FLINT_ERR_SHAPE;
  if (!aligned(x, 16) || (res && !aligned(res, 16)) || !aligned(norm_w, 16) || !aligned(gate_w, 16) || !aligned(w13, 16) ||
      !aligned(s13, 16) || !aligned(w2, 16) || !aligned(s2, 16) || (out && !aligned(out, 16)) || (res_out && !aligned(res_out, 16)) ||
      (xn_out && !aligned(xn_out, 16)) || !aligned(workspace, 16))
    return FLINT_ERR_ALIGN;
  if (res_out && !res) return FLINT_ERR_ARGUMENT;
  CUtensorMap uc, us, dc, ds;
  int rc = encode_u8_2d(&uc, w13, H / 2, n_local * 2 * I, H / 2, 128, kFBox, true);
  if (!rc) rc = encode_u8_2d(&us, s13, H / 16, n_local * 2 * I, H / 16, 16, kFBox, false);
  if (!rc) rc = encode_u8_2d(&dc, w2, I / 2, n_local * H, I / 2, 128, kFBox, true);
  if (!rc) rc = encode_u8_2d(&ds, s2, I / 16, n_local * H, I / 16, 16, kFBox, false);
  if (rc) return rc;
  MoeFusedArgs a;
  a.x = (const bf16*)x; a.ldx = ldx; a.res = (const bf16*)res; a.nw = (const bf16*)norm_w; a.eps = eps;
  a.gate_w = (const bf16*)gate_w; a.E = (int)E; a.topk = (int)topk; a.score_fn = score_fn; a.g13 = g13; a.g2 = g2;
  a.M = (int)M; a.H = (int)H; a.I = (int)I; a.out = (bf16*)out; a.res_out = (bf16*)res_out; a.xn_out = (bf16*)xn_out;
  a.logits_out = logits_out; a.ids_out = (int*)topk_ids_out; a.tw_out = topk_weights_out;
  a.ws = static_cast<MoeFusedWs*>(workspace);
  a.y_out = (bf16*)y_out;
  a.e_lo = (int)e_lo;
  a.e_hi = (y_out || ps) ? (int)(e_lo + n_local) : kNotLocal;
  a.peer = ps != nullptr;
  a.send = (const bf16*)x;
  if (ps) a.ps = *ps;
  else memset(&a.ps, 0, sizeof(a.ps));
  {
    // a CTA's down tiles (at most ceil(R tpd / grid) of them) span at most ceil(that / tpd) + 1 groups of <= 8 routes
    const long tpd = H / (2 * kFBox), tmax = (M * topk * tpd + sms - 1) / sms;
    a.nslot_cap = (int)std::min<long>(kMaxRoutes, ((tmax + tpd - 1) / tpd + 1) * 8);
  }
  // two consumer groups (16 consumer warps: the weight stream is consumer-bound with 8) and a 7-stage ring when they
  // fit beside the rows; else one group and a 4-stage ring
  if (H == 2048) {
    using L7 = EngineSmem<kFW, 7, kFBox>;
    if (moe_fused_smem(L7::ring_bytes + 2 * L7::dtile_bytes, a) + 12 * 1024 <= 227 * 1024)
      return launch_fused<7, 8, 2>(sms, uc, us, dc, ds, a, pdl, stream);
    return launch_fused<4, 8, 1>(sms, uc, us, dc, ds, a, pdl, stream);
  }
  return launch_fused<4, 16, 1>(sms, uc, us, dc, ds, a, pdl, stream);
}

extern "C" int flint_moe_fused(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps, const void* gate_w,
                               int64_t M, int64_t H, int64_t E, int64_t topk, int score_fn, const void* w13, const void* s13,
                               const float* g13, const void* w2, const void* s2, const float* g2, int64_t I, void* out,
                               void* res_out, void* xn_out, float* logits_out, int32_t* topk_ids_out,
                               float* topk_weights_out, void* workspace, int pdl, void* stream) {
  if (!out) return FLINT_ERR_ARGUMENT;
  return moe_fused_launch(x, ldx, res, norm_w, eps, gate_w, M, H, E, topk, score_fn, w13, s13, g13, w2, s2, g2, I, 0, E,
                          out, nullptr, res_out, xn_out, logits_out, topk_ids_out, topk_weights_out, workspace, pdl,
                          stream);
}

extern "C" int flint_moe_fused_ep(const void* x, int64_t ldx, const void* res, const void* norm_w, float eps,
                                  const void* gate_w, int64_t M, int64_t H, int64_t E, int64_t topk, int score_fn,
                                  const void* w13, const void* s13, const float* g13, const void* w2, const void* s2,
                                  const float* g2, int64_t I, int64_t expert_lo, int64_t n_local, void* y_out,
                                  void* res_out, float* logits_out, int32_t* topk_ids_out, float* topk_weights_out,
                                  void* workspace, int pdl, void* stream) {
  if (!y_out) return FLINT_ERR_ARGUMENT;
  return moe_fused_launch(x, ldx, res, norm_w, eps, gate_w, M, H, E, topk, score_fn, w13, s13, g13, w2, s2, g2, I,
                          expert_lo, n_local, nullptr, y_out, res_out, nullptr, logits_out, topk_ids_out,
                          topk_weights_out, workspace, pdl, stream);
}

extern "C" int flint_moe_fused_dp_peer(const void* send, const void* norm_w, float eps, const void* gate_w, int64_t H,
                                       int64_t E, int64_t topk, int score_fn, const void* w13, const void* s13,
                                       const float* g13, const void* w2, const void* s2, const float* g2, int64_t I,
                                       int64_t expert_lo, int64_t n_local, const void* const* peers, int rank,
                                       int world, void* res_out, float* logits_out, int32_t* topk_ids_out,
                                       float* topk_weights_out, void* workspace, int pdl, void* stream) {
  if (!send || !topk_ids_out || !topk_weights_out) return FLINT_ERR_ARGUMENT;
  if (topk > kPeerSlots) return FLINT_ERR_SHAPE;
  PeerSet ps;
  const int rc = peer_set(peers, rank, world, &ps);
  if (rc) return rc;
  // the M = world tokens come from the token tables; send's two rows (H apart) pass the launch's argument checks
  return moe_fused_launch(send, H, (const bf16*)send + H, norm_w, eps, gate_w, world, H, E, topk, score_fn, w13, s13,
                          g13, w2, s2, g2, I, expert_lo, n_local, nullptr, nullptr, res_out, nullptr, logits_out,
                          topk_ids_out, topk_weights_out, workspace, pdl, stream, &ps);
}
