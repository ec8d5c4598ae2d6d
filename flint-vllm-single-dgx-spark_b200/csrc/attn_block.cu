// (3) Fused decode attention block: add + RMSNorm -> NVFP4 QKV GEMV -> q/k RMSNorm + RoPE + KV write -> paged
// split-K GQA attention -> NVFP4 O projection, in ONE cooperative persistent launch (one CTA per SM).
// Replaces the reference's qkv_head_kernel and o_gemv_kernel (fast/attn_gemv2.cu:170-289) together with the decode
// attention between them (the Flint PR's CuTe _FlintDecodeAttention, patch:1741-2415); the numerics are those of
// attn_proj.cu and decode_attention.cu (same rounding points), only the summation partition differs.
//
// Work of CTA c (grid G = #SMs, 8 consumer warps + 1 TMA producer warp):
//  prologue  before the PDL wait the producer loads the CTA's QKV row groups (16 rows x K each) and O row groups into
//            shared memory, where they stay for the whole launch; after the wait it streams the CTA's KV pages
//            (8 KB: 16 tokens x [K | V] of one kv head) into a ring of np slots, so at short context every page is in
//            flight while phase A runs.
//  A  every CTA recomputes the add + RMSNorm (same bits everywhere; CTA 0 publishes res_out), stages it as f16 and
//     computes y = bf16(acc * gs) for its QKV rows: the K slices are split over the 8 warps and the partial tiles
//     summed in warp order.  y is published as epoch-tagged words (tagged.cuh); no grid barrier follows.
//  B  the pages of all (request, kv head) segments, in linear order, are cut into G contiguous ranges.  For each
//     segment piece of its range the CTA polls its q heads' words, normalises + ropes them; the warp that holds the
//     current token's page normalises + ropes the new k, writes k and v to the cache slot and patches its shared copy
//     of the page; each warp runs the online softmax over its pages (S = K q, exp2, P rounded to bf16, O += P V); the
//     CTA merges its warps (fixed order) and, unless it owns the whole segment (then it publishes the output),
//     writes one partial record and takes an arrival ticket for the segment.
//  B2 the CTAs with the last min(n, Gq) tickets of a segment merge its records once all n have arrived: per q head,
//     record weights exp2(m_r c - m c), the records' O folded by 8 warps in record order mod 8 and the 8 warp
//     results in warp order (sinks in the denominator); the output is published as tagged words.
//  C  every CTA stages the attention output (polling its tagged words) as f16 and computes its O rows from the
//     resident weights.  The kernel has no grid barrier.
#include "common.cuh"
#include "gridsync.cuh"
#include "tagged.cuh"
#include "nvfp4_tile.cuh"
#include "runtime.cuh"
#include "tma.cuh"
#include "timeline.cuh"

#include <algorithm>
#include <stdio.h>

// phase stamps of development builds (-DFLINT_TIMELINE): 0 entry, 1 PDL wait done, 2 norm staged, 3 QKV rows
// published, 4 page partition known, 5 first q heads fetched, 6 own pages done, 7 merges done, 8 O rows written,
// 12 norm computed (before the consumer barrier), 13 QKV weights resident, 14 QKV sums done;
// producer: 10 first page requested, 11 last page requested
FLINT_TL_BUFFER

namespace flint {

constexpr int kBW = 8;                       // consumer warps
constexpr int kBThreads = (kBW + 1) * 32;
constexpr int kBCons = kBW * 32;
constexpr int kBD = 128;                     // head dim
constexpr int kBPage = 16;                   // tokens per KV page
constexpr int kBPageBytes = kBPage * 2 * kBD * 2;
constexpr int kBUnitBytes = 2048 + 256;      // one 16-row x 256-k unit of an NVFP4 matrix: codes + scales
constexpr int kBMaxSeg = 64;                 // requests x kv heads
constexpr int kBMaxSlots = 16;
constexpr int kBGQ = 3;                      // max QKV row groups per CTA
constexpr int kBGO = 2;                      // max O row groups per CTA
constexpr float kBLog2e = 1.4426950408889634f;

struct BlockWs {
  GridSync gs;
  unsigned status;
  unsigned epoch;                    // launches so far: this launch tags its published words with epoch + 1
  unsigned pad[30];
  unsigned seg_cnt[kBMaxSeg];         // per split segment: pieces whose record is written (tickets taken)
  unsigned seg_done[kBMaxSeg];        // per split segment: merges finished (the last one resets both counters)
  // followed by: QKV output as tagged words [8][Nqkv / 2], attention output as tagged words [8][Ko / 2], records
};

struct BlockArgs {
  const bf16* x;
  int64_t ldx;
  const int* tokens;                 // optional embedding gather (row m of x = x[tokens[m]])
  const bf16* res;
  int64_t ldr;                       // row stride of res / res_out / out
  const bf16* nw;
  float eps;
  int M, H, Nqkv, nq, nkv, Gq;
  const float* gs_qkv;
  const bf16* q_w;
  const bf16* k_w;
  float eps_head;
  const int64_t* positions;
  const float* cos_sin;              // [max_pos, 128] (cos | sin), or null: no RoPE
  int64_t cs_stride;
  bf16* kv;                          // HND [blocks, nkv, 16, 256]
  int64_t st_block, st_head;         // elements
  const int* bt;
  int64_t bt_stride;
  int max_blocks;
  const int* seq_lens;
  const int64_t* slots;
  const float* sinks;
  int window;
  float c;                           // scale * log2(e)
  int Ko, No;
  const float* gs_o;
  bf16* out;
  bf16* res_out;
  bf16* q_out;                       // optional
  bf16* attn;                        // optional plain copy of the attention output [M][Ko] (the caller's)
  unsigned long long* attn_tag;      // workspace: attention output as tagged words [8][Ko / 2] (tagged.cuh)
  unsigned long long* y_tag;         // workspace: raw QKV output as tagged words of row pairs [8][Nqkv / 2]
  float* rec;                        // workspace: partial records
  int gq_total, go_total;            // row groups of 16
  int nks_q, nks_o;                  // 256-k slices
  int np;                            // page ring slots
  uint32_t off_ring, off_wo, off_xs, off_red, wq_scale_off, wo_scale_off;
  BlockWs* ws;
};

// record r: o [8][128] fp32, then (m, l) [8] float2
constexpr int kBRecFloats = 8 * kBD + 16;

__device__ __forceinline__ void cons_sync() { asm volatile("bar.sync 1, %0;" ::"r"(kBCons) : "memory"); }
// consumer barrier that also ANDs a predicate over the 256 consumer threads (uniform decisions after bounded waits)
__device__ __forceinline__ bool cons_sync_and(bool pred) {
  int r;
  asm volatile("{\n.reg .pred p, q;\nsetp.ne.s32 p, %1, 0;\nbar.red.and.pred q, 1, %2, p;\nselp.s32 %0, 1, 0, q;\n}"
               : "=r"(r) : "r"((int)pred), "r"(kBCons) : "memory");
  return r != 0;
}

__device__ __forceinline__ void st_shared_u16(uint32_t addr, unsigned short v) {
  asm volatile("st.shared.u16 [%0], %1;" ::"r"(addr), "h"(v) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
// shared address of the 16-byte unit (token row, dim unit) of a page held as four 128B-swizzled boxes K0 K1 V0 V1
__device__ __forceinline__ uint32_t bpage_unit(uint32_t page, int box, int row, int unit) {
  return page + box * 2048 + row * 128 + ((unit ^ (row & 7)) << 4);
}

// Resident NVFP4 GEMV: ng row groups x nks slices in shared memory (unit (gi, ks) codes at wc + (gi*nks+ks)*2048,
// scales at wsc + (gi*nks+ks)*256); warp w takes slices w, w+8, ...; partial tiles to red[gi][w][16][8].
// One out-of-line copy serves both projections (QKV in phase A, O in phase C), so the O projection finds its code
// already in the instruction caches.
__device__ __noinline__ void gemv_resident(const uint8_t* wc, const uint8_t* wsc, int ng, int nks, const __half* xs, int K,
                                           int M, float* red, int warp, int lane) {
  const int g = lane >> 2, t = lane & 3;
  const bool active = g < M;
  const __half* xrow = xs + (active ? g : 0) * xs_stride(K);
  const int r0 = tile_phi(g), r1 = r0 + 8, n0 = 2 * t, n1 = 2 * t + 1;
  // one row group at a time, slice loop rolled: the tile code appears once; the per-group sums are unchanged
#pragma unroll 1
  for (int gi = 0; gi < ng; ++gi) {
    float acc[4][4];
    zero_acc(acc);
#pragma unroll 1
    for (int ks = warp; ks < nks; ks += kBW)
      consume_stage(wc + (gi * nks + ks) * 2048, wsc + (gi * nks + ks) * 256, 0, g, t, ks, xrow, active, acc);
    float d[4];
    sum_acc(acc, d);
    float* rt = red + (gi * kBW + warp) * 128;
    rt[r0 * 8 + n0] = d[0];
    rt[r0 * 8 + n1] = d[1];
    rt[r1 * 8 + n0] = d[2];
    rt[r1 * 8 + n1] = d[3];
  }
}

// O projection streamed over the attention output (tagged words, src[m * src_words + k / 2]): warp w takes K slices
// w, w + 8, ... (256 k = two heads each) and stages each one as soon as its words carry `ep` -- per token with the
// slice's own power-of-two shift (the rule of stage_rows_f16 over the slice) -- so a warp starts while other heads are
// still being merged.  Each slice's partial tile is rescaled by 2^-shift before it joins the warp's sum; partial
// tiles go to red[gi][w][16][8] with the scales applied (finish with zero shifts).
__device__ __noinline__ void gemv_stream_o(const uint8_t* wc, const uint8_t* wsc, int ng, int nks,
                                           const unsigned long long* src, int64_t src_words, unsigned ep, __half* xs,
                                           int K, int M, float* red, int warp, int lane, unsigned* status) {
  const int g = lane >> 2, t = lane & 3;
  const bool active = g < M;
  const __half* xrow = xs + (active ? g : 0) * xs_stride(K);
  float tot[kBGO][4];
#pragma unroll
  for (int gi = 0; gi < kBGO; ++gi) tot[gi][0] = tot[gi][1] = tot[gi][2] = tot[gi][3] = 0.f;
#pragma unroll 1
  for (int ks = warp; ks < nks; ks += kBW) {
    int my_sh = 0;                                     // lane m < M: the shift of token m for this slice
#pragma unroll 1
    for (int m = 0; m < M; ++m) {
      const unsigned long long* p = src + (int64_t)m * src_words + ks * 128 + lane * 4;
      ulonglong2 w0, w1;
      unsigned it = 0;
#pragma unroll 1
      for (;; ++it) {
        w0 = ld_tagged2(p);
        w1 = ld_tagged2(p + 2);
        if (tag_is(w0.x, ep) && tag_is(w0.y, ep) && tag_is(w1.x, ep) && tag_is(w1.y, ep)) break;
        if (it == FLINT_WAIT_LIMIT) {
          atomicOr(status, STATUS_WAIT_TIMEOUT);
          break;
        }
        poll_pause();
      }
      const uint4 v = make_uint4((uint32_t)w0.x, (uint32_t)w0.y, (uint32_t)w1.x, (uint32_t)w1.y);
      float f[8];
      bf16x8_to_f32(v, f);
      unsigned mxb = 0u;
#pragma unroll
      for (int j = 0; j < 8; ++j) mxb = max(mxb, __float_as_uint(fabsf(f[j])));
      mxb = __reduce_max_sync(0xffffffffu, mxb);
      const float mx = __uint_as_float(mxb);
      int sh = 0;
      if (mx > 0.f && !(mx != mx) && mx <= 3.0e38f) sh = 14 - ((int)((mxb >> 23) & 0xFF) - 127);
      if (lane == m) my_sh = sh;
      uint32_t h[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        __half2 hv = __floats2half2_rn(scale_pow2(f[2 * j], sh), scale_pow2(f[2 * j + 1], sh));
        h[j] = *reinterpret_cast<uint32_t*>(&hv);
      }
      *reinterpret_cast<uint4*>(xs + m * xs_stride(K) + xs_perm(ks * 256 + lane * 8)) = make_uint4(h[0], h[1], h[2], h[3]);
    }
    __syncwarp();
    const int c0 = 2 * t, c1 = 2 * t + 1;              // this lane's tile columns (tokens)
    const int sh0 = __shfl_sync(0xffffffffu, my_sh, c0 & 31), sh1 = __shfl_sync(0xffffffffu, my_sh, c1 & 31);
#pragma unroll
    for (int gi = 0; gi < kBGO; ++gi) {
      if (gi >= ng) break;
      float acc[4][4];
      zero_acc(acc);
      consume_stage(wc + (gi * nks + ks) * 2048, wsc + (gi * nks + ks) * 256, 0, g, t, ks, xrow, active, acc);
      float d[4];
      sum_acc(acc, d);
      tot[gi][0] += scale_pow2(d[0], -sh0);
      tot[gi][1] += scale_pow2(d[1], -sh1);
      tot[gi][2] += scale_pow2(d[2], -sh0);
      tot[gi][3] += scale_pow2(d[3], -sh1);
    }
    __syncwarp();
  }
  const int r0 = tile_phi(g), r1 = r0 + 8, n0 = 2 * t, n1 = 2 * t + 1;
#pragma unroll
  for (int gi = 0; gi < kBGO; ++gi) {
    if (gi >= ng) break;
    float* rt = red + (gi * kBW + warp) * 128;
    rt[r0 * 8 + n0] = tot[gi][0];
    rt[r0 * 8 + n1] = tot[gi][1];
    rt[r1 * 8 + n0] = tot[gi][2];
    rt[r1 * 8 + n1] = tot[gi][3];
  }
}

// out[m][row0 + 16 gi + r] = bf16(sum_w red[gi][w][r][m] * gs * 2^-shift[m]); consumer threads.
__device__ __forceinline__ void gemv_finish(const float* red, int ng, int M, float gs, const int* shift, bf16* out,
                                            int64_t ld, int row0) {
  for (int idx = threadIdx.x; idx < ng * 16 * M; idx += kBCons) {
    const int gi = idx / (16 * M), rem = idx - gi * 16 * M, r = rem / M, m = rem - r * M;
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kBW; ++w) s += red[(gi * kBW + w) * 128 + r * 8 + m];
    out[(int64_t)m * ld + row0 + gi * 16 + r] = __float2bfloat16_rn(s * ldexpf(gs, -shift[m]));
  }
}

// out[m][row0 + 16 gi + r] for the QKV rows, as tagged words of row pairs (same per-row sums and rounding as
// gemv_finish): word (row0 + 16 gi + r) / 2 of row m carries rows r, r + 1 (r even).
__device__ __forceinline__ void gemv_finish_tagged(const float* red, int ng, int M, float gs, const int* shift,
                                                   unsigned long long* out, int64_t ld_words, int row0, unsigned ep) {
  for (int idx = threadIdx.x; idx < ng * 8 * M; idx += kBCons) {
    const int gi = idx / (8 * M), rem = idx - gi * 8 * M, r = 2 * (rem / M), m = rem - (r / 2) * M;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int w = 0; w < kBW; ++w) {
      s0 += red[(gi * kBW + w) * 128 + r * 8 + m];
      s1 += red[(gi * kBW + w) * 128 + (r + 1) * 8 + m];
    }
    const float sc = ldexpf(gs, -shift[m]);
    st_tagged(out + (int64_t)m * ld_words + (row0 + gi * 16 + r) / 2, ep, pack_bf16x2(s0 * sc, s1 * sc));
  }
}

// A lane's 4 dims of a 128-dim head in the pair layout of the tagged QKV words: 2 lane, 2 lane + 1, 64 + 2 lane,
// 65 + 2 lane (so RoPE partners d and d + 64 sit in one lane, as i and i + 2).
__device__ __forceinline__ int pdim(int lane, int i) { return (i & 2) * 32 + 2 * lane + (i & 1); }

// The lane's 4 values of head `head` of a tagged QKV row, once they carry this launch's tag (bounded poll).
__device__ __forceinline__ void fetch_head(const unsigned long long* yrow, int head, unsigned ep, float (&v)[4], int lane,
                                           unsigned* status) {
  const unsigned long long* p = yrow + head * (kBD / 2) + lane;
  unsigned long long w0 = 0, w1 = 0;
  unsigned it = 0;
#pragma unroll 1
  for (;; ++it) {
    w0 = ld_tagged(p);
    w1 = ld_tagged(p + 32);
    if (tag_is(w0, ep) && tag_is(w1, ep)) break;
    if (it == FLINT_WAIT_LIMIT) {
      atomicOr(status, STATUS_WAIT_TIMEOUT);
      break;
    }
    poll_pause();
  }
  v[0] = bf16_bits_to_f32((uint32_t)w0 & 0xFFFFu);
  v[1] = bf16_bits_to_f32(((uint32_t)w0) >> 16);
  v[2] = bf16_bits_to_f32((uint32_t)w1 & 0xFFFFu);
  v[3] = bf16_bits_to_f32(((uint32_t)w1) >> 16);
}

// q / k head finish (attn_proj.cu's epilogue): y (4 values per lane, dims pdim(lane, i)) -> bf16(rmsnorm(y) * w) ->
// RoPE (rotate-half: d with d + 64).
__device__ __forceinline__ void head_norm_rope(float (&v)[4], const bf16* w, float eps, const float* cs, int lane) {
  float v2 = v[0] * v[0] + v[1] * v[1] + v[2] * v[2] + v[3] * v[3];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v2 += __shfl_xor_sync(0xffffffffu, v2, off);
  const float rs = rsqrtf(v2 / (float)kBD + eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = bf16r(v[i] * rs * __bfloat162float(w[pdim(lane, i)]));
  if (cs) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int r = 2 * lane + i;
      const float c = cs[r], s = cs[64 + r];
      const float n1 = v[i], n2 = v[i + 2];
      v[i] = fmaf(n1, c, -(n2 * s));
      v[i + 2] = fmaf(n2, c, n1 * s);
    }
  }
}

// attention output of request b, columns col .. col + 2 n - 1 (n bf16 pairs, col even): tagged words for the O
// projection of this launch, plus the caller's plain copy when one was asked for
__device__ __forceinline__ void publish_attn(const BlockArgs& a, unsigned ep, int b, int col, const uint32_t* pk, int n) {
  for (int i = 0; i < n; ++i) st_tagged(a.attn_tag + (int64_t)b * (a.Ko / 2) + col / 2 + i, ep, pk[i]);
  if (a.attn)
    for (int i = 0; i < n; ++i) reinterpret_cast<uint32_t*>(a.attn + (int64_t)b * a.Ko + col)[i] = pk[i];
}

// MC > 0: the batch size fixed at compile time (MC = 1 is the single-stream decode: every per-token loop collapses,
// which shrinks the code each launch has to fetch into the instruction caches); MC = 0: M = a.M at run time.
template <int MC>
__global__ void __launch_bounds__(kBThreads, 1)
attn_block_kernel(const __grid_constant__ CUtensorMap mqc, const __grid_constant__ CUtensorMap mqs,
                  const __grid_constant__ CUtensorMap moc, const __grid_constant__ CUtensorMap mos,
                  const __grid_constant__ CUtensorMap mkv, const BlockArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t full[kBMaxSlots], empty[kBMaxSlots], bar_wq, bar_wo, bar_tab;
  __shared__ int shift[8];
  __shared__ float red_n[kBW * 8 + 8];
  __shared__ int s_pf[8], s_npg[8], s_seq[8], s_start[8], s_pre[9];
  // per segment (request x kv head): first page slot A in the flattened page list, first owning CTA, number of
  // owning CTAs (partial records) and first record; plus the flattened page count P
  __shared__ int s_segA[kBMaxSeg], s_first[kBMaxSeg], s_nparts[kBMaxSeg], s_recb[kBMaxSeg], s_P;
  __shared__ int s_tk_seg[kBMaxSeg], s_tk[kBMaxSeg], s_ntk, s_go;   // this CTA's merge tickets
  __shared__ int s_lo, s_hi;                                          // this CTA's flattened page range
  __shared__ __align__(16) bf16 q_tile[8][kBD];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int G = gridDim.x, cta = blockIdx.x;
  const int M = MC > 0 ? MC : a.M;
  if (threadIdx.x == 0) FLINT_TL(0);
  unsigned* status = &a.ws->status;
  uint8_t* ring = smem + a.off_ring;
  uint8_t* wq = smem;                                  // QKV weights (phase A), then warp partials (phase B)
  uint8_t* wo = smem + a.off_wo;
  __half* xs = reinterpret_cast<__half*>(smem + a.off_xs);
  float* red = reinterpret_cast<float*>(smem + a.off_red);
  __half* xs_o = reinterpret_cast<__half*>(smem);       // phase C: over the QKV weights and the page ring

  const int gq0 = (int)((int64_t)cta * a.gq_total / G), ngq = (int)((int64_t)(cta + 1) * a.gq_total / G) - gq0;
  const int go0 = (int)((int64_t)cta * a.go_total / G), ngo = (int)((int64_t)(cta + 1) * a.go_total / G) - go0;

  if (threadIdx.x == 0) {
    for (int i = 0; i < a.np; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&bar_wq, 1);
    mbar_init(&bar_wo, 1);
    mbar_init(&bar_tab, 1);
    fence_mbar_init();
  }
  __syncthreads();

  // ---- prologue: resident weights (independent of the previous kernel) ----
  if (warp == kBW && lane == 0) {
    tma_prefetch_desc(&mqc);
    tma_prefetch_desc(&mqs);
    tma_prefetch_desc(&mkv);
    // one 3-D box per 16-row group: all K slices at once, landing as [slice][16 rows][128 B] (codes, swizzled) and
    // [slice][16 rows][16 B] (scales)
    if (ngq > 0) {
      mbar_arrive_expect_tx(&bar_wq, ngq * a.nks_q * kBUnitBytes);
      for (int gi = 0; gi < ngq; ++gi) {
        tma_load_3d(wq + gi * a.nks_q * 2048, &mqc, 0, (gq0 + gi) * 16, 0, &bar_wq);
        tma_load_3d(wq + a.wq_scale_off + gi * a.nks_q * 256, &mqs, 0, (gq0 + gi) * 16, 0, &bar_wq);
      }
    }
    if (ngo > 0) {
      mbar_arrive_expect_tx(&bar_wo, ngo * a.nks_o * kBUnitBytes);
      for (int gi = 0; gi < ngo; ++gi) {
        tma_load_3d(wo + gi * a.nks_o * 2048, &moc, 0, (go0 + gi) * 16, 0, &bar_wo);
        tma_load_3d(wo + a.wo_scale_off + gi * a.nks_o * 256, &mos, 0, (go0 + gi) * 16, 0, &bar_wo);
      }
    }
  }
  // the consumers' norm weights (8 per thread) do not depend on the previous kernel either
  const uint4 nwc = warp < kBW && (int)threadIdx.x < (a.H >> 3) ? reinterpret_cast<const uint4*>(a.nw)[threadIdx.x]
                                                                : make_uint4(0u, 0u, 0u, 0u);
  pdl_wait();
  if (threadIdx.x == 0) FLINT_TL(1);
  unsigned ep;                                         // this launch's tag (the last CTA to retire advances it)
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(ep) : "l"(&a.ws->epoch) : "memory");
  ep += 1u;
  const int S = M * a.nkv;
  if (warp == kBW) {
    // ---- producer: the page partition inputs from the sequence lengths, right after the wait (the consumers run
    // the norm meanwhile; they read these tables only once bar_tab has been released) ----
    if (lane == 0) {
      int pre = 0;
      for (int b = 0; b < M; ++b) {
        const int seq = a.seq_lens[b];
        const int start = a.window > 0 ? max(0, seq - a.window) : 0;
        const int pf = start / kBPage;
        int pe = (seq + kBPage - 1) / kBPage;
        if (pe > a.max_blocks) {
          atomicOr(status, 4u);
          pe = a.max_blocks;
        }
        s_seq[b] = seq;
        s_start[b] = start;
        s_pf[b] = pf;
        s_npg[b] = max(0, pe - pf);
        s_pre[b] = pre;
        pre += s_npg[b];
      }
      s_pre[M] = pre;
      s_P = a.nkv * pre;
      s_ntk = 0;
    }
    __syncwarp();
  } else {
    // ---- A (first half), consumers: add + RMSNorm ----
    if (a.H / 8 <= kBCons)
      norm_stage_f16_1w(a.x, a.ldx, a.tokens, a.res, a.ldr, nwc, a.eps, M, a.H, xs, shift, red_n,
                        cta == 0 ? a.res_out : nullptr, kBCons, 1);
    else
      norm_stage_f16(a.x, a.ldx, a.tokens, a.res, a.ldr, a.nw, a.eps, M, a.H, xs, shift, red_n,
                     cta == 0 ? a.res_out : nullptr, kBCons, 1);
    if (threadIdx.x == 0) FLINT_TL(12);
    cons_sync();
    if (threadIdx.x == 0) FLINT_TL(2);
  }

  if (warp == kBW) {
    const int P = s_P;
    // ---- producer, next: the partition, off the consumers' critical path (released to them through bar_tab).
    // Each CTA works on ONE segment: segment s gets k_s CTAs in proportion to its n_s pages (floor of n_s G / P, at
    // least 1, at most n_s; spare CTAs to the largest remainders, ties to the lower segment), which split its pages
    // evenly in CTA order; CTA c0_s + i owns pages [A_s + i n_s / k_s, A_s + (i + 1) n_s / k_s) and writes record
    // c0_s + i when k_s > 1.  Lane sg (and sg + 32) handles segment sg.  32-bit: the host keeps M * nkv * max_blocks *
    // grid below 2^32. ----
    {
      const unsigned Pu = (unsigned)P, Gu = (unsigned)G;
      int n[2], k[2], rm[2], A[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int sg = lane + 32 * h;
        n[h] = k[h] = A[h] = 0;
        rm[h] = -1;
        if (sg < S) {
          const int b = sg / a.nkv;
          n[h] = s_npg[b];
          A[h] = a.nkv * s_pre[b] + (sg - b * a.nkv) * n[h];
          if (n[h] > 0) {
            const unsigned q = (unsigned)n[h] * Gu;
            k[h] = (int)(q / Pu);
            rm[h] = (int)(q - (unsigned)k[h] * Pu);
            if (k[h] == 0) {
              k[h] = 1;
              rm[h] = -1;
            }
            if (k[h] >= n[h]) {
              k[h] = n[h];
              rm[h] = -1;
            }
          }
        }
      }
      auto warp_total = [&]() {
        int t = k[0] + k[1];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        return t;
      };
      int tot = warp_total();
      if (tot < G) {                                               // spare CTAs: largest remainders first
        int rank[2] = {0, 0};
#pragma unroll 1
        for (int jj = 0; jj < 64; ++jj) {
          const int rj = __shfl_sync(0xffffffffu, jj < 32 ? rm[0] : rm[1], jj & 31);
#pragma unroll
          for (int h = 0; h < 2; ++h)
            if (rj > rm[h] || (rj == rm[h] && jj < lane + 32 * h)) ++rank[h];
        }
#pragma unroll
        for (int h = 0; h < 2; ++h)
          if (rm[h] >= 0 && rank[h] < G - tot) ++k[h];
        tot = warp_total();
      }
#pragma unroll 1
      for (int guard = 0; tot > G && guard < 64; ++guard) {        // segments bumped to one CTA: give back the largest
        unsigned best = 0u;
#pragma unroll
        for (int h = 0; h < 2; ++h)
          if (k[h] > 1) best = max(best, ((unsigned)k[h] << 8) | (unsigned)(lane + 32 * h));
        best = __reduce_max_sync(0xffffffffu, best);
        if (best == 0u) break;
#pragma unroll
        for (int h = 0; h < 2; ++h)
          if (k[h] > 1 && (((unsigned)k[h] << 8) | (unsigned)(lane + 32 * h)) == best) --k[h];
        --tot;
      }
      int inc0 = k[0], inc1 = k[1];                                // first CTA of each segment: exclusive scan
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int v0 = __shfl_up_sync(0xffffffffu, inc0, o), v1 = __shfl_up_sync(0xffffffffu, inc1, o);
        if (lane >= o) {
          inc0 += v0;
          inc1 += v1;
        }
      }
      const int tot0 = __shfl_sync(0xffffffffu, inc0, 31);
      const int c0[2] = {inc0 - k[0], tot0 + inc1 - k[1]};
      if (lane == 0) s_lo = s_hi = 0;                              // a CTA without a segment has no pages
      __syncwarp();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int sg = lane + 32 * h;
        if (sg < S) {
          s_segA[sg] = A[h];
          s_first[sg] = c0[h];
          s_nparts[sg] = k[h];
          s_recb[sg] = c0[h];
          if (k[h] > 0 && cta >= c0[h] && cta < c0[h] + k[h]) {
            const int i = cta - c0[h];
            s_lo = A[h] + i * n[h] / k[h];
            s_hi = A[h] + (i + 1) * n[h] / k[h];
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar_tab);
    }
    const int lo = s_lo, hi = s_hi;
    // ---- producer: this CTA's pages, in the order the consumers take them, from the start: the ring fills
    // while the norm and the QKV GEMV run (the resident weights were requested before the wait) ----
    if (lane == 0) {
      FLINT_TL(10);
      int j = 0;
      for (int s = 0; s < S; ++s) {
        const int b = s / a.nkv, kvh = s - b * a.nkv;
        const int A = s_segA[s], from = max(A, lo), to = min(A + s_npg[b], hi);
        const int* btb = a.bt + (int64_t)b * a.bt_stride;
        for (int L = from; L < to; ++L, ++j) {
          const int slot = j % a.np, round = j / a.np;
          if (!mbar_wait(&empty[slot], (round & 1) ^ 1u, status)) return;
          const int blk = btb[s_pf[b] + (L - A)];
          mbar_arrive_expect_tx(&full[slot], kBPageBytes);
          // the whole page in one 5-D box: [K0 K1 V0 V1][16 rows][64 dims], each quarter 128B-swizzled
          tma_load_5d(ring + slot * kBPageBytes, &mkv, 0, 0, 0, kvh, blk, &full[slot]);
        }
      }
      FLINT_TL(11);
    }
    return;
  }

  // ================= consumers (256 threads) =================
  // ---- A (second half): QKV rows ----
  if (ngq > 0 && cons_sync_and(mbar_wait(&bar_wq, 0, status))) {
    if (threadIdx.x == 0) FLINT_TL(13);
    gemv_resident(wq, wq + a.wq_scale_off, ngq, a.nks_q, xs, a.H, M, red, warp, lane);
    cons_sync();
    if (threadIdx.x == 0) FLINT_TL(14);
    gemv_finish_tagged(red, ngq, M, a.gs_qkv[0], shift, a.y_tag, a.Nqkv / 2, gq0 * 16, ep);
  }
  if (threadIdx.x == 0) FLINT_TL(3);
  const bool have_tab = cons_sync_and(mbar_wait(&bar_tab, 0, status));   // segment tables from the producer warp
  if (threadIdx.x == 0) FLINT_TL(4);
  const int lo = s_lo, hi = s_hi;

  // ---- B: attention ----
  const int tid = threadIdx.x, g = lane >> 2, t4 = lane & 3;
  const float c = a.c;
  float* wo_p = reinterpret_cast<float*>(wq);                     // [8 warps][8 heads][128]
  float* wm = wo_p + kBW * 8 * kBD;                               // [8][16]
  float* wl = wm + kBW * 16;
  // empty segments (no pages): zero output, KV write of the slot (by CTA s % G)
  for (int s = cta; s < S; s += G) {
    const int b = s / a.nkv, kvh = s - b * a.nkv;
    if (s_npg[b] != 0) continue;
    if (tid < a.Gq * 16) {
      const int hh = tid >> 4, d0 = (tid & 15) * 8;
      const uint32_t zero[4] = {0u, 0u, 0u, 0u};
      publish_attn(a, ep, b, (kvh * a.Gq + hh) * kBD + d0, zero, 4);
    }
    if (a.q_out && warp < a.Gq) {                                 // q of the empty request still goes out
      const int qh = kvh * a.Gq + warp;
      float q[4];
      fetch_head(a.y_tag + (int64_t)b * (a.Nqkv / 2), qh, ep, q, lane, status);
      head_norm_rope(q, a.q_w, a.eps_head, a.cos_sin ? a.cos_sin + a.positions[b] * a.cs_stride : nullptr, lane);
#pragma unroll
      for (int i = 0; i < 4; ++i) a.q_out[(int64_t)b * a.nq * kBD + qh * kBD + pdim(lane, i)] = __float2bfloat16_rn(q[i]);
    }
    if (warp == 0 && a.slots && a.slots[b] >= 0) {
      const unsigned long long* yrow = a.y_tag + (int64_t)b * (a.Nqkv / 2);
      float k[4], v[4];
      fetch_head(yrow, a.nq + kvh, ep, k, lane, status);
      fetch_head(yrow, a.nq + a.nkv + kvh, ep, v, lane, status);
      head_norm_rope(k, a.k_w, a.eps_head, a.cos_sin ? a.cos_sin + a.positions[b] * a.cs_stride : nullptr, lane);
      const int64_t slot = a.slots[b];
      bf16* dst = a.kv + (slot / kBPage) * a.st_block + (int64_t)kvh * a.st_head + (slot % kBPage) * (2 * kBD);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        dst[pdim(lane, i)] = __float2bfloat16_rn(k[i]);
        dst[kBD + pdim(lane, i)] = __float2bfloat16_rn(v[i]);
      }
    }
  }

  int j = 0;                                                       // CTA page sequence (matches the producer)
  for (int s = 0; have_tab && s < S; ++s) {
    const int b = s / a.nkv, kvh = s - b * a.nkv;
    const int A = s_segA[s], n = s_npg[b];
    const int from = max(A, lo), to = min(A + n, hi);
    if (from >= to) continue;
    const int c_first = s_first[s], n_parts = s_nparts[s];
    const int seq = s_seq[b], start = s_start[b], last_page = (seq - 1) / kBPage;
    const unsigned long long* yrow = a.y_tag + (int64_t)b * (a.Nqkv / 2);
    const float* cs = a.cos_sin ? a.cos_sin + a.positions[b] * a.cs_stride : nullptr;
    // q heads of this segment: warp hh, once the QKV rows carry this launch's tag (no grid barrier)
    {
      float q[4] = {0.f, 0.f, 0.f, 0.f};
      if (warp < a.Gq) {
        const int qh = kvh * a.Gq + warp;
        fetch_head(yrow, qh, ep, q, lane, status);
        head_norm_rope(q, a.q_w, a.eps_head, cs, lane);
        if (a.q_out && cta == c_first) {
#pragma unroll
          for (int i = 0; i < 4; ++i) a.q_out[(int64_t)b * a.nq * kBD + qh * kBD + pdim(lane, i)] = __float2bfloat16_rn(q[i]);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) q_tile[warp][pdim(lane, i)] = __float2bfloat16_rn(q[i]);
    }
    cons_sync();
    if (threadIdx.x == 0 && j == 0) FLINT_TL(5);
    uint32_t qa[8][2];
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      qa[kk][0] = *reinterpret_cast<const uint32_t*>(&q_tile[g][16 * kk + 2 * t4]);
      qa[kk][1] = *reinterpret_cast<const uint32_t*>(&q_tile[g][16 * kk + 8 + 2 * t4]);
    }
    float o[16][4];
#pragma unroll
    for (int dt = 0; dt < 16; ++dt)
#pragma unroll
      for (int e = 0; e < 4; ++e) o[dt][e] = 0.f;
    float m_run = -INFINITY, l_run = 0.f;

    for (int L = from; L < to; ++L, ++j) {
      if (j % kBW != warp) continue;
      const int slot = j % a.np;
      if (!mbar_wait(&full[slot], (j / a.np) & 1, status)) break;
      const uint32_t page = smem_u32(ring + slot * kBPageBytes);
      const int p = s_pf[b] + (L - A);                             // page index within the request
      if (p == last_page) {
        // the current token: new k (normalised + roped) and v, to the cache slot and into this page's shared copy
        float k[4], v[4];
        fetch_head(yrow, a.nq + kvh, ep, k, lane, status);
        fetch_head(yrow, a.nq + a.nkv + kvh, ep, v, lane, status);
        head_norm_rope(k, a.k_w, a.eps_head, cs, lane);
        const int64_t slot_b = a.slots ? a.slots[b] : -1;
        if (slot_b >= 0) {
          bf16* dst = a.kv + (slot_b / kBPage) * a.st_block + (int64_t)kvh * a.st_head + (slot_b % kBPage) * (2 * kBD);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            dst[pdim(lane, i)] = __float2bfloat16_rn(k[i]);
            dst[kBD + pdim(lane, i)] = __float2bfloat16_rn(v[i]);
          }
          const int row = (seq - 1) % kBPage;
          const int64_t here = (int64_t)a.bt[(int64_t)b * a.bt_stride + p] * kBPage + row;
          if (slot_b == here) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              const int d = pdim(lane, i);
              const uint32_t off = (d & 7) * 2;
              st_shared_u16(bpage_unit(page, d >> 6, row, (d & 63) >> 3) + off,
                            __bfloat16_as_ushort(__float2bfloat16_rn(k[i])));
              st_shared_u16(bpage_unit(page, 2 + (d >> 6), row, (d & 63) >> 3) + off,
                            __bfloat16_as_ushort(__float2bfloat16_rn(v[i])));
            }
            fence_proxy_async();                                  // ordered before the slot's next TMA fill
          }
        }
        __syncwarp();
      }
      // ---- S = K q ----
      float sc[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) sc[nt][e] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const int mat = lane >> 3, r = lane & 7;
        const int row = 8 * (mat >> 1) + r;
        const int dim = 16 * kk + 8 * (mat & 1);
        uint32_t k0, k1, k2, k3;
        ldsm_x4(bpage_unit(page, dim >> 6, row, (dim & 63) >> 3), k0, k1, k2, k3);
        const uint32_t aq[4] = {qa[kk][0], 0u, qa[kk][1], 0u};
        mma_bf16(sc[0], aq, k0, k1);
        mma_bf16(sc[1], aq, k2, k3);
      }
      // ---- mask + online softmax (row g = head g; lane holds tokens 8nt + 2t4 + {0,1}) ----
      float sv[4] = {sc[0][0], sc[0][1], sc[1][0], sc[1][1]};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int tok = p * kBPage + 8 * (i >> 1) + 2 * t4 + (i & 1);
        if (tok >= seq || tok < start) sv[i] = -INFINITY;
      }
      float mx = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run, mx);
      const float alpha = m_run == -INFINITY ? 0.f : exp2f(m_run * c - m_new * c);
      float pv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pv[i] = sv[i] == -INFINITY ? 0.f : exp2f(sv[i] * c - m_new * c);
      l_run = l_run * alpha + ((pv[0] + pv[1]) + (pv[2] + pv[3]));
      m_run = m_new;
#pragma unroll
      for (int dt = 0; dt < 16; ++dt) {
        o[dt][0] *= alpha;
        o[dt][1] *= alpha;
      }
      // ---- O += P V ----
      const uint32_t pa[4] = {pack_bf16x2(pv[0], pv[1]), 0u, pack_bf16x2(pv[2], pv[3]), 0u};
#pragma unroll
      for (int dp = 0; dp < 8; ++dp) {
        const int mat = lane >> 3, r = lane & 7;
        const int row = 8 * (mat & 1) + r;
        const int dim = 16 * dp + 8 * (mat >> 1);
        uint32_t v0, v1, v2, v3;
        ldsm_x4_t(bpage_unit(page, 2 + (dim >> 6), row, (dim & 63) >> 3), v0, v1, v2, v3);
        mma_bf16(o[2 * dp], pa, v0, v1);
        mma_bf16(o[2 * dp + 1], pa, v2, v3);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[slot]);
    }

    // ---- merge the warps (fixed order) ----
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
    l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
    if (t4 == 0) {
      wm[warp * 16 + g] = m_run;
      wl[warp * 16 + g] = l_run;
    }
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      wo_p[(warp * 8 + g) * kBD + 8 * dt + 2 * t4] = o[dt][0];
      wo_p[(warp * 8 + g) * kBD + 8 * dt + 2 * t4 + 1] = o[dt][1];
    }
    cons_sync();
    if (tid < 128) {
      const int hh = tid >> 4, d0 = (tid & 15) * 8;
      float mc = -INFINITY;
#pragma unroll
      for (int w = 0; w < kBW; ++w) mc = fmaxf(mc, wm[w * 16 + hh]);
      float lc = 0.f, oc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) oc[i] = 0.f;
#pragma unroll
      for (int w = 0; w < kBW; ++w) {
        const float mw = wm[w * 16 + hh];
        if (mw == -INFINITY) continue;
        const float f = exp2f(mw * c - mc * c);
        lc += wl[w * 16 + hh] * f;
#pragma unroll
        for (int i = 0; i < 8; ++i) oc[i] += wo_p[(w * 8 + hh) * kBD + d0 + i] * f;
      }
      if (n_parts == 1) {
        if (hh < a.Gq) {
          const int qh = kvh * a.Gq + hh;
          float den = lc;
          if (a.sinks && mc != -INFINITY) den += exp2f(a.sinks[qh] * kBLog2e - mc * c);
          const float inv = den > 0.f ? 1.0f / den : 0.f;
          uint32_t pk[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) pk[i] = pack_bf16x2(oc[2 * i] * inv, oc[2 * i + 1] * inv);
          publish_attn(a, ep, b, qh * kBD + d0, pk, 4);
        }
      } else {
        float* rec = a.rec + (int64_t)(s_recb[s] + cta - c_first) * kBRecFloats;
        __stcg(reinterpret_cast<float4*>(rec + hh * kBD + d0), make_float4(oc[0], oc[1], oc[2], oc[3]));
        __stcg(reinterpret_cast<float4*>(rec + hh * kBD + d0) + 1, make_float4(oc[4], oc[5], oc[6], oc[7]));
        if ((tid & 15) == 0) __stcg(reinterpret_cast<float2*>(rec + 8 * kBD) + hh, make_float2(mc, lc));
        __threadfence();                                           // this thread's record before the ticket
      }
    }
    cons_sync();                                                   // warp partials are reused by the next piece
    if (n_parts > 1 && tid == 0) {                                 // ticket: order of arrival among the pieces
      s_tk_seg[s_ntk] = s;
      s_tk[s_ntk] = (int)atomicAdd(&a.ws->seg_cnt[s], 1u);
      ++s_ntk;
    }
  }
  cons_sync();
  if (threadIdx.x == 0) FLINT_TL(6);

  // ---- B2: merge the partial records of each split segment without a grid barrier.  The CTAs holding the last
  // nm = min(n, Gq) of the segment's n tickets merge it, merger j taking q heads j, j + nm, ...; each waits until all
  // n pieces have taken their tickets (records written), then warp w folds records r = w, w + 8, ... (loaded
  // together) with the online softmax rule and the 8 warp results are folded in warp order.  Fixed order throughout,
  // so the result does not depend on which CTA merges.  The last merger to finish resets the segment's counters. ----
  {
    constexpr int kMR = 8;                                         // records per warp per round
    float* part = reinterpret_cast<float*>(wq);                    // [8 warps][128]
    float* wml = part + kBW * kBD;                                 // [8 warps][2]: m, l
    const int ntk = s_ntk;
    for (int k = 0; k < ntk; ++k) {
      const int s = s_tk_seg[k], n = s_nparts[s], nm = min(n, a.Gq), jm = s_tk[k] - (n - nm);
      if (jm < 0) continue;                                          // not one of the last nm tickets
      if (tid == 0) {                                                // every piece's record is written
        int ok = 1;
        unsigned it = 0;
#pragma unroll 1
        while ((int)ld_acquire_u32(&a.ws->seg_cnt[s]) < n) {
          if (++it > FLINT_WAIT_LIMIT) {
            atomicOr(status, STATUS_WAIT_TIMEOUT);
            ok = 0;
            break;
          }
          poll_pause();
        }
        __threadfence();
        s_go = ok;
      }
      cons_sync();
      const bool go = s_go != 0;
      for (int hh = jm; go && hh < a.Gq; hh += nm) {
        const int b = s / a.nkv, kvh = s - b * a.nkv;
        const float* r0 = a.rec + (int64_t)s_recb[s] * kBRecFloats;
        const int d0 = lane * 4;
        float m_w = -INFINITY, l_w = 0.f, acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 1
        for (int base = 0; base < n; base += kBW * kMR) {
          float4 v[kMR];
          float2 ml[kMR];
#pragma unroll
          for (int i = 0; i < kMR; ++i) {
            const int r = base + warp + kBW * i;
            if (r < n) {
              const float* rec = r0 + (int64_t)r * kBRecFloats;
              v[i] = __ldcg(reinterpret_cast<const float4*>(rec + hh * kBD + d0));
              ml[i] = __ldcg(reinterpret_cast<const float2*>(rec + 8 * kBD) + hh);
            } else {
              v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
              ml[i] = make_float2(-INFINITY, 0.f);
            }
          }
          float m_new = m_w;
#pragma unroll
          for (int i = 0; i < kMR; ++i) m_new = fmaxf(m_new, ml[i].x);
          if (m_new != -INFINITY) {
            const float sc = m_w == -INFINITY ? 0.f : exp2f(m_w * c - m_new * c);
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[e] *= sc;
            l_w *= sc;
#pragma unroll
            for (int i = 0; i < kMR; ++i) {
              const float f = ml[i].x == -INFINITY ? 0.f : exp2f(ml[i].x * c - m_new * c);
              acc[0] = fmaf(v[i].x, f, acc[0]);
              acc[1] = fmaf(v[i].y, f, acc[1]);
              acc[2] = fmaf(v[i].z, f, acc[2]);
              acc[3] = fmaf(v[i].w, f, acc[3]);
              l_w = fmaf(ml[i].y, f, l_w);
            }
            m_w = m_new;
          }
        }
        *reinterpret_cast<float4*>(part + warp * kBD + d0) = make_float4(acc[0], acc[1], acc[2], acc[3]);
        if (lane == 0) {
          wml[2 * warp] = m_w;
          wml[2 * warp + 1] = l_w;
        }
        cons_sync();
        if (tid < 32) {
          float m = -INFINITY;
#pragma unroll
          for (int w = 0; w < kBW; ++w) m = fmaxf(m, wml[2 * w]);
          float ov[4] = {0.f, 0.f, 0.f, 0.f}, den = 0.f;
          if (m != -INFINITY) {
#pragma unroll
            for (int w = 0; w < kBW; ++w) {
              const float mw = wml[2 * w];
              const float f = mw == -INFINITY ? 0.f : exp2f(mw * c - m * c);
              const float4 pv = *reinterpret_cast<const float4*>(part + w * kBD + d0);
              ov[0] = fmaf(pv.x, f, ov[0]);
              ov[1] = fmaf(pv.y, f, ov[1]);
              ov[2] = fmaf(pv.z, f, ov[2]);
              ov[3] = fmaf(pv.w, f, ov[3]);
              den = fmaf(wml[2 * w + 1], f, den);
            }
          }
          const int qh = kvh * a.Gq + hh;
          if (a.sinks && m != -INFINITY) den += exp2f(a.sinks[qh] * kBLog2e - m * c);
          const float inv = den > 0.f ? 1.0f / den : 0.f;
          const uint32_t pk[2] = {pack_bf16x2(ov[0] * inv, ov[1] * inv), pack_bf16x2(ov[2] * inv, ov[3] * inv)};
          publish_attn(a, ep, b, qh * kBD + d0, pk, 2);
        }
        cons_sync();
      }
      // the last merger to finish resets the counters for the next launch
      if (tid == 0 && atomicAdd(&a.ws->seg_done[s], 1u) == (unsigned)(nm - 1)) {
        atomicExch(&a.ws->seg_cnt[s], 0u);
        atomicExch(&a.ws->seg_done[s], 0u);
      }
      cons_sync();                                                   // s_go is rewritten for the next ticket
    }
  }
  if (threadIdx.x == 0) FLINT_TL(7);
  pdl_trigger();

  // ---- C: O projection from the resident weights, each warp's K slices staged as their heads arrive ----
  if (ngo > 0) {
    cons_sync();                                                   // xs_o overlays the merge scratch of B2
    if (tid < 8) shift[tid] = 0;                                   // the slices' scales are applied in the sums
    if (cons_sync_and(mbar_wait(&bar_wo, 0, status))) {
      gemv_stream_o(wo, wo + a.wo_scale_off, ngo, a.nks_o, a.attn_tag, a.Ko / 2, ep, xs_o, a.Ko, M, red, warp, lane,
                    status);
      cons_sync();
      gemv_finish(red, ngo, M, a.gs_o[0], shift, a.out, a.ldr, go0 * 16);
    }
  }
  if (threadIdx.x == 0) FLINT_TL(8);
  grid_sync_retire(&a.ws->gs, G, &a.ws->epoch);
}

struct BlockLayout {
  size_t wq_bytes, wo_bytes, xs_bytes, red_bytes, ring_off, wo_off, xs_off, red_off, total;
  int np;
};

static BlockLayout block_layout(int M, int H, int Ko, int gq_per, int go_per, int nks_q, int nks_o, int sms) {
  BlockLayout L{};
  auto up = [](size_t v, size_t a) { return (v + a - 1) / a * a; };
  const size_t wq = up((size_t)gq_per * nks_q * 2048, 1024) + up((size_t)gq_per * nks_q * 256, 1024);
  // phase B over region A: warp partials [8][8][128] fp32, (m, l) [8][16] x 2, merge tables
  const size_t partials = (size_t)kBW * 8 * kBD * 4 + (size_t)kBW * 16 * 8 + (size_t)sms * 64 + 64;
  const size_t xs_o = (size_t)M * xs_stride(Ko) * 2;
  L.wq_bytes = up(std::max(wq, partials), 1024);
  L.wo_bytes = up((size_t)go_per * nks_o * 2048, 1024) + up((size_t)go_per * nks_o * 256, 1024);
  L.xs_bytes = up((size_t)M * xs_stride(H) * 2, 1024);
  L.red_bytes = up((size_t)std::max(kBGQ, kBGO) * kBW * 128 * 4, 1024);
  const size_t budget = 227 * 1024 - 4096;           // dynamic shared memory left beside the static arrays
  const size_t fixed = 1024 + L.wq_bytes + L.wo_bytes + L.xs_bytes + L.red_bytes;
  L.np = 0;
  if (fixed < budget) L.np = (int)std::min<size_t>(kBMaxSlots, (budget - fixed) / kBPageBytes);
  if (L.np >= 2 && L.wq_bytes + (size_t)L.np * kBPageBytes < xs_o) {   // phase C staging must fit over A + ring
    const size_t extra = up(xs_o - L.wq_bytes - (size_t)L.np * kBPageBytes, 1024);
    L.wq_bytes += extra;
    const size_t fixed2 = fixed + extra;
    L.np = fixed2 < budget ? (int)std::min<size_t>(kBMaxSlots, (budget - fixed2) / kBPageBytes) : 0;
  }
  L.ring_off = L.wq_bytes;
  L.wo_off = L.ring_off + (size_t)L.np * kBPageBytes;
  L.xs_off = L.wo_off + L.wo_bytes;
  L.red_off = L.xs_off + L.xs_bytes;
  L.total = 1024 + L.red_off + L.red_bytes;
  return L;
}

static size_t block_ws_bytes(int64_t Nqkv, int64_t Ko, int sms) {
  return sizeof(BlockWs) + (size_t)8 * (Nqkv / 2) * 8 + (size_t)8 * (Ko / 2) * 8 +
         (size_t)(sms + kBMaxSeg) * kBRecFloats * 4 + 512;
}

}  // namespace flint

using namespace flint;

int64_t flint::status_offset_attn_block() { return (int64_t)offsetof(BlockWs, status); }

extern "C" int64_t flint_attn_block_workspace_bytes(int64_t n_qkv, int64_t k_o) {
  const int sms = num_sms();
  return (int64_t)block_ws_bytes(n_qkv, k_o, sms > 0 ? sms : 148);
}

extern "C" int flint_attn_block(const void* x, int64_t ldx, const int32_t* tokens, const void* res, int64_t ldr,
                                const void* norm_w, float eps, int64_t M, int64_t H, const void* Wqkv, const void* Sqkv,
                                const float* gs_qkv, int64_t num_q_heads, int64_t num_kv_heads, const void* q_norm_w,
                                const void* k_norm_w, float eps_head, const int64_t* positions, const float* cos_sin,
                                int64_t cs_stride, void* kv_cache, int64_t num_blocks, int64_t stride_block,
                                int64_t stride_head, const int32_t* block_tables, int64_t bt_stride, int64_t max_blocks,
                                const int32_t* seq_lens, const int64_t* slots, const float* sinks, int64_t window,
                                float scale, const void* Wo, const void* So, const float* gs_o, int64_t n_o, void* out,
                                void* res_out, void* q_out, void* attn_out, void* workspace, int pdl, void* stream) {
  if (!x || !norm_w || !Wqkv || !Sqkv || !gs_qkv || !q_norm_w || !k_norm_w || !kv_cache || !block_tables || !seq_lens ||
      !Wo || !So || !gs_o || !out || !res_out || !workspace || (cos_sin && !positions))
    return FLINT_ERR_ARGUMENT;
  const int sms = num_sms();
  if (sms <= 0 || sms > 256) return FLINT_ERR_DEVICE;
  if (M < 1 || M > 8 || H < kSliceK || H % kSliceK != 0 || H > 8192 || num_kv_heads < 1 || num_q_heads % num_kv_heads != 0 ||
      num_q_heads / num_kv_heads > 8 || M * num_kv_heads > kBMaxSeg || ldx < H || ldr < H || n_o < 16 || n_o % 16 != 0 ||
      num_blocks < 1 || max_blocks < 1 || window < 0 || stride_head < 2 * kBD || stride_block < num_kv_heads * stride_head)
    return FLINT_ERR_SHAPE;
  const int64_t Nqkv = (num_q_heads + 2 * num_kv_heads) * kBD, Ko = num_q_heads * kBD;
  if (Ko % kSliceK != 0 || Ko > 8192) return FLINT_ERR_SHAPE;
  // every (request, kv head) segment gets a CTA of its own
  if (M * num_kv_heads > sms) return FLINT_ERR_SHAPE;
  // the kernel's page partition runs in 32-bit arithmetic: pages x (grid + 1) must stay below 2^32
  if ((uint64_t)M * (uint64_t)num_kv_heads * (uint64_t)max_blocks * (uint64_t)(sms + 1) >= (1ull << 32))
    return FLINT_ERR_SHAPE;
  if (!aligned(x, 16) || ldx % 8 != 0 || ldr % 8 != 0 || (res && !aligned(res, 16)) || !aligned(norm_w, 16) ||
      !aligned(out, 16) || !aligned(res_out, 16) || !aligned(Wqkv, 16) || !aligned(Sqkv, 16) || !aligned(Wo, 16) ||
      !aligned(So, 16) || !aligned(kv_cache, 16) || stride_block % 8 != 0 || stride_head % 8 != 0 ||
      (attn_out && !aligned(attn_out, 16)) || !aligned(workspace, 256))
    return FLINT_ERR_ALIGN;
  const int gq_total = (int)(Nqkv / 16), go_total = (int)(n_o / 16);
  const int gq_per = (gq_total + sms - 1) / sms, go_per = (go_total + sms - 1) / sms;
  if (gq_per > kBGQ || go_per > kBGO) return FLINT_ERR_SHAPE;
  const int nks_q = (int)(H / kSliceK), nks_o = (int)(Ko / kSliceK);
  const BlockLayout L = block_layout((int)M, (int)H, (int)Ko, gq_per, go_per, nks_q, nks_o, sms);
  if (L.np < 2 || L.total > 227 * 1024) return FLINT_ERR_SHAPE;

  // weights as 3-D views [slice][row][bytes of the slice] so one box carries a 16-row group over all of K
  CUtensorMap mqc, mqs, moc, mos, mkv;
  auto enc3 = [](CUtensorMap* m, const void* base, uint64_t inner, uint64_t rows, uint64_t row_bytes, uint64_t nks,
                 bool swz) {
    const uint64_t d[3] = {inner, rows, nks};
    const uint64_t st[2] = {row_bytes, inner};
    const uint32_t bx[3] = {(uint32_t)inner, 16u, (uint32_t)nks};
    return encode_u8_3d(m, base, d, st, bx, swz);
  };
  int rc = enc3(&mqc, Wqkv, 128, Nqkv, H / 2, H / kSliceK, true);
  if (!rc) rc = enc3(&mqs, Sqkv, 16, Nqkv, H / 16, H / kSliceK, false);
  if (!rc) rc = enc3(&moc, Wo, 128, n_o, Ko / 2, Ko / kSliceK, true);
  if (!rc) rc = enc3(&mos, So, 16, n_o, Ko / 16, Ko / kSliceK, false);
  if (rc) return rc;
  // KV pages as a 5-D view [block][head][quarter K0 K1 V0 V1][16 rows][64 dims]: one box per page
  const uint64_t dims[5] = {64, kBPage, 4, (uint64_t)num_kv_heads, (uint64_t)num_blocks};
  const uint64_t strides[4] = {2 * kBD * 2, 128, (uint64_t)stride_head * 2, (uint64_t)stride_block * 2};
  const uint32_t box[5] = {64, kBPage, 4, 1, 1};
  rc = encode_bf16_5d(&mkv, kv_cache, dims, strides, box);
  if (rc) return rc;

  uint8_t* wsb = static_cast<uint8_t*>(workspace);
  BlockArgs a{};
  a.x = (const bf16*)x; a.ldx = ldx; a.tokens = tokens; a.res = (const bf16*)res; a.ldr = ldr; a.nw = (const bf16*)norm_w;
  a.eps = eps; a.M = (int)M; a.H = (int)H; a.Nqkv = (int)Nqkv; a.nq = (int)num_q_heads; a.nkv = (int)num_kv_heads;
  a.Gq = (int)(num_q_heads / num_kv_heads); a.gs_qkv = gs_qkv; a.q_w = (const bf16*)q_norm_w; a.k_w = (const bf16*)k_norm_w;
  a.eps_head = eps_head; a.positions = positions; a.cos_sin = cos_sin; a.cs_stride = cs_stride; a.kv = (bf16*)kv_cache;
  a.st_block = stride_block; a.st_head = stride_head; a.bt = block_tables; a.bt_stride = bt_stride;
  a.max_blocks = (int)max_blocks; a.seq_lens = seq_lens; a.slots = slots; a.sinks = sinks; a.window = (int)window;
  a.c = scale * kBLog2e; a.Ko = (int)Ko; a.No = (int)n_o; a.gs_o = gs_o; a.out = (bf16*)out; a.res_out = (bf16*)res_out;
  a.q_out = (bf16*)q_out;
  a.y_tag = reinterpret_cast<unsigned long long*>(wsb + sizeof(BlockWs));
  a.attn_tag = reinterpret_cast<unsigned long long*>(
      (reinterpret_cast<uintptr_t>(a.y_tag + 8 * (Nqkv / 2)) + 255) & ~uintptr_t(255));
  a.attn = (bf16*)attn_out;
  a.rec = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(a.attn_tag + 8 * (Ko / 2)) + 255) & ~uintptr_t(255));
  a.gq_total = gq_total; a.go_total = go_total; a.nks_q = nks_q; a.nks_o = nks_o; a.np = L.np;
  a.off_ring = (uint32_t)L.ring_off; a.off_wo = (uint32_t)L.wo_off; a.off_xs = (uint32_t)L.xs_off;
  a.off_red = (uint32_t)L.red_off;
  a.wq_scale_off = (uint32_t)(((size_t)gq_per * nks_q * 2048 + 1023) / 1024 * 1024);
  a.wo_scale_off = (uint32_t)(((size_t)go_per * nks_o * 2048 + 1023) / 1024 * 1024);
  a.ws = reinterpret_cast<BlockWs*>(wsb);

  // one CTA per SM must be resident (cooperative launch): give back ring slots until the occupancy query agrees
  void (*kern)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, BlockArgs) =
      M == 1 ? attn_block_kernel<1> : attn_block_kernel<0>;
  set_max_carveout(kern);
  size_t smem = L.total;
  int np = L.np;
  for (;;) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return record_cuda(cudaGetLastError(), FLINT_ERR_LAUNCH);
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kBThreads, smem) != cudaSuccess)
      return record_cuda(cudaGetLastError(), FLINT_ERR_LAUNCH);
    if (per_sm >= 1) break;
    if (np <= 2) {
      cudaFuncAttributes fa{};
      cudaFuncGetAttributes(&fa, kern);
      char msg[160];
      snprintf(msg, sizeof(msg), "attn_block: no CTA fits an SM (regs %d, static smem %zu, dynamic smem %zu)", fa.numRegs,
               fa.sharedSizeBytes, smem);
      record_message(msg);
      return FLINT_ERR_LAUNCH;
    }
    --np;
    smem -= kBPageBytes;
  }
  a.np = np;
  a.off_wo = (uint32_t)(L.ring_off + (size_t)np * kBPageBytes);
  a.off_xs = a.off_wo + (uint32_t)L.wo_bytes;
  a.off_red = a.off_xs + (uint32_t)L.xs_bytes;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3(kBThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute at[2];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  at[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = at;
  cfg.numAttrs = pdl ? 2 : 1;
  return record_cuda(cudaLaunchKernelEx(&cfg, kern, mqc, mqs, moc, mos, mkv, a), FLINT_ERR_LAUNCH);
}

FLINT_TL_READER(flint_timeline_attn_block)
