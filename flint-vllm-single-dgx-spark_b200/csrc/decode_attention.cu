// (3) Paged split-K GQA decode attention, one query token per request.  Replaces the Flint PR's CuTe
// _FlintDecodeAttention (patch:1741-2415, entry flint_decode_attention patch:2539-2605) and, at batch 1, the
// FlashInfer decode the GB10 recipe falls back to.
//
// KV cache: FlashInfer HND bf16 [num_blocks, num_kv_heads, 16, 2*D] with K in [..., :D] and V in [..., D:], D = 128.
// Grid (splits, kv_heads, batch); each CTA owns a contiguous page range of its (request, kv head) and its warps take
// pages round robin.  A page (16 tokens x [K | V], 8 KB) arrives in four 128B-swizzled TMA boxes (K lo/hi, V lo/hi)
// in the warp's private ring; pages not holding the current token are prefetched before the PDL wait.
// Per page: S = K q (mma.sync, query heads padded 8 -> 16 rows), online softmax in fp32 as exp2(S*c - m*c) with
// c = scale*log2(e), P rounded to bf16 for O += P V (the S accumulators are reused as P fragments), l sums the fp32 p.
// The number of active splits follows the context (at least 8 pages each).  Warps, then splits, merge their (m, l, O)
// in fixed order (deterministic); the last CTA of a (request, kv head) to finish merges the splits and adds the sink term exp2(sink*log2e - m*c) to the denominator
// (numerics of patch:1444-1464).
#include "common.cuh"
#include "runtime.cuh"
#include "tma.cuh"

namespace flint {

constexpr int kAttnD = 128;
constexpr int kPage = 16;
constexpr int kAttnWarps = 4;
constexpr int kAttnStages = 3;
constexpr int kPageBytes = kPage * 2 * kAttnD * 2;       // 8 KB
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMinPagesPerSplit = 8;

struct AttnWorkspace {
  unsigned status;
  unsigned pad[31];
  unsigned counter[1024];          // per (request, kv head)
  // followed by split partials: fp32 o [B*Hkv*splits][16][D], m/l [B*Hkv*splits][16][2]
};

struct AttnArgs {
  const bf16* q;
  int64_t q_stride_b;              // elements between requests
  const int* block_tables;
  int64_t bt_stride;
  const int* seq_lens;
  const float* sinks;
  int window;
  float c;                          // scale * log2(e)
  bf16* out;
  int64_t out_stride_b;
  int B, Hkv, G, splits, max_blocks;
  AttnWorkspace* ws;
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(addr));
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
// shared address of the 16-byte unit (token row, dim) inside a page: box = dim / 64 of the 4 boxes (K0 K1 V0 V1),
// each box 16 rows x 128 B with the 128-byte swizzle
__device__ __forceinline__ uint32_t page_unit(uint32_t page, int box, int row, int unit) {
  return page + box * 2048 + row * 128 + ((unit ^ (row & 7)) << 4);
}

__global__ void __launch_bounds__(kAttnWarps * 32, 2)
decode_attn_kernel(const __grid_constant__ CUtensorMap kv, const AttnArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bars[kAttnWarps][kAttnStages];
  __shared__ float wm[kAttnWarps][16], wl[kAttnWarps][16];
  __shared__ float wo[kAttnWarps][8][kAttnD];
  __shared__ int s_last;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int g = lane >> 2, t4 = lane & 3;
  const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int G = a.G;

  const int seq = a.seq_lens[b];
  const int start = a.window > 0 ? max(0, seq - a.window) : 0;
  const int p_first = start / kPage, p_end = (seq + kPage - 1) / kPage;
  const int npages = max(0, p_end - p_first);
  // active splits follow the context: at least kMinPagesPerSplit pages each (fewer partials to merge when short)
  const int n_act = max(1, min(a.splits, npages / kMinPagesPerSplit));
  if (split >= n_act) return;
  const int pps = (npages + n_act - 1) / n_act;
  const int pb = p_first + split * pps, pe = min(p_end, pb + pps);
  const int last_page = p_end - 1;                          // holds the current token (written by the previous kernel)
  const int* bt = a.block_tables + (int64_t)b * a.bt_stride;
  uint8_t* ring = smem + warp * kAttnStages * kPageBytes;
  unsigned* status = &a.ws->status;

  const int my_n = pb + warp < pe ? (pe - pb - warp + kAttnWarps - 1) / kAttnWarps : 0;
  if (lane == 0) {
    for (int s = 0; s < kAttnStages; ++s) mbar_init(&bars[warp][s], 1);
    fence_mbar_init();
  }
  __syncwarp();
  auto issue = [&](int j) {                                  // page j of this warp into slot j % stages
    const int p = pb + warp + j * kAttnWarps;
    const int blk = bt[p];
    const int slot = j % kAttnStages;
    uint64_t* bar = &bars[warp][slot];
    mbar_arrive_expect_tx(bar, kPageBytes);
    uint8_t* dst = ring + slot * kPageBytes;
#pragma unroll
    for (int bx = 0; bx < 4; ++bx) tma_load_4d(dst + bx * 2048, &kv, bx * 64, 0, h, blk, bar);
  };
  int issued = 0;
  if (lane == 0) {
    while (issued < my_n && issued < kAttnStages && pb + warp + issued * kAttnWarps != last_page) issue(issued++);
  }
  pdl_wait();
  if (lane == 0)
    while (issued < my_n && issued < kAttnStages) issue(issued++);

  // query fragments (rows = heads g of this kv head; rows 8..15 are padding)
  uint32_t qa[8][2];
  {
    const bf16* qp = a.q + (int64_t)b * a.q_stride_b + (int64_t)(h * G + g) * kAttnD;
    const bool qv = g < G;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      qa[kk][0] = qv ? *reinterpret_cast<const uint32_t*>(qp + 16 * kk + 2 * t4) : 0u;
      qa[kk][1] = qv ? *reinterpret_cast<const uint32_t*>(qp + 16 * kk + 8 + 2 * t4) : 0u;
    }
  }
  float o[16][4];
#pragma unroll
  for (int dt = 0; dt < 16; ++dt)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[dt][e] = 0.f;
  float m_run = -INFINITY, l_run = 0.f;
  const float c = a.c;

  for (int j = 0; j < my_n; ++j) {
    const int slot = j % kAttnStages;
    if (!mbar_wait(&bars[warp][slot], (j / kAttnStages) & 1, status)) break;
    const uint32_t page = smem_u32(ring + slot * kPageBytes);
    const int p = pb + warp + j * kAttnWarps;
    // ---- S = K q: 2 token tiles x 8 dim steps; ldmatrix x4 = (tokens 0-7, 8-15) x (dims lo, hi) of a 16-dim step
    float s[2][4];
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) s[nt][e] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int mat = lane >> 3, r = lane & 7;
      const int row = 8 * (mat >> 1) + r;                  // token
      const int dim = 16 * kk + 8 * (mat & 1);
      uint32_t k0, k1, k2, k3;
      ldsm_x4(page_unit(page, dim >> 6, row, (dim & 63) >> 3), k0, k1, k2, k3);
      const uint32_t aq[4] = {qa[kk][0], 0u, qa[kk][1], 0u};
      asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                   : "+f"(s[0][0]), "+f"(s[0][1]), "+f"(s[0][2]), "+f"(s[0][3])
                   : "r"(aq[0]), "r"(aq[1]), "r"(aq[2]), "r"(aq[3]), "r"(k0), "r"(k1));
      asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                   : "+f"(s[1][0]), "+f"(s[1][1]), "+f"(s[1][2]), "+f"(s[1][3])
                   : "r"(aq[0]), "r"(aq[1]), "r"(aq[2]), "r"(aq[3]), "r"(k2), "r"(k3));
    }
    // ---- mask, online softmax (row g: head g; this lane holds tokens 8nt + 2t4 + {0,1}) ----
    float sv[4] = {s[0][0], s[0][1], s[1][0], s[1][1]};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int tok = p * kPage + 8 * (i >> 1) + 2 * t4 + (i & 1);
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
    // ---- O += P V: P (rows = heads) as the A operand, V^T tiles via ldmatrix.trans ----
    const uint32_t pa[4] = {pack_bf16(pv[0], pv[1]), 0u, pack_bf16(pv[2], pv[3]), 0u};
#pragma unroll
    for (int dp = 0; dp < 8; ++dp) {                       // two 8-dim tiles per ldmatrix x4.trans
      const int mat = lane >> 3, r = lane & 7;
      const int row = 8 * (mat & 1) + r;                   // token
      const int dim = 16 * dp + 8 * (mat >> 1);
      uint32_t v0, v1, v2, v3;
      ldsm_x4_t(page_unit(page, 2 + (dim >> 6), row, (dim & 63) >> 3), v0, v1, v2, v3);
      asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                   : "+f"(o[2 * dp][0]), "+f"(o[2 * dp][1]), "+f"(o[2 * dp][2]), "+f"(o[2 * dp][3])
                   : "r"(pa[0]), "r"(pa[1]), "r"(pa[2]), "r"(pa[3]), "r"(v0), "r"(v1));
      asm volatile("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
                   : "+f"(o[2 * dp + 1][0]), "+f"(o[2 * dp + 1][1]), "+f"(o[2 * dp + 1][2]), "+f"(o[2 * dp + 1][3])
                   : "r"(pa[0]), "r"(pa[1]), "r"(pa[2]), "r"(pa[3]), "r"(v2), "r"(v3));
    }
    __syncwarp();
    if (lane == 0 && issued < my_n) issue(issued++);        // the slot just consumed
  }
  pdl_trigger();

  // ---- merge the warps of this CTA (fixed warp order) ----
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  if (t4 == 0) {
    wm[warp][g] = m_run;
    wl[warp][g] = l_run;
  }
  if (g < 8) {
#pragma unroll
    for (int dt = 0; dt < 16; ++dt) {
      wo[warp][g][8 * dt + 2 * t4] = o[dt][0];
      wo[warp][g][8 * dt + 2 * t4 + 1] = o[dt][1];
    }
  }
  __syncthreads();
  const int nb = a.B * a.Hkv;
  const int bh = b * a.Hkv + h;
  float* part_o = reinterpret_cast<float*>(a.ws + 1);
  float* part_ml = part_o + (size_t)nb * a.splits * 8 * kAttnD;
  // thread -> (head, dims): 128 threads x 8 dims = 8 heads x 128 dims
  const int hh = threadIdx.x >> 4, d0 = (threadIdx.x & 15) * 8;
  float mc = -INFINITY;
#pragma unroll
  for (int w = 0; w < kAttnWarps; ++w) mc = fmaxf(mc, wm[w][hh]);
  float lc = 0.f, oc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) oc[i] = 0.f;
#pragma unroll
  for (int w = 0; w < kAttnWarps; ++w) {
    if (wm[w][hh] == -INFINITY) continue;
    const float f = exp2f(wm[w][hh] * c - mc * c);
    lc += wl[w][hh] * f;
#pragma unroll
    for (int i = 0; i < 8; ++i) oc[i] += wo[w][hh][d0 + i] * f;
  }
  auto finish = [&](float m, float l, const float* ov) {
    if (hh >= G) return;
    const int qh = h * G + hh;
    float den = l;
    if (a.sinks && m != -INFINITY) den += exp2f(a.sinks[qh] * kLog2e - m * c);
    const float inv = den > 0.f ? 1.0f / den : 0.f;
    uint32_t pk[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) pk[i] = pack_bf16(ov[2 * i] * inv, ov[2 * i + 1] * inv);
    *reinterpret_cast<uint4*>(a.out + (int64_t)b * a.out_stride_b + (int64_t)qh * kAttnD + d0) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  };
  if (n_act == 1) {
    finish(mc, lc, oc);
    return;
  }
  // split partials, laid out [(request, kv head, head)][split] so the merging CTA reads each head's splits contiguously
  const size_t row = (size_t)bh * 8 + hh;
  float* po = part_o + (row * a.splits + split) * kAttnD + d0;
  __stcg(reinterpret_cast<float4*>(po), make_float4(oc[0], oc[1], oc[2], oc[3]));
  __stcg(reinterpret_cast<float4*>(po) + 1, make_float4(oc[4], oc[5], oc[6], oc[7]));
  if ((threadIdx.x & 15) == 0) __stcg(reinterpret_cast<float2*>(part_ml) + row * a.splits + split, make_float2(mc, lc));
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    s_last = atomicAdd(&a.ws->counter[bh], 1u) == (unsigned)n_act - 1;
    if (s_last) atomicExch(&a.ws->counter[bh], 0u);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const float2* ml = reinterpret_cast<const float2*>(part_ml) + row * a.splits;
  float m = -INFINITY;
#pragma unroll 8
  for (int sp = 0; sp < n_act; ++sp) m = fmaxf(m, __ldcg(ml + sp).x);
  float l = 0.f, ov[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) ov[i] = 0.f;
#pragma unroll 4
  for (int sp = 0; sp < n_act; ++sp) {
    const float2 v = __ldcg(ml + sp);
    const float4* o4 = reinterpret_cast<const float4*>(part_o + (row * a.splits + sp) * kAttnD + d0);
    const float4 u0 = __ldcg(o4), u1 = __ldcg(o4 + 1);
    const float f = v.x == -INFINITY ? 0.f : exp2f(v.x * c - m * c);
    l += v.y * f;
    ov[0] += u0.x * f; ov[1] += u0.y * f; ov[2] += u0.z * f; ov[3] += u0.w * f;
    ov[4] += u1.x * f; ov[5] += u1.y * f; ov[6] += u1.z * f; ov[7] += u1.w * f;
  }
  finish(m, l, ov);
}

static size_t attn_ws_bytes(int B, int Hkv, int splits) {
  return sizeof(AttnWorkspace) + (size_t)B * Hkv * splits * 8 * (kAttnD + 2) * sizeof(float);
}

}  // namespace flint

using namespace flint;

extern "C" int64_t flint_decode_attention_splits(int64_t batch, int64_t num_kv_heads) {
  const int sms = num_sms();
  const int64_t n = (sms > 0 ? 2 * sms : 296) / (batch * num_kv_heads);
  return n < 1 ? 1 : (n > 256 ? 256 : n);
}

int64_t flint::status_offset_decode_attention() { return (int64_t)offsetof(AttnWorkspace, status); }

extern "C" int64_t flint_decode_attention_workspace_bytes(int64_t batch, int64_t num_kv_heads, int64_t splits) {
  return (int64_t)attn_ws_bytes((int)batch, (int)num_kv_heads, (int)splits);
}

extern "C" int flint_decode_attention(const void* q, int64_t q_stride_b, const void* kv_cache, int64_t num_blocks,
                                      int64_t num_kv_heads, int64_t stride_block, int64_t stride_head,
                                      const int32_t* block_tables, int64_t bt_stride, int64_t max_blocks,
                                      const int32_t* seq_lens, const float* sinks, int64_t window, float scale,
                                      int64_t batch, int64_t num_q_heads, void* out, int64_t out_stride_b, int64_t splits,
                                      void* workspace, int pdl, void* stream) {
  if (!q || !kv_cache || !block_tables || !seq_lens || !out || !workspace) return FLINT_ERR_ARGUMENT;
  if (batch < 1 || num_kv_heads < 1 || num_q_heads % num_kv_heads != 0 || num_q_heads / num_kv_heads > 8 ||
      batch * num_kv_heads > 1024 || splits < 1 || splits > 256 || num_blocks < 1 || max_blocks < 1 || window < 0)
    return FLINT_ERR_SHAPE;
  if (!aligned(kv_cache, 16) || stride_block % 8 != 0 || stride_head % 8 != 0 || !aligned(out, 16) || !aligned(q, 4) ||
      out_stride_b % 8 != 0)
    return FLINT_ERR_ALIGN;
  if (num_sms() <= 0) return FLINT_ERR_DEVICE;
  CUtensorMap map;
  const uint64_t dims[4] = {2 * kAttnD, kPage, (uint64_t)num_kv_heads, (uint64_t)num_blocks};
  const uint64_t strides[3] = {2 * kAttnD * 2, (uint64_t)stride_head * 2, (uint64_t)stride_block * 2};
  const uint32_t box[4] = {64, kPage, 1, 1};
  int rc = encode_bf16_4d(&map, kv_cache, dims, strides, box);
  if (rc) return rc;
  AttnArgs a;
  a.q = (const bf16*)q; a.q_stride_b = q_stride_b; a.block_tables = (const int*)block_tables; a.bt_stride = bt_stride;
  a.seq_lens = (const int*)seq_lens; a.sinks = sinks; a.window = (int)window; a.c = scale * kLog2e; a.out = (bf16*)out;
  a.out_stride_b = out_stride_b; a.B = (int)batch; a.Hkv = (int)num_kv_heads; a.G = (int)(num_q_heads / num_kv_heads);
  a.splits = (int)splits; a.max_blocks = (int)max_blocks; a.ws = static_cast<AttnWorkspace*>(workspace);
  const size_t smem = 1024 + (size_t)kAttnWarps * kAttnStages * kPageBytes;
  if (cudaFuncSetAttribute(decode_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return FLINT_ERR_LAUNCH;
  return launch(decode_attn_kernel, dim3((int)splits, (int)num_kv_heads, (int)batch), dim3(kAttnWarps * 32), smem, stream,
                pdl, map, a);
}
