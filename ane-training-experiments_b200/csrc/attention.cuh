// attention.cuh -- paged KV-cache attention for decode (and block-causal prefill).
//
// Reference: ane/stories/infer.go:267-299 (attend: scores q.k/sqrt(hd) over t <= pos,
// softmaxPrefix, PV) with the GQA head map kv_head = q_head / group of
// training/training_dynamic/io.h:434-455.
//
// KV layout in HBM: pages of 16 positions; for (layer, page, kv_head) one contiguous block
// [K: 16 x hd][V: 16 x hd] of the activation type, each of them laid out by kv_off
// (common.cuh): 64-element row halves as 128-byte rows of 16 x 128 B sub-blocks, 16-byte chunk
// c of row s at c ^ (s & 7), so ldmatrix reads of 8 rows are bank-conflict free and a
// sub-block is a 128B-swizzled K-major tcgen05 operand.  A block table maps (sequence, logical
// page) -> physical page.
//
// One CTA = (query block, kv_head, split).  A query block is up to 8/group consecutive
// query positions of one sequence (1 for decode); its columns c = qi*group + h cover every
// q head of the GQA group, so each KV page is read from HBM once per kv head.  The 4 warps
// take pages round-robin; each warp owns a STAGES-deep ring of page buffers filled by the
// TMA bulk-copy engine (one cp.async.bulk per page, completion on an mbarrier) and runs
//   S^T[16 tok x 8 col] = K[16 x hd] . Q^T        (mma.m16n8k16, K via ldmatrix)
//   online softmax per column (max via 3 xor shuffles, exp2 with log2e folded in)
//   O^T[hd x 8]        += V^T[hd x 16] . P^T       (V via ldmatrix.trans; P split into two
//                         activation-type terms, each moved into B fragments by 4 shuffles)
// Warps merge through shared memory; splits > 1 merge through a workspace, the last CTA of
// a (block, kv_head) combining the splits in order.  All mbarrier waits are bounded.
#pragma once
#include "common.cuh"

namespace llm {

struct AttnParams {
  const void* q;              // [rows][n_heads][HD] act type
  const void* kv_pool;        // see layout above
  const int* block_table;     // [max_seqs][max_pages_per_seq]
  int max_pages_per_seq;
  const int* seq_ids;         // [rows]
  const int* positions;       // [rows]
  const int* blk_row0;        // [n_blocks] first row of each query block (nullptr: row = block)
  const int* blk_nq;          // [n_blocks] rows in the block (nullptr: 1)
  int n_blocks;
  int n_heads, n_kv_heads, layer, n_pages;
  int splits;
  float scale_log2;           // log2(e) / sqrt(hd)
  void* out;                  // [rows][n_heads][HD] act type, or fp32 when out_f32
  int out_f32;
  float* ws;                  // splits > 1: [n_blocks][n_kv_heads][splits][8][HD + 2]
  int* counters;              // splits > 1: [n_blocks][n_kv_heads]
  // optional fused per-token int8 quantisation of the fp32 output (out_f32 only): the last
  // CTA to finish a row (row_counters, zero between launches) quantises it
  int8_t* q8;                 // [rows][n_heads * HD]
  float* q8_scale;            // [rows]
  int* row_counters;          // [rows]
  int* err;
  TraceRec* trace;            // llm_trace_step
};

constexpr int kAttnWarps = 4;

// Page-ring depth per warp (pages of 16 positions in flight per warp).
// Two pages (64 KB per CTA, three CTAs per SM) measured faster than three (96 KB, two per SM):
// 235.7 vs 240.6 us per Qwen3 layer at 256 sequences x 1536 positions (6.92 vs 6.78 TB/s).
#ifndef LLM_ATTN_STAGES_HD128
#define LLM_ATTN_STAGES_HD128 2
#endif
// head_dim 64: two pages as well (32 KB per CTA): 28.4 vs 36.3 us per Stories110M layer at 256
// sequences x ~160 positions against four pages (short contexts want more CTAs per SM).
#ifndef LLM_ATTN_STAGES_HD64
#define LLM_ATTN_STAGES_HD64 2
#endif

template <typename T, int HD>
struct AttnCfg {
  static constexpr int PAGE_BYTES = 2 * 16 * HD * (int)sizeof(T);
  static constexpr int STAGES = HD >= 128 ? LLM_ATTN_STAGES_HD128 : LLM_ATTN_STAGES_HD64;
  static constexpr int WARP_BYTES = STAGES * PAGE_BYTES;
  static constexpr int SMEM = kAttnWarps * WARP_BYTES;
  static_assert(WARP_BYTES >= 8 * HD * 4 + 64 * 4, "merge area must fit in a warp's ring");
};

// Fused per-token quantisation: called by every CTA after it stored its rows' fp32 outputs.
// The CTA that completes a row (the last of its n_kv_heads producers) reads the whole row back
// from L2 and applies the bridge quantiser exactly as the row kernel in norm.cuh does.
template <int HD>
__device__ void attn_quant_rows(const AttnParams& p, int r0, int nq, int group, int* s_rowlast, float* s_wmax) {
  if (p.q8 == nullptr) return;
  const int nrows = min(nq, 8);  // rows r0..r0+nq-1 (nq <= 8 / group)
  __threadfence();
  __syncthreads();
  if (threadIdx.x < nrows) {
    const int prev = atomicAdd(p.row_counters + r0 + threadIdx.x, 1);
    s_rowlast[threadIdx.x] = prev == p.n_kv_heads - 1;
  }
  __syncthreads();
  const int cols = p.n_heads * HD;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = 0; i < nrows; ++i) {
    if (!s_rowlast[i]) continue;  // uniform across the CTA
    __threadfence();
    const int row = r0 + i;
    const float* src = reinterpret_cast<const float*>(p.out) + static_cast<size_t>(row) * cols;
    float mx = 0.0f;
    for (int c = 4 * threadIdx.x; c < cols; c += 4 * kAttnWarps * 32) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(src + c));
      mx = fmaxf(fmaxf(fmaxf(mx, fabsf(v.x)), fmaxf(fabsf(v.y), fabsf(v.z))), fabsf(v.w));
    }
    mx = warp_max(mx);
    if (lane == 0) s_wmax[warp] = mx;
    __syncthreads();
    mx = s_wmax[0];
#pragma unroll
    for (int w = 1; w < kAttnWarps; ++w) mx = fmaxf(mx, s_wmax[w]);
    float sc = __fdiv_rn(mx, 127.0f);
    if (sc == 0.0f) sc = 1.0f;
    const float inv = __fdiv_rn(1.0f, sc);
    int8_t* qo = p.q8 + static_cast<size_t>(row) * cols;
    for (int c = 4 * threadIdx.x; c < cols; c += 4 * kAttnWarps * 32) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(src + c));
      char4 q;
      q.x = quant_bridge_fast(v.x, sc, inv);
      q.y = quant_bridge_fast(v.y, sc, inv);
      q.z = quant_bridge_fast(v.z, sc, inv);
      q.w = quant_bridge_fast(v.w, sc, inv);
      *reinterpret_cast<char4*>(qo + c) = q;
    }
    if (threadIdx.x == 0) {
      p.q8_scale[row] = sc;
      p.row_counters[row] = 0;
    }
    __syncthreads();
  }
}

template <typename T, int HD>
__global__ void __launch_bounds__(kAttnWarps * 32) attn_kernel(AttnParams p) {
  using Cfg = AttnCfg<T, HD>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int PB = Cfg::PAGE_BYTES;
  constexpr int KS = HD / 16;
  constexpr int ROWB = HD * (int)sizeof(T);

  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[kAttnWarps][STAGES];
  __shared__ int s_last;
  __shared__ int s_rowlast[8];
  __shared__ float s_wmax[kAttnWarps];

  griddep_launch_dependents();
  trace_start(p.trace);
  griddep_wait();
  const int blk = blockIdx.x, kvh = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int group = p.n_heads / p.n_kv_heads;

  const int r0 = p.blk_row0 ? p.blk_row0[blk] : blk;
  const int nq = p.blk_nq ? p.blk_nq[blk] : 1;
  const int seq = p.seq_ids[r0];
  const int pos0 = p.positions[r0];
  const int ctx = pos0 + nq;
  const int n_pg = (ctx + 15) >> 4;
  const int chunk = (n_pg + p.splits - 1) / p.splits;
  const int p_begin = split * chunk;
  const int p_end = min(n_pg, p_begin + chunk);

  // Q^T fragments: column g of the B operand is (query g/group, head g%group).
  uint32_t qb[KS][2];
  {
    const int qi = g / group, h = g % group;
    const bool ok = qi < nq;
    const T* qrow = reinterpret_cast<const T*>(p.q) +
                    (static_cast<size_t>(r0 + (ok ? qi : 0)) * p.n_heads + kvh * group + h) * HD;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      qb[ks][0] = ok ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 2 * t) : 0u;
      qb[ks][1] = ok ? *reinterpret_cast<const uint32_t*>(qrow + ks * 16 + 8 + 2 * t) : 0u;
    }
  }
  // causal limits of this lane's two score columns (2t, 2t+1); invalid columns mask all
  const int c0 = 2 * t, c1 = 2 * t + 1;
  const int lim0 = (c0 / group) < nq ? pos0 + c0 / group : -1;
  const int lim1 = (c1 / group) < nq ? pos0 + c1 / group : -1;

  uint8_t* wbuf = smem + warp * Cfg::WARP_BYTES;
  const uint32_t wbase = smem_u32(wbuf);
  const uint32_t bar0 = smem_u32(&bars[warp][0]);
  const T* pool = reinterpret_cast<const T*>(p.kv_pool);
  const int* bt = p.block_table + static_cast<size_t>(seq) * p.max_pages_per_seq;

  auto page_src = [&](int lp) -> const T* {
    int phys = bt[lp];
    if (phys < 0 || phys >= p.n_pages) {
      if (p.err) atomicExch(p.err, kDevBadPage);
      phys = 0;
    }
    return pool + ((static_cast<size_t>(p.layer) * p.n_pages + phys) * p.n_kv_heads + kvh) * (2 * 16 * HD);
  };

  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) mbar_init(bar0 + 8 * s, 1);
    fence_mbar_init();
  }
  __syncwarp();
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      const int lp = p_begin + warp + kAttnWarps * s;
      if (lp < p_end) {
        mbar_arrive_expect_tx(bar0 + 8 * s, PB);
        bulk_g2s(wbase + s * PB, page_src(lp), PB, bar0 + 8 * s);
      }
    }
  }

  float m_run0 = -INFINITY, m_run1 = -INFINITY, l_run0 = 0.f, l_run1 = 0.f;
  float o[KS][4];
#pragma unroll
  for (int i = 0; i < KS; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  bool timed_out = false;
  int it = 0;
  for (;; ++it) {
    const int lp = p_begin + warp + kAttnWarps * it;
    if (lp >= p_end) break;
    const int s = it % STAGES;
    const uint32_t parity = (it / STAGES) & 1;
    if (!mbar_wait_bounded(bar0 + 8 * s, parity)) {
      if (lane == 0 && p.err) atomicExch(p.err, kDevWaitTimeout);
      timed_out = true;
      break;
    }
    const uint32_t kb = wbase + s * PB;
    const uint32_t vb = kb + 16 * ROWB;
    const int tok_base = lp * 16;
    if (tok_base + 16 > ctx) {
      // zero V rows past the context so 0-weight x stale data can never produce NaN
      uint8_t* vblk = wbuf + s * PB + 16 * ROWB;
      for (int i = lane; i < 16 * HD / 8; i += 32) {
        const int rr = i / (HD / 8), c = i % (HD / 8);
        if (tok_base + rr >= ctx) *reinterpret_cast<uint4*>(vblk + kv_off(rr, c)) = make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    }
    float sacc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      uint32_t a[4];
      const int row = (lane & 7) + 8 * ((lane >> 3) & 1);
      ldmatrix_x4(a, kb + kv_off(row, 2 * ks + (lane >> 4)));
      mma_16816(sacc, a, qb[ks][0], qb[ks][1], T());
    }
    const int tk0 = tok_base + g, tk1 = tk0 + 8;
    const float s0 = tk0 <= lim0 ? sacc[0] * p.scale_log2 : -INFINITY;
    const float s1 = tk0 <= lim1 ? sacc[1] * p.scale_log2 : -INFINITY;
    const float s2 = tk1 <= lim0 ? sacc[2] * p.scale_log2 : -INFINITY;
    const float s3 = tk1 <= lim1 ? sacc[3] * p.scale_log2 : -INFINITY;
    float pm0 = fmaxf(s0, s2), pm1 = fmaxf(s1, s3);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      pm0 = fmaxf(pm0, __shfl_xor_sync(0xffffffffu, pm0, off));
      pm1 = fmaxf(pm1, __shfl_xor_sync(0xffffffffu, pm1, off));
    }
    const float mn0 = fmaxf(m_run0, pm0), mn1 = fmaxf(m_run1, pm1);
    const float mu0 = mn0 == -INFINITY ? 0.f : mn0, mu1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = exp2f(m_run0 - mu0), al1 = exp2f(m_run1 - mu1);
    const float p0 = exp2f(s0 - mu0), p1 = exp2f(s1 - mu1), p2 = exp2f(s2 - mu0), p3 = exp2f(s3 - mu1);
    l_run0 = l_run0 * al0 + (p0 + p2);
    l_run1 = l_run1 * al1 + (p1 + p3);
    m_run0 = mn0;
    m_run1 = mn1;
#pragma unroll
    for (int i = 0; i < KS; ++i) {
      o[i][0] *= al0; o[i][1] *= al1; o[i][2] *= al0; o[i][3] *= al1;
    }
    // P^T fragments for column g, tokens (2t,2t+1) and (2t+8,2t+9).  P is carried as a
    // two-term split hi + lo (both in the activation type) so the PV product sees P with
    // ~16 mantissa bits instead of the activation type's 8 or 11.
    const uint32_t ph01 = ActTraits<T>::pack2(p0, p1);
    const uint32_t ph23 = ActTraits<T>::pack2(p2, p3);
    const float2 h01 = ActTraits<T>::unpack2(ph01), h23 = ActTraits<T>::unpack2(ph23);
    const uint32_t pl01 = ActTraits<T>::pack2(p0 - h01.x, p1 - h01.y);
    const uint32_t pl23 = ActTraits<T>::pack2(p2 - h23.x, p3 - h23.y);
    const int srcA = 8 * t + (g >> 1), srcB = srcA + 4;
    const int sh = (g & 1) ? 16 : 0;
    auto gather = [&](uint32_t v01, uint32_t v23, uint32_t& b0, uint32_t& b1) {
      const uint32_t xa01 = __shfl_sync(0xffffffffu, v01, srcA);
      const uint32_t xa23 = __shfl_sync(0xffffffffu, v23, srcA);
      const uint32_t xb01 = __shfl_sync(0xffffffffu, v01, srcB);
      const uint32_t xb23 = __shfl_sync(0xffffffffu, v23, srcB);
      b0 = ((xa01 >> sh) & 0xffffu) | (((xb01 >> sh) & 0xffffu) << 16);
      b1 = ((xa23 >> sh) & 0xffffu) | (((xb23 >> sh) & 0xffffu) << 16);
    };
    uint32_t bh0, bh1, bl0, bl1;
    gather(ph01, ph23, bh0, bh1);
    gather(pl01, pl23, bl0, bl1);
#pragma unroll
    for (int mt = 0; mt < KS; ++mt) {
      uint32_t a[4];
      const int row = (lane & 7) + 8 * (lane >> 4);
      ldmatrix_x4_trans(a, vb + kv_off(row, 2 * mt + ((lane >> 3) & 1)));
      mma_16816(o[mt], a, bh0, bh1, T());
      mma_16816(o[mt], a, bl0, bl1, T());
    }
    __syncwarp();
    if (lane == 0) {
      const int nlp = lp + kAttnWarps * STAGES;
      if (nlp < p_end) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(bar0 + 8 * s, PB);
        bulk_g2s(kb, page_src(nlp), PB, bar0 + 8 * s);
      }
    }
  }
  if (timed_out) {
    // drain copies still in flight into this warp's ring (bounded), contribute nothing
    for (int j = it + 1; j < it + STAGES; ++j) {
      const int lp = p_begin + warp + kAttnWarps * j;
      if (lp >= p_end) break;
      mbar_wait_bounded(bar0 + 8 * (j % STAGES), (j / STAGES) & 1);
    }
    m_run0 = m_run1 = -INFINITY;
    l_run0 = l_run1 = 0.f;
#pragma unroll
    for (int i = 0; i < KS; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  }
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l_run0 += __shfl_xor_sync(0xffffffffu, l_run0, off);
    l_run1 += __shfl_xor_sync(0xffffffffu, l_run1, off);
  }
  // ---- per-warp results into this warp's ring: m[8], l[8], O[8][HD]
  __syncwarp();
  float* wm_ = reinterpret_cast<float*>(wbuf);
  float* wl_ = wm_ + 8;
  float* wo_ = wm_ + 64;
  if (g == 0) {
    wm_[c0] = m_run0; wm_[c1] = m_run1;
    wl_[c0] = l_run0; wl_[c1] = l_run1;
  }
#pragma unroll
  for (int mt = 0; mt < KS; ++mt) {
    const int d = mt * 16 + g;
    wo_[c0 * HD + d] = o[mt][0];
    wo_[c1 * HD + d] = o[mt][1];
    wo_[c0 * HD + d + 8] = o[mt][2];
    wo_[c1 * HD + d + 8] = o[mt][3];
  }
  __syncthreads();

  // ---- merge the 4 warps (and, with splits, the splits)
  const int ncols = min(8, nq * group);
  const bool multi = p.splits > 1;
  float* part = nullptr;
  if (multi)
    part = p.ws + ((static_cast<size_t>(blk) * p.n_kv_heads + kvh) * p.splits + split) * 8 * (HD + 2);
  for (int i = threadIdx.x; i < ncols * HD; i += kAttnWarps * 32) {
    const int c = i / HD, d = i % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w)
      M = fmaxf(M, reinterpret_cast<float*>(smem + w * Cfg::WARP_BYTES)[c]);
    const float Mu = M == -INFINITY ? 0.f : M;
    float acc = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < kAttnWarps; ++w) {
      const float* b = reinterpret_cast<float*>(smem + w * Cfg::WARP_BYTES);
      const float f = exp2f(b[c] - Mu);
      acc += f * b[64 + c * HD + d];
      L += f * b[8 + c];
    }
    if (!multi) {
      const int row = r0 + c / group, head = kvh * group + c % group;
      const float v = L > 0.f ? acc / L : 0.f;
      const size_t oi = (static_cast<size_t>(row) * p.n_heads + head) * HD + d;
      if (p.out_f32) reinterpret_cast<float*>(p.out)[oi] = v;
      else reinterpret_cast<T*>(p.out)[oi] = ActTraits<T>::from_f(v);
    } else {
      __stcg(part + c * (HD + 2) + d, acc);
      if (d == 0) {
        __stcg(part + c * (HD + 2) + HD, M);
        __stcg(part + c * (HD + 2) + HD + 1, L);
      }
    }
  }
  if (!multi) {
    attn_quant_rows<HD>(p, r0, nq, group, s_rowlast, s_wmax);
    trace_end(p.trace);
    return;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(p.counters + blk * p.n_kv_heads + kvh, 1);
    s_last = prev == p.splits - 1;
  }
  __syncthreads();
  if (!s_last) {
    trace_end(p.trace);
    return;
  }
  __threadfence();
  const float* base = p.ws + (static_cast<size_t>(blk) * p.n_kv_heads + kvh) * p.splits * 8 * (HD + 2);
  for (int i = threadIdx.x; i < ncols * HD; i += kAttnWarps * 32) {
    const int c = i / HD, d = i % HD;
    float M = -INFINITY;
    for (int s = 0; s < p.splits; ++s) M = fmaxf(M, __ldcg(base + (s * 8 + c) * (HD + 2) + HD));
    const float Mu = M == -INFINITY ? 0.f : M;
    float acc = 0.f, L = 0.f;
    for (int s = 0; s < p.splits; ++s) {
      const float* b = base + (s * 8 + c) * (HD + 2);
      const float f = exp2f(__ldcg(b + HD) - Mu);
      acc += f * __ldcg(b + d);
      L += f * __ldcg(b + HD + 1);
    }
    const int row = r0 + c / group, head = kvh * group + c % group;
    const float v = L > 0.f ? acc / L : 0.f;
    const size_t oi = (static_cast<size_t>(row) * p.n_heads + head) * HD + d;
    if (p.out_f32) reinterpret_cast<float*>(p.out)[oi] = v;
    else reinterpret_cast<T*>(p.out)[oi] = ActTraits<T>::from_f(v);
  }
  if (threadIdx.x == 0) p.counters[blk * p.n_kv_heads + kvh] = 0;
  attn_quant_rows<HD>(p, r0, nq, group, s_rowlast, s_wmax);
  trace_end(p.trace);
}

}  // namespace llm
