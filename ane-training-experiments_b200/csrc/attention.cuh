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
//   online softmax per column (max via 3 xor shuffles, exp2_det with log2e folded in)
//   O^T[hd x 8]        += V^T[hd x 16] . P^T       (V via ldmatrix.trans; P split into two
//                         activation-type terms, each moved into B fragments by 4 shuffles)
//
// Fixed reduction order (independent of the split count, hence of the batch): the context's
// pages form segments of kAttnSegPages pages.  Inside a segment warp w takes pages w, w+4, ...
// with its own online-softmax state; at the segment's end the four warp states are folded as
// (w0 + w1) + (w2 + w3), and the segment states are folded left to right, starting from the
// empty state.  A fold of states (m, l, o) and (m', l', o') is M = max(m, m'), a = 2^(m - M),
// b = 2^(m' - M), l = b*l' + a*l, o = b*o' + a*o (fused multiply-add of the second term onto
// the rounded first).  With one CTA per (block, kv head) the segment states fold in registers;
// with splits the CTAs own whole segments, write every segment state to the workspace, and the
// last CTA of a (block, kv head) folds them in segment order.  Every arithmetic step is an
// explicit round-to-nearest operation or a tensor-core MMA, so the CPU oracle restates it.
// All mbarrier waits are bounded.
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
  int splits;                 // CTAs per (query block, kv head); a block uses at most one per segment
  float scale_log2;           // log2(e) / sqrt(hd)
  void* out;                  // [rows][n_heads][HD] act type, or fp32 when out_f32
  int out_f32;
  float* ws;                  // splits > 1: [n_blocks][n_kv_heads][ws_segs][8][HD + 2] segment states
  int ws_segs;                // segment stride of ws (>= the segments of the longest context)
  int* counters;              // splits > 1: [n_blocks][n_kv_heads]
  // optional fused per-token int8 quantisation of the fp32 output (out_f32 only): the last
  // CTA to finish a row (row_counters, zero between launches) quantises it
  int8_t* q8;                 // [rows][n_heads * HD]
  float* q8_scale;            // [rows]
  int* row_counters;          // [rows]
  // Nonzero when nothing the preceding kernels of this launch chain write can change the
  // block tables, positions, sequence ids or the K/V pages before each block's first query
  // position (decode steps whose inputs were complete before the step began): those pages are
  // then requested before the programmatic wait for the preceding kernel (the QKV projection),
  // which writes only q and the K/V at the query positions.
  int early_kv;
  int* err;
  TraceRec* trace;            // llm_trace_step
};

constexpr int kAttnWarps = 4;
// Pages per segment of the fixed reduction order (512 positions).  Fewer, larger segments mean
// fewer four-warp folds per CTA: 16 / 32 / 64 pages measured 259 / 255 / 249 us per Qwen3 layer at
// 256 sequences x 1536 positions; 32 keeps splits of 512 positions for small batches.
#ifndef LLM_ATTN_SEG_PAGES
#define LLM_ATTN_SEG_PAGES 32
#endif
constexpr int kAttnSegPages = LLM_ATTN_SEG_PAGES;
// Resident CTAs per SM the register budget is sized for (head_dim 128: the shared-memory ring
// allows three; head_dim 64: five).
#ifndef LLM_ATTN_MINB_HD64
#define LLM_ATTN_MINB_HD64 5
#endif
template <int HD>
constexpr int attn_min_blocks() { return HD >= 128 ? 3 : LLM_ATTN_MINB_HD64; }

// Page-ring depth per warp (pages of 16 positions in flight per warp).
// Two pages (64 KB per CTA, three CTAs per SM) measured faster than three (96 KB, two per SM):
// 235.7 vs 240.6 us per Qwen3 layer at 256 sequences x 1536 positions (6.92 vs 6.78 TB/s).
#ifndef LLM_ATTN_STAGES_HD128
#define LLM_ATTN_STAGES_HD128 2
#endif
// head_dim 64: two pages as well (32 KB per CTA): 28.4 vs 36.3 us per Stories110M layer at 256
// sequences x ~160 positions against four pages (short contexts want more CTAs per SM); three
// pages at four CTAs per SM measured slower too (Stories W8A8 decode step 0.925 vs 0.904 ms).
#ifndef LLM_ATTN_STAGES_HD64
#define LLM_ATTN_STAGES_HD64 2
#endif

template <typename T, int HD>
struct AttnCfg {
  static constexpr int PAGE_BYTES = 2 * 16 * HD * (int)sizeof(T);
  static constexpr int STAGES = HD >= 128 ? LLM_ATTN_STAGES_HD128 : LLM_ATTN_STAGES_HD64;
  static constexpr int WARP_BYTES = STAGES * PAGE_BYTES;
  static constexpr int KS = HD / 16;
  // one warp's state in fragment order, value k of lane l at [k * 32 + l]: m0 m1 l0 l1 o[KS][4]
  static constexpr int SLOT_FLOATS = 32 * (4 + 4 * KS);
  static constexpr int FOLD_BYTES = 2 * SLOT_FLOATS * 4;  // two slots for the segment fold
  static constexpr int SMEM = kAttnWarps * WARP_BYTES + FOLD_BYTES;
  static_assert(FOLD_BYTES >= (8 * HD + 8) * 4, "output staging must fit in the fold area");
};

// Online-softmax state of one warp in mma fragment order: lane (g, t) holds columns c0 = 2t and
// c1 = 2t + 1; o[i][0..3] are (dim 16i + g, c0), (16i + g, c1), (16i + g + 8, c0), (16i + g + 8, c1).
template <int KS>
struct WarpState {
  float m0, m1, l0, l1;
  float o[KS][4];
  __device__ __forceinline__ void clear() {
    m0 = m1 = -INFINITY;
    l0 = l1 = 0.f;
#pragma unroll
    for (int i = 0; i < KS; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  }
};

// Scale factors of a fold of maxima ma (kept state) and mb (added state).
__device__ __forceinline__ void fold_scales(float ma, float mb, float& M, float& fa, float& fb) {
  M = fmaxf(ma, mb);
  const float mu = M == -INFINITY ? 0.f : M;
  const float2 f = exp2_det_lo2(sub2_rn(make_float2(ma, mb), make_float2(mu, mu)));
  fa = f.x;
  fb = f.y;
}
__device__ __forceinline__ float fold_val(float fa, float a, float fb, float b) {
  return __fmaf_rn(fb, b, __fmul_rn(fa, a));
}

// a = fold(a, state stored in `slot` by the same lane positions)
template <int KS>
__device__ __forceinline__ void fold_from_slot(WarpState<KS>& a, const float* slot, int lane) {
  float M0, fa0, fb0, M1, fa1, fb1;
  fold_scales(a.m0, slot[0 * 32 + lane], M0, fa0, fb0);
  fold_scales(a.m1, slot[1 * 32 + lane], M1, fa1, fb1);
  a.l0 = fold_val(fa0, a.l0, fb0, slot[2 * 32 + lane]);
  a.l1 = fold_val(fa1, a.l1, fb1, slot[3 * 32 + lane]);
#pragma unroll
  for (int i = 0; i < KS; ++i) {
    const float* s = slot + (4 + 4 * i) * 32 + lane;
    a.o[i][0] = fold_val(fa0, a.o[i][0], fb0, s[0]);
    a.o[i][1] = fold_val(fa1, a.o[i][1], fb1, s[32]);
    a.o[i][2] = fold_val(fa0, a.o[i][2], fb0, s[64]);
    a.o[i][3] = fold_val(fa1, a.o[i][3], fb1, s[96]);
  }
  a.m0 = M0;
  a.m1 = M1;
}
template <int KS>
__device__ __forceinline__ void fold_state(WarpState<KS>& a, const WarpState<KS>& b) {
  float M0, fa0, fb0, M1, fa1, fb1;
  fold_scales(a.m0, b.m0, M0, fa0, fb0);
  fold_scales(a.m1, b.m1, M1, fa1, fb1);
  a.l0 = fold_val(fa0, a.l0, fb0, b.l0);
  a.l1 = fold_val(fa1, a.l1, fb1, b.l1);
#pragma unroll
  for (int i = 0; i < KS; ++i) {
    a.o[i][0] = fold_val(fa0, a.o[i][0], fb0, b.o[i][0]);
    a.o[i][1] = fold_val(fa1, a.o[i][1], fb1, b.o[i][1]);
    a.o[i][2] = fold_val(fa0, a.o[i][2], fb0, b.o[i][2]);
    a.o[i][3] = fold_val(fa1, a.o[i][3], fb1, b.o[i][3]);
  }
  a.m0 = M0;
  a.m1 = M1;
}
template <int KS>
__device__ __forceinline__ void store_slot(float* slot, const WarpState<KS>& a, int lane) {
  slot[0 * 32 + lane] = a.m0;
  slot[1 * 32 + lane] = a.m1;
  slot[2 * 32 + lane] = a.l0;
  slot[3 * 32 + lane] = a.l1;
#pragma unroll
  for (int i = 0; i < KS; ++i) {
    float* s = slot + (4 + 4 * i) * 32 + lane;
    s[0] = a.o[i][0];
    s[32] = a.o[i][1];
    s[64] = a.o[i][2];
    s[96] = a.o[i][3];
  }
}

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
__global__ void __launch_bounds__(kAttnWarps * 32, attn_min_blocks<HD>()) attn_kernel(AttnParams p) {
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
  if (!p.early_kv) griddep_wait();
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
  const int n_seg = (n_pg + kAttnSegPages - 1) / kAttnSegPages;
  // whole segments per CTA: this block uses at most one CTA per segment
  const int want = min(p.splits, n_seg);
  const int per = (n_seg + want - 1) / want;
  const int n_cta = (n_seg + per - 1) / per;
  if (split >= n_cta) {
    trace_end(p.trace);
    return;
  }
  const bool multi = n_cta > 1;
  const int seg0 = split * per, seg1 = min(n_seg, seg0 + per);
  const int p_begin = seg0 * kAttnSegPages, p_end = min(n_pg, seg1 * kAttnSegPages);

  // causal limits of this lane's two score columns (2t, 2t+1); invalid columns mask all
  const int c0 = 2 * t, c1 = 2 * t + 1;
  const int lim0 = (c0 / group) < nq ? pos0 + c0 / group : -1;
  const int lim1 = (c1 / group) < nq ? pos0 + c1 / group : -1;

  uint8_t* wbuf = smem + warp * Cfg::WARP_BYTES;
  float* const fold_area = reinterpret_cast<float*>(smem + kAttnWarps * Cfg::WARP_BYTES);
  float* const slot0 = fold_area;
  float* const slot1 = fold_area + Cfg::SLOT_FLOATS;
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
  // The ring's first pages: with early_kv those wholly before the first query position go out
  // before the wait for the preceding kernel, the rest after it.
  const int stable_end = p.early_kv ? min(p_end, pos0 >> 4) : 0;
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      const int lp = p_begin + warp + kAttnWarps * s;
      if (lp < stable_end) {
        mbar_arrive_expect_tx(bar0 + 8 * s, PB);
        bulk_g2s(wbase + s * PB, page_src(lp), PB, bar0 + 8 * s);
      }
    }
  }
  if (p.early_kv) griddep_wait();
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < STAGES; ++s) {
      const int lp = p_begin + warp + kAttnWarps * s;
      if (lp >= stable_end && lp < p_end) {
        mbar_arrive_expect_tx(bar0 + 8 * s, PB);
        bulk_g2s(wbase + s * PB, page_src(lp), PB, bar0 + 8 * s);
      }
    }
  }
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

  WarpState<KS> run;  // warp 0: fold of this CTA's segments so far
  run.clear();
  int it = 0;         // this warp's pages consumed so far (ring position)
  int fail_it = -1;   // ring position of an expired wait
  for (int sg = seg0; sg < seg1; ++sg) {
    WarpState<KS> st;
    st.clear();
    const int sp_end = min(n_pg, (sg + 1) * kAttnSegPages);
    for (int lp = sg * kAttnSegPages + warp; lp < sp_end; lp += kAttnWarps, ++it) {
      if (fail_it >= 0) continue;
      const int s = it % STAGES;
      const uint32_t parity = (it / STAGES) & 1;
      if (!mbar_wait_bounded(bar0 + 8 * s, parity)) {
        if (lane == 0 && p.err) atomicExch(p.err, kDevWaitTimeout);
        fail_it = it;
        continue;
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
      const float s0 = tk0 <= lim0 ? __fmul_rn(sacc[0], p.scale_log2) : -INFINITY;
      const float s1 = tk0 <= lim1 ? __fmul_rn(sacc[1], p.scale_log2) : -INFINITY;
      const float s2 = tk1 <= lim0 ? __fmul_rn(sacc[2], p.scale_log2) : -INFINITY;
      const float s3 = tk1 <= lim1 ? __fmul_rn(sacc[3], p.scale_log2) : -INFINITY;
      float pm0 = fmaxf(s0, s2), pm1 = fmaxf(s1, s3);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        pm0 = fmaxf(pm0, __shfl_xor_sync(0xffffffffu, pm0, off));
        pm1 = fmaxf(pm1, __shfl_xor_sync(0xffffffffu, pm1, off));
      }
      const float mn0 = fmaxf(st.m0, pm0), mn1 = fmaxf(st.m1, pm1);
      const float mu0 = mn0 == -INFINITY ? 0.f : mn0, mu1 = mn1 == -INFINITY ? 0.f : mn1;
      const float2 mu01 = make_float2(mu0, mu1);
      const float2 al = exp2_det_lo2(sub2_rn(make_float2(st.m0, st.m1), mu01));
      const float2 p01 = exp2_det_lo2(sub2_rn(make_float2(s0, s1), mu01));
      const float2 p23 = exp2_det_lo2(sub2_rn(make_float2(s2, s3), mu01));
      const float al0 = al.x, al1 = al.y, p0 = p01.x, p1 = p01.y, p2 = p23.x, p3 = p23.y;
      st.l0 = __fmaf_rn(st.l0, al0, __fadd_rn(p0, p2));
      st.l1 = __fmaf_rn(st.l1, al1, __fadd_rn(p1, p3));
      st.m0 = mn0;
      st.m1 = mn1;
#pragma unroll
      for (int i = 0; i < KS; ++i) {
        st.o[i][0] = __fmul_rn(st.o[i][0], al0);
        st.o[i][1] = __fmul_rn(st.o[i][1], al1);
        st.o[i][2] = __fmul_rn(st.o[i][2], al0);
        st.o[i][3] = __fmul_rn(st.o[i][3], al1);
      }
      // P^T fragments for column g, tokens (2t,2t+1) and (2t+8,2t+9).  P is carried as a
      // two-term split hi + lo (both in the activation type; lo = p - hi is exact) so the PV
      // product sees P with ~16 mantissa bits instead of the activation type's 8 or 11.
      const uint32_t ph01 = ActTraits<T>::pack2(p0, p1);
      const uint32_t ph23 = ActTraits<T>::pack2(p2, p3);
      const float2 h01 = ActTraits<T>::unpack2(ph01), h23 = ActTraits<T>::unpack2(ph23);
      const uint32_t pl01 = ActTraits<T>::pack2(__fsub_rn(p0, h01.x), __fsub_rn(p1, h01.y));
      const uint32_t pl23 = ActTraits<T>::pack2(__fsub_rn(p2, h23.x), __fsub_rn(p3, h23.y));
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
        mma_16816(st.o[mt], a, bh0, bh1, T());
        mma_16816(st.o[mt], a, bl0, bl1, T());
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
    if (fail_it >= 0) st.clear();  // an expired wait contributes nothing (the error is recorded)
    // the warp's row sums: lanes of a column hold partial sums over their token pairs
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      st.l0 = __fadd_rn(st.l0, __shfl_xor_sync(0xffffffffu, st.l0, off));
      st.l1 = __fadd_rn(st.l1, __shfl_xor_sync(0xffffffffu, st.l1, off));
    }
    // segment state = (w0 + w1) + (w2 + w3)
    if (warp == 1) store_slot(slot0, st, lane);
    if (warp == 3) store_slot(slot1, st, lane);
    __syncthreads();
    if (warp == 0) fold_from_slot(st, slot0, lane);
    if (warp == 2) {
      fold_from_slot(st, slot1, lane);
      store_slot(slot1, st, lane);  // each lane rewrites only the values it read
    }
    __syncthreads();
    if (warp == 0) {
      fold_from_slot(st, slot1, lane);
      if (!multi) {
        fold_state(run, st);
      } else {
        float* part = p.ws + ((static_cast<size_t>(blk) * p.n_kv_heads + kvh) * p.ws_segs + sg) * 8 * (HD + 2);
#pragma unroll
        for (int mt = 0; mt < KS; ++mt) {
          const int d = mt * 16 + g;
          __stcg(part + c0 * (HD + 2) + d, st.o[mt][0]);
          __stcg(part + c1 * (HD + 2) + d, st.o[mt][1]);
          __stcg(part + c0 * (HD + 2) + d + 8, st.o[mt][2]);
          __stcg(part + c1 * (HD + 2) + d + 8, st.o[mt][3]);
        }
        if (g == 0) {
          __stcg(part + c0 * (HD + 2) + HD, st.m0);
          __stcg(part + c0 * (HD + 2) + HD + 1, st.l0);
          __stcg(part + c1 * (HD + 2) + HD, st.m1);
          __stcg(part + c1 * (HD + 2) + HD + 1, st.l1);
        }
      }
    }
    __syncthreads();  // the slots are rewritten at the next segment's end
  }
  if (fail_it >= 0) {
    // drain copies still in flight into this warp's ring (bounded)
    for (int j = fail_it + 1; j < fail_it + STAGES; ++j) {
      const int lp = p_begin + warp + kAttnWarps * j;
      if (lp >= p_end) break;
      mbar_wait_bounded(bar0 + 8 * (j % STAGES), (j / STAGES) & 1);
    }
  }

  const int ncols = min(8, nq * group);
  if (!multi) {
    // out = o / l: o and l staged through the fold area, then every thread divides and stores
    // its own elements (only the block's ncols valid columns), coalesced along the rows
    float* stage = fold_area;
    float* stage_l = fold_area + 8 * HD;
    if (warp == 0) {
#pragma unroll
      for (int mt = 0; mt < KS; ++mt) {
        const int d = mt * 16 + g;
        stage[c0 * HD + d] = run.o[mt][0];
        stage[c1 * HD + d] = run.o[mt][1];
        stage[c0 * HD + d + 8] = run.o[mt][2];
        stage[c1 * HD + d + 8] = run.o[mt][3];
      }
      if (g == 0) {  // every lane of a column holds the same row sum
        stage_l[c0] = run.l0;
        stage_l[c1] = run.l1;
      }
    }
    __syncthreads();
    for (int i = threadIdx.x; i < ncols * HD; i += kAttnWarps * 32) {
      const int c = i / HD, d = i % HD;
      const float l = stage_l[c];
      const float v = l > 0.f ? __fdiv_rn(stage[i], l) : 0.f;
      const int row = r0 + c / group, head = kvh * group + c % group;
      const size_t oi = (static_cast<size_t>(row) * p.n_heads + head) * HD + d;
      if (p.out_f32) reinterpret_cast<float*>(p.out)[oi] = v;
      else reinterpret_cast<T*>(p.out)[oi] = ActTraits<T>::from_f(v);
    }
    attn_quant_rows<HD>(p, r0, nq, group, s_rowlast, s_wmax);
    trace_end(p.trace);
    return;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(p.counters + blk * p.n_kv_heads + kvh, 1);
    s_last = prev == n_cta - 1;
  }
  __syncthreads();
  if (!s_last) {
    trace_end(p.trace);
    return;
  }
  __threadfence();
  // the last CTA folds every segment state in segment order, starting from the empty state
  const float* base = p.ws + (static_cast<size_t>(blk) * p.n_kv_heads + kvh) * p.ws_segs * 8 * (HD + 2);
  for (int i = threadIdx.x; i < ncols * HD; i += kAttnWarps * 32) {
    const int c = i / HD, d = i % HD;
    float M = -INFINITY, L = 0.f, O = 0.f;
    for (int sg = 0; sg < n_seg; ++sg) {
      const float* b = base + (static_cast<size_t>(sg) * 8 + c) * (HD + 2);
      float Mn, fa, fb;
      fold_scales(M, __ldcg(b + HD), Mn, fa, fb);
      O = fold_val(fa, O, fb, __ldcg(b + d));
      L = fold_val(fa, L, fb, __ldcg(b + HD + 1));
      M = Mn;
    }
    const int row = r0 + c / group, head = kvh * group + c % group;
    const float v = L > 0.f ? __fdiv_rn(O, L) : 0.f;
    const size_t oi = (static_cast<size_t>(row) * p.n_heads + head) * HD + d;
    if (p.out_f32) reinterpret_cast<float*>(p.out)[oi] = v;
    else reinterpret_cast<T*>(p.out)[oi] = ActTraits<T>::from_f(v);
  }
  if (threadIdx.x == 0) p.counters[blk * p.n_kv_heads + kvh] = 0;
  attn_quant_rows<HD>(p, r0, nq, group, s_rowlast, s_wmax);
  trace_end(p.trace);
}

}  // namespace llm
