// attn_prefill.cuh -- causal attention of prefill tiles over the paged KV cache.
//
// Reference: ane/stories/infer.go:267-299 (attend: scores q.k/sqrt(hd) over t <= pos,
// softmaxPrefix, PV), evaluated for many query positions of one sequence at once, with the GQA
// head map kv_head = q_head / group of training/training_dynamic/io.h:434-455.
//
// One CTA = (query tile, kv head).  A query tile is up to QT = 128/group consecutive query
// positions of one sequence; its 128 score rows are (head h of the kv head's group, position
// i) -> row h*QT + i, 16 rows per warp (8 warps).  The CTA streams the sequence's K/V pages
// (16 positions x [K | V], swizzled rows, see attention.cuh) 64 positions at a time through a
// STAGES-deep ring filled by the bulk-copy engine (one cp.async.bulk per page, completion on
// an mbarrier), and every warp runs, per 64-position tile:
//   S[16 x 64]  = Q[16 x hd] . K^T           (mma.m16n8k16, Q fragments in registers,
//                                             K fragments by ldmatrix)
//   online softmax per row (quad shuffles, exp2 with log2(e)/sqrt(hd) folded in, causal mask)
//   O[16 x hd] += P[16 x 64] . V[64 x hd]     (P from the S accumulators without shuffles,
//                                             carried as two activation-type terms hi + lo
//                                             like the decode kernel; V by ldmatrix.trans)
// A CTA stops at the last tile its query positions can see (causal), and tiles are numbered
// longest-first so the heaviest CTAs start first.  All waits are bounded.
#pragma once
#include "common.cuh"

namespace llm {

struct PrefillAttnParams {
  const void* q;            // [rows][n_heads][HD] act type
  const void* kv_pool;
  const int* block_table;   // [max_seqs][max_pages_per_seq]
  int max_pages_per_seq;
  const int* seq_ids;       // [rows]
  const int* positions;     // [rows]
  const int* tile_row0;     // [n_tiles] first row of each query tile
  const int* tile_nq;       // [n_tiles] rows in the tile (<= 128 / group)
  int n_tiles;
  int n_heads, n_kv_heads, layer, n_pages;
  float scale_log2;         // log2(e) / sqrt(hd)
  void* out;                // [rows][n_heads][HD] act type, or fp32 when out_f32
  int out_f32;
  int* err;
  TraceRec* trace;
};

constexpr int kPrefillWarps = 8;
constexpr int kPrefillRows = 16 * kPrefillWarps;  // score rows per CTA

template <typename T, int HD>
struct PrefillCfg {
  static constexpr int PAGE_BYTES = 2 * 16 * HD * (int)sizeof(T);
  static constexpr int TILE_PAGES = 4;  // 64 positions per tile
  static constexpr int STAGE_BYTES = TILE_PAGES * PAGE_BYTES;
  static constexpr int STAGES = HD >= 128 ? 3 : 4;
  static constexpr int SMEM = STAGES * STAGE_BYTES;
};

template <typename T, int HD>
__global__ void __launch_bounds__(kPrefillWarps * 32, 1) attn_prefill_kernel(PrefillAttnParams p) {
  using Cfg = PrefillCfg<T, HD>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int PB = Cfg::PAGE_BYTES;
  constexpr int KS = HD / 16;      // k-steps over the head dimension
  constexpr int NO = HD / 8;       // n-tiles of the output
  constexpr int ROWB = HD * (int)sizeof(T);

  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ __align__(8) uint64_t bars[STAGES];

  griddep_launch_dependents();
  trace_start(p.trace);
  griddep_wait();
  // 1-D grid, kv head fastest: the host lists tiles longest context first, so every kv
  // head's longest tiles start in the first wave
  const int tile = static_cast<int>(blockIdx.x) / p.n_kv_heads;
  const int kvh = static_cast<int>(blockIdx.x) % p.n_kv_heads;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int group = p.n_heads / p.n_kv_heads;
  const int QT = kPrefillRows / group;

  const int r0 = p.tile_row0[tile];
  const int nq = p.tile_nq[tile];
  const int seq = p.seq_ids[r0];
  const int pos0 = p.positions[r0];
  const int ctx = pos0 + nq;                   // positions 0 .. ctx-1 are visible to the tile
  const int n_tiles_kv = (ctx + 63) >> 6;

  // this warp's 16 rows: head h = (warp*16)/QT of the group, positions i0 .. i0+15
  const int row_base = warp * 16;
  const int h = row_base / QT;
  const int i0 = row_base % QT;
  const int qa = i0 + g, qb = i0 + g + 8;      // this lane's two query positions (tile-relative)
  const bool va = qa < nq, vb = qb < nq;
  const int lim_a = va ? pos0 + qa : -1, lim_b = vb ? pos0 + qb : -1;
  const int head = kvh * group + h;

  uint32_t qf[KS][4];
  {
    const T* qra = reinterpret_cast<const T*>(p.q) + (static_cast<size_t>(r0 + (va ? qa : 0)) * p.n_heads + head) * HD;
    const T* qrb = reinterpret_cast<const T*>(p.q) + (static_cast<size_t>(r0 + (vb ? qb : 0)) * p.n_heads + head) * HD;
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
      qf[ks][0] = va ? *reinterpret_cast<const uint32_t*>(qra + ks * 16 + 2 * t) : 0u;
      qf[ks][1] = vb ? *reinterpret_cast<const uint32_t*>(qrb + ks * 16 + 2 * t) : 0u;
      qf[ks][2] = va ? *reinterpret_cast<const uint32_t*>(qra + ks * 16 + 8 + 2 * t) : 0u;
      qf[ks][3] = vb ? *reinterpret_cast<const uint32_t*>(qrb + ks * 16 + 8 + 2 * t) : 0u;
    }
  }

  const uint32_t sbase = smem_u32(smem);
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
  const int n_pages_ctx = (ctx + 15) >> 4;
  // thread 0 fills stage s with the pages of kv tile kt
  auto issue = [&](int kt, int s) {
    const int first = kt * Cfg::TILE_PAGES;
    const int np = min(Cfg::TILE_PAGES, n_pages_ctx - first);
    const uint32_t bar = smem_u32(&bars[s]);
    mbar_arrive_expect_tx(bar, np * PB);
    for (int j = 0; j < np; ++j) bulk_g2s(sbase + s * Cfg::STAGE_BYTES + j * PB, page_src(first + j), PB, bar);
  };
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) mbar_init(smem_u32(&bars[s]), 1);
    fence_mbar_init();
    for (int s = 0; s < STAGES && s < n_tiles_kv; ++s) issue(s, s);
  }
  __syncthreads();

  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  float o[NO][4];
#pragma unroll
  for (int i = 0; i < NO; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;

  bool timed_out = false;
  int kt = 0;
  for (; kt < n_tiles_kv; ++kt) {
    const int s = kt % STAGES;
    const bool ok = mbar_wait_bounded(smem_u32(&bars[s]), (kt / STAGES) & 1);
    if (__syncthreads_or(!ok)) {  // the CTA agrees, so no thread is left waiting at a barrier
      timed_out = true;
      break;
    }
    const int kbase = kt * 64;
    const uint32_t st = sbase + s * Cfg::STAGE_BYTES;
    // pages of the tile past the context were not loaded: zero their V rows so 0-weight x
    // stale shared memory cannot produce NaN (their scores are masked)
    const int valid = ctx - kbase;  // positions of this tile that exist (>= 1)
    if (valid < 64) {
      for (int i = threadIdx.x; i < (64 - valid) * (HD / 8); i += kPrefillWarps * 32) {
        const int pr = valid + i / (HD / 8);  // tile-relative position
        const int c = i % (HD / 8);
        uint4* dst = reinterpret_cast<uint4*>(smem + s * Cfg::STAGE_BYTES + (pr >> 4) * PB + 16 * ROWB + kv_off(pr & 15, c));
        *dst = make_uint4(0, 0, 0, 0);
      }
      __syncthreads();
    }
    // warps whose rows cannot see this tile skip the math (warp-uniform; they still take
    // part in the CTA barriers)
    const bool active = i0 < nq && kbase <= pos0 + min(nq - 1, i0 + 15);
    if (active) {
      float sc[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
      // k-steps outer, pages inner: eight independent accumulators per k-step
#pragma unroll
      for (int ks = 0; ks < KS; ++ks) {
#pragma unroll
        for (int pg = 0; pg < 4; ++pg) {
          uint32_t b[4];
          const int mi = lane >> 3;
          const int row = ((mi >> 1) << 3) + (lane & 7);
          ldmatrix_x4(b, st + pg * PB + kv_off(row, 2 * ks + (mi & 1)));
          mma_16816(sc[2 * pg], qf[ks], b[0], b[1], T());
          mma_16816(sc[2 * pg + 1], qf[ks], b[2], b[3], T());
        }
      }
      // scale, causal mask, running max
      float mx_a = -INFINITY, mx_b = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c0 = kbase + 8 * j + 2 * t, c1 = c0 + 1;
        sc[j][0] = c0 <= lim_a ? sc[j][0] * p.scale_log2 : -INFINITY;
        sc[j][1] = c1 <= lim_a ? sc[j][1] * p.scale_log2 : -INFINITY;
        sc[j][2] = c0 <= lim_b ? sc[j][2] * p.scale_log2 : -INFINITY;
        sc[j][3] = c1 <= lim_b ? sc[j][3] * p.scale_log2 : -INFINITY;
        mx_a = fmaxf(mx_a, fmaxf(sc[j][0], sc[j][1]));
        mx_b = fmaxf(mx_b, fmaxf(sc[j][2], sc[j][3]));
      }
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 1));
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, 2));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 1));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, 2));
      const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
      const float mu_a = mn_a == -INFINITY ? 0.f : mn_a, mu_b = mn_b == -INFINITY ? 0.f : mn_b;
      const float al_a = exp2_det(m_a - mu_a), al_b = exp2_det(m_b - mu_b);
      m_a = mn_a;
      m_b = mn_b;
      float rs_a = 0.f, rs_b = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        sc[j][0] = exp2_det(sc[j][0] - mu_a);
        sc[j][1] = exp2_det(sc[j][1] - mu_a);
        sc[j][2] = exp2_det(sc[j][2] - mu_b);
        sc[j][3] = exp2_det(sc[j][3] - mu_b);
        rs_a += sc[j][0] + sc[j][1];
        rs_b += sc[j][2] + sc[j][3];
      }
      l_a = l_a * al_a + rs_a;
      l_b = l_b * al_b + rs_b;
#pragma unroll
      for (int i = 0; i < NO; ++i) {
        o[i][0] *= al_a; o[i][1] *= al_a; o[i][2] *= al_b; o[i][3] *= al_b;
      }
      // O += P . V, one page (16 positions) per k-step; P as hi + lo activation-type terms
#pragma unroll
      for (int pg = 0; pg < 4; ++pg) {
        uint32_t ah[4], al[4];
        {
          const float* s0 = sc[2 * pg];
          const float* s1 = sc[2 * pg + 1];
          ah[0] = ActTraits<T>::pack2(s0[0], s0[1]);
          ah[1] = ActTraits<T>::pack2(s0[2], s0[3]);
          ah[2] = ActTraits<T>::pack2(s1[0], s1[1]);
          ah[3] = ActTraits<T>::pack2(s1[2], s1[3]);
          const float2 h0 = ActTraits<T>::unpack2(ah[0]), h1 = ActTraits<T>::unpack2(ah[1]);
          const float2 h2 = ActTraits<T>::unpack2(ah[2]), h3 = ActTraits<T>::unpack2(ah[3]);
          al[0] = ActTraits<T>::pack2(s0[0] - h0.x, s0[1] - h0.y);
          al[1] = ActTraits<T>::pack2(s0[2] - h1.x, s0[3] - h1.y);
          al[2] = ActTraits<T>::pack2(s1[0] - h2.x, s1[1] - h2.y);
          al[3] = ActTraits<T>::pack2(s1[2] - h3.x, s1[3] - h3.y);
        }
        const uint32_t vb = st + pg * PB + 16 * ROWB;
#pragma unroll
        for (int nt = 0; nt < NO; nt += 2) {
          uint32_t b[4];
          const int row = (lane & 7) + 8 * ((lane >> 3) & 1);
          ldmatrix_x4_trans(b, vb + kv_off(row, nt + (lane >> 4)));
          mma_16816(o[nt], ah, b[0], b[1], T());
          mma_16816(o[nt], al, b[0], b[1], T());
          mma_16816(o[nt + 1], ah, b[2], b[3], T());
          mma_16816(o[nt + 1], al, b[2], b[3], T());
        }
      }
    }
    __syncthreads();  // every warp is done with stage s
    if (threadIdx.x == 0 && kt + STAGES < n_tiles_kv) {
      fence_proxy_async_smem();
      issue(kt + STAGES, s);
    }
  }
  if (timed_out) {
    if (p.err) atomicExch(p.err, kDevWaitTimeout);
    // drain the copies still in flight into the ring (bounded) before the CTA exits
    for (int j = kt + 1; j < kt + STAGES && j < n_tiles_kv; ++j) mbar_wait_bounded(smem_u32(&bars[j % STAGES]), (j / STAGES) & 1);
    trace_end(p.trace);
    return;
  }
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 1);
  l_a += __shfl_xor_sync(0xffffffffu, l_a, 2);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 1);
  l_b += __shfl_xor_sync(0xffffffffu, l_b, 2);
  const float inv_a = l_a > 0.f ? 1.0f / l_a : 0.f, inv_b = l_b > 0.f ? 1.0f / l_b : 0.f;
#pragma unroll
  for (int nt = 0; nt < NO; ++nt) {
    const int d = nt * 8 + 2 * t;
    if (va) {
      const size_t oi = (static_cast<size_t>(r0 + qa) * p.n_heads + head) * HD + d;
      if (p.out_f32) *reinterpret_cast<float2*>(reinterpret_cast<float*>(p.out) + oi) = make_float2(o[nt][0] * inv_a, o[nt][1] * inv_a);
      else *reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(p.out) + oi) = ActTraits<T>::pack2(o[nt][0] * inv_a, o[nt][1] * inv_a);
    }
    if (vb) {
      const size_t oi = (static_cast<size_t>(r0 + qb) * p.n_heads + head) * HD + d;
      if (p.out_f32) *reinterpret_cast<float2*>(reinterpret_cast<float*>(p.out) + oi) = make_float2(o[nt][2] * inv_b, o[nt][3] * inv_b);
      else *reinterpret_cast<uint32_t*>(reinterpret_cast<T*>(p.out) + oi) = ActTraits<T>::pack2(o[nt][2] * inv_b, o[nt][3] * inv_b);
    }
  }
  trace_end(p.trace);
}

}  // namespace llm
