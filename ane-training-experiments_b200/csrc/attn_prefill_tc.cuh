// attn_prefill_tc.cuh -- causal prefill attention on the 5th-generation tensor cores.
//
// Reference: ane/stories/infer.go:267-299 (attend: scores q.k/sqrt(hd) over t <= pos,
// softmaxPrefix, PV) for many query positions of one sequence at once, with the GQA head map
// kv_head = q_head / group of training/training_dynamic/io.h:434-455.
//
// One CTA = (query tile, kv head): 128 score rows, row = h * (128/group) + i for head h of the
// kv head's group and query position i of the tile; TMEM lane = row.  The sequence's cached
// K/V pages are streamed 64 positions at a time through separate K and V rings (bulk copies of
// the pages' 16 x 128 B sub-blocks, see kv_off in common.cuh, placed so that a 64-position tile
// of every 64-element half of K and V is one 128B-swizzled operand).  Per tile t:
//   MMA warp:      S_t[128 x 64] = Q . K_t^T   (tcgen05.mma kind::f16, Q and K K-major in shared
//                                               memory, f32 accumulator in TMEM, two buffers)
//   softmax warps: one thread per row reads its 64 scores from TMEM, applies scale and the
//                  causal mask, accumulates the row sum against a reference max, and writes P
//                  as two activation-type terms hi + lo (the decode kernel's ~16-bit softmax
//                  weights) back into the same TMEM columns
//   MMA warp:      O[128 x hd] += P_hi . V_t + P_lo . V_t   (A = P from TMEM, V MN-major)
// The reference max of a row moves only when a tile's max exceeds it by more than 2^8 (log2
// domain 8): P <= 256 stays exact in the hi + lo split, and the O rescale -- the one step that
// has to wait for the previous PV -- becomes rare.  S_{t+1} runs on the tensor core while the
// softmax of t runs, and two CTAs share an SM (~97 KB shared memory, 256 TMEM columns each), so
// one CTA's softmax overlaps the other's MMAs.  Warp 0 = bulk-copy producer, warp 1 = TMEM
// allocator + MMA issuer (one thread), warps 2..5 = softmax / epilogue.  Every wait is bounded;
// on expiry the CTA records kDevWaitTimeout, drains its copies and MMAs and still frees its TMEM.
#pragma once
#include "attn_prefill.cuh"
#include "common.cuh"
#include "umma.cuh"

namespace llm {

template <typename T, int HD>
struct PrefillTcCfg {
  static constexpr int HALVES = HD / 64;              // 64-element halves of a K / V row
  static constexpr int SUB = 16 * 128;                // one page's half sub-block (bytes)
  static constexpr int REGION = 4 * SUB;              // 64 positions of one half (bytes)
  static constexpr int TILE_BYTES = HALVES * REGION;  // K (or V) of one 64-position tile
  static constexpr int K_STAGES = HD == 64 ? 3 : 2;
  static constexpr int V_STAGES = HD == 64 ? 3 : 2;
  static constexpr int Q_BYTES = HALVES * 128 * 128;  // 128 rows x HD, K-major halves
  static constexpr int SMEM = Q_BYTES + (K_STAGES + V_STAGES) * TILE_BYTES + 1024;
  static constexpr uint32_t TMEM_COLS = 256;          // S/P: 2 x 64 columns, O: HD columns at 128
  static constexpr float RESCALE_LOG2 = 8.0f;         // reference max moves beyond this gap
};

template <typename T, int HD>
__global__ void __launch_bounds__(192, 2) attn_prefill_tc_kernel(PrefillAttnParams p) {
  using Cfg = PrefillTcCfg<T, HD>;
  constexpr int KS = Cfg::K_STAGES, VS = Cfg::V_STAGES;
  constexpr int HALVES = Cfg::HALVES;
  constexpr int SUB = Cfg::SUB;
  constexpr int REGION = Cfg::REGION;
  constexpr int ROWB = HD * (int)sizeof(T);  // bytes of one K or V row in the page block
  // MN-major V: the second 64-element chunk of hd is the next half's region; with one half
  // the offset is never applied and stays inside the tile
  constexpr uint32_t V_LBO = HALVES > 1 ? REGION : 1024;

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t k_full[KS], k_empty[KS], v_full[VS], v_empty[VS], s_full[2], p_ready[2],
      pv_done, q_ready, drain;
  __shared__ uint32_t s_tmem;

  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t q_s = sbase;
  const uint32_t k_ring = q_s + Cfg::Q_BYTES;
  const uint32_t v_ring = k_ring + KS * Cfg::TILE_BYTES;
  uint8_t* const gbase = smem_raw + (sbase - smem_u32(smem_raw));  // generic pointer of sbase

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 1-D grid, kv head fastest: the host lists tiles longest context first, so every kv
  // head's longest tiles start in the first wave
  const int tile = static_cast<int>(blockIdx.x) / p.n_kv_heads;
  const int kvh = static_cast<int>(blockIdx.x) % p.n_kv_heads;
  const int group = p.n_heads / p.n_kv_heads;
  const int QT = 128 / group;

  trace_start(p.trace);
  if (threadIdx.x == 0) {
    for (int s = 0; s < KS; ++s) {
      mbar_init(smem_u32(&k_full[s]), 1);
      mbar_init(smem_u32(&k_empty[s]), 1);
    }
    for (int s = 0; s < VS; ++s) {
      mbar_init(smem_u32(&v_full[s]), 1);
      mbar_init(smem_u32(&v_empty[s]), 1);
    }
    mbar_init(smem_u32(&s_full[0]), 1);
    mbar_init(smem_u32(&s_full[1]), 1);
    mbar_init(smem_u32(&p_ready[0]), 128);
    mbar_init(smem_u32(&p_ready[1]), 128);
    mbar_init(smem_u32(&pv_done), 1);
    mbar_init(smem_u32(&q_ready), 128);
    mbar_init(smem_u32(&drain), 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&s_tmem), Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;
  // dependents launch only after every CTA of this grid holds its TMEM columns
  griddep_launch_dependents();
  griddep_wait();

  const int r0 = p.tile_row0[tile];
  const int nq = p.tile_nq[tile];
  const int seq = p.seq_ids[r0];
  const int pos0 = p.positions[r0];
  const int ctx = pos0 + nq;
  const int nkv = (ctx + 63) >> 6;            // 64-position K/V tiles the CTA needs
  const int n_pages_ctx = (ctx + 15) >> 4;
  bool failed = false;

  if (warp == 0) {
    // ------------------------------------------------------------ bulk-copy producer
    // The whole warp reads the block table, 32 pages (8 tiles) per coalesced load, one batch
    // ahead of use; lane 0 issues the copies.  Waits run on every lane and are made uniform.
    const T* pool = reinterpret_cast<const T*>(p.kv_pool);
    const int* bt = p.block_table + static_cast<size_t>(seq) * p.max_pages_per_seq;
    auto entries = [&](int first_page) -> int {
      const int pg = first_page + lane;
      if (pg >= n_pages_ctx) return 0;
      int e = bt[pg];
      if (e < 0 || e >= p.n_pages) {
        if (p.err) atomicExch(p.err, kDevBadPage);
        e = 0;
      }
      return e;
    };
    int ent = entries(0), ent_next = entries(32);
    // one tile of K (v = 0) or V (v = 1): its pages' half sub-blocks into one ring stage
    auto load = [&](int t, int v, uint32_t dst, uint32_t bar) {
      const int np = min(4, n_pages_ctx - 4 * t);
      int phys[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) phys[j] = __shfl_sync(0xffffffffu, ent, ((t & 7) << 2) + j);
      if (lane == 0) {
        mbar_arrive_expect_tx(bar, np * HALVES * SUB);
        for (int j = 0; j < np; ++j) {
          const uint8_t* blk = reinterpret_cast<const uint8_t*>(
                                   pool + ((static_cast<size_t>(p.layer) * p.n_pages + phys[j]) * p.n_kv_heads + kvh) *
                                              (2 * 16 * HD)) +
                               v * 16 * ROWB;
          for (int hh = 0; hh < HALVES; ++hh) bulk_g2s(dst + hh * REGION + j * SUB, blk + hh * SUB, SUB, bar);
        }
      }
    };
    int k_issued = 0, v_issued = 0;
    for (int t = 0; t < nkv; ++t) {
      if (t > 0 && (t & 7) == 0) {
        ent = ent_next;
        ent_next = entries(4 * t + 32);
      }
      if (t >= KS && !__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&k_empty[t % KS]), ((t / KS) + 1) & 1))) {
        failed = true;
        break;
      }
      load(t, 0, k_ring + (t % KS) * Cfg::TILE_BYTES, smem_u32(&k_full[t % KS]));
      k_issued = t + 1;
      if (t >= VS && !__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&v_empty[t % VS]), ((t / VS) + 1) & 1))) {
        failed = true;
        break;
      }
      load(t, 1, v_ring + (t % VS) * Cfg::TILE_BYTES, smem_u32(&v_full[t % VS]));
      v_issued = t + 1;
    }
    // copies still in flight must land before the CTA's shared memory goes away
    if (lane == 0) {
      for (int t = max(0, k_issued - KS); t < k_issued; ++t) mbar_wait_bounded(smem_u32(&k_full[t % KS]), (t / KS) & 1);
      for (int t = max(0, v_issued - VS); t < v_issued; ++t) mbar_wait_bounded(smem_u32(&v_full[t % VS]), (t / VS) & 1);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc<T>(128, 64);
      constexpr uint32_t idesc_pv = umma_idesc<T>(128, HD) | (1u << 16);  // B (V) MN-major
      const uint32_t o_tmem = tmem + 128;
      // S_t into TMEM columns (t & 1) * 64; frees the K stage when the MMAs complete
      auto issue_s = [&](int t) -> bool {
        const int s = t % KS;
        if (!mbar_wait_bounded(smem_u32(&k_full[s]), (t / KS) & 1)) return false;
        tc_fence_after();
        const uint32_t kst = k_ring + s * Cfg::TILE_BYTES;
        const uint32_t d = tmem + (t & 1) * 64;
#pragma unroll
        for (int k = 0; k < HD / 16; ++k) {
          const int hh = k >> 2, kk = k & 3;
          umma<false>(d, sw128_desc(q_s + hh * 128 * 128 + 32 * kk), sw128_desc(kst + hh * REGION + 32 * kk), idesc_s,
                      k > 0 ? 1u : 0u);
        }
        tc_commit(smem_u32(&k_empty[s]));
        tc_commit(smem_u32(&s_full[t & 1]));
        return true;
      };
      bool ok = mbar_wait_bounded(smem_u32(&q_ready), 0);
      if (ok) ok = issue_s(0);
      if (ok && nkv > 1) ok = issue_s(1);
      for (int t = 0; ok && t < nkv; ++t) {
        if (!mbar_wait_bounded(smem_u32(&p_ready[t & 1]), (t >> 1) & 1) ||
            !mbar_wait_bounded(smem_u32(&v_full[t % VS]), (t / VS) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t vst = v_ring + (t % VS) * Cfg::TILE_BYTES;
        const uint32_t pa = tmem + (t & 1) * 64;  // P_hi at +0, P_lo at +32 (16-bit pairs)
#pragma unroll
        for (int term = 0; term < 2; ++term) {
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)  // 16 positions per MMA
            umma_ts(o_tmem, pa + term * 32 + kk * 8, sw128_desc_mn(vst + kk * 2048, V_LBO, 1024), idesc_pv,
                    (t > 0 || term > 0 || kk > 0) ? 1u : 0u);
        }
        tc_commit(smem_u32(&v_empty[t % VS]));
        tc_commit(smem_u32(&pv_done));
        if (t + 2 < nkv) {
          // S_{t+2} overwrites the columns P_t is read from: PV_t must be complete
          if (!mbar_wait_bounded(smem_u32(&pv_done), t & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          ok = issue_s(t + 2);
        }
      }
      if (!ok) failed = true;
      // every MMA this thread issued has completed before O is read and TMEM is freed
      tc_commit(smem_u32(&drain));
      mbar_wait_bounded(smem_u32(&drain), 0);
    }
  } else {
    // ------------------------------------------------------------ softmax / epilogue warps
    const int q = warp & 3;
    const int tl = q * 32 + lane;              // score row = TMEM lane
    const int h = tl / QT, i = tl % QT;
    const bool row_ok = i < nq;
    const int lim = row_ok ? pos0 + i : -1;    // last visible position of this row
    const int head = kvh * group + h;
    const uint32_t trow = tmem + (static_cast<uint32_t>(q * 32) << 16);

    // Q row -> shared memory, K-major 128B-swizzled halves
    {
      const uint4* src = reinterpret_cast<const uint4*>(reinterpret_cast<const T*>(p.q) +
                                                        (static_cast<size_t>(r0 + (row_ok ? i : 0)) * p.n_heads + head) * HD);
#pragma unroll
      for (int c = 0; c < HD / 8; ++c) {
        const uint4 v = row_ok ? src[c] : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(gbase + (c >> 3) * 128 * 128 + tl * 128 + (((c & 7) ^ (tl & 7)) << 4)) = v;
      }
      fence_proxy_async_smem();
      mbar_arrive(smem_u32(&q_ready));
    }

    const float sl2 = p.scale_log2;
    float m_ref = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int t = 0; t < nkv; ++t) {
      // wait results are made warp-uniform: the TMEM accesses below are warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&s_full[t & 1]), (t >> 1) & 1))) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t scol = trow + (t & 1) * 64;
      float sv[64];
      {
        uint32_t ra[32], rb[32];
        tmem_ld32(scol, ra);
        tmem_ld32(scol + 32, rb);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          sv[j] = __uint_as_float(ra[j]);
          sv[32 + j] = __uint_as_float(rb[j]);
        }
      }
      const int kbase = t * 64;
      // causal / ragged mask: only tiles reaching past some row's last visible position
      if (__any_sync(0xffffffffu, kbase + 63 > lim)) {
#pragma unroll
        for (int j = 0; j < 64; ++j)
          if (kbase + j > lim) sv[j] = -INFINITY;
      }
      float m8[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) m8[j] = sv[j];
#pragma unroll
      for (int j = 8; j < 64; ++j) m8[j & 7] = fmaxf(m8[j & 7], sv[j]);
      const float mx = __fmul_rn(fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                                       fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7]))), sl2);  // scale > 0
      // move the reference max only past the gap; the first visible tile always sets it
      const bool move = mx > __fadd_rn(m_ref, Cfg::RESCALE_LOG2);
      const float m_new = move ? mx : m_ref;
      const float mu = m_new == -INFINITY ? 0.f : m_new;
      const float alpha = move ? exp2_det_lo(__fsub_rn(m_ref, mu)) : 1.0f;
      // p = 2^(s * scale - ref) two positions at a time (packed f32 pairs); the row sum in 8
      // interleaved partials r8[j & 7] (pairs r4[k] = (r8[2k], r8[2k + 1]))
      float2 r4[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) r4[k] = make_float2(0.f, 0.f);
      {
        const float2 sl22 = make_float2(sl2, sl2), nmu = make_float2(-mu, -mu);
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float2 pe = exp2_det_lo2(fma2_rn(make_float2(sv[2 * e], sv[2 * e + 1]), sl22, nmu));
          sv[2 * e] = pe.x;
          sv[2 * e + 1] = pe.y;
          r4[e & 3] = add2_rn(r4[e & 3], pe);
        }
      }
      const float rs = __fadd_rn(__fadd_rn(__fadd_rn(r4[0].x, r4[0].y), __fadd_rn(r4[1].x, r4[1].y)),
                                 __fadd_rn(__fadd_rn(r4[2].x, r4[2].y), __fadd_rn(r4[3].x, r4[3].y)));
      l_run = __fmaf_rn(l_run, alpha, rs);
      m_ref = m_new;

      // O holds PV of tiles < t: rescale rows whose reference moved, after PV_{t-1} completed
      // (tile 0's PV overwrites O, so nothing to rescale before it)
      if (t > 0 && __any_sync(0xffffffffu, move)) {
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&pv_done), (t - 1) & 1))) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < HD / 32; ++c) {
          uint32_t r[32];
          tmem_ld32(trow + 128 + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(__fmul_rn(__uint_as_float(r[j]), alpha));
          tmem_st32(trow + 128 + c * 32, r);
        }
      }
      // the tile's V rows past the context were not loaded (or are stale): zero them so a
      // zero weight times stale shared memory cannot make NaN (only the last tile is ragged;
      // its V copies land first)
      const int valid = ctx - kbase;
      if (valid < 64) {
        if (!__all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&v_full[t % VS]), (t / VS) & 1))) {
          ok = false;
          break;
        }
        uint8_t* vreg = gbase + (v_ring - sbase) + (t % VS) * Cfg::TILE_BYTES;
        for (int idx = tl; idx < (64 - valid) * HALVES * 8; idx += 128) {
          const int rr = valid + idx / (HALVES * 8), rem = idx % (HALVES * 8);
          *reinterpret_cast<uint4*>(vreg + (rem >> 3) * REGION + rr * 128 + ((rem & 7) << 4)) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
      }
      // P row (64 positions) as hi + lo activation-type terms over the S columns just read
      {
        uint32_t hi[32], lo[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float a = sv[2 * e], b = sv[2 * e + 1];
          hi[e] = ActTraits<T>::pack2(a, b);
          const float2 hv = ActTraits<T>::unpack2(hi[e]);
          lo[e] = ActTraits<T>::pack2(a - hv.x, b - hv.y);
        }
        tmem_st32(scol, hi);
        tmem_st32(scol + 32, lo);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(smem_u32(&p_ready[t & 1]));
    }
    if (ok) {
      ok = __all_sync(0xffffffffu, mbar_wait_bounded(smem_u32(&drain), 0));
      tc_fence_after();
    }
    if (!ok) failed = true;
    // O row / l -> output row (fp32, or the activation type)
    const float inv = l_run > 0.f ? __fdiv_rn(1.0f, l_run) : 0.f;
#pragma unroll
    for (int c = 0; c < HD / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(trow + 128 + c * 32, r);
      tmem_wait_ld();
      if (!row_ok || !ok) continue;
      const size_t oi = (static_cast<size_t>(r0 + i) * p.n_heads + head) * HD + c * 32;
      if (p.out_f32) {
        float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + oi);
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          dst[j / 4] = make_float4(__fmul_rn(__uint_as_float(r[j]), inv), __fmul_rn(__uint_as_float(r[j + 1]), inv),
                                   __fmul_rn(__uint_as_float(r[j + 2]), inv), __fmul_rn(__uint_as_float(r[j + 3]), inv));
      } else {
        uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<T*>(p.out) + oi);
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          uint4 v;
          v.x = ActTraits<T>::pack2(__fmul_rn(__uint_as_float(r[j]), inv), __fmul_rn(__uint_as_float(r[j + 1]), inv));
          v.y = ActTraits<T>::pack2(__fmul_rn(__uint_as_float(r[j + 2]), inv), __fmul_rn(__uint_as_float(r[j + 3]), inv));
          v.z = ActTraits<T>::pack2(__fmul_rn(__uint_as_float(r[j + 4]), inv), __fmul_rn(__uint_as_float(r[j + 5]), inv));
          v.w = ActTraits<T>::pack2(__fmul_rn(__uint_as_float(r[j + 6]), inv), __fmul_rn(__uint_as_float(r[j + 7]), inv));
          dst[j / 8] = v;
        }
      }
    }
  }
  if (failed && p.err) atomicExch(p.err, kDevWaitTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::TMEM_COLS);
  }
  trace_end(p.trace);
}

}  // namespace llm
