// umma_persist.cuh -- persistent tcgen05 GEMM for prefill-sized projections.
//
// Same products and epilogues as umma_gemm_kernel (umma.cuh) for the projections of a prefill
// chunk (QKV with QK-norm + RoPE + paged K/V write, residual add, SwiGLU), restated as one CTA
// per SM that walks a static list of 128 x BN output tiles:
//   warp 0       TMA producer: streams every tile's K slices through one STAGES-deep ring
//                without draining between tiles
//   warp 1       TMEM allocator + MMA issuer: accumulates tile i into TMEM buffer i & 1
//   warps 2..17  epilogue: one warp per (TMEM lane quadrant, 32-column chunk); for QKV and
//                SwiGLU two groups of 8 warps, group g draining buffer g (every other tile),
//                for the residual projections one group of 16
// so the epilogue of one tile overlaps the mainloop of the next (and, with two groups, the
// epilogue of the other buffer's tile), and the ring stays full.  Each group's coalesced-store
// staging area is its own shared-memory region (the ring is never idle).
// Per-element arithmetic is that of umma_gemm_kernel, so the outputs are bit-identical.
// Reference: the projections of ane/stories/infer.go:213-262 (forwardLayer) for many rows.
#pragma once
#include "umma.cuh"

namespace llm {

// Named barrier `id` over the NT threads of one epilogue group; the _and form also ANDs a
// predicate across them (a wait that expired on any thread ends the group's tile loop on all
// of its threads together).
template <int NT>
__device__ __forceinline__ void epi_bar_n(int id) {
  asm volatile("bar.sync %0, %1;\n" ::"r"(id), "n"(NT) : "memory");
}
template <int NT>
__device__ __forceinline__ bool epi_bar_and(int id, bool v) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n bar.red.and.pred q, %2, %3, p;\n selp.u32 %0, 1, 0, q;\n}\n"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v)), "r"(id), "n"(NT)
      : "memory");
  return r != 0;
}

template <int BN, int EPI>
struct PersistCfg {
  static constexpr int A_BYTES = kUmmaTokens * 128;
  static constexpr int B_BYTES = BN * 128;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int OUT_COLS = EPI == EPI_SWIGLU ? BN / 2 : BN;
  static constexpr int SP = OUT_COLS + 4;  // staging pitch (floats)
  static constexpr int RP = BN / 2 + 4;    // RoPE staging pitch (floats)
  static constexpr int STG_BYTES = EPI == EPI_QKV ? kUmmaTokens * RP * 4 * 2 : kUmmaTokens * SP * 4;
  // Epilogue groups: with two, group g owns TMEM buffer g (every other tile), so two tiles'
  // epilogues run at once and hide each other's latency; the residual projections (long K,
  // few tiles per SM) keep one group and a deeper ring.
  static constexpr int GROUPS = EPI == EPI_RESID ? 1 : 2;
  static constexpr int NCH = BN / 32;
  // warps per group: one per (TMEM lane quadrant, 32-column chunk), at most 16 / GROUPS (a
  // warp then takes every (GW/4)-th chunk)
  static constexpr int GW = 4 * NCH > 16 / GROUPS ? 16 / GROUPS : 4 * NCH;
  static constexpr int CPW = 4 * NCH / GW;  // chunks per epilogue warp
  static constexpr int GT = 32 * GW;        // threads per group
  static constexpr int EPI_THREADS = GROUPS * GT;
  static constexpr int THREADS = 64 + EPI_THREADS;
  static constexpr int BUDGET = 216 * 1024;  // dynamic shared memory (static arrays need the rest)
  static constexpr int STAGES_RAW = (BUDGET - GROUPS * STG_BYTES - 1024) / STAGE_BYTES;
  static constexpr int STAGES = STAGES_RAW > 8 ? 8 : STAGES_RAW;
  static constexpr int SMEM = STAGES * STAGE_BYTES + GROUPS * STG_BYTES + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulator buffers
  static_assert(STAGES >= 2, "ring too shallow");
  static_assert(TMEM_COLS == 128 || TMEM_COLS == 256 || TMEM_COLS == 512, "TMEM allocation");
};

template <typename InT, typename OutT, int BN, int EPI>
__global__ void __launch_bounds__(PersistCfg<BN, EPI>::THREADS, 1)
    umma_persist_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, GemmParams p) {
  using Cfg = PersistCfg<BN, EPI>;
  static_assert(EPI == EPI_QKV || EPI == EPI_RESID || EPI == EPI_SWIGLU, "prefill epilogues");
  constexpr bool I8 = sizeof(InT) == 1;
  constexpr int STAGES = Cfg::STAGES;
  constexpr int A_BYTES = Cfg::A_BYTES;
  constexpr int STAGE_BYTES = Cfg::STAGE_BYTES;
  constexpr int ESZ = sizeof(InT);
  constexpr int KSTEP_BYTES = 32;
  constexpr int NCH = BN / 32;
  constexpr int GROUPS = Cfg::GROUPS, GT = Cfg::GT;

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[STAGES], empty_bar[STAGES], acc_full[2], acc_empty[2];
  __shared__ uint32_t s_tmem;
  __shared__ float s_bsc[GROUPS][BN];
  __shared__ float s_nw[GROUPS][BN];
  __shared__ double s_ss[GROUPS][EPI == EPI_QKV ? NCH : 1][kUmmaTokens];  // QK-norm partial sums per chunk
  __shared__ int s_rowpage[GROUPS][EPI == EPI_QKV ? kUmmaTokens : 1];      // QKV: a row's K/V page (-1: none)
  __shared__ int s_rowpos[GROUPS][EPI == EPI_QKV ? kUmmaTokens : 1];       // QKV: a row's position

  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  float* const stg = reinterpret_cast<float*>(smem_raw + (sbase - smem_u32(smem_raw)) + STAGES * STAGE_BYTES);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int num_m = (p.M + kUmmaTokens - 1) / kUmmaTokens;
  const int n_tiles = num_m * ((p.N + BN - 1) / BN);
  const int nkt = p.K * ESZ / 128;

  griddep_launch_dependents();
  trace_start(p.trace);
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(smem_u32(&acc_full[b]), 1);
      mbar_init(smem_u32(&acc_empty[b]), GT);  // the threads of the group that drains buffer b
    }
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
  bool failed = false;

  if (warp == 0) {
    // ---------------------------------------------------------------- TMA producer
    if (lane == 0) {
      asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
      asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
      // the first tile's weight slices do not depend on the preceding kernel
      const int first = blockIdx.x;
      const int pre = first < n_tiles ? min(nkt, STAGES) : 0;
      const int ch_first = first < n_tiles ? (first / num_m) * BN : 0;
      for (int i = 0; i < pre; ++i) {
        mbar_arrive_expect_tx(smem_u32(&full_bar[i]), STAGE_BYTES);
        tma_load_2d(sbase + i * STAGE_BYTES + A_BYTES, &tmW, i * (128 / ESZ), ch_first, smem_u32(&full_bar[i]));
      }
      griddep_wait();
      int g = 0;  // k slices issued over all tiles of this CTA
      for (int tile = first; tile < n_tiles && !failed; tile += gridDim.x) {
        const int tok0 = (tile % num_m) * kUmmaTokens, ch0 = (tile / num_m) * BN;
        for (int i = 0; i < nkt; ++i, ++g) {
          const int s = g % STAGES;
          const uint32_t st = sbase + s * STAGE_BYTES;
          const int kx = i * (128 / ESZ);
          if (g < pre) {  // weights already in flight
            tma_load_2d(st, &tmX, kx, tok0, smem_u32(&full_bar[s]));
            continue;
          }
          if (g >= STAGES && !mbar_wait_bounded(smem_u32(&empty_bar[s]), ((g / STAGES) & 1) ^ 1)) {
            failed = true;
            break;
          }
          mbar_arrive_expect_tx(smem_u32(&full_bar[s]), STAGE_BYTES);
          tma_load_2d(st + A_BYTES, &tmW, kx, ch0, smem_u32(&full_bar[s]));
          tma_load_2d(st, &tmX, kx, tok0, smem_u32(&full_bar[s]));
        }
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc<InT>(kUmmaTokens, BN);
      int g = 0, lt = 0;
      for (int tile = blockIdx.x; tile < n_tiles && !failed; tile += gridDim.x, ++lt) {
        const int buf = lt & 1;
        if (lt >= 2 && !mbar_wait_bounded(smem_u32(&acc_empty[buf]), ((lt >> 1) & 1) ^ 1)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + buf * BN;
        for (int i = 0; i < nkt; ++i, ++g) {
          const int s = g % STAGES;
          if (!mbar_wait_bounded(smem_u32(&full_bar[s]), (g / STAGES) & 1)) {
            failed = true;
            break;
          }
          tc_fence_after();
          const uint32_t a = sbase + s * STAGE_BYTES, b = a + A_BYTES;
#pragma unroll
          for (int k = 0; k < 128 / KSTEP_BYTES; ++k)
            umma<I8>(acc, sw128_desc(a + k * KSTEP_BYTES), sw128_desc(b + k * KSTEP_BYTES), idesc,
                     (i > 0 || k > 0) ? 1u : 0u);
          tc_commit(smem_u32(&empty_bar[s]));
        }
        if (failed) break;
        tc_commit(smem_u32(&acc_full[buf]));
      }
    }
  } else {
    // ---------------------------------------------------------------- epilogue
    // Epilogue warp ew = warp - 2 belongs to group g = ew / GW, which takes tiles lt = g, g +
    // GROUPS, ... (TMEM buffer lt & 1).  Warp w reads TMEM lanes 32 * (w % 4) .. + 31 (its
    // quadrant) and chunks cb, cb + GW/4, ... (cb = (ew % GW) / 4).
    constexpr int GW = Cfg::GW, CPW = Cfg::CPW;
    const int ew = warp - 2;
    const int g = ew / GW;
    const int q = warp & 3;
    const int cb = (ew % GW) >> 2;       // first 32-column chunk of this warp
    const int gt = threadIdx.x - 64 - g * GT;  // 0 .. GT-1 within the group
    const int tl = q * 32 + lane;        // token within the tile (= TMEM lane)
    const int bar_id = 1 + g;
    float* const gstg = stg + g * (Cfg::STG_BYTES / 4);
    float* const bsc = s_bsc[g];
    float* const nwv = s_nw[g];
    griddep_wait();  // positions, scales and the residual come from earlier kernels
    for (int tile = blockIdx.x + g * gridDim.x, lt = g; tile < n_tiles; tile += GROUPS * gridDim.x, lt += GROUPS) {
      const int buf = lt & 1;
      const int tok0 = (tile % num_m) * kUmmaTokens, ch0 = (tile / num_m) * BN;
      const int tok = tok0 + tl;
      const bool tok_ok = tok < p.M;
      const int tokc = tok_ok ? tok : p.M - 1;
      const uint32_t tcol = tmem + buf * BN + (static_cast<uint32_t>(q * 32) << 16);  // + 32 * chunk

      epi_bar_n<GT>(bar_id);  // the group's previous tile's readers of its shared arrays are done
      float a_s = 1.0f;
      if constexpr (I8) a_s = p.a_scale[tokc];
      for (int j = gt; j < BN; j += GT) {
        const int ch = ch0 + j;
        if constexpr (I8) bsc[j] = ch < p.N ? p.b_scale[ch] : 0.0f;
      }
      int region = 0, head = 0, pos = 0, page = 0;
      if constexpr (EPI == EPI_QKV) {
        const int hd = p.head_dim;  // == BN
        const int q_dim = p.n_heads * hd, kv_dim = p.n_kv_heads * hd;
        if (ch0 < q_dim) { region = 0; head = ch0 / hd; }
        else if (ch0 < q_dim + kv_dim) { region = 1; head = (ch0 - q_dim) / hd; }
        else { region = 2; head = (ch0 - q_dim - kv_dim) / hd; }
        if (tok_ok) {
          pos = p.positions[tok];
          if (region > 0) page = p.block_table[static_cast<size_t>(p.seq_ids[tok]) * p.max_pages_per_seq + (pos >> 4)];
        }
        if (region < 2 && p.qk_norm) {
          const float* nw = region == 0 ? p.q_norm : p.k_norm;
          for (int j = gt; j < BN; j += GT) nwv[j] = nw[j];
        }
        if (region < 2) {
          // the tile's RoPE rows, coalesced: cos at gstg[row * RP], sin at gstg[(128 + row) * RP]
          constexpr int RP = Cfg::RP, H4 = BN / 8;  // float4 per half-row
#pragma unroll 4
          for (int idx = gt; idx < kUmmaTokens * H4; idx += GT) {
            const int row = idx / H4, c4 = idx % H4;
            const int t = min(tok0 + row, p.M - 1);
            const size_t off = static_cast<size_t>(p.positions[t]) * (BN / 2) + 4 * c4;
            *reinterpret_cast<float4*>(gstg + row * RP + 4 * c4) = *reinterpret_cast<const float4*>(p.rope_cos + off);
            *reinterpret_cast<float4*>(gstg + (kUmmaTokens + row) * RP + 4 * c4) =
                *reinterpret_cast<const float4*>(p.rope_sin + off);
          }
        }
      }
      // the residual does not depend on this GEMM: its loads overlap the wait for the accumulator
      constexpr int RPT = kUmmaTokens * (BN / 4) / GT;  // residual float4 per thread
      float4 rpre[EPI == EPI_RESID ? RPT : 1];
      if constexpr (EPI == EPI_RESID) {
#pragma unroll
        for (int u = 0; u < RPT; ++u) {
          const int idx = gt + u * GT;
          const int row = idx / (BN / 4), col = 4 * (idx % (BN / 4));
          const int t = tok0 + row, ch = ch0 + col;
          rpre[u] = (t < p.M && ch < p.N) ? *reinterpret_cast<const float4*>(p.resid + static_cast<size_t>(t) * p.ldo + ch)
                                          : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      const bool ok = epi_bar_and<GT>(bar_id, mbar_wait_bounded(smem_u32(&acc_full[buf]), (lt >> 1) & 1));
      if (!ok) failed = true;
      tc_fence_after();
      // this warp's chunks, dequantised (the tile's scales / norm weights / RoPE rows are
      // visible: the barrier above also orders them)
      float vv[CPW][32];
#pragma unroll
      for (int w = 0; w < CPW; ++w) {
        const int cc = cb + w * (GW / 4);
        uint32_t r[32];
        tmem_ld32(tcol + cc * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          if constexpr (I8) vv[w][j] = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[j])), a_s), bsc[cc * 32 + j]);
          else vv[w][j] = __uint_as_float(r[j]);
          if (!ok) vv[w][j] = 0.f;
        }
      }
      // the accumulator buffer is free for the MMAs of tile lt + 2 once every chunk is read
      tc_fence_before();
      mbar_arrive(smem_u32(&acc_empty[buf]));
      constexpr int SP = Cfg::SP;

      if constexpr (EPI == EPI_RESID) {
#pragma unroll
        for (int w = 0; w < CPW; ++w) {
          const int cc = cb + w * (GW / 4);
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<float4*>(gstg + tl * SP + cc * 32 + j) = make_float4(vv[w][j], vv[w][j + 1], vv[w][j + 2], vv[w][j + 3]);
        }
        epi_bar_n<GT>(bar_id);
        // out may alias resid (in-place residual): each element is read (above, before the
        // accumulator) and written by one thread
        constexpr int C4 = BN / 4;
#pragma unroll
        for (int u = 0; u < RPT; ++u) {
          const int idx = gt + u * GT;
          const int row = idx / C4, col = 4 * (idx % C4);
          const int t = tok0 + row, ch = ch0 + col;
          if (t >= p.M || ch >= p.N) continue;
          const float4 y = *reinterpret_cast<const float4*>(gstg + row * SP + col);
          *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + static_cast<size_t>(t) * p.ldo + ch) =
              make_float4(resid_add(y.x, rpre[u].x, p.resid_scale), resid_add(y.y, rpre[u].y, p.resid_scale),
                          resid_add(y.z, rpre[u].z, p.resid_scale), resid_add(y.w, rpre[u].w, p.resid_scale));
        }
      } else if constexpr (EPI == EPI_SWIGLU) {
#pragma unroll
        for (int w = 0; w < CPW; ++w) {
          const int cc = cb + w * (GW / 4);
          float gg[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) gg[i] = swiglu_pair(vv[w][2 * i], vv[w][2 * i + 1], p.silu_form);
#pragma unroll
          for (int i = 0; i < 16; i += 4)
            *reinterpret_cast<float4*>(gstg + tl * SP + cc * 16 + i) = make_float4(gg[i], gg[i + 1], gg[i + 2], gg[i + 3]);
        }
        epi_bar_n<GT>(bar_id);
        constexpr int OUT_COLS = Cfg::OUT_COLS;
        const int F = p.N / 2, j0 = ch0 / 2;
        if (p.swiglu_f32) {
          constexpr int C4 = OUT_COLS / 4;
          for (int idx = gt; idx < kUmmaTokens * C4; idx += GT) {
            const int row = idx / C4, col = 4 * (idx % C4);
            const int t = tok0 + row;
            if (t >= p.M || j0 + col >= F) continue;
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + static_cast<size_t>(t) * F + j0 + col) =
                *reinterpret_cast<const float4*>(gstg + row * SP + col);
          }
        } else {
          constexpr int C8 = OUT_COLS / 8;
          for (int idx = gt; idx < kUmmaTokens * C8; idx += GT) {
            const int row = idx / C8, col = 8 * (idx % C8);
            const int t = tok0 + row;
            if (t >= p.M || j0 + col >= F) continue;
            const float4 a = *reinterpret_cast<const float4*>(gstg + row * SP + col);
            const float4 b = *reinterpret_cast<const float4*>(gstg + row * SP + col + 4);
            uint4 pk;
            pk.x = ActTraits<OutT>::pack2(a.x, a.y);
            pk.y = ActTraits<OutT>::pack2(a.z, a.w);
            pk.z = ActTraits<OutT>::pack2(b.x, b.y);
            pk.w = ActTraits<OutT>::pack2(b.z, b.w);
            *reinterpret_cast<uint4*>(reinterpret_cast<OutT*>(p.out) + static_cast<size_t>(t) * F + j0 + col) = pk;
          }
        }
      } else {  // EPI_QKV: one head per tile (BN == head_dim)
        constexpr int hd = BN;
        constexpr int RP = Cfg::RP;
        float rr = 1.0f;
        if (region < 2 && p.qk_norm) {
          // sum of squares in f64: per chunk in order, then the chunks in order
#pragma unroll
          for (int w = 0; w < CPW; ++w) {
            double sc = 0.0;
#pragma unroll
            for (int j = 0; j < 32; ++j) sc = __dadd_rn(sc, __dmul_rn((double)vv[w][j], (double)vv[w][j]));
            s_ss[g][cb + w * (GW / 4)][tl] = sc;
          }
          epi_bar_n<GT>(bar_id);
          double ss = s_ss[g][0][tl];
#pragma unroll
          for (int cc = 1; cc < NCH; ++cc) ss = __dadd_rn(ss, s_ss[g][cc][tl]);
          rr = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)hd), p.eps))));
        }
        if (region > 0 && tok_ok && !(page >= 0 && page < p.n_pages) && cb == 0 && p.err) atomicExch(p.err, kDevBadPage);
        uint4 pk[CPW][4];
#pragma unroll
        for (int w = 0; w < CPW; ++w) {
          float (&v)[32] = vv[w];
          const int d0 = (cb + w * (GW / 4)) * 32;  // first head dimension of the chunk
          if (region < 2) {
            if (p.qk_norm) {
#pragma unroll
              for (int j = 0; j < 32; ++j) v[j] = __fmul_rn(__fmul_rn(v[j], rr), nwv[d0 + j]);
            }
            float cs[16], sn[16];
#pragma unroll
            for (int i = 0; i < 16; i += 4) {
              const float4 a = *reinterpret_cast<const float4*>(gstg + tl * RP + d0 / 2 + i);
              const float4 b = *reinterpret_cast<const float4*>(gstg + (kUmmaTokens + tl) * RP + d0 / 2 + i);
              cs[i] = a.x; cs[i + 1] = a.y; cs[i + 2] = a.z; cs[i + 3] = a.w;
              sn[i] = b.x; sn[i + 1] = b.y; sn[i + 2] = b.z; sn[i + 3] = b.w;
            }
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float a0 = v[2 * i], a1 = v[2 * i + 1];
              v[2 * i] = __fsub_rn(__fmul_rn(a0, cs[i]), __fmul_rn(a1, sn[i]));
              v[2 * i + 1] = __fadd_rn(__fmul_rn(a0, sn[i]), __fmul_rn(a1, cs[i]));
            }
          }
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            pk[w][h].x = ActTraits<OutT>::pack2(v[8 * h + 0], v[8 * h + 1]);
            pk[w][h].y = ActTraits<OutT>::pack2(v[8 * h + 2], v[8 * h + 3]);
            pk[w][h].z = ActTraits<OutT>::pack2(v[8 * h + 4], v[8 * h + 5]);
            pk[w][h].w = ActTraits<OutT>::pack2(v[8 * h + 6], v[8 * h + 7]);
          }
        }
        // Coalesced stores: the tile's packed rows go through the group's staging area (its RoPE
        // rows are no longer read once every thread has passed this barrier), then 16-byte
        // pieces of each row are stored by consecutive threads, to q or to the row's K/V page.
        constexpr int OP = BN * 2 + 16;  // staged row pitch (bytes): 16 B bank offset per row
        constexpr int U = BN * 2 / 16;   // 16-byte pieces per row
        uint8_t* const ost = reinterpret_cast<uint8_t*>(gstg);
        epi_bar_n<GT>(bar_id);
#pragma unroll
        for (int w = 0; w < CPW; ++w) {
          const int d0 = (cb + w * (GW / 4)) * 32;
#pragma unroll
          for (int h = 0; h < 4; ++h) *reinterpret_cast<uint4*>(ost + tl * OP + d0 * 2 + h * 16) = pk[w][h];
        }
        if (cb == 0) {  // the warps of chunk 0 cover all 128 rows
          s_rowpage[g][tl] = (region > 0 && tok_ok && page >= 0 && page < p.n_pages) ? page : -1;
          s_rowpos[g][tl] = pos;
        }
        epi_bar_n<GT>(bar_id);
        for (int idx = gt; idx < kUmmaTokens * U; idx += GT) {
          const int row = idx / U, cu = idx % U;
          const int t = tok0 + row;
          if (t >= p.M) continue;
          const uint4 val = *reinterpret_cast<const uint4*>(ost + row * OP + cu * 16);
          if (region == 0) {
            *reinterpret_cast<uint4*>(reinterpret_cast<OutT*>(p.q_out) + (static_cast<size_t>(t) * p.n_heads + head) * hd + cu * 8) = val;
          } else {
            const int pg = s_rowpage[g][row];
            if (pg < 0) continue;
            const size_t blk = ((static_cast<size_t>(p.layer) * p.n_pages + pg) * p.n_kv_heads + head) * 2 + (region - 1);
            uint8_t* kv_base = reinterpret_cast<uint8_t*>(reinterpret_cast<OutT*>(p.kv_pool) + blk * 16 * hd);
            *reinterpret_cast<uint4*>(kv_base + kv_off(s_rowpos[g][row] & 15, cu)) = val;
          }
        }
      }
      if (!ok) break;
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
