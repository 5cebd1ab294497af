// gemm.cuh -- projection GEMMs of the token loop with fused epilogues.
//
//   C[M x N] = A[M x K] . B[N x K]^T
//   A = activations (row-major, K contiguous; bf16/fp16, or int8 with per-row scales)
//   B = weights in the reference's [out, in] row-major layout (ane/stories/weights.go:13-17)
//
// One CTA (8 warps, 2 x 4) computes a BM x BN tile; K is streamed in 128-byte slices
// through a STAGES-deep cp.async ring with an XOR swizzle so ldmatrix is conflict-free.
// 16-bit inputs use mma.m16n8k16 (f32 accumulate); int8 uses mma.m16n8k32 (s32
// accumulate, exact).  The byte layout of a k-step is the same for both, so one data path
// serves both element types.
//
// Split-K is deterministic: every split writes its partial tile to a workspace in a
// per-thread fragment order, the last CTA to arrive (per-tile counter) sums the partials in
// split order, resets the counter and runs the epilogue.
//
// Epilogues (reference operation they fuse, ane/stories/infer.go):
//   EPI_F32     store fp32 (logits / debug)
//   EPI_S32     store the raw int32 accumulators (bit-exact int8 GEMM check)
//   EPI_RESID   out = resid + y                       (:225-228, :236-239)
//               or resid + a * y (ane/storiesane/residual.go:9, a = 1/sqrt(2 * layers))
//   EPI_SWIGLU  g_j = silu(h1_j) * h3_j on interleaved W1/W3 rows   (:231-235)
//               or (h1 * sigmoid(h1)) * h3 (ane/storiesane/accel_other.go:66-71)
//   EPI_QKV     per-head QK-norm, RoPE (:222, :247-265), q store, paged K/V write (:223)
//   EPI_ARGMAX  per-row (max, first index) partial per N tile for the greedy token (:373-383)
#pragma once
#include "common.cuh"

namespace llm {

enum EpiKind : int { EPI_F32 = 0, EPI_S32 = 1, EPI_RESID = 2, EPI_SWIGLU = 3, EPI_QKV = 4, EPI_ARGMAX = 5 };

struct GemmParams {
  const void* A;
  const void* B;
  int M, N, K;                 // K in elements
  int k_splits;                // >= 1
  int k_tiles_per_split;
  float* ws;                   // split-K workspace (fp32 or int32 bit patterns)
  int* counters;               // per output tile, zero between launches
  const float* a_scale;        // [M] int8 dequant
  const float* b_scale;        // [N] int8 dequant
  // EPI_F32 / EPI_S32 / EPI_RESID
  void* out;
  int ldo;
  const float* resid;
  // EPI_SWIGLU: g [M][N/2] act type, or fp32 when swiglu_f32
  int swiglu_f32;
  // EPI_QKV
  void* q_out;                 // [M][n_heads][head_dim] act type
  void* kv_pool;               // [layer][page][kv_head][2][16][head_dim] act type (swizzled rows)
  const int* block_table;      // [max_seqs][max_pages_per_seq]
  const int* seq_ids;          // [M]
  const int* positions;        // [M]
  const float* q_norm;         // [head_dim] or nullptr
  const float* k_norm;
  const float* rope_cos;       // [max_pos][head_dim/2]
  const float* rope_sin;
  int layer, n_pages, max_pages_per_seq, n_heads, n_kv_heads, head_dim, qk_norm;
  double eps;
  // EPI_ARGMAX
  unsigned long long* argmax_part;  // [M][argmax_parts]: one (value, index) key per channel tile
  int argmax_parts;
  float* logits;                    // optional [M][ld_logits]
  int ld_logits;
  int* err;
  // tcgen05 GEMM: stage-ring depth (0 = the kernel's maximum); fewer stages need less shared
  // memory, which lets a GEMM CTA share an SM with an attention CTA
  int stages;
  // tcgen05 QKV: token rows per tile (64 or 0 = 128)
  int a_rows;
  TraceRec* trace;  // llm_trace_step (tcgen05 GEMM only)
  // storiesane arithmetic (ane/storiesane/residual.go:9, accel_other.go:60-71):
  // EPI_RESID out = resid + resid_scale * y when resid_scale != 0 (0 = out = y + resid);
  // EPI_SWIGLU silu_form 1 = (h1 * f32(1 / (1 + exp(-h1)))) * h3 (0 = h1 / (1 + exp(-h1)) * h3)
  float resid_scale;
  int silu_form;
};

// SiLU gate of one (h1, h3) pair in the selected form (see GemmParams::silu_form), built from
// IEEE round-to-nearest steps only so that the CPU oracle restates it bit for bit:
// e = exp(-h1) as exp2_det(-h1 * f32(log2 e)); form 0 (stories.Decoder's silu, infer.go:324-326)
// h1 / (1 + e) * h3, form 1 (storiesane, accel_other.go:66-71) (h1 * (1 / (1 + e))) * h3.
__device__ __forceinline__ float swiglu_pair(float h1, float up, int form) {
  const float e = exp2_det(__fmul_rn(h1, -1.4426950408889634f));
  const float d = __fadd_rn(1.0f, e);
  if (form == 0) return __fmul_rn(__fdiv_rn(h1, d), up);
  return __fmul_rn(__fmul_rn(h1, __fdiv_rn(1.0f, d)), up);
}
// Residual update of one element (see GemmParams::resid_scale).
__device__ __forceinline__ float resid_add(float y, float r, float scale) {
  return scale == 0.0f ? __fadd_rn(y, r) : __fadd_rn(r, __fmul_rn(scale, y));
}

template <typename InT> struct GemmAcc { using type = float; };
template <> struct GemmAcc<int8_t> { using type = int; };

constexpr int kGemmThreads = 256;

template <int BM, int BN, int STAGES>
constexpr int gemm_smem_bytes() {
  return STAGES * (BM + BN) * 128;
}

template <typename InT, typename OutT, int BM, int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(kGemmThreads) gemm_kernel(GemmParams p) {
  using Acc = typename GemmAcc<InT>::type;
  constexpr int WARPS_M = 2, WARPS_N = 4;
  constexpr int WTM = BM / WARPS_M, WTN = BN / WARPS_N;
  constexpr int MT = WTM / 16, NT = WTN / 8;
  static_assert(NT % 2 == 0, "n tiles are loaded in pairs");
  constexpr int ESZ = sizeof(InT);
  constexpr int BK = 128 / ESZ;  // elements per 128-byte k slice
  constexpr int STAGE_BYTES = (BM + BN) * 128;
  constexpr int CHUNKS = (BM + BN) * 8;
  static_assert(CHUNKS % kGemmThreads == 0, "tile chunks must divide the CTA");

  extern __shared__ __align__(1024) uint8_t smem[];
  griddep_launch_dependents();
  griddep_wait();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = warp / WARPS_N, wn = warp % WARPS_N;
  const int m_tile = blockIdx.x, n_tile = blockIdx.y, split = blockIdx.z;
  const int m0 = m_tile * BM, n0 = n_tile * BN;
  const int k_tiles = p.K / BK;
  const int kt_begin = split * p.k_tiles_per_split;
  const int kt_end = min(k_tiles, kt_begin + p.k_tiles_per_split);
  const int nkt = max(0, kt_end - kt_begin);
  const size_t row_bytes = static_cast<size_t>(p.K) * ESZ;
  const uint8_t* Ab = reinterpret_cast<const uint8_t*>(p.A);
  const uint8_t* Bb = reinterpret_cast<const uint8_t*>(p.B);
  const uint32_t sbase = smem_u32(smem);

  auto load_stage = [&](int stage, int kt) {
    const uint32_t st = sbase + stage * STAGE_BYTES;
    const size_t kbyte = static_cast<size_t>(kt) * 128;
#pragma unroll
    for (int i = 0; i < CHUNKS / kGemmThreads; ++i) {
      const int c = tid + i * kGemmThreads;
      const int r = c >> 3, ch = c & 7;
      if (r < BM) {
        const int gm = m0 + r;
        const bool ok = gm < p.M;
        const uint8_t* src = Ab + (ok ? gm * row_bytes + kbyte + ch * 16 : 0);
        cp_async_16(st + swz(r, ch, 128), src, ok ? 16 : 0);
      } else {
        const int rb = r - BM;
        const int gn = n0 + rb;
        const bool ok = gn < p.N;
        const uint8_t* src = Bb + (ok ? gn * row_bytes + kbyte + ch * 16 : 0);
        cp_async_16(st + BM * 128 + swz(rb, ch, 128), src, ok ? 16 : 0);
      }
    }
  };

  Acc acc[MT][NT][4];
#pragma unroll
  for (int a = 0; a < MT; ++a)
#pragma unroll
    for (int b = 0; b < NT; ++b)
#pragma unroll
      for (int c = 0; c < 4; ++c) acc[a][b][c] = 0;

#pragma unroll
  for (int s = 0; s < STAGES - 1; ++s) {
    if (s < nkt) load_stage(s, kt_begin + s);
    cp_async_commit();
  }

  for (int it = 0; it < nkt; ++it) {
    cp_async_wait<STAGES - 2>();
    __syncthreads();
    {
      const int nxt = it + STAGES - 1;
      if (nxt < nkt) load_stage(nxt % STAGES, kt_begin + nxt);
      cp_async_commit();
    }
    const uint32_t sA = sbase + (it % STAGES) * STAGE_BYTES;
    const uint32_t sB = sA + BM * 128;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t af[MT][4];
      uint32_t bf[NT][2];
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int r = wm * WTM + mt * 16 + (lane & 7) + 8 * ((lane >> 3) & 1);
        ldmatrix_x4(af[mt], sA + swz(r, 2 * kk + (lane >> 4), 128));
      }
#pragma unroll
      for (int np = 0; np < NT / 2; ++np) {
        const int r = wn * WTN + np * 16 + (lane & 7) + 8 * (lane >> 4);
        uint32_t t4[4];
        ldmatrix_x4(t4, sB + swz(r, 2 * kk + ((lane >> 3) & 1), 128));
        bf[2 * np][0] = t4[0];
        bf[2 * np][1] = t4[1];
        bf[2 * np + 1][0] = t4[2];
        bf[2 * np + 1][1] = t4[3];
      }
#pragma unroll
      for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          if constexpr (ESZ == 1) {
            mma_16832_s8(acc[mt][nt], af[mt], bf[nt][0], bf[nt][1]);
          } else {
            mma_16816(acc[mt][nt], af[mt], bf[nt][0], bf[nt][1], InT());
          }
        }
    }
  }
  cp_async_wait<0>();
  __syncthreads();

  // ------------------------------------------------------------------ split-K reduction
  if (p.k_splits > 1) {
    const int tiles = gridDim.x * gridDim.y;
    const int tile = n_tile * gridDim.x + m_tile;
    constexpr int PER = MT * NT * 4;
    float* wsb = p.ws + (static_cast<size_t>(split) * tiles + tile) * (BM * BN);
    int j = 0;
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
      for (int b = 0; b < NT; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c, ++j) {
          float v;
          if constexpr (ESZ == 1) v = __int_as_float(acc[a][b][c]);
          else v = acc[a][b][c];
          __stcg(wsb + j * kGemmThreads + tid, v);
        }
    __threadfence();
    __syncthreads();
    __shared__ int s_last;
    if (tid == 0) {
      const int prev = atomicAdd(p.counters + tile, 1);
      s_last = (prev == p.k_splits - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    (void)PER;
    // Sum the partials split-major so every thread keeps PER independent loads in flight
    // (a split-minor loop would serialise one L2 round trip per split and element).
#pragma unroll
    for (int a = 0; a < MT; ++a)
#pragma unroll
      for (int b = 0; b < NT; ++b)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[a][b][c] = 0;
    for (int s = 0; s < p.k_splits; ++s) {
      const float* src = p.ws + (static_cast<size_t>(s) * tiles + tile) * (BM * BN) + tid;
      j = 0;
#pragma unroll
      for (int a = 0; a < MT; ++a)
#pragma unroll
        for (int b = 0; b < NT; ++b)
#pragma unroll
          for (int c = 0; c < 4; ++c, ++j) {
            const float v = __ldcg(src + j * kGemmThreads);
            if constexpr (ESZ == 1) acc[a][b][c] += __float_as_int(v);
            else acc[a][b][c] = __fadd_rn(acc[a][b][c], v);
          }
    }
    if (tid == 0) p.counters[tile] = 0;
  }

  // ------------------------------------------------------------------ epilogues
  const int g = lane >> 2, t = lane & 3;
  auto row_of = [&](int mt, int c) { return m0 + wm * WTM + mt * 16 + g + (c >= 2 ? 8 : 0); };
  auto col_of = [&](int nt, int c) { return n0 + wn * WTN + nt * 8 + 2 * t + (c & 1); };
  auto value = [&](int mt, int nt, int c) -> float {
    if constexpr (ESZ == 1) {
      const int r = row_of(mt, c), cl = col_of(nt, c);
      const float sa = r < p.M ? p.a_scale[r] : 0.0f;
      const float sb = cl < p.N ? p.b_scale[cl] : 0.0f;
      return __fmul_rn(__fmul_rn(__int2float_rn(acc[mt][nt][c]), sa), sb);
    } else {
      return acc[mt][nt][c];
    }
  };

  if constexpr (EPI == EPI_S32) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int r = row_of(mt, c), cl = col_of(nt, c);
          if (r < p.M && cl < p.N) {
            int v;
            if constexpr (ESZ == 1) v = acc[mt][nt][c];
            else v = __float2int_rn(acc[mt][nt][c]);
            reinterpret_cast<int*>(p.out)[static_cast<size_t>(r) * p.ldo + cl] = v;
          }
        }
  } else if constexpr (EPI == EPI_F32 || EPI == EPI_RESID) {
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = row_of(mt, 2 * h), cl = col_of(nt, 0);
          if (r >= p.M) continue;
          float v0 = value(mt, nt, 2 * h), v1 = value(mt, nt, 2 * h + 1);
          float* o = reinterpret_cast<float*>(p.out) + static_cast<size_t>(r) * p.ldo + cl;
          if constexpr (EPI == EPI_RESID) {
            const float* rs = p.resid + static_cast<size_t>(r) * p.ldo + cl;
            if (cl + 1 < p.N) {
              float2 rv = *reinterpret_cast<const float2*>(rs);
              *reinterpret_cast<float2*>(o) =
                  make_float2(resid_add(v0, rv.x, p.resid_scale), resid_add(v1, rv.y, p.resid_scale));
            } else if (cl < p.N) {
              o[0] = resid_add(v0, rs[0], p.resid_scale);
            }
          } else {
            if (cl < p.N) o[0] = v0;
            if (cl + 1 < p.N) o[1] = v1;
          }
        }
  } else if constexpr (EPI == EPI_SWIGLU) {
    const int F = p.N / 2;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = row_of(mt, 2 * h), cl = col_of(nt, 0);
          if (r >= p.M || cl >= p.N) continue;
          const float h1 = value(mt, nt, 2 * h), h3 = value(mt, nt, 2 * h + 1);
          const float gv = swiglu_pair(h1, h3, p.silu_form);
          const size_t idx = static_cast<size_t>(r) * F + (cl >> 1);
          if (p.swiglu_f32) reinterpret_cast<float*>(p.out)[idx] = gv;
          else reinterpret_cast<OutT*>(p.out)[idx] = ActTraits<OutT>::from_f(gv);
        }
  } else if constexpr (EPI == EPI_ARGMAX) {
    // per-row best over this thread's columns, then over the 4 lanes of a row group,
    // then over the WARPS_N warps through shared memory.
    __shared__ unsigned long long s_best[WARPS_N][BM];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int r = row_of(mt, 2 * h);
        unsigned long long best = 0ull;
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const int cl = col_of(nt, c);
            if (cl < p.N && r < p.M) {
              const float v = value(mt, nt, 2 * h + c);
              if (p.logits) p.logits[static_cast<size_t>(r) * p.ld_logits + cl] = v;
              const unsigned long long k = argmax_key(v, cl);
              best = k > best ? k : best;
            }
          }
#pragma unroll
        for (int o = 1; o <= 2; o <<= 1) {
          const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
          best = other > best ? other : best;
        }
        if (t == 0) s_best[wn][wm * WTM + mt * 16 + g + 8 * h] = best;
      }
    __syncthreads();
    for (int r = tid; r < BM; r += kGemmThreads) {
      unsigned long long best = s_best[0][r];
#pragma unroll
      for (int w = 1; w < WARPS_N; ++w) best = s_best[w][r] > best ? s_best[w][r] : best;
      if (m0 + r < p.M) p.argmax_part[static_cast<size_t>(m0 + r) * p.argmax_parts + n_tile] = best;
    }
  } else if constexpr (EPI == EPI_QKV) {
    // Stage the dequantised tile in shared memory, then process whole heads per row.
    constexpr int LDS = BN + 4;
    float* sC = reinterpret_cast<float*>(smem);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int rl = wm * WTM + mt * 16 + g + (c >= 2 ? 8 : 0);
          const int cl = wn * WTN + nt * 8 + 2 * t + (c & 1);
          sC[rl * LDS + cl] = value(mt, nt, c);
        }
    // per-row position and physical KV page, resolved once per tile (one thread per row)
    // so the head jobs below carry no dependent global-load chains
    __shared__ int s_pos[BM], s_page[BM];
    for (int rl = tid; rl < BM; rl += kGemmThreads) {
      const int r = m0 + rl;
      int pos = 0, page = 0;
      if (r < p.M) {
        pos = p.positions[r];
        page = p.block_table[static_cast<size_t>(p.seq_ids[r]) * p.max_pages_per_seq + (pos >> 4)];
      }
      s_pos[rl] = pos;
      s_page[rl] = page;
    }
    __syncthreads();
    const int hd = p.head_dim;
    const int E = hd / 32;  // values per lane (2 or 4)
    const int q_dim = p.n_heads * hd, kv_dim = p.n_kv_heads * hd;
    const int heads_in_tile = BN / hd;
    for (int job = warp; job < BM * heads_in_tile; job += kGemmThreads / 32) {
      const int rl = job / heads_in_tile, hh = job % heads_in_tile;
      const int r = m0 + rl;
      const int col0 = n0 + hh * hd;
      if (r >= p.M || col0 >= p.N) continue;
      int region, head;
      if (col0 < q_dim) { region = 0; head = col0 / hd; }
      else if (col0 < q_dim + kv_dim) { region = 1; head = (col0 - q_dim) / hd; }
      else { region = 2; head = (col0 - q_dim - kv_dim) / hd; }
      float v[4];
      const int d0 = lane * E;
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (e < E) v[e] = sC[rl * LDS + hh * hd + d0 + e];
      const int pos = s_pos[rl];
      if (region < 2) {
        if (p.qk_norm) {
          const float* nw = region == 0 ? p.q_norm : p.k_norm;
          double a = 0.0;
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (e < E) a = __dadd_rn(a, __dmul_rn((double)v[e], (double)v[e]));
          const double tot = warp_sum_f64(a);
          const float rr = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(tot, (double)hd), p.eps))));
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (e < E) v[e] = __fmul_rn(__fmul_rn(v[e], rr), nw[d0 + e]);
        }
        const float* cs = p.rope_cos + static_cast<size_t>(pos) * (hd / 2);
        const float* sn = p.rope_sin + static_cast<size_t>(pos) * (hd / 2);
#pragma unroll
        for (int e = 0; e < 4; e += 2)
          if (e < E) {
            const int i = (d0 + e) >> 1;
            const float c = cs[i], s = sn[i];
            const float a0 = v[e], a1 = v[e + 1];
            v[e] = __fsub_rn(__fmul_rn(a0, c), __fmul_rn(a1, s));
            v[e + 1] = __fadd_rn(__fmul_rn(a0, s), __fmul_rn(a1, c));
          }
      }
      if (region == 0) {
        OutT* qo = reinterpret_cast<OutT*>(p.q_out) + (static_cast<size_t>(r) * p.n_heads + head) * hd + d0;
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (e < E) qo[e] = ActTraits<OutT>::from_f(v[e]);
      } else {
        const int page = s_page[rl];
        if (page < 0 || page >= p.n_pages) {
          if (p.err) atomicExch(p.err, kDevBadPage);
          continue;
        }
        const int slot = pos & 15;
        const size_t blk = ((static_cast<size_t>(p.layer) * p.n_pages + page) * p.n_kv_heads + head) * 2 + (region - 1);
        OutT* base = reinterpret_cast<OutT*>(p.kv_pool) + blk * 16 * hd;
        // element d of row `slot` lives in chunk d/8 placed by kv_off (common.cuh)
        OutT* dst = reinterpret_cast<OutT*>(reinterpret_cast<uint8_t*>(base) + kv_off(slot, d0 >> 3)) + (d0 & 7);
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (e < E) dst[e] = ActTraits<OutT>::from_f(v[e]);
      }
    }
  }
}

}  // namespace llm
