// umma.cuh -- tcgen05 (5th-generation tensor core) GEMM for the token loop's projections.
//
//   D[n, m] = sum_k W[n, k] * X[m, k]     (W = weights [N_out x K], X = activations [M x K])
//
// The weight tile is the UMMA "A" operand (M_umma = 128 output channels) and the token tile
// the "B" operand (N_umma = BT tokens, up to 256), so at decode one CTA covers every token
// of the step and each weight byte is streamed from HBM once.  Both operands are K-major
// 128-byte-swizzled tiles written by TMA (cp.async.bulk.tensor, no multicast); the fp32/s32
// accumulator lives in tensor memory.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM allocator + MMA issuer
// (one elected thread), warps 2..5 = epilogue.  Epilogue warp w reads TMEM lanes
// 32*(w%4)..+31, i.e. thread = output channel, and walks the token columns 32 at a time.
// A STAGES-deep ring of (full, empty) mbarriers connects producer and MMA; tcgen05.commit
// releases a stage when its MMAs have consumed it and signals the epilogue after the last.
// Every mbarrier wait is bounded: on expiry the kernel records kDevWaitTimeout, skips the
// remaining work and still reaches the TMEM deallocation.
//
// Split-K (residual epilogue only, p.k_splits > 1): the splits of one output tile are one
// thread-block cluster along z.  Each CTA parks its partial accumulator tile in its own (now
// idle) stage memory; after a cluster barrier CTA rank r sums token slice r of all ranks'
// partials through distributed shared memory, in rank order, and runs the epilogue on it; a
// second cluster barrier keeps every CTA's shared memory alive until its peers are done.
#pragma once
#include <cuda.h>

#include "common.cuh"
#include "gemm.cuh"

namespace llm {

// ----------------------------------------------------------------------------- PTX wrappers
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void tmem_alloc(uint32_t smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_dst), "r"(ncols));
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar) : "memory");
}
template <bool I8>
__device__ __forceinline__ void umma(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  if constexpr (I8) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
  } else {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc));
  }
}
// 32 lanes x 32 columns of 32-bit: thread t receives columns col..col+31 of lane (base lane + t)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;\n" ::: "memory"); }
// Thread-block cluster barrier (every thread of every CTA of the cluster arrives), with
// release/acquire ordering of shared-memory writes across the cluster.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
// 32-bit load from CTA `rank`'s shared memory at the address this CTA uses for `saddr`.
// Not volatile: the loads only follow the cluster barrier (which orders them), so the
// compiler may batch them.
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t saddr, uint32_t rank) {
  uint32_t remote;
  asm("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(remote) : "r"(saddr), "r"(rank));
  return remote;
}
__device__ __forceinline__ uint32_t ld_dsmem(uint32_t remote) {
  uint32_t v;
  asm("ld.shared::cluster.u32 %0, [%1];\n" : "=r"(v) : "r"(remote));
  return v;
}

// Shared-memory matrix descriptor for a K-major operand tile whose rows are 128 bytes,
// written by TMA with 128-byte swizzle: 8-row core groups 1024 bytes apart (SBO), layout
// type 2 (SWIZZLE_128B), descriptor version 1.  The start address of the k-th 32-byte
// slice of the swizzle atom is base + 32*k.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3fff);
  d |= static_cast<uint64_t>(1) << 16;            // leading byte offset (16 B, unused for SW128 K-major)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;    // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;            // version
  d |= static_cast<uint64_t>(2) << 61;            // SWIZZLE_128B
  return d;
}
// Instruction descriptor: K-major A and B, D format f32 (kind::f16) or s32 (kind::i8).
template <typename InT>
__host__ __device__ constexpr uint32_t umma_idesc(int m, int n) {
  uint32_t c_fmt = sizeof(InT) == 1 ? 2u : 1u;
  uint32_t ab_fmt = 0;
  if constexpr (sizeof(InT) == 1) ab_fmt = 1;  // signed int8
  else if constexpr (std::is_same<InT, __nv_bfloat16>::value) ab_fmt = 1;
  else ab_fmt = 0;  // fp16
  return (c_fmt << 4) | (ab_fmt << 7) | (ab_fmt << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

constexpr int kUmmaThreads = 192;

template <int BT, int STAGES>
constexpr int umma_smem_bytes() {
  return STAGES * (128 + BT) * 128 + 1024;  // + alignment slack
}

template <typename InT, typename OutT, int BT, int STAGES, int EPI>
__global__ void __launch_bounds__(kUmmaThreads, 1)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmX, GemmParams p) {
  constexpr bool I8 = sizeof(InT) == 1;
  constexpr int A_BYTES = 128 * 128;
  constexpr int B_BYTES = BT * 128;
  constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = BT < 32 ? 32 : BT;
  constexpr int ESZ = sizeof(InT);
  constexpr int KSTEP_BYTES = 32;  // one UMMA consumes 32 bytes of K (16 x 16-bit or 32 x 8-bit)

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[STAGES], empty_bar[STAGES], accum_bar;
  __shared__ uint32_t s_tmem;
  __shared__ int s_pos[BT], s_page[BT];
  __shared__ double s_ss[4][32];
  __shared__ unsigned long long s_best[4][32];

  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_tile = blockIdx.x, m_tile = blockIdx.y;
  const int n0 = n_tile * 128, m0 = m_tile * BT;
  const int k_tiles = p.K * ESZ / 128;
  const int kt_begin = blockIdx.z * p.k_tiles_per_split;
  const int kt_end = min(k_tiles, kt_begin + p.k_tiles_per_split);
  const int nkt = max(0, kt_end - kt_begin);

  griddep_launch_dependents();
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    mbar_init(smem_u32(&accum_bar), 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(&s_tmem), TMEM_COLS);
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
      asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
      asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
      // The weights do not depend on the preceding kernel: stream the first stages' weight
      // tiles while it drains, then wait for it before touching the activations.
      const int pre = min(nkt, STAGES);
      for (int i = 0; i < pre; ++i) {
        const uint32_t st = sbase + i * STAGE_BYTES;
        mbar_arrive_expect_tx(smem_u32(&full_bar[i]), STAGE_BYTES);
        tma_load_2d(st, &tmW, (kt_begin + i) * (128 / ESZ), n0, smem_u32(&full_bar[i]));
      }
      griddep_wait();
      for (int i = 0; i < pre; ++i)
        tma_load_2d(sbase + i * STAGE_BYTES + A_BYTES, &tmX, (kt_begin + i) * (128 / ESZ), m0,
                    smem_u32(&full_bar[i]));
      for (int i = pre; i < nkt; ++i) {
        const int s = i % STAGES;
        const uint32_t par = ((i / STAGES) & 1) ^ 1;
        if (!mbar_wait_bounded(smem_u32(&empty_bar[s]), par)) {
          failed = true;
          break;
        }
        const uint32_t st = sbase + s * STAGE_BYTES;
        const int kx = (kt_begin + i) * (128 / ESZ);  // element coordinate of the K slice
        mbar_arrive_expect_tx(smem_u32(&full_bar[s]), STAGE_BYTES);
        tma_load_2d(st, &tmW, kx, n0, smem_u32(&full_bar[s]));
        tma_load_2d(st + A_BYTES, &tmX, kx, m0, smem_u32(&full_bar[s]));
      }
    }
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc<InT>(128, BT);
      for (int i = 0; i < nkt; ++i) {
        const int s = i % STAGES;
        if (!mbar_wait_bounded(smem_u32(&full_bar[s]), (i / STAGES) & 1)) {
          failed = true;
          break;
        }
        tc_fence_after();
        const uint32_t a = sbase + s * STAGE_BYTES, b = a + A_BYTES;
#pragma unroll
        for (int k = 0; k < 128 / KSTEP_BYTES; ++k)
          umma<I8>(tmem, sw128_desc(a + k * KSTEP_BYTES), sw128_desc(b + k * KSTEP_BYTES), idesc,
                   (i > 0 || k > 0) ? 1u : 0u);
        tc_commit(smem_u32(&empty_bar[s]));
      }
      tc_commit(smem_u32(&accum_bar));
    }
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5)
    const int q = warp & 3;                 // TMEM lane quadrant
    const int et = threadIdx.x - 64;        // 0..127 among epilogue threads
    const int nl = q * 32 + lane;           // channel within the tile
    const int n = n0 + nl;
    griddep_wait();  // positions, scales and the residual come from earlier kernels
    if constexpr (EPI == EPI_QKV) {
      for (int j = et; j < BT; j += 128) {
        const int m = m0 + j;
        int pos = 0, page = 0;
        if (m < p.M) {
          pos = p.positions[m];
          page = p.block_table[static_cast<size_t>(p.seq_ids[m]) * p.max_pages_per_seq + (pos >> 4)];
        }
        s_pos[j] = pos;
        s_page[j] = page;
      }
    }
    const float sw = (I8 && n < p.N) ? p.b_scale[n] : 1.0f;
    // 32 x 33 transpose buffers of the epilogue warps live in the stage ring, which is idle
    // once the accumulator is complete (every TMA write and MMA read has finished)
    float(*s_tr)[32 * 33] = reinterpret_cast<float(*)[32 * 33]>(smem_raw + (sbase - smem_u32(smem_raw)));
    bool ok = nkt > 0 && mbar_wait_bounded(smem_u32(&accum_bar), 0);
    if (!ok && nkt > 0) failed = true;
    tc_fence_after();
    if constexpr (EPI == EPI_QKV) epi_bar();  // s_pos / s_page visible to all epilogue warps
    const int mcount = min(BT, p.M - m0);
    const bool split = EPI == EPI_RESID && p.k_splits > 1;
    if (split) {
      // stage this split's partial tile [128 channels][BT tokens] (+1 column of padding)
      uint32_t* part = reinterpret_cast<uint32_t*>(smem_raw + (sbase - smem_u32(smem_raw)));
      for (int c0 = 0; c0 < BT; c0 += 32) {
        uint32_t r[32];
        tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) part[nl * (BT + 1) + c0 + j] = ok ? r[j] : 0u;
      }
    }
    for (int c0 = 0; c0 < BT && !split; c0 += 32) {
      if (c0 >= mcount) break;  // uniform across the epilogue warps
      uint32_t r[32];
      tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + c0, r);
      tmem_wait_ld();
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if constexpr (I8) {
          const int m = min(m0 + c0 + j, p.M - 1);
          v[j] = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[j])), p.a_scale[m]), sw);
        } else {
          v[j] = __uint_as_float(r[j]);
        }
      }
      if (!ok) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = 0.f;
      }
      if constexpr (EPI == EPI_S32 || EPI == EPI_F32 || EPI == EPI_RESID) {
        // out may alias resid (in-place residual): read the whole chunk before any store
        float rs[32];
        if constexpr (EPI == EPI_RESID) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int m = m0 + c0 + j;
            rs[j] = (m < p.M && n < p.N) ? p.resid[static_cast<size_t>(m) * p.ldo + n] : 0.f;
          }
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int m = m0 + c0 + j;
          if (m < p.M && n < p.N) {
            const size_t idx = static_cast<size_t>(m) * p.ldo + n;
            if constexpr (EPI == EPI_S32) reinterpret_cast<int*>(p.out)[idx] = static_cast<int>(r[j]);
            else if constexpr (EPI == EPI_F32) reinterpret_cast<float*>(p.out)[idx] = v[j];
            else reinterpret_cast<float*>(p.out)[idx] = __fadd_rn(v[j], rs[j]);
          }
        }
      } else if constexpr (EPI == EPI_SWIGLU) {
        // rows interleaved (W1[j], W3[j]): lane 2i holds the gate, lane 2i+1 the up value of
        // channel pair i for 32 tokens.  The even lane finishes tokens 0..15, the odd lane
        // tokens 16..31, each receiving the missing operand from its neighbour.
        const int F = p.N / 2;
        const bool odd = lane & 1;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float sent = __shfl_xor_sync(0xffffffffu, odd ? v[j] : v[j + 16], 1);
          const float h1 = odd ? sent : v[j];
          const float up = odd ? v[j + 16] : sent;
          const int m = m0 + c0 + j + (odd ? 16 : 0);
          const int ch = n & ~1;
          if (m < p.M && ch < p.N) {
            const float gv = __fmul_rn(__fdiv_rn(h1, __fadd_rn(1.0f, expf(-h1))), up);
            const size_t idx = static_cast<size_t>(m) * F + (ch >> 1);
            if (p.swiglu_f32) reinterpret_cast<float*>(p.out)[idx] = gv;
            else reinterpret_cast<OutT*>(p.out)[idx] = ActTraits<OutT>::from_f(gv);
          }
        }
      } else if constexpr (EPI == EPI_ARGMAX) {
        if (p.logits) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int m = m0 + c0 + j;
            if (n < p.N && m < p.M) p.logits[static_cast<size_t>(m) * p.ld_logits + n] = v[j];
          }
        }
        // transpose the 32 channels x 32 tokens block so thread `lane` scans token lane's
        // 32 channels in ascending order (first maximum wins), then combine the 4 warps
        float* tb = s_tr[q];
#pragma unroll
        for (int j = 0; j < 32; ++j) tb[j * 33 + lane] = v[j];
        __syncwarp();
        unsigned long long best = 0ull;
        const int nbase = n0 + q * 32;
#pragma unroll
        for (int c = 0; c < 32; ++c) {
          if (nbase + c < p.N) {
            const unsigned long long k = argmax_key(tb[lane * 33 + c], nbase + c);
            best = k > best ? k : best;
          }
        }
        s_best[q][lane] = best;
        epi_bar();
        if (et < 32) {
          unsigned long long b = s_best[0][et];
#pragma unroll
          for (int w = 1; w < 4; ++w) b = s_best[w][et] > b ? s_best[w][et] : b;
          const int m = m0 + c0 + et;
          if (m < p.M) p.argmax_part[static_cast<size_t>(n_tile) * p.M + m] = b;
        }
        epi_bar();
      } else if constexpr (EPI == EPI_QKV) {
        // Transpose the warp's 32 channels x 32 tokens block through shared memory so each
        // thread owns one token's 32 consecutive channels of a head.
        const int hd = p.head_dim;
        const int q_dim = p.n_heads * hd, kv_dim = p.n_kv_heads * hd;
        int region, head0;
        if (n0 < q_dim) { region = 0; head0 = n0 / hd; }
        else if (n0 < q_dim + kv_dim) { region = 1; head0 = (n0 - q_dim) / hd; }
        else { region = 2; head0 = (n0 - q_dim - kv_dim) / hd; }
        float* tb = s_tr[q];
#pragma unroll
        for (int j = 0; j < 32; ++j) tb[j * 33 + lane] = v[j];
        __syncwarp();
        float x[32];
#pragma unroll
        for (int c = 0; c < 32; ++c) x[c] = tb[lane * 33 + c];
        const int tok = c0 + lane;              // this thread's token within the tile
        const int m = m0 + tok;
        const int cbase = q * 32;               // first channel of this warp within the tile
        const int head = head0 + cbase / hd;
        const int d0 = cbase % hd;              // first head dimension held by this thread
        const int wph = hd / 32;                // warps per head
        if (region < 2 && p.qk_norm) {
          double ss = 0.0;
#pragma unroll
          for (int c = 0; c < 32; ++c) ss = __dadd_rn(ss, __dmul_rn((double)x[c], (double)x[c]));
          s_ss[q][lane] = ss;
          epi_bar();
          const int qh0 = (q / wph) * wph;
          double tot = 0.0;
          for (int w = 0; w < wph; ++w) tot = __dadd_rn(tot, s_ss[qh0 + w][lane]);
          const float rr = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(tot, (double)hd), p.eps))));
          const float* nw = region == 0 ? p.q_norm : p.k_norm;
#pragma unroll
          for (int c = 0; c < 32; ++c) x[c] = __fmul_rn(__fmul_rn(x[c], rr), nw[d0 + c]);
          epi_bar();
        }
        const int pos = s_pos[tok];
        if (region < 2) {
          const float* cs = p.rope_cos + static_cast<size_t>(pos) * (hd / 2) + d0 / 2;
          const float* sn = p.rope_sin + static_cast<size_t>(pos) * (hd / 2) + d0 / 2;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float c = cs[i], s = sn[i];
            const float a0 = x[2 * i], a1 = x[2 * i + 1];
            x[2 * i] = __fsub_rn(__fmul_rn(a0, c), __fmul_rn(a1, s));
            x[2 * i + 1] = __fadd_rn(__fmul_rn(a0, s), __fmul_rn(a1, c));
          }
        }
        if (m < p.M && n0 + cbase < p.N) {
          uint4 pk[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            pk[c].x = ActTraits<OutT>::pack2(x[8 * c + 0], x[8 * c + 1]);
            pk[c].y = ActTraits<OutT>::pack2(x[8 * c + 2], x[8 * c + 3]);
            pk[c].z = ActTraits<OutT>::pack2(x[8 * c + 4], x[8 * c + 5]);
            pk[c].w = ActTraits<OutT>::pack2(x[8 * c + 6], x[8 * c + 7]);
          }
          if (region == 0) {
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<OutT*>(p.q_out) +
                                                  (static_cast<size_t>(m) * p.n_heads + head) * hd + d0);
#pragma unroll
            for (int c = 0; c < 4; ++c) dst[c] = pk[c];
          } else {
            const int page = s_page[tok];
            if (page < 0 || page >= p.n_pages) {
              if (p.err) atomicExch(p.err, kDevBadPage);
            } else {
              const int slot = pos & 15;
              const size_t blk =
                  ((static_cast<size_t>(p.layer) * p.n_pages + page) * p.n_kv_heads + head) * 2 + (region - 1);
              OutT* base = reinterpret_cast<OutT*>(p.kv_pool) + blk * 16 * hd + slot * hd;
#pragma unroll
              for (int c = 0; c < 4; ++c) {
                const int chunk = ((d0 >> 3) + c) ^ (slot & 7);
                *reinterpret_cast<uint4*>(base + chunk * 8) = pk[c];
              }
            }
          }
        }
        __syncwarp();
      }
    }
  }
  if constexpr (EPI == EPI_RESID) {
    if (p.k_splits > 1) {
      __syncwarp();
      cluster_sync_all();  // every split's partial tile is in its shared memory
      if (warp >= 2) {
        const int q = warp & 3, nl = q * 32 + lane, n = n0 + nl;
        const float sw = (I8 && n < p.N) ? p.b_scale[n] : 1.0f;
        const uint32_t rank = cluster_rank();
        const int S = p.k_splits;
        const int per = BT / S;
        uint32_t base[4];  // the partial tile of every rank (same offset in each CTA)
#pragma unroll
        for (int sr = 0; sr < 4; ++sr) base[sr] = sr < S ? dsmem_addr(sbase, sr) : 0u;
        // token slice in batches of 8: issue the batch's remote loads of every rank, then sum
        for (int jb = 0; jb < per; jb += 8) {
          uint32_t raw[4][8];
#pragma unroll
          for (int sr = 0; sr < 4; ++sr)
#pragma unroll
            for (int jj = 0; jj < 8; ++jj)
              if (sr < S && jb + jj < per)
                raw[sr][jj] =
                    ld_dsmem(base[sr] + 4u * static_cast<uint32_t>(nl * (BT + 1) + static_cast<int>(rank) * per + jb + jj));
#pragma unroll
          for (int jj = 0; jj < 8; ++jj) {
            const int j = static_cast<int>(rank) * per + jb + jj;
            const int m = m0 + j;
            if (jb + jj >= per || m >= p.M || n >= p.N) continue;
            float v;
            if constexpr (I8) {
              int acc = 0;
#pragma unroll
              for (int sr = 0; sr < 4; ++sr)
                if (sr < S) acc += static_cast<int>(raw[sr][jj]);
              v = __fmul_rn(__fmul_rn(__int2float_rn(acc), p.a_scale[m]), sw);
            } else {
              float acc = 0.f;
#pragma unroll
              for (int sr = 0; sr < 4; ++sr)
                if (sr < S) acc = __fadd_rn(acc, __uint_as_float(raw[sr][jj]));
              v = acc;
            }
            const size_t idx = static_cast<size_t>(m) * p.ldo + n;
            reinterpret_cast<float*>(p.out)[idx] = __fadd_rn(v, p.resid[idx]);
          }
        }
      }
      __syncwarp();
      cluster_sync_all();  // peers may still be reading this CTA's partial tile
    }
  }
  if (failed && p.err) atomicExch(p.err, kDevWaitTimeout);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

}  // namespace llm
