// umma.cuh -- tcgen05 (5th-generation tensor core) GEMM for the token loop's projections.
//
//   D[m, n] = sum_k X[m, k] * W[n, k]     (X = activations [M x K], W = weights [N x K])
//
// Token-major tiles: the UMMA "A" operand is a 128-token tile of X and the "B" operand a
// BN-channel tile of W (BN = 16..256), both K-major and 128-byte swizzled, written by TMA
// (cp.async.bulk.tensor, each CTA loading its own tiles).  The fp32/s32 accumulator lives in tensor memory
// with TMEM lane = token and column = output channel, so in the epilogue every thread owns
// one token and walks that token's channels in registers: QK-norm, RoPE, SwiGLU pairing and
// the greedy argmax are per-thread loops over contiguous channels, and every store is a
// contiguous run of one output row.
//
// Decode shapes (a few hundred tokens) are latency-bound per SM, so the host picks BN such
// that the grid is about one CTA per SM and every CTA streams its share of W through a
// ~192 KB stage ring (4..11 stages) with all stages in flight.  Grid x = token tile (fastest,
// so the CTAs that share a weight tile run side by side and the second one reads it from
// L2), y = channel tile.  One SM streams only ~50 GB/s into shared memory, and a decode CTA
// loads the whole activation tile for its few channels, so the long-K narrow-N residual
// projections of the 16-bit models split K over a thread-block cluster (z = split, SPLIT
// instantiation): each CTA runs its own MMA chain over a contiguous range of K slices, and after
// a cluster barrier finishes 128/S rows of the tile by adding the S partial tiles, read from
// the CTAs' shared memory through the cluster, in rank order (splitk_reduce).
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM allocator + MMA issuer
// (one elected thread), warps 2..5 = epilogue.  Epilogue warp w reads TMEM lanes
// 32*(w%4)..+31.  A STAGES-deep ring of (full, empty) mbarriers connects producer and MMA;
// tcgen05.commit releases a stage when its MMAs have consumed it and signals the epilogue
// after the last.  Everything the epilogue needs besides the accumulator (token scales and
// positions, channel scales, norm weights, residual rows, RoPE rows) is loaded while the
// mainloop runs.  Every mbarrier wait is bounded: on expiry the kernel records
// kDevWaitTimeout, skips the remaining work and still reaches the TMEM deallocation.
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
// kind::f16 MMA whose A operand (M lanes x K 16-bit elements, two per 32-bit column, row m in
// lane m) is read from tensor memory at tmem_a; B from shared memory as in umma().
__device__ __forceinline__ void umma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                        uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(acc));
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
// 32 lanes x 32 columns of 32-bit from registers: thread t writes columns col..col+31 of lane
// (base lane + t)
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }
// Shared-memory descriptor of an MN-major operand written in 128-byte-swizzle atoms (64
// elements of MN contiguous per 128-byte row, 8 rows of K per 1024-byte atom): lbo = byte
// distance between 64-element MN chunks, sbo = byte distance between 8-row K groups.
__device__ __forceinline__ uint64_t sw128_desc_mn(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3fff);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3fff) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3fff) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // version
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;\n" ::: "memory"); }
// Cluster-wide barrier (every thread of every CTA of the cluster), release / acquire ordering
// of shared-memory writes before it and distributed shared-memory reads after it.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire;\n" ::: "memory");
}
// Address of the same shared-memory location in cluster CTA `rank`.
__device__ __forceinline__ uint32_t dsmem_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ uint4 ld_dsmem_u4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared::cluster.v4.u32 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}
__device__ __forceinline__ void prefetch_l2(const void* ptr) { asm volatile("prefetch.global.L2 [%0];\n" ::"l"(ptr)); }

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
constexpr int kUmmaTokens = 128;  // token rows per tile (UMMA M)

// Stage ring of ~192 KB: one CTA per SM, all stages in flight.
#ifndef LLM_UMMA_MAX_STAGES
#define LLM_UMMA_MAX_STAGES 11
#endif
template <int BN>
constexpr int umma_stages() {
  return (192 * 1024) / ((kUmmaTokens + BN) * 128) > LLM_UMMA_MAX_STAGES ? LLM_UMMA_MAX_STAGES
                                                                          : (192 * 1024) / ((kUmmaTokens + BN) * 128);
}
template <int BN>
constexpr int umma_smem_bytes() {
  return umma_stages<BN>() * (kUmmaTokens + BN) * 128 + 1024;  // + alignment slack
}
// Dynamic shared memory of a launch with `stages` ring stages (0 = the maximum).
template <int BN>
constexpr int umma_smem_bytes_for(int stages) {
  return (stages > 0 && stages < umma_stages<BN>() ? stages : umma_stages<BN>()) * (kUmmaTokens + BN) * 128 + 1024;
}
template <int BN>
constexpr uint32_t umma_tmem_cols() {
  return BN < 32 ? 32u : static_cast<uint32_t>(BN);
}

// Monotone 32-bit key of a float (the high half of argmax_key): unsigned order of the keys
// is the order of the values, with distinct keys for distinct bit patterns.
__device__ __forceinline__ uint32_t float_key_fast(float f) {
  const uint32_t u = __float_as_uint(f);
  return u ^ (static_cast<uint32_t>(static_cast<int>(u) >> 31) | 0x80000000u);
}

// Split-K reduction of one cluster CTA's rows: rows row0 .. row0+rp-1 of the tile, summed over
// the S partial tiles (pitch PP floats at part_s in every CTA of the cluster) in rank order
// (int32 exactly, fp32 rounded to nearest at each addition), written to this CTA's red_s
// (same pitch, rp rows).  Each of the 128 epilogue threads keeps 16 distributed-shared-memory
// loads in flight.
template <int S, bool I8, int PP>
__device__ __forceinline__ void splitk_reduce(uint32_t part_s, uint32_t red_s, int row0, int rp, int c4, int et) {
  constexpr int G = 16 / S;  // items per batch
  const int total = rp * c4;
  for (int base = et; base < total; base += 128 * G) {
    uint4 v[G][S];
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int idx = base + g * 128;
      if (idx < total) {
        const uint32_t off = part_s + ((row0 + idx / c4) * PP + 4 * (idx % c4)) * 4;
#pragma unroll
        for (int z = 0; z < S; ++z) v[g][z] = ld_dsmem_u4(dsmem_addr(off, static_cast<uint32_t>(z)));
      }
    }
#pragma unroll
    for (int g = 0; g < G; ++g) {
      const int idx = base + g * 128;
      if (idx >= total) continue;
      uint32_t r[4] = {v[g][0].x, v[g][0].y, v[g][0].z, v[g][0].w};
#pragma unroll
      for (int z = 1; z < S; ++z) {
        const uint32_t w[4] = {v[g][z].x, v[g][z].y, v[g][z].z, v[g][z].w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          if constexpr (I8) r[j] = static_cast<uint32_t>(static_cast<int>(r[j]) + static_cast<int>(w[j]));
          else r[j] = __float_as_uint(__fadd_rn(__uint_as_float(r[j]), __uint_as_float(w[j])));
        }
      }
      asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};\n" ::"r"(red_s + ((idx / c4) * PP + 4 * (idx % c4)) * 4),
                   "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3])
                   : "memory");
    }
  }
}

// SPLIT: the split-K cluster form (k_splits > 1); a separate instantiation, so the whole-K
// kernels carry none of its registers.
template <typename InT, typename OutT, int BN, int EPI, bool SPLIT = false>
__global__ void __launch_bounds__(kUmmaThreads, 2)
    umma_gemm_kernel(const __grid_constant__ CUtensorMap tmX, const __grid_constant__ CUtensorMap tmW, GemmParams p) {
  constexpr bool I8 = sizeof(InT) == 1;
  static_assert(!SPLIT || EPI == EPI_RESID || EPI == EPI_F32 || EPI == EPI_S32, "split-K: elementwise epilogues");
  constexpr int MAX_STAGES = umma_stages<BN>();
  const int STAGES = p.stages > 0 && p.stages < MAX_STAGES ? p.stages : MAX_STAGES;
  constexpr int A_BYTES = kUmmaTokens * 128;
  constexpr int B_BYTES = BN * 128;
  constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  constexpr uint32_t TMEM_COLS = umma_tmem_cols<BN>();
  constexpr int ESZ = sizeof(InT);
  constexpr int KSTEP_BYTES = 32;  // one UMMA consumes 32 bytes of K (16 x 16-bit or 32 x 8-bit)
  constexpr int NCH = (BN + 31) / 32;  // 32-column chunks of the accumulator

  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[MAX_STAGES], empty_bar[MAX_STAGES], accum_bar;
  __shared__ uint32_t s_tmem;
  __shared__ float s_bsc[BN];   // per-channel weight scales (int8)
  __shared__ float s_nw[BN];    // QK-norm weights of this tile's head

  const uint32_t sbase = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // QKV tiles of 64 tokens (a_rows == 64, chosen when the grid has SMs to spare): the CTA loads
  // only its 64 activation rows per K slice (a 64-row box), the MMA still forms 128 rows, and
  // rows 64..127 of the accumulator are never read.
  const int TR = EPI == EPI_QKV && p.a_rows == 64 ? 64 : kUmmaTokens;
  const uint32_t LOAD_BYTES = TR * 128 + BN * 128;
  const int tok0 = blockIdx.x * TR, ch0 = blockIdx.y * BN;
  // Split-K (k_splits > 1): the CTAs blockIdx.z = 0 .. k_splits-1 of one cluster take
  // contiguous ranges of the 128-byte K slices and exchange their partial tiles through
  // distributed shared memory (splitk_reduce and the split epilogue below).
  const int n_split = SPLIT && p.k_splits > 1 ? p.k_splits : 1;
  const int nkt_all = p.K * ESZ / 128;
  const int kt0 = static_cast<int>(blockIdx.z) * nkt_all / n_split;
  const int nkt = (static_cast<int>(blockIdx.z) + 1) * nkt_all / n_split - kt0;  // this CTA's slices

  griddep_launch_dependents();
  trace_start(p.trace);
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
      asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&tmX)) : "memory");
      asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(&tmW)) : "memory");
      // The weights do not depend on the preceding kernel: start streaming the first
      // stages' weight tiles while it drains, then wait for it before the activations.
      const int pre = min(nkt, STAGES);
      for (int i = 0; i < pre; ++i) {
        const uint32_t st = sbase + i * STAGE_BYTES;
        mbar_arrive_expect_tx(smem_u32(&full_bar[i]), LOAD_BYTES);
        tma_load_2d(st + A_BYTES, &tmW, (kt0 + i) * (128 / ESZ), ch0, smem_u32(&full_bar[i]));
      }
      griddep_wait();
      for (int i = 0; i < pre; ++i)
        tma_load_2d(sbase + i * STAGE_BYTES, &tmX, (kt0 + i) * (128 / ESZ), tok0, smem_u32(&full_bar[i]));
      for (int i = pre; i < nkt; ++i) {
        const int s = i % STAGES;
        const uint32_t par = ((i / STAGES) & 1) ^ 1;
        if (!mbar_wait_bounded(smem_u32(&empty_bar[s]), par)) {
          failed = true;
          break;
        }
        const uint32_t st = sbase + s * STAGE_BYTES;
        const int kx = (kt0 + i) * (128 / ESZ);  // element coordinate of the K slice
        mbar_arrive_expect_tx(smem_u32(&full_bar[s]), LOAD_BYTES);
        tma_load_2d(st + A_BYTES, &tmW, kx, ch0, smem_u32(&full_bar[s]));
        tma_load_2d(st, &tmX, kx, tok0, smem_u32(&full_bar[s]));
      }
    }
    __syncwarp();
    if (SPLIT && n_split > 1) cluster_sync_all();  // partial tiles written (splitk epilogue)
  } else if (warp == 1) {
    // ---------------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc<InT>(kUmmaTokens, BN);
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
    __syncwarp();
    if (SPLIT && n_split > 1) cluster_sync_all();
  } else {
    // ---------------------------------------------------------------- epilogue (warps 2..5)
    const int q = warp & 3;              // TMEM lane quadrant
    const int et = threadIdx.x - 64;     // 0..127 among epilogue threads
    // Split-K: cluster CTA z finishes rows z*RP .. z*RP+RP-1 of the tile (RP = 128 / k_splits)
    // from every CTA's partial.
    const bool split = SPLIT && n_split > 1;
    const int RP = kUmmaTokens / n_split;
    const int tl = q * 32 + lane;        // token within the tile (= TMEM lane)
    const int tok = tok0 + tl;
    const bool tok_ok = tl < TR && tok < p.M;
    const int tokc = tok_ok ? tok : p.M - 1;
    const uint32_t trow = tmem + (static_cast<uint32_t>(q * 32) << 16);
    griddep_wait();  // positions, scales and the residual come from earlier kernels

    // ---- loads that only depend on earlier kernels, overlapped with the mainloop
    float a_s = 1.0f;
    if constexpr (I8) a_s = p.a_scale[tokc];
    for (int j = et; j < BN; j += 128) {
      const int ch = ch0 + j;
      if constexpr (I8) s_bsc[j] = ch < p.N ? p.b_scale[ch] : 0.0f;
    }
    float rs[32];  // residual of the first chunk
    if constexpr (EPI == EPI_RESID) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        rs[j] = (j < BN && tok_ok && ch0 + j < p.N) ? p.resid[static_cast<size_t>(tok) * p.ldo + ch0 + j] : 0.f;
    }
    int region = 0, head = 0, pos = 0, page = 0;
    const float* cs_row = nullptr;
    const float* sn_row = nullptr;
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
      cs_row = p.rope_cos + static_cast<size_t>(pos) * (hd / 2);
      sn_row = p.rope_sin + static_cast<size_t>(pos) * (hd / 2);
      for (int b = 0; b < hd * 2; b += 128) {
        prefetch_l2(reinterpret_cast<const uint8_t*>(cs_row) + b);
        prefetch_l2(reinterpret_cast<const uint8_t*>(sn_row) + b);
      }
      if (region < 2 && p.qk_norm) {
        const float* nw = region == 0 ? p.q_norm : p.k_norm;
        for (int j = et; j < BN; j += 128) s_nw[j] = nw[j];
      }
    }

    bool ok = nkt > 0 && mbar_wait_bounded(smem_u32(&accum_bar), 0);
    if (!ok && nkt > 0) failed = true;
    tc_fence_after();
    epi_bar();  // s_bsc / s_nw visible to all epilogue threads

    // Split-K partial tiles: each CTA's accumulator rows, TMEM lane = token, are written to its
    // idle stage ring (pitch PP floats); after the cluster barrier a row's chunk is the sum of the
    // CTAs' partials in rank order (int32 exactly, fp32 rounded to nearest at each addition).
    constexpr int PP = BN + 4;
    const uint32_t part_s = sbase;
    const uint32_t red_s = sbase + kUmmaTokens * PP * 4;  // this CTA's summed rows (split-K)
    if (split) {
      if (STAGES * STAGE_BYTES < (kUmmaTokens + RP) * PP * 4) {  // the host sizes the ring for this
        if (p.err) atomicExch(p.err, kDevWaitTimeout);
        ok = false;
      }
      const int tr = q * 32 + lane;  // this thread's TMEM lane
      for (int c = 0; c < NCH && ok; ++c) {
        uint32_t r[32];
        tmem_ld32(trow + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          if (c * 32 + j < BN)
            asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};\n" ::"r"(part_s + (tr * PP + c * 32 + j) * 4),
                         "r"(r[j]), "r"(r[j + 1]), "r"(r[j + 2]), "r"(r[j + 3])
                         : "memory");
      }
      cluster_sync_all();
      const int row0 = static_cast<int>(blockIdx.z) * RP;
      if constexpr (SPLIT) {
        if (ok) {
          if (n_split == 2) splitk_reduce<2, I8, PP>(part_s, red_s, row0, RP, BN / 4, et);
          else if (n_split == 4) splitk_reduce<4, I8, PP>(part_s, red_s, row0, RP, BN / 4, et);
          else splitk_reduce<8, I8, PP>(part_s, red_s, row0, RP, BN / 4, et);
        }
      }
      epi_bar();  // the summed rows are visible to every epilogue thread
    }
    // the summed partials of columns col..col+3 of tile row `row` of this CTA (split-K)
    auto split_sum4 = [&](int row, int col, uint32_t (&r)[4]) {
      uint4 v;
      asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];\n"
                   : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                   : "r"(red_s + ((row - static_cast<int>(blockIdx.z) * RP) * PP + col) * 4)
                   : "memory");
      r[0] = v.x; r[1] = v.y; r[2] = v.z; r[3] = v.w;
    };

    // dequantised chunk c (columns 32c..32c+31 of this token's row)
    auto load_chunk = [&](int c, float (&v)[32]) {
      uint32_t r[32];
      tmem_ld32(trow + c * 32, r);
      tmem_wait_ld();
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        if constexpr (I8) v[j] = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[j])), a_s), s_bsc[(c * 32 + j) % BN]);
        else v[j] = __uint_as_float(r[j]);
        if (!ok) v[j] = 0.f;
      }
    };

    // Coalesced output: the stage ring is idle once the accumulator is complete (every MMA has
    // read its stages and no copy is outstanding), so a tile of per-token rows is written there
    // and then stored row by row with 16-byte vectors, consecutive threads on consecutive
    // columns, instead of each thread storing its own row (32 rows per warp instruction).
    float* const stg = reinterpret_cast<float*>(smem_raw + (sbase - smem_u32(smem_raw)));
    constexpr int OUT_COLS = EPI == EPI_SWIGLU ? BN / 2 : BN;  // values per token row of the tile
    constexpr int SP = OUT_COLS + 4;                             // staging pitch (floats)
    const bool staged = STAGES * STAGE_BYTES >= kUmmaTokens * SP * 4 &&
                        (EPI == EPI_RESID || EPI == EPI_F32 || EPI == EPI_S32 || EPI == EPI_SWIGLU);
    auto stage4 = [&](int col, float a, float b, float c_, float d) {
      *reinterpret_cast<float4*>(stg + tl * SP + col) = make_float4(a, b, c_, d);
    };

    if (split) {
      // Split-K residual / plain outputs: elementwise over this CTA's RP rows, four consecutive
      // channels per item (consecutive threads on consecutive channels: coalesced).
      if constexpr (SPLIT) {
        constexpr int C4 = BN / 4;
        for (int idx = et; idx < RP * C4; idx += 128) {
          const int row = static_cast<int>(blockIdx.z) * RP + idx / C4, col = 4 * (idx % C4);
          const int t = tok0 + row, ch = ch0 + col;
          if (t >= p.M || ch >= p.N) continue;
          uint32_t r[4];
          split_sum4(row, col, r);
          if constexpr (EPI == EPI_S32) {  // the int32 accumulators
            *reinterpret_cast<uint4*>(reinterpret_cast<int*>(p.out) + static_cast<size_t>(t) * p.ldo + ch) =
                ok ? make_uint4(r[0], r[1], r[2], r[3]) : make_uint4(0u, 0u, 0u, 0u);
            continue;
          }
          float v[4];
          const float as = I8 ? p.a_scale[t] : 1.0f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if constexpr (I8) v[j] = __fmul_rn(__fmul_rn(__int2float_rn(static_cast<int>(r[j])), as), s_bsc[col + j]);
            else v[j] = __uint_as_float(r[j]);
            if (!ok) v[j] = 0.f;
          }
          if constexpr (EPI == EPI_F32) {
            *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + static_cast<size_t>(t) * p.ldo + ch) =
                make_float4(v[0], v[1], v[2], v[3]);
          } else if constexpr (EPI == EPI_RESID) {
            float* dst = reinterpret_cast<float*>(p.out) + static_cast<size_t>(t) * p.ldo + ch;
            const float4 rv = *reinterpret_cast<const float4*>(p.resid + static_cast<size_t>(t) * p.ldo + ch);
            *reinterpret_cast<float4*>(dst) =
                make_float4(resid_add(v[0], rv.x, p.resid_scale), resid_add(v[1], rv.y, p.resid_scale),
                            resid_add(v[2], rv.z, p.resid_scale), resid_add(v[3], rv.w, p.resid_scale));
          }
        }
      }
    } else if (staged && (EPI == EPI_RESID || EPI == EPI_F32 || EPI == EPI_S32)) {
      for (int c = 0; c < NCH; ++c) {
        float v[32];
        if constexpr (EPI == EPI_S32) {
          uint32_t r[32];
          tmem_ld32(trow + c * 32, r);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(ok ? r[j] : 0u);
        } else {
          load_chunk(c, v);
        }
#pragma unroll
        for (int j = 0; j < 32; j += 4)
          if (c * 32 + j < BN) stage4(c * 32 + j, v[j], v[j + 1], v[j + 2], v[j + 3]);
      }
      epi_bar();
      // out may alias resid (in-place residual): each element is read and written by one thread.
      // The residual is read UNR vectors at a time so their L2 round trips overlap.
      constexpr int C4 = BN / 4;
      constexpr int PER_THREAD = kUmmaTokens * C4 / 128;
      constexpr int UNR = PER_THREAD >= 8 ? 8 : PER_THREAD;
      for (int it0 = 0; it0 < PER_THREAD; it0 += UNR) {
        float4 r[UNR];
        if constexpr (EPI == EPI_RESID) {
#pragma unroll
          for (int u = 0; u < UNR; ++u) {
            const int idx = et + (it0 + u) * 128;
            const int row = idx / C4, col = 4 * (idx % C4);
            const int t = tok0 + row, ch = ch0 + col;
            r[u] = (t < p.M && ch < p.N) ? *reinterpret_cast<const float4*>(p.resid + static_cast<size_t>(t) * p.ldo + ch)
                                         : make_float4(0.f, 0.f, 0.f, 0.f);
          }
        }
#pragma unroll
        for (int u = 0; u < UNR; ++u) {
          const int idx = et + (it0 + u) * 128;
          const int row = idx / C4, col = 4 * (idx % C4);
          const int t = tok0 + row, ch = ch0 + col;
          if (t >= p.M || ch >= p.N) continue;
          const float4 y = *reinterpret_cast<const float4*>(stg + row * SP + col);
          float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + static_cast<size_t>(t) * p.ldo + ch);
          if constexpr (EPI == EPI_RESID) {
            *dst = make_float4(resid_add(y.x, r[u].x, p.resid_scale), resid_add(y.y, r[u].y, p.resid_scale),
                               resid_add(y.z, r[u].z, p.resid_scale), resid_add(y.w, r[u].w, p.resid_scale));
          } else {
            *dst = y;  // fp32 values, or the int32 accumulators' bit patterns
          }
        }
      }
    } else if (staged && EPI == EPI_SWIGLU) {
      for (int c = 0; c < NCH; ++c) {
        float v[32];
        load_chunk(c, v);
        float g[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) g[i] = swiglu_pair(v[2 * i], v[2 * i + 1], p.silu_form);
#pragma unroll
        for (int i = 0; i < 16; i += 4)
          if (c * 16 + i < OUT_COLS) stage4(c * 16 + i, g[i], g[i + 1], g[i + 2], g[i + 3]);
      }
      epi_bar();
      const int F = p.N / 2, j0 = ch0 / 2;
      if (p.swiglu_f32) {
        constexpr int C4 = OUT_COLS / 4;
        for (int idx = et; idx < kUmmaTokens * C4; idx += 128) {
          const int row = idx / C4, col = 4 * (idx % C4);
          const int t = tok0 + row;
          if (t >= p.M || j0 + col >= F) continue;
          *reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + static_cast<size_t>(t) * F + j0 + col) =
              *reinterpret_cast<const float4*>(stg + row * SP + col);
        }
      } else {
        constexpr int C8 = OUT_COLS / 8;
        for (int idx = et; idx < kUmmaTokens * C8; idx += 128) {
          const int row = idx / C8, col = 8 * (idx % C8);
          const int t = tok0 + row;
          if (t >= p.M || j0 + col >= F) continue;
          const float4 a = *reinterpret_cast<const float4*>(stg + row * SP + col);
          const float4 b = *reinterpret_cast<const float4*>(stg + row * SP + col + 4);
          uint4 pk;
          pk.x = ActTraits<OutT>::pack2(a.x, a.y);
          pk.y = ActTraits<OutT>::pack2(a.z, a.w);
          pk.z = ActTraits<OutT>::pack2(b.x, b.y);
          pk.w = ActTraits<OutT>::pack2(b.z, b.w);
          *reinterpret_cast<uint4*>(reinterpret_cast<OutT*>(p.out) + static_cast<size_t>(t) * F + j0 + col) = pk;
        }
      }
    } else if constexpr (EPI == EPI_S32) {
      for (int c = 0; c < NCH; ++c) {
        uint32_t r[32];
        tmem_ld32(trow + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int ch = ch0 + c * 32 + j;
          if (c * 32 + j < BN && tok_ok && ch < p.N)
            reinterpret_cast<int*>(p.out)[static_cast<size_t>(tok) * p.ldo + ch] = ok ? static_cast<int>(r[j]) : 0;
        }
      }
    } else if constexpr (EPI == EPI_F32) {
      for (int c = 0; c < NCH; ++c) {
        float v[32];
        load_chunk(c, v);
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int ch = ch0 + c * 32 + j;
          if (c * 32 + j < BN && tok_ok && ch < p.N) reinterpret_cast<float*>(p.out)[static_cast<size_t>(tok) * p.ldo + ch] = v[j];
        }
      }
    } else if constexpr (EPI == EPI_RESID) {
      // out may alias resid (in-place residual): every element is read before it is written,
      // by the same thread
      for (int c = 0; c < NCH; ++c) {
        float v[32];
        load_chunk(c, v);
        if (c > 0) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int ch = ch0 + c * 32 + j;
            rs[j] = (tok_ok && ch < p.N) ? p.resid[static_cast<size_t>(tok) * p.ldo + ch] : 0.f;
          }
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int ch = ch0 + c * 32 + j;
          if (c * 32 + j < BN && tok_ok && ch < p.N)
            reinterpret_cast<float*>(p.out)[static_cast<size_t>(tok) * p.ldo + ch] = resid_add(v[j], rs[j], p.resid_scale);
        }
      }
    } else if constexpr (EPI == EPI_SWIGLU) {
      // interleaved rows: channel 2i is W1 row i (gate), 2i+1 is W3 row i (up)
      const int F = p.N / 2;
      for (int c = 0; c < NCH; ++c) {
        float v[32];
        load_chunk(c, v);
        float g[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          g[i] = swiglu_pair(v[2 * i], v[2 * i + 1], p.silu_form);
        }
        const int j0 = (ch0 + c * 32) / 2;  // first output channel of the chunk
        if (tok_ok) {
          if (p.swiglu_f32) {
            float* dst = reinterpret_cast<float*>(p.out) + static_cast<size_t>(tok) * F + j0;
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (c * 32 + 2 * i < BN && j0 + i < F) dst[i] = g[i];
          } else if (c * 32 + 32 <= BN && j0 + 16 <= F && (F % 8) == 0) {
            uint4 pk[2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              pk[h].x = ActTraits<OutT>::pack2(g[8 * h + 0], g[8 * h + 1]);
              pk[h].y = ActTraits<OutT>::pack2(g[8 * h + 2], g[8 * h + 3]);
              pk[h].z = ActTraits<OutT>::pack2(g[8 * h + 4], g[8 * h + 5]);
              pk[h].w = ActTraits<OutT>::pack2(g[8 * h + 6], g[8 * h + 7]);
            }
            uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<OutT*>(p.out) + static_cast<size_t>(tok) * F + j0);
            dst[0] = pk[0];
            dst[1] = pk[1];
          } else {
            OutT* dst = reinterpret_cast<OutT*>(p.out) + static_cast<size_t>(tok) * F + j0;
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (c * 32 + 2 * i < BN && j0 + i < F) dst[i] = ActTraits<OutT>::from_f(g[i]);
          }
        }
      }
    } else if constexpr (EPI == EPI_ARGMAX) {
      // (key desc, channel asc) over this token's BN channels: two interleaved running
      // maxima (even / odd columns) break the dependency chain, then merge.
      uint32_t bk[2] = {0u, 0u};
      int bi[2] = {ch0, ch0};
      for (int c = 0; c < NCH; ++c) {
        float v[32];
        load_chunk(c, v);
        if (p.logits && tok_ok) {
          float* dst = p.logits + static_cast<size_t>(tok) * p.ld_logits + ch0 + c * 32;
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (c * 32 + j < BN && ch0 + c * 32 + j < p.N) dst[j] = v[j];
        }
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const int ch = ch0 + c * 32 + j;
          const uint32_t k = (c * 32 + j < BN && ch < p.N) ? float_key_fast(v[j]) : 0u;
          if (k > bk[j & 1]) {
            bk[j & 1] = k;
            bi[j & 1] = ch;
          }
        }
      }
      const int w = (bk[1] > bk[0] || (bk[1] == bk[0] && bi[1] < bi[0])) ? 1 : 0;
      if (tok_ok)
        p.argmax_part[static_cast<size_t>(tok) * p.argmax_parts + blockIdx.y] =
            (static_cast<unsigned long long>(bk[w]) << 32) | (0xffffffffu - static_cast<uint32_t>(bi[w]));
    } else if constexpr (EPI == EPI_QKV) {
      // One head per tile (BN == head_dim): QK-norm over the whole head (sum of squares in
      // f64), RoPE on adjacent pairs, then the head's row is stored to q or to its K/V page.
      const int hd = BN;
      float rr = 1.0f;
      if (region < 2 && p.qk_norm) {
        // sum of squares in f64: per 32-column chunk in order, then the chunks in order
        double ss = 0.0;
        for (int c = 0; c < NCH; ++c) {
          float v[32];
          load_chunk(c, v);
          double sc = 0.0;
#pragma unroll
          for (int j = 0; j < 32; ++j) sc = __dadd_rn(sc, __dmul_rn((double)v[j], (double)v[j]));
          ss = c == 0 ? sc : __dadd_rn(ss, sc);
        }
        rr = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(__dadd_rn(__ddiv_rn(ss, (double)hd), p.eps))));
      }
      const int slot = pos & 15;
      OutT* kv_base = nullptr;
      if (region > 0 && tok_ok) {
        if (page < 0 || page >= p.n_pages) {
          if (p.err) atomicExch(p.err, kDevBadPage);
        } else {
          const size_t blk =
              ((static_cast<size_t>(p.layer) * p.n_pages + page) * p.n_kv_heads + head) * 2 + (region - 1);
          kv_base = reinterpret_cast<OutT*>(p.kv_pool) + blk * 16 * hd;  // the page's K or V block
        }
      }
      for (int c = 0; c < NCH; ++c) {
        float x[32];
        load_chunk(c, x);
        const int d0 = c * 32;  // first head dimension of the chunk
        if (region < 2) {
          if (p.qk_norm) {
#pragma unroll
            for (int j = 0; j < 32; ++j) x[j] = __fmul_rn(__fmul_rn(x[j], rr), s_nw[d0 + j]);
          }
          float cs[16], sn[16];
#pragma unroll
          for (int i = 0; i < 16; i += 4) {
            const float4 a = *reinterpret_cast<const float4*>(cs_row + d0 / 2 + i);
            const float4 b = *reinterpret_cast<const float4*>(sn_row + d0 / 2 + i);
            cs[i] = a.x; cs[i + 1] = a.y; cs[i + 2] = a.z; cs[i + 3] = a.w;
            sn[i] = b.x; sn[i + 1] = b.y; sn[i + 2] = b.z; sn[i + 3] = b.w;
          }
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float a0 = x[2 * i], a1 = x[2 * i + 1];
            x[2 * i] = __fsub_rn(__fmul_rn(a0, cs[i]), __fmul_rn(a1, sn[i]));
            x[2 * i + 1] = __fadd_rn(__fmul_rn(a0, sn[i]), __fmul_rn(a1, cs[i]));
          }
        }
        uint4 pk[4];
#pragma unroll
        for (int h = 0; h < 4; ++h) {
          pk[h].x = ActTraits<OutT>::pack2(x[8 * h + 0], x[8 * h + 1]);
          pk[h].y = ActTraits<OutT>::pack2(x[8 * h + 2], x[8 * h + 3]);
          pk[h].z = ActTraits<OutT>::pack2(x[8 * h + 4], x[8 * h + 5]);
          pk[h].w = ActTraits<OutT>::pack2(x[8 * h + 6], x[8 * h + 7]);
        }
        if (!tok_ok) continue;
        if (region == 0) {
          uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<OutT*>(p.q_out) +
                                                (static_cast<size_t>(tok) * p.n_heads + head) * hd + d0);
#pragma unroll
          for (int h = 0; h < 4; ++h) dst[h] = pk[h];
        } else if (kv_base) {
#pragma unroll
          for (int h = 0; h < 4; ++h)
            *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(kv_base) + kv_off(slot, (d0 >> 3) + h)) = pk[h];
        }
      }
    }
  }
  if (failed && p.err) atomicExch(p.err, kDevWaitTimeout);
  // split-K: no CTA leaves while another may still read its partial tile
  if (SPLIT && n_split > 1) cluster_sync_all();
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
  trace_end(p.trace);
}

}  // namespace llm
