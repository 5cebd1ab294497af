// llm_cuda.cu -- the C ABI of include/llm_cuda.h: context, weights, paged KV cache,
// the token-loop orchestration (prefill / decode step / device-resident generate with CUDA
// graphs), the stories.Decoder host mirror, and the bit-exact debug hooks.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <cerrno>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <numeric>
#include <string>
#include <thread>
#include <tuple>
#include <vector>

#include "../../include/llm_cuda.h"
#include "attention.cuh"
#include "attn_prefill.cuh"
#include "attn_prefill_tc.cuh"
#include "umma_persist.cuh"
#include "common.cuh"
#include "gemm.cuh"
#include "norm.cuh"
#include "sample.cuh"
#include "umma.cuh"

using namespace llm;

// ============================================================================ errors
namespace {
thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define CU(call)                                                                                   \
  do {                                                                                             \
    cudaError_t e_ = (call);                                                                       \
    if (e_ != cudaSuccess) return fail(LLM_ERR_CUDA, "%s failed: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

#define RC(call)                \
  do {                          \
    int rc_ = (call);           \
    if (rc_ != LLM_OK) return rc_; \
  } while (0)
}  // namespace

// Lets the library's other translation units record the thread's last error.
int llm_detail_fail(int code, const char* msg) { return fail(code, "%s", msg); }

extern "C" int llm_last_error(char* buf, size_t n) {
  if (buf && n) {
    size_t k = std::min(n - 1, g_last_error.size());
    memcpy(buf, g_last_error.data(), k);
    buf[k] = 0;
  }
  return static_cast<int>(g_last_error.size());
}

// ============================================================================ synthetic weights
namespace {
inline uint64_t splitmix64(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}
}  // namespace

extern "C" uint64_t llm_synth_stream(int layer, int kind) {
  if (kind == 7) return 1;
  if (kind == 8) return 2;
  return 100ull + 16ull * static_cast<uint64_t>(layer) + static_cast<uint64_t>(kind);
}

extern "C" void llm_synth_normal(float* dst, uint64_t n, uint64_t seed, uint64_t stream, double stddev,
                                 double scale) {
  const uint64_t key = splitmix64(seed ^ splitmix64(stream * 0xD1B54A32D192ED03ull + 0x8CB92BA72F3D8DD7ull));
  const double mult = stddev * scale;
  const uint64_t pairs = (n + 1) / 2;
  auto work = [&](uint64_t p0, uint64_t p1) {
    const double two_pi = 6.283185307179586476925286766559;
    for (uint64_t j = p0; j < p1; ++j) {
      const uint64_t a = splitmix64(key + 2 * j), b = splitmix64(key + 2 * j + 1);
      const double u1 = (static_cast<double>(a >> 11) + 0.5) * (1.0 / 9007199254740992.0);
      const double u2 = static_cast<double>(b >> 11) * (1.0 / 9007199254740992.0);
      const double r = std::sqrt(-2.0 * std::log(u1));
      const double z0 = r * std::cos(two_pi * u2), z1 = r * std::sin(two_pi * u2);
      dst[2 * j] = static_cast<float>(mult * z0);
      if (2 * j + 1 < n) dst[2 * j + 1] = static_cast<float>(mult * z1);
    }
  };
  unsigned nt = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
  if (pairs < (1u << 16)) nt = 1;
  std::vector<std::thread> th;
  const uint64_t per = (pairs + nt - 1) / nt;
  for (unsigned i = 0; i < nt; ++i) {
    const uint64_t p0 = i * per, p1 = std::min(pairs, p0 + per);
    if (p0 < p1) th.emplace_back(work, p0, p1);
  }
  for (auto& t : th) t.join();
}

// ============================================================================ small kernels
namespace {

struct FinishParams {
  const unsigned long long* part;  // [M][n_tiles]
  int M, n_tiles;
  int* next;                       // [M]
  int* tok_io;                     // optional: tokens <- next
  int* pos_io;                     // optional: positions += 1
  const int* gen_start;            // optional with gen_out
  int* gen_out;                    // [cap][M]
  int gen_cap;
  const int* sampled;              // optional [M]: tokens drawn by sample_kernel replace the argmax
};

// Greedy token per row: max over the lm_head tiles' (value, first index) partials.
__global__ void __launch_bounds__(256) finish_kernel(FinishParams f) {
  griddep_launch_dependents();
  griddep_wait();
  const int row = blockIdx.x * 8 + threadIdx.x / 32, lane = threadIdx.x & 31;
  if (row >= f.M) return;
  unsigned long long best = 0ull;
  const unsigned long long* pr = f.part + static_cast<size_t>(row) * f.n_tiles;
#pragma unroll 4
  for (int t = lane; t < f.n_tiles; t += 32) {
    const unsigned long long k = pr[t];
    best = k > best ? k : best;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
    best = other > best ? other : best;
  }
  if (lane == 0) {
    const int idx = f.sampled ? f.sampled[row] : argmax_key_index(best);
    f.next[row] = idx;
    if (f.tok_io) f.tok_io[row] = idx;
    if (f.gen_out) {
      const int step = f.pos_io[row] - f.gen_start[row];
      if (step >= 0 && step < f.gen_cap) f.gen_out[static_cast<size_t>(step) * f.M + row] = idx;
    }
    if (f.pos_io) f.pos_io[row] += 1;
  }
}

// Read one cached K or V row (un-swizzled) as fp32.
template <typename T>
__global__ void read_kv_kernel(const T* pool, int layer, int n_pages, int n_kv_heads, int hd, int page, int slot,
                               float* k, float* v) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  const int kv_dim = n_kv_heads * hd;
  if (i >= 2 * kv_dim) return;
  const int which = i / kv_dim, j = i % kv_dim, head = j / hd, d = j % hd;
  const size_t blk = ((static_cast<size_t>(layer) * n_pages + page) * n_kv_heads + head) * 2 + which;
  const T* base = pool + blk * 16 * hd;
  const float val =
      ActTraits<T>::to_f(*(reinterpret_cast<const T*>(reinterpret_cast<const uint8_t*>(base) + kv_off(slot, d >> 3)) + (d & 7)));
  (which ? v : k)[j] = val;
}

template <typename T>
__global__ void f32_to_act_kernel(const float* src, T* dst, size_t n) {
  size_t i = blockIdx.x * static_cast<size_t>(blockDim.x) + threadIdx.x;
  if (i < n) dst[i] = ActTraits<T>::from_f(src[i]);
}

// ---------------------------------------------------------------------------- launchers
// Launch with programmatic stream serialisation (see griddep_* in common.cuh) unless the
// calling context disabled it (llm_set_option LLM_OPT_PDL); the flag is per host thread.
thread_local bool t_use_pdl = true;
// Scheduling priority of the next launches (0 = the stream's own).  The overlapped decode
// schedule raises it for the projection and row kernels so their CTAs are dispatched ahead of
// the other micro-batch's pending attention CTAs.
thread_local int t_prio = 0;
// When set, the next launch records this event once all its CTAs have begun execution
// (launch completion); the overlapped schedule chains the micro-batches' attention launches on it.
thread_local cudaEvent_t t_lc_event = nullptr;
// When > 1, the next launch groups its CTAs in clusters of this many along grid z.
thread_local int t_cluster_z = 1;
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[4];
  int na = 0;
  if (t_cluster_z > 1) {
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = 1;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = static_cast<unsigned>(t_cluster_z);
    ++na;
  }
  if (t_lc_event != nullptr) {
    attr[na].id = cudaLaunchAttributeLaunchCompletionEvent;
    attr[na].val.launchCompletionEvent.event = t_lc_event;
    attr[na].val.launchCompletionEvent.flags = 0;
    ++na;
  }
  if (t_use_pdl) {
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (t_prio != 0) {
    attr[na].id = cudaLaunchAttributePriority;
    attr[na].val.priority = t_prio;
    ++na;
  }
  cfg.attrs = attr;
  cfg.numAttrs = na;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}
template <typename InT, typename OutT, int BM, int EPI>
cudaError_t gemm_launch_t(const GemmParams& p, dim3 grid, cudaStream_t s, bool prepare) {
  constexpr int BN = 128, ST = 4;
  constexpr int smem = gemm_smem_bytes<BM, BN, ST>();
  auto k = gemm_kernel<InT, OutT, BM, BN, ST, EPI>;
  if (prepare) return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  (void)cudaGetLastError();
  k<<<grid, kGemmThreads, smem, s>>>(p);
  return cudaGetLastError();
}

template <typename InT, typename OutT>
cudaError_t gemm_dispatch(const GemmParams& p, int epi, int bm, dim3 grid, cudaStream_t s, bool prepare) {
#define LLM_GEMM_CASE(E)                                                                    \
  case E:                                                                                   \
    return bm == 64 ? gemm_launch_t<InT, OutT, 64, E>(p, grid, s, prepare)                  \
                    : gemm_launch_t<InT, OutT, 128, E>(p, grid, s, prepare);
  switch (epi) {
    LLM_GEMM_CASE(EPI_F32)
    LLM_GEMM_CASE(EPI_S32)
    LLM_GEMM_CASE(EPI_RESID)
    LLM_GEMM_CASE(EPI_SWIGLU)
    LLM_GEMM_CASE(EPI_QKV)
    LLM_GEMM_CASE(EPI_ARGMAX)
  }
#undef LLM_GEMM_CASE
  return cudaErrorInvalidValue;
}

// act: 1 = fp16, 2 = bf16; in8: int8 A/B
cudaError_t gemm_any(int act, bool in8, const GemmParams& p, int epi, int bm, dim3 grid, cudaStream_t s,
                     bool prepare) {
  if (in8) return act == 1 ? gemm_dispatch<int8_t, __half>(p, epi, bm, grid, s, prepare)
                           : gemm_dispatch<int8_t, __nv_bfloat16>(p, epi, bm, grid, s, prepare);
  return act == 1 ? gemm_dispatch<__half, __half>(p, epi, bm, grid, s, prepare)
                  : gemm_dispatch<__nv_bfloat16, __nv_bfloat16>(p, epi, bm, grid, s, prepare);
}

template <typename T, int HD>
cudaError_t attn_launch_t(const AttnParams& p, cudaStream_t s, bool prepare) {
  auto k = attn_kernel<T, HD>;
  constexpr int smem = AttnCfg<T, HD>::SMEM;
  if (prepare) return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  dim3 grid(p.n_blocks, p.n_kv_heads, p.splits);
  (void)cudaGetLastError();
  return launch_pdl(k, grid, dim3(kAttnWarps * 32), smem, s, p);
}

template <typename T, int HD>
cudaError_t attn_prefill_launch_t(const PrefillAttnParams& p, cudaStream_t s, bool prepare) {
  auto k = attn_prefill_kernel<T, HD>;
  constexpr int smem = PrefillCfg<T, HD>::SMEM;
  if (prepare) return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  (void)cudaGetLastError();
  return launch_pdl(k, dim3(p.n_tiles * p.n_kv_heads), dim3(kPrefillWarps * 32), smem, s, p);
}

cudaError_t attn_prefill_any(int act, int hd, const PrefillAttnParams& p, cudaStream_t s, bool prepare) {
  if (act == 1) return hd == 64 ? attn_prefill_launch_t<__half, 64>(p, s, prepare) : attn_prefill_launch_t<__half, 128>(p, s, prepare);
  return hd == 64 ? attn_prefill_launch_t<__nv_bfloat16, 64>(p, s, prepare)
                  : attn_prefill_launch_t<__nv_bfloat16, 128>(p, s, prepare);
}

template <typename T, int HD>
cudaError_t attn_prefill_tc_launch_t(const PrefillAttnParams& p, cudaStream_t s, bool prepare) {
  auto k = attn_prefill_tc_kernel<T, HD>;
  constexpr int smem = PrefillTcCfg<T, HD>::SMEM;
  if (prepare) return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  (void)cudaGetLastError();
  return launch_pdl(k, dim3(p.n_tiles * p.n_kv_heads), dim3(192), smem, s, p);
}

cudaError_t attn_prefill_tc_any(int act, int hd, const PrefillAttnParams& p, cudaStream_t s, bool prepare) {
  if (act == 1)
    return hd == 64 ? attn_prefill_tc_launch_t<__half, 64>(p, s, prepare) : attn_prefill_tc_launch_t<__half, 128>(p, s, prepare);
  return hd == 64 ? attn_prefill_tc_launch_t<__nv_bfloat16, 64>(p, s, prepare)
                  : attn_prefill_tc_launch_t<__nv_bfloat16, 128>(p, s, prepare);
}

cudaError_t attn_any(int act, int hd, const AttnParams& p, cudaStream_t s, bool prepare) {
  if (act == 1) return hd == 64 ? attn_launch_t<__half, 64>(p, s, prepare) : attn_launch_t<__half, 128>(p, s, prepare);
  return hd == 64 ? attn_launch_t<__nv_bfloat16, 64>(p, s, prepare)
                  : attn_launch_t<__nv_bfloat16, 128>(p, s, prepare);
}

template <typename T, bool Q>
cudaError_t norm_launch(const NormParams& p, cudaStream_t s) {
  (void)cudaGetLastError();
  const int G = norm_groups_per_thread(p.D), W = norm_threads(p.D) / 32;
  const dim3 wgrid((p.rows + kNormWarpRows - 1) / kNormWarpRows), wblock(kNormWarpRows * 32);
  // One warp per row for prefill-sized RMSNorms (measured: 4096 rows x 1024, 14.4 -> 8.2 us); the
  // CTA-per-row kernel for decode-sized launches and the quantise-only rows, where its shorter
  // per-thread float64 chains measured faster (Stories W8A8 decode step 0.99 vs 1.07 ms, SwiGLU
  // output 3072 wide: 16.7 vs 28 us; a two-pass warp-per-row quantiser without the float64
  // layout was slower as well: Qwen3 W8A8 prefill of 16 x 1024 tokens 28.5 vs 25.9 ms).
  if (p.w != nullptr && p.rows >= 1024) {
#define LLM_NORM_WARP(g, w) \
  if (G == g && W == w) return launch_pdl(norm_rows_warp_kernel<T, Q, g, w>, wgrid, wblock, 0, s, p);
  LLM_NORM_WARP(1, 1) LLM_NORM_WARP(1, 2) LLM_NORM_WARP(1, 3)
  LLM_NORM_WARP(2, 2) LLM_NORM_WARP(2, 3) LLM_NORM_WARP(2, 4) LLM_NORM_WARP(2, 6) LLM_NORM_WARP(2, 8)
  LLM_NORM_WARP(2, 12)
#undef LLM_NORM_WARP
  }
  const dim3 block(norm_threads(p.D));
  if (G == 2) return launch_pdl(norm_rows_kernel<T, Q, 2>, dim3(p.rows), block, 0, s, p);
  return launch_pdl(norm_rows_kernel<T, Q, 1>, dim3(p.rows), block, 0, s, p);
}

cudaError_t norm_any(int act, bool quant, const NormParams& p, cudaStream_t s) {
  if (p.D > kNormMaxD || p.D % (4 * norm_groups_per_thread(p.D)) || norm_threads(p.D) % 32 || p.rows <= 0)
    return cudaErrorInvalidValue;
  if (act == 1) return quant ? norm_launch<__half, true>(p, s) : norm_launch<__half, false>(p, s);
  return quant ? norm_launch<__nv_bfloat16, true>(p, s) : norm_launch<__nv_bfloat16, false>(p, s);
}

// ---------------------------------------------------------------------------- tcgen05 GEMM
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_tiled() {
  static EncodeTiledFn fn = nullptr;
  static bool tried = false;
  if (!tried) {
    tried = true;
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  }
  return fn;
}

// 2-D K-major tensor map: rows x k_elems elements of `esz` bytes (act type when esz == 2),
// box = 128 bytes of K x box_rows rows, 128-byte swizzle, zero fill out of bounds.
int make_kmajor_map(CUtensorMap* map, const void* ptr, int esz, bool bf16, int k_elems, int rows, int box_rows) {
  EncodeTiledFn fn = encode_tiled();
  if (!fn) return fail(LLM_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  const CUtensorMapDataType dt = esz == 1 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                                          : (bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(k_elems), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(k_elems) * esz};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(128 / esz), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, dt, 2, const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(LLM_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d) rows=%d k=%d box=%d", (int)r, rows, k_elems, box_rows);
  return LLM_OK;
}

template <typename InT, typename OutT, int BN, int EPI>
cudaError_t umma_launch_t(const CUtensorMap& tx, const CUtensorMap& tw, const GemmParams& p, dim3 grid, cudaStream_t s,
                          bool prepare) {
  constexpr int smem = umma_smem_bytes<BN>();
  static_assert(smem <= 200 * 1024, "stage ring exceeds the shared-memory budget");
  // split-K clusters (k_splits > 1) run their own instantiation: residual and plain outputs
  constexpr bool kSplittable = EPI == EPI_RESID || EPI == EPI_F32 || EPI == EPI_S32;
  auto k = umma_gemm_kernel<InT, OutT, BN, EPI, false>;
  if constexpr (kSplittable) {
    auto ks = umma_gemm_kernel<InT, OutT, BN, EPI, true>;
    if (prepare) {
      const cudaError_t e = cudaFuncSetAttribute(ks, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
      if (e != cudaSuccess) return e;
    } else if (p.k_splits > 1) {
      (void)cudaGetLastError();
      return launch_pdl(ks, grid, dim3(kUmmaThreads), umma_smem_bytes_for<BN>(p.stages), s, tx, tw, p);
    }
  } else {
    if (!prepare && p.k_splits > 1) return cudaErrorInvalidValue;
  }
  if (prepare) return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  (void)cudaGetLastError();  // launch errors below must be this launch's own
  return launch_pdl(k, grid, dim3(kUmmaThreads), umma_smem_bytes_for<BN>(p.stages), s, tx, tw, p);
}

// Channel-tile widths each epilogue is built for (QKV: one head per tile; argmax: 256).
bool umma_bn_supported(int epi, int bn) {
  switch (epi) {
    case EPI_QKV: return bn == 64 || bn == 128;
    case EPI_ARGMAX: return bn == 256;
    case EPI_SWIGLU: return bn == 32 || bn == 64 || bn == 128 || bn == 256;
    default: return bn == 16 || bn == 32 || bn == 64 || bn == 128 || bn == 256;
  }
}

template <typename InT, typename OutT, int BN, int EPI>
cudaError_t umma_persist_launch_t(const CUtensorMap& tx, const CUtensorMap& tw, const GemmParams& p, dim3 grid,
                                  cudaStream_t s, bool prepare) {
  constexpr int smem = PersistCfg<BN, EPI>::SMEM;
  auto k = umma_persist_kernel<InT, OutT, BN, EPI>;
  if (prepare) return cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  (void)cudaGetLastError();
  return launch_pdl(k, grid, dim3(PersistCfg<BN, EPI>::THREADS), smem, s, tx, tw, p);
}

// Persistent prefill projections: QKV (one head per tile), residual and SwiGLU at 128 columns.
bool umma_persist_supported(int epi, int bn) {
  return (epi == EPI_QKV && (bn == 64 || bn == 128)) || ((epi == EPI_RESID || epi == EPI_SWIGLU) && bn == 128);
}

template <typename InT, typename OutT>
cudaError_t umma_persist_dispatch(const CUtensorMap& tx, const CUtensorMap& tw, const GemmParams& p, int epi, int bn,
                                  dim3 grid, cudaStream_t s, bool prepare) {
  if (epi == EPI_QKV && bn == 64) return umma_persist_launch_t<InT, OutT, 64, EPI_QKV>(tx, tw, p, grid, s, prepare);
  if (epi == EPI_QKV && bn == 128) return umma_persist_launch_t<InT, OutT, 128, EPI_QKV>(tx, tw, p, grid, s, prepare);
  if (epi == EPI_RESID && bn == 128) return umma_persist_launch_t<InT, OutT, 128, EPI_RESID>(tx, tw, p, grid, s, prepare);
  if (epi == EPI_SWIGLU && bn == 128) return umma_persist_launch_t<InT, OutT, 128, EPI_SWIGLU>(tx, tw, p, grid, s, prepare);
  return cudaErrorInvalidValue;
}

cudaError_t umma_persist_any(int act, bool in8, const CUtensorMap& tx, const CUtensorMap& tw, const GemmParams& p,
                             int epi, int bn, dim3 grid, cudaStream_t s, bool prepare) {
  if (in8) return act == 1 ? umma_persist_dispatch<int8_t, __half>(tx, tw, p, epi, bn, grid, s, prepare)
                           : umma_persist_dispatch<int8_t, __nv_bfloat16>(tx, tw, p, epi, bn, grid, s, prepare);
  return act == 1 ? umma_persist_dispatch<__half, __half>(tx, tw, p, epi, bn, grid, s, prepare)
                  : umma_persist_dispatch<__nv_bfloat16, __nv_bfloat16>(tx, tw, p, epi, bn, grid, s, prepare);
}

template <typename InT, typename OutT, int EPI>
cudaError_t umma_dispatch_bn(const CUtensorMap& tx, const CUtensorMap& tw, const GemmParams& p, int bn, dim3 grid,
                             cudaStream_t s, bool prepare) {
  if constexpr (EPI == EPI_QKV) {
    if (bn == 64) return umma_launch_t<InT, OutT, 64, EPI>(tx, tw, p, grid, s, prepare);
    if (bn == 128) return umma_launch_t<InT, OutT, 128, EPI>(tx, tw, p, grid, s, prepare);
  } else if constexpr (EPI == EPI_ARGMAX) {
    if (bn == 256) return umma_launch_t<InT, OutT, 256, EPI>(tx, tw, p, grid, s, prepare);
  } else {
    if constexpr (EPI != EPI_SWIGLU)
      if (bn == 16) return umma_launch_t<InT, OutT, 16, EPI>(tx, tw, p, grid, s, prepare);
    if (bn == 32) return umma_launch_t<InT, OutT, 32, EPI>(tx, tw, p, grid, s, prepare);
    if (bn == 64) return umma_launch_t<InT, OutT, 64, EPI>(tx, tw, p, grid, s, prepare);
    if (bn == 128) return umma_launch_t<InT, OutT, 128, EPI>(tx, tw, p, grid, s, prepare);
    if (bn == 256) return umma_launch_t<InT, OutT, 256, EPI>(tx, tw, p, grid, s, prepare);
  }
  return cudaErrorInvalidValue;
}

template <typename InT, typename OutT>
cudaError_t umma_dispatch(const CUtensorMap& tx, const CUtensorMap& tw, const GemmParams& p, int epi, int bn, dim3 grid,
                          cudaStream_t s, bool prepare) {
  switch (epi) {
    case EPI_F32: return umma_dispatch_bn<InT, OutT, EPI_F32>(tx, tw, p, bn, grid, s, prepare);
    case EPI_S32: return umma_dispatch_bn<InT, OutT, EPI_S32>(tx, tw, p, bn, grid, s, prepare);
    case EPI_RESID: return umma_dispatch_bn<InT, OutT, EPI_RESID>(tx, tw, p, bn, grid, s, prepare);
    case EPI_SWIGLU: return umma_dispatch_bn<InT, OutT, EPI_SWIGLU>(tx, tw, p, bn, grid, s, prepare);
    case EPI_QKV: return umma_dispatch_bn<InT, OutT, EPI_QKV>(tx, tw, p, bn, grid, s, prepare);
    case EPI_ARGMAX: return umma_dispatch_bn<InT, OutT, EPI_ARGMAX>(tx, tw, p, bn, grid, s, prepare);
  }
  return cudaErrorInvalidValue;
}

cudaError_t umma_any(int act, bool in8, const CUtensorMap& tx, const CUtensorMap& tw, const GemmParams& p, int epi,
                     int bn, dim3 grid, cudaStream_t s, bool prepare) {
  if (in8) return act == 1 ? umma_dispatch<int8_t, __half>(tx, tw, p, epi, bn, grid, s, prepare)
                           : umma_dispatch<int8_t, __nv_bfloat16>(tx, tw, p, epi, bn, grid, s, prepare);
  return act == 1 ? umma_dispatch<__half, __half>(tx, tw, p, epi, bn, grid, s, prepare)
                  : umma_dispatch<__nv_bfloat16, __nv_bfloat16>(tx, tw, p, epi, bn, grid, s, prepare);
}

// Channel-tile width of a tcgen05 projection: QKV one head, argmax 256; otherwise the
// narrowest tile that still keeps the grid within one CTA per SM (decode: the most SMs
// streaming weights), or 256 when even that grid is larger (prefill).
int umma_bn_for(int M, int N, int epi, int head_dim, int n_sm, int max_bn = 256) {
  if (epi == EPI_QKV) return head_dim;
  if (epi == EPI_ARGMAX) return 256;
  const long long tm = (M + kUmmaTokens - 1) / kUmmaTokens;
  for (int bn : {16, 32, 64, 128, 256}) {
    if (!umma_bn_supported(epi, bn) || bn > max_bn) continue;
    if (tm * ((N + bn - 1) / bn) <= n_sm || bn == max_bn) return bn;
  }
  return max_bn;
}

// The greedy-argmax partials: one key per (row, lm_head channel tile).
int argmax_tile_width(bool umma) { return umma ? 256 : 128; }

struct GemmPlan {
  int bm = 128, splits = 1, kts = 1, tiles = 1;
  dim3 grid;
  size_t ws_floats = 0;
};

GemmPlan plan_gemm(int M, int N, int K, int esz, int n_sm, int force_splits, size_t ws_cap_floats) {
  GemmPlan pl;
  pl.bm = M <= 64 ? 64 : 128;
  const int mt = (M + pl.bm - 1) / pl.bm, nt = (N + 127) / 128;
  pl.tiles = mt * nt;
  const int k_tiles = K * esz / 128;
  const int occ = pl.bm == 64 ? 2 : 1;
  const int target = n_sm * occ;
  int splits = force_splits > 0 ? force_splits
                                : (pl.tiles >= target ? 1 : std::max(1, std::min(16, target / pl.tiles)));
  splits = std::max(1, std::min(splits, k_tiles));
  for (;;) {
    pl.kts = (k_tiles + splits - 1) / splits;
    pl.splits = (k_tiles + pl.kts - 1) / pl.kts;
    pl.ws_floats = pl.splits > 1 ? static_cast<size_t>(pl.splits) * pl.tiles * pl.bm * 128 : 0;
    if (pl.ws_floats <= ws_cap_floats || splits == 1) break;
    --splits;
  }
  if (pl.splits > 1 && pl.ws_floats > ws_cap_floats) {
    pl.splits = 1;
    pl.kts = k_tiles;
    pl.ws_floats = 0;
  }
  pl.grid = dim3(mt, nt, pl.splits);
  return pl;
}

}  // namespace

// Micro-batches of the overlapped decode schedule: at most kMaxParts, each >= 32 rows.
constexpr int kMaxParts = 4;
constexpr int kOverlapMinPartRows = 32;
// Split-attention tile counters (device array length).
constexpr int kCounters = 65536;

// ============================================================================ context
struct LayerW {
  void* wqkv = nullptr;  // [(q_dim + 2 kv_dim) x D]
  float* sqkv = nullptr;
  void* wo = nullptr;    // [D x q_dim]
  float* so = nullptr;
  void* w13 = nullptr;   // [2F x D], rows interleaved (W1[j], W3[j])
  float* s13 = nullptr;
  void* w2 = nullptr;    // [D x F]
  float* s2 = nullptr;
  float *rms_att = nullptr, *rms_ffn = nullptr, *q_norm = nullptr, *k_norm = nullptr;
};

#ifndef LLM_QKV_TILE64_DEFAULT
#define LLM_QKV_TILE64_DEFAULT 1
#endif
struct GraphKey {
  int n, splits, mode;  // mode: 0 = step, 1 = step + logits, 2 = generate
  bool operator<(const GraphKey& o) const { return std::tie(n, splits, mode) < std::tie(o.n, o.splits, o.mode); }
};

struct llm_ctx {
  llm_model_config cfg{};
  int dtype = 0, device = 0, act = 2, n_sm = 148;
  bool in8 = false;
  int q_dim = 0, kv_dim = 0, group = 1;
  cudaStream_t stream = nullptr;
  std::vector<void*> allocs;
  uint64_t bytes_weights = 0, bytes_kv = 0, bytes_other = 0;

  // weights
  bool weights_loaded = false;
  void* embed = nullptr;
  void* lm_head = nullptr;
  float* rms_final = nullptr;
  std::vector<LayerW> layers;
  float *rope_cos = nullptr, *rope_sin = nullptr;

  // paged KV
  bool kv_ready = false;
  void* kv_pool = nullptr;
  int n_pages = 0, max_seqs = 0, max_pos = 0, max_pages_per_seq = 0;
  int* d_block_table = nullptr;
  std::vector<int> h_block_table, seq_npages, free_pages;
  std::vector<uint32_t> seq_stamp;  // duplicate-sequence check: seq_stamp[s] == stamp_gen once seen
  uint32_t stamp_gen = 0;

  // activations (max_rows rows)
  int max_rows = 0;
  float* x = nullptr;
  void* xn = nullptr;
  int8_t* xq = nullptr;
  float* xs = nullptr;
  void* qbuf = nullptr;
  void* attn = nullptr;  // act or fp32
  int8_t* aq = nullptr;
  float* as = nullptr;
  void* gbuf = nullptr;  // act or fp32
  int8_t* gq = nullptr;
  float* gs = nullptr;
  void* xf = nullptr;
  unsigned long long* argmax_part = nullptr;
  float* logits = nullptr;
  size_t logits_rows = 0;
  float* logits_t = nullptr;  // llm_eval_window: channel-first logits [vocab][window]
  size_t logits_t_rows = 0;
  int *d_seq = nullptr, *d_tok = nullptr, *d_pos = nullptr, *d_next = nullptr, *d_gen_start = nullptr;
  int *d_blk_row0 = nullptr, *d_blk_nq = nullptr, *d_final = nullptr;
  int* d_gen_out = nullptr;
  size_t gen_out_cap = 0;
  int32_t* h_pin = nullptr;  // pinned staging
  size_t h_pin_ints = 0;
  float* ws = nullptr;
  size_t ws_floats = 0;
  int* counters = nullptr;
  int* row_counters = nullptr;  // [max_rows] fused attention-output quantisation
  int* d_err = nullptr;

  // generate state
  int gen_n = 0, gen_steps_done = 0, gen_max_steps = 0, gen_splits = 1;
  std::vector<int> gen_seq, gen_pos0;

  std::map<GraphKey, cudaGraphExec_t> graphs;
  bool use_graphs = true;
  bool use_umma = true;  // tcgen05 GEMMs (false: the warp-level mma.sync GEMMs)
  // programmatic dependent launch between the kernels of single-stream steps and prefill:
  // measured 2-8% faster on latency-bound steps (Stories110M fp16 x 64: 0.749 -> 0.692 ms;
  // Qwen3 bf16 x 128 at context 768: 3.79 -> 3.65 ms).  Overlapped steps do not use it (a
  // waiting dependent CTA holds SM resources the other micro-batches' attention needs), unless
  // chain_pdl.
  bool use_pdl = true;
  // Overlapped decode: the batch runs as micro-batches on their own streams whose attention
  // launches form a chain, so one micro-batch's projections and row kernels (latency-bound)
  // run while the others' attention (HBM-bound) streams the KV cache.
  int overlap = 1;  // 0 off, 1 when the step's K/V time covers the host launches, 2 always
  int overlap_ring_kb = 64;   // tcgen05 stage ring in overlap mode: fits beside two attention CTAs
  int attn_splits = 0;        // decode attention splits per sequence (0 = chosen per batch)
  bool decode_splitk = true;  // LLM_OPT_DECODE_SPLITK
  bool qkv_tile64 = LLM_QKV_TILE64_DEFAULT;  // 64-token QKV tiles when the grid allows
  bool null_tokens = false;   // llm_eval_window: token id -1 = a zero embedding row
  // how one micro-batch's attention launch waits for the other's: 0 = its completion,
  // 1 = all of its CTAs having started (launch-completion event)
  int attn_chain = 1;
  bool prefill_tiles = true;  // prefill attention by query tiles (attn_prefill_kernel)
  bool prefill_tc = true;     // ... on the tcgen05 tensor cores (attn_prefill_tc_kernel)
  bool prefill_persist = true;  // prefill projections on umma_persist_kernel
  // tcgen05 stage ring of prefill-sized GEMMs (0 = the full ring) and their channel tile
  // (0 = the widest supported): two 64 KB CTAs per SM measured fastest (Qwen3 W8A8 prefill of
  // 256 x 1516 tokens 1441 -> 1270 ms; Qwen3 bf16 306 -> 266 ms; Stories W8A8 33.2 -> 28.9 ms)
  int prefill_ring_kb = 64;
  int prefill_bn = 128;
  // layer arithmetic of the forward pass (llm_eval_window selects storiesane's for one call):
  // residual scale (0 = plain residual) and SiLU gate form, see GemmParams
  float resid_scale = 0.f;
  int silu_form = 0;
  // temperature sampling (llm_set_sampling): temperature <= 1e-6 = greedy
  float sample_temp = 0.f;
  double sample_inv_t = 0.0;
  uint64_t sample_seed = 0;
  unsigned long long* d_draws = nullptr;  // [max_seqs] draws so far per sequence slot
  int* d_sampled = nullptr;               // [max_rows]
  // llm_trace_step: per-launch timeline records (device) and their labels (host)
  bool tracing = false;
  TraceRec* d_trace = nullptr;
  std::vector<std::string> trace_labels;
  int micro_batches = 4;      // micro-batches of the overlapped schedule (2..kMaxParts)
  double step_kv_positions = 0;  // sum over the step's rows of their context lengths
  bool overlap_graphs = false;  // capture overlapped steps in CUDA graphs (eager launches measured faster)
  bool chain_pdl = false;       // overlap mode: programmatic dependent launch within projection chains
  cudaStream_t xstream[3] = {nullptr, nullptr, nullptr};  // micro-batches 1.. (0 runs on `stream`)
  cudaEvent_t ev_fork = nullptr, ev_join = nullptr, ev_att[4] = {nullptr, nullptr, nullptr, nullptr};
  int prio_hi = 0;  // greatest stream priority of the device
  std::map<std::tuple<const void*, int, int, int, int>, CUtensorMap> tmaps;

  // llm_profile_step: when non-null, enqueue_forward records an event after each launch
  std::vector<std::pair<const char*, cudaEvent_t>>* trace = nullptr;
};

namespace {

int dalloc(llm_ctx* c, void** p, size_t bytes, uint64_t* counter) {
  if (bytes == 0) bytes = 16;
  cudaError_t e = cudaMalloc(p, bytes);
  if (e != cudaSuccess) return fail(LLM_ERR_OOM, "cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
  c->allocs.push_back(*p);
  if (counter) *counter += bytes;
  return LLM_OK;
}
template <typename P>
int dalloc_t(llm_ctx* c, P** p, size_t bytes, uint64_t* counter) {
  void* v = nullptr;
  int rc = dalloc(c, &v, bytes, counter);
  *p = static_cast<P*>(v);
  return rc;
}

size_t act_bytes(const llm_ctx* c) { return 2; }

int set_device(const llm_ctx* c) {
  CU(cudaSetDevice(c->device));
  return LLM_OK;
}

int check_device_error(llm_ctx* c) {
  int h = 0;
  CU(cudaMemcpyAsync(&h, c->d_err, sizeof(int), cudaMemcpyDeviceToHost, c->stream));
  CU(cudaStreamSynchronize(c->stream));
  if (h != kDevOk) {
    CU(cudaMemsetAsync(c->d_err, 0, sizeof(int), c->stream));
    CU(cudaStreamSynchronize(c->stream));
    return fail(LLM_ERR_DEVICE, "kernel reported device error %d (%s)", h,
                h == kDevWaitTimeout ? "bounded wait expired" : (h == kDevBadPage ? "bad page index" : "unknown"));
  }
  return LLM_OK;
}

int prepare_kernels(llm_ctx* c) {
  const int epis[] = {EPI_F32, EPI_S32, EPI_RESID, EPI_SWIGLU, EPI_QKV, EPI_ARGMAX};
  GemmParams gp{};
  for (int e : epis)
    for (int bm : {64, 128}) {
      CU(gemm_any(c->act, false, gp, e, bm, dim3(1), c->stream, true));
      if (c->in8) CU(gemm_any(c->act, true, gp, e, bm, dim3(1), c->stream, true));
    }
  AttnParams ap{};
  CU(attn_any(c->act, c->cfg.head_dim, ap, c->stream, true));
  PrefillAttnParams pp{};
  CU(attn_prefill_any(c->act, c->cfg.head_dim, pp, c->stream, true));
  CU(attn_prefill_tc_any(c->act, c->cfg.head_dim, pp, c->stream, true));
  CUtensorMap dummy{};
  for (int e : epis)
    for (int bn : {16, 32, 64, 128, 256}) {
      if (!umma_bn_supported(e, bn)) continue;
      CU(umma_any(c->act, false, dummy, dummy, gp, e, bn, dim3(1), c->stream, true));
      if (c->in8) CU(umma_any(c->act, true, dummy, dummy, gp, e, bn, dim3(1), c->stream, true));
    }
  for (int e : epis)
    for (int bn : {64, 128, 256}) {
      if (!umma_persist_supported(e, bn)) continue;
      CU(umma_persist_any(c->act, false, dummy, dummy, gp, e, bn, dim3(1), c->stream, true));
      if (c->in8) CU(umma_persist_any(c->act, true, dummy, dummy, gp, e, bn, dim3(1), c->stream, true));
    }
  return LLM_OK;
}

}  // namespace

extern "C" int llm_ctx_create(const llm_model_config* cfg, int dtype, int device, llm_ctx** out) {
  if (!cfg || !out) return fail(LLM_ERR_INVALID, "nil config or output handle");
  *out = nullptr;
  const llm_model_config& k = *cfg;
  if (dtype < LLM_DTYPE_F16 || dtype > LLM_DTYPE_W8A8_BF16) return fail(LLM_ERR_INVALID, "unknown dtype %d", dtype);
  if (k.dim <= 0 || k.hidden <= 0 || k.n_layers <= 0 || k.n_heads <= 0 || k.n_kv_heads <= 0 || k.vocab <= 0 ||
      k.max_seq <= 0)
    return fail(LLM_ERR_INVALID, "config dimensions must be positive");
  if (k.head_dim != 64 && k.head_dim != 128) return fail(LLM_ERR_UNSUPPORTED, "head_dim=%d (supported: 64, 128)", k.head_dim);
  if (k.n_heads % k.n_kv_heads) return fail(LLM_ERR_INVALID, "heads=%d not a multiple of kv_heads=%d", k.n_heads, k.n_kv_heads);
  const int group = k.n_heads / k.n_kv_heads;
  if (group > 8) return fail(LLM_ERR_UNSUPPORTED, "GQA group %d > 8", group);
  const int q_dim = k.n_heads * k.head_dim, kv_dim = k.n_kv_heads * k.head_dim;
  if (k.dim % 128 || k.hidden % 128 || q_dim % 128 || kv_dim % 128)
    return fail(LLM_ERR_UNSUPPORTED, "dim, hidden, heads*head_dim and kv_heads*head_dim must be multiples of 128");
  if (k.dim > kNormMaxD || k.hidden > kNormMaxD || q_dim > kNormMaxD)
    return fail(LLM_ERR_UNSUPPORTED, "rows wider than %d elements are not supported", kNormMaxD);
  if (!(k.norm_eps > 0)) return fail(LLM_ERR_INVALID, "norm_eps must be positive");
  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
    return fail(LLM_ERR_CUDA, "no CUDA device available (the token loop has no CPU fallback)");
  if (device < 0 || device >= ndev) return fail(LLM_ERR_INVALID, "device %d out of range (have %d)", device, ndev);

  llm_ctx* c = new llm_ctx();
  c->cfg = k;
  c->dtype = dtype;
  c->device = device;
  c->act = (dtype == LLM_DTYPE_F16 || dtype == LLM_DTYPE_W8A8_F16) ? 1 : 2;
  c->in8 = dtype >= LLM_DTYPE_W8A8_F16;
  c->q_dim = q_dim;
  c->kv_dim = kv_dim;
  c->group = group;
  auto bail = [&](int rc) {
    llm_ctx_destroy(c);
    return rc;
  };
  if (cudaSetDevice(device) != cudaSuccess) return bail(fail(LLM_ERR_CUDA, "cudaSetDevice(%d) failed", device));
  cudaDeviceProp prop{};
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return bail(fail(LLM_ERR_CUDA, "device query failed"));
  if (prop.major < 10) return bail(fail(LLM_ERR_UNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a", device, prop.major, prop.minor));
  c->n_sm = prop.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess)
    return bail(fail(LLM_ERR_CUDA, "stream create failed"));
  for (cudaStream_t& xs : c->xstream)
    if (cudaStreamCreateWithFlags(&xs, cudaStreamNonBlocking) != cudaSuccess)
      return bail(fail(LLM_ERR_CUDA, "stream create failed"));
  for (cudaEvent_t* e : {&c->ev_fork, &c->ev_join, &c->ev_att[0], &c->ev_att[1], &c->ev_att[2], &c->ev_att[3]})
    if (cudaEventCreateWithFlags(e, cudaEventDisableTiming) != cudaSuccess)
      return bail(fail(LLM_ERR_CUDA, "event create failed"));
  {
    int least = 0, greatest = 0;
    if (cudaDeviceGetStreamPriorityRange(&least, &greatest) == cudaSuccess) c->prio_hi = greatest;
  }
  // RoPE tables in float64, as ane/stories/infer.go:97-107
  const int half = k.head_dim / 2;
  std::vector<float> hc(static_cast<size_t>(k.max_seq) * half), hs(hc.size());
  for (int pos = 0; pos < k.max_seq; ++pos)
    for (int i = 0; i < half; ++i) {
      const double freq = static_cast<double>(pos) / std::pow(k.rope_theta, static_cast<double>(2 * i) / k.head_dim);
      hc[static_cast<size_t>(pos) * half + i] = static_cast<float>(std::cos(freq));
      hs[static_cast<size_t>(pos) * half + i] = static_cast<float>(std::sin(freq));
    }
  int rc = dalloc_t(c, &c->rope_cos, hc.size() * 4, &c->bytes_other);
  if (!rc) rc = dalloc_t(c, &c->rope_sin, hs.size() * 4, &c->bytes_other);
  if (!rc) rc = dalloc_t(c, &c->d_err, 4, &c->bytes_other);
  if (rc) return bail(rc);
  // every upload is ordered on the context's (non-blocking) stream: a synchronous copy on the
  // legacy stream may still be in flight when that stream's kernels start
  if (cudaMemcpyAsync(c->rope_cos, hc.data(), hc.size() * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
      cudaMemcpyAsync(c->rope_sin, hs.data(), hs.size() * 4, cudaMemcpyHostToDevice, c->stream) != cudaSuccess ||
      cudaMemsetAsync(c->d_err, 0, 4, c->stream) != cudaSuccess || cudaStreamSynchronize(c->stream) != cudaSuccess)
    return bail(fail(LLM_ERR_CUDA, "table upload failed"));
  rc = prepare_kernels(c);
  if (rc) return bail(rc);
  *out = c;
  return LLM_OK;
}

extern "C" int llm_ctx_destroy(llm_ctx* c) {
  if (!c) return fail(LLM_ERR_INVALID, "nil context");
  cudaSetDevice(c->device);
  if (c->stream) cudaStreamSynchronize(c->stream);
  for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second);
  for (void* p : c->allocs) cudaFree(p);
  if (c->h_pin) cudaFreeHost(c->h_pin);
  for (cudaStream_t xs : c->xstream)
    if (xs) cudaStreamSynchronize(xs);
  for (cudaEvent_t e : {c->ev_fork, c->ev_join, c->ev_att[0], c->ev_att[1], c->ev_att[2], c->ev_att[3]})
    if (e) cudaEventDestroy(e);
  for (cudaStream_t xs : c->xstream)
    if (xs) cudaStreamDestroy(xs);
  if (c->stream) cudaStreamDestroy(c->stream);
  delete c;
  return LLM_OK;
}

// ============================================================================ weights
namespace {

// Convert one fp32 host tensor [rows x cols] into device storage; int8 when `quant`.
int upload_convert(llm_ctx* c, float* dtmp, const float* src, int rows, int cols, void* dst, float* dscale,
                   bool quant, int row_mul, int row_add) {
  const size_t n = static_cast<size_t>(rows) * cols;
  CU(cudaMemcpyAsync(dtmp, src, n * 4, cudaMemcpyHostToDevice, c->stream));
  ConvertParams p{dtmp, rows, cols, row_mul, row_add, dst, dscale};
  dim3 grid((rows + 7) / 8);
  if (quant) convert_rows_kernel<int8_t><<<grid, 256, 0, c->stream>>>(p);
  else if (c->act == 1) convert_rows_kernel<__half><<<grid, 256, 0, c->stream>>>(p);
  else convert_rows_kernel<__nv_bfloat16><<<grid, 256, 0, c->stream>>>(p);
  CU(cudaGetLastError());
  CU(cudaStreamSynchronize(c->stream));  // dtmp is reused by the next tensor
  return LLM_OK;
}

int upload_f32(llm_ctx* c, float** dst, const float* src, size_t n, float fill) {
  RC(dalloc_t(c, dst, n * 4, &c->bytes_weights));
  if (src) {
    CU(cudaMemcpyAsync(*dst, src, n * 4, cudaMemcpyHostToDevice, c->stream));
    CU(cudaStreamSynchronize(c->stream));
  } else {
    std::vector<float> ones(n, fill);
    CU(cudaMemcpyAsync(*dst, ones.data(), n * 4, cudaMemcpyHostToDevice, c->stream));
    CU(cudaStreamSynchronize(c->stream));
  }
  return LLM_OK;
}

// A weight file read tensor by tensor: byte offset of every tensor, the file's norm weights
// (read whole), and a reader that pulls one matrix into host memory on demand.
struct FileTensors {
  FILE* f = nullptr;
  std::string path;
  // offsets (bytes) of kind 0..6 = wq,wk,wv,wo,w1,w2,w3 per layer, embed
  std::vector<std::array<int64_t, 7>> off;
  int64_t embed_off = 0;
  std::vector<std::vector<float>> rms_att, rms_ffn;
  std::vector<float> rms_final;
  std::vector<llm_layer_weights_f32> layer_norms;
  ~FileTensors() {
    if (f) fclose(f);
  }
  int read_at(int64_t off, float* dst, size_t n, const char* what) {
    if (fseeko(f, off, SEEK_SET) != 0) return fail(LLM_ERR_INVALID, "read %s: seek failed", what);
    const size_t got = fread(dst, 4, n, f);
    if (got != n) return fail(LLM_ERR_INVALID, "read %s: %s", what, got == 0 ? "EOF" : "unexpected EOF");
    return LLM_OK;
  }
};

// Tensor source: caller fp32 pointers, a weight file, or the synthetic generator.
struct Source {
  const llm_model_weights_f32* w = nullptr;
  FileTensors* file = nullptr;
  int file_rc = LLM_OK;
  uint64_t seed = 0;
  float out_scale = 1.f;
  std::vector<float> host;  // synthetic / file scratch
  const float* get(int layer, int kind, size_t n) {
    if (file) {
      static const char* names[9] = {"wq", "wk", "wv", "wo", "w1", "w2", "w3", "embed", "lm_head"};
      if (kind == 8) return nullptr;
      host.resize(n);
      char what[32];
      snprintf(what, sizeof what, kind == 7 ? "%s" : "%s[%d]", names[kind], layer);
      const int64_t off = kind == 7 ? file->embed_off : file->off[layer][kind];
      file_rc = file->read_at(off, host.data(), n, what);
      return file_rc ? nullptr : host.data();
    }
    if (w) {
      if (kind == 7) return w->embed;
      if (kind == 8) return w->lm_head;
      const llm_layer_weights_f32& L = w->layers[layer];
      const float* t[7] = {L.wq, L.wk, L.wv, L.wo, L.w1, L.w2, L.w3};
      return t[kind];
    }
    host.resize(n);
    const double sc = (kind == 3 || kind == 5) ? out_scale : 1.0;
    llm_synth_normal(host.data(), n, seed, llm_synth_stream(layer, kind), 0.02, sc);
    return host.data();
  }
};

int load_weights(llm_ctx* c, Source& src) {
  if (c->weights_loaded) return fail(LLM_ERR_STATE, "weights already loaded");
  RC(set_device(c));
  const llm_model_config& k = c->cfg;
  const int D = k.dim, F = k.hidden, V = k.vocab, Q = c->q_dim, KV = c->kv_dim;
  const size_t ab = act_bytes(c);
  const size_t wb = c->in8 ? 1 : ab;
  size_t maxn = std::max({static_cast<size_t>(V) * D, static_cast<size_t>(F) * D, static_cast<size_t>(Q) * D});
  float* dtmp = nullptr;
  {
    void* v = nullptr;
    CU(cudaMalloc(&v, maxn * 4));
    dtmp = static_cast<float*>(v);
  }
  auto cleanup = [&](int rc) {
    cudaFree(dtmp);
    return rc;
  };
  int rc;
  if ((rc = dalloc(c, &c->embed, static_cast<size_t>(V) * D * ab, &c->bytes_weights))) return cleanup(rc);
  const float* e = src.get(0, 7, static_cast<size_t>(V) * D);
  if (!e) return cleanup(src.file_rc ? src.file_rc : fail(LLM_ERR_INVALID, "nil embed"));
  if ((rc = upload_convert(c, dtmp, e, V, D, c->embed, nullptr, false, 1, 0))) return cleanup(rc);
  if (k.tied_embed) {
    c->lm_head = c->embed;
  } else {
    const float* lh = src.get(0, 8, static_cast<size_t>(V) * D);
    if (!lh) return cleanup(fail(LLM_ERR_INVALID, "untied model needs lm_head"));
    if ((rc = dalloc(c, &c->lm_head, static_cast<size_t>(V) * D * ab, &c->bytes_weights))) return cleanup(rc);
    if ((rc = upload_convert(c, dtmp, lh, V, D, c->lm_head, nullptr, false, 1, 0))) return cleanup(rc);
  }
  const float* rms_final = src.w ? src.w->rms_final : (src.file ? src.file->rms_final.data() : nullptr);
  if ((rc = upload_f32(c, &c->rms_final, rms_final, D, 1.f))) return cleanup(rc);
  c->layers.resize(k.n_layers);
  const int NQKV = Q + 2 * KV;
  for (int l = 0; l < k.n_layers; ++l) {
    LayerW& L = c->layers[l];
    if ((rc = dalloc(c, &L.wqkv, static_cast<size_t>(NQKV) * D * wb, &c->bytes_weights))) return cleanup(rc);
    if ((rc = dalloc(c, &L.wo, static_cast<size_t>(D) * Q * wb, &c->bytes_weights))) return cleanup(rc);
    if ((rc = dalloc(c, &L.w13, static_cast<size_t>(2 * F) * D * wb, &c->bytes_weights))) return cleanup(rc);
    if ((rc = dalloc(c, &L.w2, static_cast<size_t>(D) * F * wb, &c->bytes_weights))) return cleanup(rc);
    if (c->in8) {
      if ((rc = dalloc_t(c, &L.sqkv, NQKV * 4, &c->bytes_weights))) return cleanup(rc);
      if ((rc = dalloc_t(c, &L.so, D * 4, &c->bytes_weights))) return cleanup(rc);
      if ((rc = dalloc_t(c, &L.s13, 2 * F * 4, &c->bytes_weights))) return cleanup(rc);
      if ((rc = dalloc_t(c, &L.s2, D * 4, &c->bytes_weights))) return cleanup(rc);
    }
    auto part = [&](int kind, int rows, int cols, void* base, float* sbase, int row_off, int mul, int add) -> int {
      const float* s = src.get(l, kind, static_cast<size_t>(rows) * cols);
      if (!s) return src.file_rc ? src.file_rc : fail(LLM_ERR_INVALID, "nil weight (layer %d, tensor %d)", l, kind);
      uint8_t* dst = static_cast<uint8_t*>(base) + static_cast<size_t>(row_off) * cols * wb;
      float* ds = sbase ? sbase + row_off : nullptr;
      return upload_convert(c, dtmp, s, rows, cols, dst, ds, c->in8, mul, add);
    };
    if ((rc = part(0, Q, D, L.wqkv, L.sqkv, 0, 1, 0))) return cleanup(rc);
    if ((rc = part(1, KV, D, L.wqkv, L.sqkv, Q, 1, 0))) return cleanup(rc);
    if ((rc = part(2, KV, D, L.wqkv, L.sqkv, Q + KV, 1, 0))) return cleanup(rc);
    if ((rc = part(3, D, Q, L.wo, L.so, 0, 1, 0))) return cleanup(rc);
    if ((rc = part(4, F, D, L.w13, L.s13, 0, 2, 0))) return cleanup(rc);
    if ((rc = part(6, F, D, L.w13, L.s13, 0, 2, 1))) return cleanup(rc);
    if ((rc = part(5, D, F, L.w2, L.s2, 0, 1, 0))) return cleanup(rc);
    const llm_layer_weights_f32* lw =
        src.w ? &src.w->layers[l] : (src.file ? &src.file->layer_norms[l] : nullptr);
    if ((rc = upload_f32(c, &L.rms_att, lw ? lw->rms_att : nullptr, D, 1.f))) return cleanup(rc);
    if ((rc = upload_f32(c, &L.rms_ffn, lw ? lw->rms_ffn : nullptr, D, 1.f))) return cleanup(rc);
    if (k.qk_norm) {
      if ((rc = upload_f32(c, &L.q_norm, lw ? lw->q_norm : nullptr, k.head_dim, 1.f))) return cleanup(rc);
      if ((rc = upload_f32(c, &L.k_norm, lw ? lw->k_norm : nullptr, k.head_dim, 1.f))) return cleanup(rc);
    }
    if (lw && (!lw->rms_att || !lw->rms_ffn || (k.qk_norm && (!lw->q_norm || !lw->k_norm))))
      return cleanup(fail(LLM_ERR_INVALID, "nil norm weight in layer %d", l));
  }
  c->weights_loaded = true;
  return cleanup(LLM_OK);
}

}  // namespace

extern "C" int llm_load_weights_f32(llm_ctx* c, const llm_model_weights_f32* w) {
  if (!c || !w || !w->layers || !w->embed || !w->rms_final) return fail(LLM_ERR_INVALID, "nil context or weights");
  Source s;
  s.w = w;
  return load_weights(c, s);
}

namespace {

// ane/stories/weights.go:49-122: header of 7 int32 (dim, hidden, layers, heads, kv_heads,
// vocab, seq_len; vocab < 0 = the file also holds an unshared classifier, which the reference
// does not read), embed, then each kind for all layers: rms_att, wq, wk, wv, wo, rms_ffn, w1,
// w2, w3, then rms_final.  The classifier is the embedding (infer.go:243).
int scan_llama2c(const llm_ctx* c, FileTensors& ft) {
  const llm_model_config& k = c->cfg;
  int32_t h[7];
  if (fread(h, 4, 7, ft.f) != 7) return fail(LLM_ERR_INVALID, "read config: unexpected EOF");
  const int Q = c->q_dim, KV = c->kv_dim, D = k.dim, F = k.hidden, L = k.n_layers;
  if (h[0] != D || h[1] != F || h[2] != L)
    return fail(LLM_ERR_INVALID, "config mismatch: got dim=%d hidden=%d layers=%d", h[0], h[1], h[2]);
  if (h[3] != k.n_heads || h[4] != k.n_kv_heads || std::abs(h[5]) != k.vocab)
    return fail(LLM_ERR_INVALID, "config mismatch: got heads=%d kv_heads=%d vocab=%d", h[3], h[4], std::abs(h[5]));
  if (!k.tied_embed) return fail(LLM_ERR_UNSUPPORTED, "llama2.c weight files are read with the embedding as classifier (tied)");
  int64_t o = 28;
  ft.embed_off = o;
  o += 4ll * k.vocab * D;
  const int64_t rms_att = o;
  o += 4ll * L * D;
  ft.off.assign(L, {});
  const int64_t sizes[7] = {4ll * Q * D, 4ll * KV * D, 4ll * KV * D, 4ll * D * Q, 4ll * F * D, 4ll * D * F, 4ll * F * D};
  // wq, wk, wv, wo
  for (int kind = 0; kind < 4; ++kind)
    for (int l = 0; l < L; ++l) {
      ft.off[l][kind] = o;
      o += sizes[kind];
    }
  const int64_t rms_ffn = o;
  o += 4ll * L * D;
  // w1, w2, w3 (file order)
  for (int kind : {4, 5, 6})
    for (int l = 0; l < L; ++l) {
      ft.off[l][kind] = o;
      o += sizes[kind];
    }
  const int64_t rms_final = o;
  ft.rms_att.assign(L, std::vector<float>(D));
  ft.rms_ffn.assign(L, std::vector<float>(D));
  ft.rms_final.resize(D);
  char what[32];
  for (int l = 0; l < L; ++l) {
    snprintf(what, sizeof what, "rms_att[%d]", l);
    RC(ft.read_at(rms_att + 4ll * l * D, ft.rms_att[l].data(), D, what));
    snprintf(what, sizeof what, "rms_ffn[%d]", l);
    RC(ft.read_at(rms_ffn + 4ll * l * D, ft.rms_ffn[l].data(), D, what));
  }
  RC(ft.read_at(rms_final, ft.rms_final.data(), D, "rms_final"));
  return LLM_OK;
}

// ane/stories/ckpt.go:237-447 with no optimizer state wanted: a 96-byte header (magic
// 0x424C5A54, version 2 or 3, step, total steps, layers, vocab, dim, hidden, heads, seq, lr,
// loss, three f64 timers, three int32 counters, three int32 pads), then per layer wq, wk, wv,
// wo, w1, w2, w3, rms_att, rms_ffn; then every layer's Adam moments (skipped), rms_final, its
// moments (skipped), embed.
int scan_checkpoint(const llm_ctx* c, FileTensors& ft) {
  const llm_model_config& k = c->cfg;
  int32_t h[10];
  if (fread(h, 4, 2, ft.f) != 2) return fail(LLM_ERR_INVALID, "read checkpoint header: unexpected EOF");
  if (h[0] != 0x424C5A54 || (h[1] != 2 && h[1] != 3))
    return fail(LLM_ERR_INVALID, "bad checkpoint header magic=%x version=%d", static_cast<unsigned>(h[0]), h[1]);
  if (fread(h + 2, 4, 8, ft.f) != 8) return fail(LLM_ERR_INVALID, "read checkpoint header: unexpected EOF");
  if (h[4] != k.n_layers || h[5] != k.vocab || h[6] != k.dim || h[7] != k.hidden || h[8] != k.n_heads)
    return fail(LLM_ERR_INVALID, "checkpoint config mismatch");
  if (!k.tied_embed) return fail(LLM_ERR_UNSUPPORTED, "checkpoints hold one embedding, used as the classifier (tied)");
  const int Q = c->q_dim, KV = c->kv_dim, D = k.dim, F = k.hidden, L = k.n_layers;
  const int64_t sizes[7] = {4ll * Q * D, 4ll * KV * D, 4ll * KV * D, 4ll * D * Q, 4ll * F * D, 4ll * D * F, 4ll * F * D};
  int64_t o = 96;
  ft.off.assign(L, {});
  ft.rms_att.assign(L, std::vector<float>(D));
  ft.rms_ffn.assign(L, std::vector<float>(D));
  char what[32];
  for (int l = 0; l < L; ++l) {
    for (int kind = 0; kind < 7; ++kind) {
      ft.off[l][kind] = o;
      o += sizes[kind];
    }
    snprintf(what, sizeof what, "rms_att[%d]", l);
    RC(ft.read_at(o, ft.rms_att[l].data(), D, what));
    o += 4ll * D;
    snprintf(what, sizeof what, "rms_ffn[%d]", l);
    RC(ft.read_at(o, ft.rms_ffn[l].data(), D, what));
    o += 4ll * D;
  }
  int64_t layer_opt = 0;
  for (int kind = 0; kind < 7; ++kind) layer_opt += 2 * sizes[kind];
  layer_opt += 4 * 4ll * D;
  o += L * layer_opt;
  ft.rms_final.resize(D);
  RC(ft.read_at(o, ft.rms_final.data(), D, "rms_final"));
  o += 4ll * D + 2 * 4ll * D;
  ft.embed_off = o;
  return LLM_OK;
}

}  // namespace

extern "C" int llm_load_weights_file(llm_ctx* c, const char* path, int format) {
  if (!c || !path) return fail(LLM_ERR_INVALID, "nil context or path");
  if (format != LLM_WEIGHTS_LLAMA2C && format != LLM_WEIGHTS_CHECKPOINT)
    return fail(LLM_ERR_INVALID, "unknown weight file format %d", format);
  if (c->weights_loaded) return fail(LLM_ERR_STATE, "weights already loaded");
  if (c->cfg.qk_norm) return fail(LLM_ERR_UNSUPPORTED, "weight files carry no QK-norm weights");
  FileTensors ft;
  ft.path = path;
  ft.f = fopen(path, "rb");
  if (!ft.f) return fail(LLM_ERR_INVALID, "open %s: %s", path, strerror(errno));
  RC(format == LLM_WEIGHTS_LLAMA2C ? scan_llama2c(c, ft) : scan_checkpoint(c, ft));
  ft.layer_norms.resize(c->cfg.n_layers);
  for (int l = 0; l < c->cfg.n_layers; ++l) {
    ft.layer_norms[l] = llm_layer_weights_f32{};
    ft.layer_norms[l].rms_att = ft.rms_att[l].data();
    ft.layer_norms[l].rms_ffn = ft.rms_ffn[l].data();
  }
  Source s;
  s.file = &ft;
  return load_weights(c, s);
}

extern "C" int llm_load_weights_synthetic(llm_ctx* c, uint64_t seed, float out_proj_scale) {
  if (!c) return fail(LLM_ERR_INVALID, "nil context");
  Source s;
  s.seed = seed;
  s.out_scale = out_proj_scale;
  return load_weights(c, s);
}

// ============================================================================ KV cache
extern "C" int llm_kv_alloc(llm_ctx* c, int max_seqs, int max_pos, int page_tokens) {
  if (!c) return fail(LLM_ERR_INVALID, "nil context");
  if (c->kv_ready) return fail(LLM_ERR_STATE, "KV cache already allocated");
  if (page_tokens != 16) return fail(LLM_ERR_UNSUPPORTED, "page_tokens=%d (supported: 16)", page_tokens);
  if (max_seqs <= 0 || max_pos <= 0) return fail(LLM_ERR_INVALID, "max_seqs and max_pos must be positive");
  if (max_pos > c->cfg.max_seq) return fail(LLM_ERR_INVALID, "max_pos=%d exceeds the config's max_seq=%d", max_pos, c->cfg.max_seq);
  RC(set_device(c));
  const llm_model_config& k = c->cfg;
  c->max_seqs = max_seqs;
  c->max_pos = max_pos;
  c->max_pages_per_seq = (max_pos + 15) / 16;
  c->n_pages = max_seqs * c->max_pages_per_seq;
  const size_t page_bytes = static_cast<size_t>(k.n_kv_heads) * 2 * 16 * k.head_dim * act_bytes(c);
  RC(dalloc(c, &c->kv_pool, static_cast<size_t>(k.n_layers) * c->n_pages * page_bytes, &c->bytes_kv));
  CU(cudaMemsetAsync(c->kv_pool, 0, static_cast<size_t>(k.n_layers) * c->n_pages * page_bytes, c->stream));
  RC(dalloc_t(c, &c->d_block_table, static_cast<size_t>(max_seqs) * c->max_pages_per_seq * 4, &c->bytes_other));
  c->h_block_table.assign(static_cast<size_t>(max_seqs) * c->max_pages_per_seq, -1);
  CU(cudaMemcpyAsync(c->d_block_table, c->h_block_table.data(), c->h_block_table.size() * 4, cudaMemcpyHostToDevice,
                     c->stream));
  CU(cudaStreamSynchronize(c->stream));
  c->seq_npages.assign(max_seqs, 0);
  c->seq_stamp.assign(max_seqs, 0);
  c->stamp_gen = 0;
  // free list in a scrambled order so block tables are never the identity map
  int stride = c->n_pages / 2 + 1;
  while (std::gcd(stride, c->n_pages) != 1) ++stride;
  c->free_pages.resize(c->n_pages);
  for (int i = 0; i < c->n_pages; ++i)
    c->free_pages[c->n_pages - 1 - i] = static_cast<int>((static_cast<long long>(i) * stride) % c->n_pages);

  // activation buffers
  const int R = std::max(max_seqs, 4096);
  c->max_rows = R;
  const size_t D = k.dim, F = k.hidden, Q = c->q_dim, V = k.vocab, ab = act_bytes(c);
  uint64_t* o = &c->bytes_other;
  RC(dalloc_t(c, &c->x, R * D * 4, o));
  RC(dalloc(c, &c->xn, R * D * ab, o));
  RC(dalloc_t(c, &c->xq, R * D, o));
  RC(dalloc_t(c, &c->xs, R * 4, o));
  RC(dalloc(c, &c->qbuf, R * Q * ab, o));
  RC(dalloc(c, &c->attn, R * Q * 4, o));
  RC(dalloc_t(c, &c->aq, R * Q, o));
  RC(dalloc_t(c, &c->as, R * 4, o));
  RC(dalloc(c, &c->gbuf, R * F * 4, o));
  RC(dalloc_t(c, &c->gq, R * F, o));
  RC(dalloc_t(c, &c->gs, R * 4, o));
  RC(dalloc(c, &c->xf, R * D * ab, o));
  RC(dalloc_t(c, &c->argmax_part, ((V + 127) / 128) * R * 8, o));
  for (int** p : {&c->d_seq, &c->d_tok, &c->d_pos, &c->d_next, &c->d_gen_start, &c->d_blk_row0, &c->d_blk_nq, &c->d_final,
                   &c->d_sampled})
    RC(dalloc_t(c, p, R * 4, o));
  RC(dalloc_t(c, &c->d_draws, static_cast<size_t>(max_seqs) * 8, o));
  CU(cudaMemsetAsync(c->d_draws, 0, static_cast<size_t>(max_seqs) * 8, c->stream));
  c->ws_floats = 16u << 20;  // 64 MB split-K / split-attention workspace
  RC(dalloc_t(c, &c->ws, c->ws_floats * 4, o));
  RC(dalloc_t(c, &c->counters, kCounters * 4, o));
  CU(cudaMemsetAsync(c->counters, 0, kCounters * 4, c->stream));
  RC(dalloc_t(c, &c->row_counters, static_cast<size_t>(R) * 4, o));
  CU(cudaMemsetAsync(c->row_counters, 0, static_cast<size_t>(R) * 4, c->stream));
  c->h_pin_ints = static_cast<size_t>(R) * 8;
  CU(cudaMallocHost(&c->h_pin, c->h_pin_ints * 4));
  c->kv_ready = true;
  return LLM_OK;
}

extern "C" int llm_seq_release(llm_ctx* c, int seq) {
  if (!c || !c->kv_ready) return fail(LLM_ERR_STATE, "KV cache not allocated");
  if (seq < 0 || seq >= c->max_seqs) return fail(LLM_ERR_INVALID, "sequence %d out of range", seq);
  int* row = c->h_block_table.data() + static_cast<size_t>(seq) * c->max_pages_per_seq;
  for (int i = 0; i < c->seq_npages[seq]; ++i) {
    c->free_pages.push_back(row[i]);
    row[i] = -1;
  }
  c->seq_npages[seq] = 0;
  RC(set_device(c));
  CU(cudaMemcpyAsync(c->d_block_table + static_cast<size_t>(seq) * c->max_pages_per_seq, row,
                     c->max_pages_per_seq * 4, cudaMemcpyHostToDevice, c->stream));
  CU(cudaStreamSynchronize(c->stream));
  return LLM_OK;
}

namespace {

// Make sure sequence `seq` owns pages for positions [0, upto]; uploads changed rows.
int ensure_pages(llm_ctx* c, int seq, int upto, std::vector<int>* dirty) {
  const int need = upto / 16 + 1;
  if (need > c->max_pages_per_seq) return fail(LLM_ERR_POS_RANGE, "position out of range: %d", upto);
  int* row = c->h_block_table.data() + static_cast<size_t>(seq) * c->max_pages_per_seq;
  bool changed = false;
  while (c->seq_npages[seq] < need) {
    if (c->free_pages.empty()) return fail(LLM_ERR_OOM, "KV page pool exhausted");
    row[c->seq_npages[seq]++] = c->free_pages.back();
    c->free_pages.pop_back();
    changed = true;
  }
  if (changed) dirty->push_back(seq);
  return LLM_OK;
}

int upload_dirty(llm_ctx* c, std::vector<int>& dirty);

// Pages through position upto[i] for sequence seq[i], i < n (rows already validated).  If the
// pool runs out part way, the rows changed so far are still uploaded, so the device block
// table matches the host's before the error returns (those sequences keep their new pages).
int reserve_rows(llm_ctx* c, int n, const int32_t* seq, const int* upto) {
  std::vector<int> dirty;
  for (int i = 0; i < n; ++i) {
    const int rc = ensure_pages(c, seq[i], upto[i], &dirty);
    if (rc) {
      upload_dirty(c, dirty);
      return rc;
    }
  }
  return upload_dirty(c, dirty);
}

int upload_dirty(llm_ctx* c, std::vector<int>& dirty) {
  std::sort(dirty.begin(), dirty.end());
  dirty.erase(std::unique(dirty.begin(), dirty.end()), dirty.end());
  const size_t row = c->max_pages_per_seq;
  if (dirty.size() > 4) {
    // many rows change at once (a batch crossing a page boundary together): one copy of the
    // span of rows instead of one small copy per row
    const size_t lo = dirty.front(), hi = dirty.back();
    CU(cudaMemcpyAsync(c->d_block_table + lo * row, c->h_block_table.data() + lo * row, (hi - lo + 1) * row * 4,
                       cudaMemcpyHostToDevice, c->stream));
  } else {
    for (int s : dirty)
      CU(cudaMemcpyAsync(c->d_block_table + s * row, c->h_block_table.data() + s * row, row * 4,
                         cudaMemcpyHostToDevice, c->stream));
  }
  dirty.clear();
  return LLM_OK;
}

// Duplicate-sequence check of one call: start_stamp() once, then seen_before(seq) per sequence
// (seq already range-checked) is true for its second appearance.
void start_stamp(llm_ctx* c) {
  if (++c->stamp_gen == 0) {
    std::fill(c->seq_stamp.begin(), c->seq_stamp.end(), 0u);
    c->stamp_gen = 1;
  }
}
bool seen_before(llm_ctx* c, int seq) {
  if (c->seq_stamp[seq] == c->stamp_gen) return true;
  c->seq_stamp[seq] = c->stamp_gen;
  return false;
}

int check_ready(llm_ctx* c) {
  if (!c) return fail(LLM_ERR_INVALID, "nil context");
  if (!c->weights_loaded) return fail(LLM_ERR_STATE, "weights not loaded");
  if (!c->kv_ready) return fail(LLM_ERR_STATE, "KV cache not allocated");
  return LLM_OK;
}

int validate_row(llm_ctx* c, int seq, int tok, int pos) {
  if (seq < 0 || seq >= c->max_seqs) return fail(LLM_ERR_INVALID, "sequence %d out of range", seq);
  if ((tok < 0 || tok >= c->cfg.vocab) && !(tok == -1 && c->null_tokens))
    return fail(LLM_ERR_TOKEN_RANGE, "token out of range: %d", tok);
  if (pos < 0 || pos >= c->max_pos) return fail(LLM_ERR_POS_RANGE, "position out of range: %d", pos);
  return LLM_OK;
}

// Segments of the longest context the KV cache can hold: the segment stride of the split
// attention workspace.
int attn_ws_segs(const llm_ctx* c) {
  return std::max(1, ((c->max_pos + 15) / 16 + kAttnSegPages - 1) / kAttnSegPages);
}

// CTAs per (query block, kv head) of a decode attention launch.  The attention arithmetic does
// not depend on this choice (segments fold in a fixed order); it only spreads a small batch's
// long contexts over more SMs.  Splitting needs every segment state in the workspace.
int attn_splits_for(const llm_ctx* c, int n_blocks, int max_ctx) {
  const int segs = std::max(1, ((max_ctx + 15) / 16 + kAttnSegPages - 1) / kAttnSegPages);
  const size_t need = static_cast<size_t>(n_blocks) * c->cfg.n_kv_heads * attn_ws_segs(c) * 8 * (c->cfg.head_dim + 2);
  if (need > c->ws_floats / kMaxParts) return 1;  // the workspace is divided between micro-batches
  if (c->attn_splits > 0) return std::min(c->attn_splits, segs);  // fixed by llm_set_option
  const int ctas = n_blocks * c->cfg.n_kv_heads;
  const int target = 2 * c->n_sm;
  if (ctas >= target) return 1;
  return std::max(1, std::min({(target + ctas - 1) / ctas, segs, 64}));
}

// ---------------------------------------------------------------------------- forward
struct RowsSpec {
  int R = 0;
  const int *d_blk_row0 = nullptr, *d_blk_nq = nullptr;
  int n_blocks = 0;
  int attn_splits = 1;
  const int* d_final = nullptr;  // nullptr: all rows
  int n_final = 0;
  float* d_logits = nullptr;
  int* tok_io = nullptr;
  int* pos_io = nullptr;
  const int* gen_start = nullptr;
  int* gen_out = nullptr;
  int gen_cap = 0;
  bool sample = false;  // draw the next token with sample_kernel (temperature sampling)
  bool prefill_tiles = false;  // blocks are query tiles of attn_prefill_kernel (<= 128/group rows)
  // the step's inputs (tables, positions, K/V of earlier positions) were complete before its
  // first launch: decode attention may request those pages before its programmatic wait
  bool early_kv = false;
};

const CUtensorMap* tmap(llm_ctx* c, const void* ptr, int esz, int k, int rows, int box) {
  auto key = std::make_tuple(ptr, esz, k, rows, box);
  auto it = c->tmaps.find(key);
  if (it != c->tmaps.end()) return &it->second;
  CUtensorMap m{};
  if (make_kmajor_map(&m, ptr, esz, c->act == 2, k, rows, box) != LLM_OK) return nullptr;
  return &c->tmaps.emplace(key, m).first->second;
}

// CTAs of one wave of split-K clusters of 4 or 8 (decode_splits).
constexpr int kSplitPlanSMs = 128;
// Rows from which a projection runs on the persistent kernel (prefill chunks).
constexpr int kPersistMinRows = 1024;

// ring_kb > 0: cap the tcgen05 stage ring at that many KB of shared memory.
int gemm(llm_ctx* c, bool in8, int epi, GemmParams p, cudaStream_t stream = nullptr, int ring_kb = 0) {
  if (!stream) stream = c->stream;
  const int esz = in8 ? 1 : 2;
  p.argmax_parts = (p.N + argmax_tile_width(c->use_umma) - 1) / argmax_tile_width(c->use_umma);
  if (c->use_umma) {
    // Prefill chunks: the persistent kernel (tiles streamed through one ring per SM, epilogue
    // of one tile overlapping the next tile's mainloop)
    const int pbn = epi == EPI_QKV ? c->cfg.head_dim : 128;
    if (c->prefill_persist && p.M >= kPersistMinRows && umma_persist_supported(epi, pbn)) {
      const CUtensorMap* tx = tmap(c, p.A, esz, p.K, p.M, kUmmaTokens);
      const CUtensorMap* tw = tmap(c, p.B, esz, p.K, p.N, pbn);
      if (!tw || !tx) return LLM_ERR_CUDA;
      p.k_splits = 1;
      p.k_tiles_per_split = p.K * esz / 128;
      p.err = c->d_err;
      const int tiles = ((p.M + kUmmaTokens - 1) / kUmmaTokens) * ((p.N + pbn - 1) / pbn);
      CU(umma_persist_any(c->act, in8, *tx, *tw, p, epi, pbn, dim3(std::min(tiles, c->n_sm)), stream, false));
      return LLM_OK;
    }
    // split-K over a cluster of k_splits CTAs (decode rows): the narrowest channel tile whose
    // grid, times the splits, still fits one CTA per SM
    const int ksplit = p.k_splits > 1 && epi == EPI_RESID ? p.k_splits : 1;
    // (two splits: tiles up to 128 channels, so the partial and summed tiles fit the ring)
    // (one wave: clusters of two pack 144 of the 148 SMs, larger ones 128)
    const int wave = ksplit == 1 ? c->n_sm : std::min(c->n_sm, ksplit == 2 ? 144 : kSplitPlanSMs);
    int bn = umma_bn_for(p.M, p.N, epi, c->cfg.head_dim, std::max(1, wave / ksplit), ksplit == 2 ? 128 : 256);
    // Prefill-sized GEMMs (more tiles than SMs): a smaller stage ring lets two CTAs share an SM,
    // so one CTA's epilogue overlaps the other's mainloop; 128-wide channel tiles keep the
    // staged (coalesced) epilogue within that ring.
    const long long tm = (p.M + kUmmaTokens - 1) / kUmmaTokens;
    if (ksplit == 1 && c->prefill_ring_kb > 0 && tm * ((p.N + 255) / 256) > c->n_sm) {
      if (c->prefill_bn > 0 && umma_bn_supported(epi, c->prefill_bn) && epi != EPI_QKV && epi != EPI_ARGMAX)
        bn = c->prefill_bn;
      if (ring_kb <= 0) ring_kb = c->prefill_ring_kb;
    }
    if (ring_kb > 0) p.stages = std::max(2, (ring_kb * 1024 - 1024) / ((kUmmaTokens + bn) * 128));
    if (ksplit > 1) {
      // a ring of this CTA's K slices (less shared memory: two CTAs may share an SM), large
      // enough for the partial and summed tiles written to it once idle
      const int stage = (kUmmaTokens + bn) * 128;
      const int need = ((kUmmaTokens + kUmmaTokens / ksplit) * (bn + 4) * 4 + stage - 1) / stage;
      const int slices = (p.K * esz / 128 + ksplit - 1) / ksplit;
      const int want = std::max(need, p.stages > 0 ? std::min(p.stages, slices) : slices);
      p.stages = std::max(2, want);
    }
    // QKV of more than 64 tokens: 64-token tiles when twice the grid still fits one CTA per
    // SM (each CTA then loads half the activation bytes per K slice)
    const long long tiles_n = (p.N + bn - 1) / bn;
    p.a_rows = epi == EPI_QKV && c->qkv_tile64 && p.M > 64 && (p.M + 63) / 64 * tiles_n <= c->n_sm ? 64 : kUmmaTokens;
    const CUtensorMap* tx = tmap(c, p.A, esz, p.K, p.M, p.a_rows);
    const CUtensorMap* tw = tmap(c, p.B, esz, p.K, p.N, bn);
    if (!tw || !tx) return LLM_ERR_CUDA;
    p.k_splits = ksplit;
    p.k_tiles_per_split = p.K * esz / 128 / ksplit;
    p.err = c->d_err;
    dim3 grid((p.M + p.a_rows - 1) / p.a_rows, (p.N + bn - 1) / bn, ksplit);
    t_cluster_z = ksplit;
    const cudaError_t e = umma_any(c->act, in8, *tx, *tw, p, epi, bn, grid, stream, false);
    t_cluster_z = 1;
    CU(e);
    return LLM_OK;
  }
  GemmPlan pl = plan_gemm(p.M, p.N, p.K, esz, c->n_sm, 0, c->ws_floats);
  p.k_splits = pl.splits;
  p.k_tiles_per_split = pl.kts;
  p.ws = c->ws;
  p.counters = c->counters;
  p.err = c->d_err;
  CU(gemm_any(c->act, in8, p, epi, pl.bm, pl.grid, stream, false));
  return LLM_OK;
}

// Rows [r0, r0 + n) of a forward pass, enqueued on stream s.  idx selects the half of the
// split workspace a micro-batch's attention may use.
struct Part {
  int r0 = 0, n = 0, idx = 0;
  cudaStream_t s = nullptr;
};


// Micro-batches a decode step over R rows runs as (1 = the single-stream schedule): up to
// LLM_OPT_MICRO_BATCHES, each at least kOverlapMinPartRows rows, and only as many as the step
// can afford.  Overlapped steps launch eagerly, so the host must enqueue a step's launches
// faster than the device streams its K/V cache: with ~kEagerLaunchUs of host time per launch,
// a k-part step needs k * (launches per part) * kEagerLaunchUs <= (K/V bytes of the step at
// kHbmBytesPerUs) / kOverlapHostMargin.  Shorter contexts keep the single-stream graph.
constexpr double kEagerLaunchUs = 4.0;
constexpr double kHbmBytesPerUs = 6.5e6;
constexpr double kOverlapHostMargin = 1.2;
int overlap_parts(const llm_ctx* c, int R, bool decode_rows) {
  if (!c->overlap || !c->use_umma || !decode_rows) return 1;
  const int kmax = std::min(std::min(c->micro_batches, kMaxParts), R / kOverlapMinPartRows);
  const int L = c->cfg.n_layers;
  const int per_part = 1 + L * (6 + (c->in8 ? 1 : 0)) + (L - 1);
  const double kv_us = c->step_kv_positions * 2.0 * c->kv_dim * act_bytes(c) * L / kHbmBytesPerUs;
  for (int k = kmax; k >= 2; --k)
    if (c->overlap == 2 || (k * per_part + 3) * kEagerLaunchUs * kOverlapHostMargin <= kv_us) return k;
  return 1;
}
bool overlap_applies(const llm_ctx* c, int R, bool decode_rows) { return overlap_parts(c, R, decode_rows) > 1; }
// Split-K of a decode step's residual projections (Wo, W2) over a cluster
// (LLM_OPT_DECODE_SPLITK).  A decode-sized CTA loads the whole activation tile (128 rows x K)
// for its few output channels, and one SM streams only ~50 GB/s into shared memory, so these
// long-K, narrow-N projections take their per-CTA bytes / 50 GB/s; splitting K divides them.
// Fixed per model and projection (never by the batch or the device), so a row's arithmetic
// does not depend on either: the power of two <= min(LLM_SPLITK_MAX, K slices / 2) and
// <= 128 / (channel tiles at the widest tile) (128: the CTAs of one wave of 4- or 8-CTA
// clusters at one CTA per SM on B200's graphics processing clusters).  Restated by the oracle
// (oracle_decode_splits).  Measured (Qwen3 bf16, 128 rows): step 3.63 -> 3.23 ms with at most
// four CTAs per cluster (3.46 ms with eight: larger clusters wait longer for whole groups of
// free SMs); QKV and W1/W3 (short K, wide N) measured no faster, and the int8 projections
// (half the bytes) slower, so they stay whole.
#ifndef LLM_SPLITK_MAX
#define LLM_SPLITK_MAX 4
#endif
int decode_splits(const llm_ctx* c, int epi, int N, int K, bool overlapped) {
  (void)overlapped;
  if (!c->use_umma || !c->decode_splitk || c->in8 || epi != EPI_RESID) return 1;
  const int nkt = K * (c->in8 ? 1 : 2) / 128;
  const int bnmax = epi == EPI_QKV ? c->cfg.head_dim : 256;
  const int tiles = (N + bnmax - 1) / bnmax;
  const int lim = std::min({LLM_SPLITK_MAX, nkt / 2, kSplitPlanSMs / std::max(1, tiles)});
  int sk = 1;
  while (sk * 2 <= lim) sk *= 2;
  return sk;
}
// Temperature sampling replaces the greedy argmax (sampleFromLogits, infer.go:347-349).
bool sampling_on(const llm_ctx* c) { return c->sample_temp > 1e-6f; }
// Launch timeline records one traced step may use.
constexpr size_t kTraceCap = 1024;

int enqueue_forward(llm_ctx* c, const RowsSpec& rs) {
  t_use_pdl = c->use_pdl;
  t_prio = 0;
  const llm_model_config& k = c->cfg;
  const int R = rs.R, D = k.dim, F = k.hidden, Q = c->q_dim, KV = c->kv_dim;
  const bool i8 = c->in8;
  const size_t ab = act_bytes(c);
  cudaStream_t s = c->stream;
  auto mark = [&](const char* name) -> int {
    if (!c->trace) return LLM_OK;
    cudaEvent_t e;
    CU(cudaEventCreate(&e));
    CU(cudaEventRecord(e, s));
    c->trace->emplace_back(name, e);
    return LLM_OK;
  };
  RC(mark("start"));

  // Decode batches (one query row per attention block) split into micro-batches on their own
  // streams whose attention launches form a chain: part 0 (layer l), part 1 (l), ..., part k-1
  // (l), part 0 (l + 1), ...  Each attention launch may start once every CTA of the previous
  // one in the chain has started, so consecutive attention launches fill each other's tail
  // waves, and everything a micro-batch runs between two of its attention launches (Wo, norm,
  // W1/W3, W2, norm, QKV: latency-bound) runs while the others' attention streams the KV
  // cache.  The split workspace is divided between the micro-batches.
  const bool decode_rows = rs.d_blk_row0 == nullptr && rs.n_blocks == R;
  const int kparts = overlap_parts(c, R, decode_rows);
  const bool overlap = kparts > 1 && !c->trace;
  Part parts[kMaxParts];
  int np = 1;
  if (overlap) {
    // near-equal parts of whole 16-row groups; the last part takes the remainder rows
    const int units = R / 16;
    int r0 = 0;
    for (int h = 0; h < kparts; ++h) {
      const int u = units / kparts + (h < units % kparts ? 1 : 0);
      const int n = h == kparts - 1 ? R - r0 : 16 * u;
      parts[h] = {r0, n, h, h == 0 ? c->stream : c->xstream[h - 1]};
      r0 += n;
    }
    np = kparts;
    CU(cudaEventRecord(c->ev_fork, c->stream));
    for (int h = 1; h < np; ++h) CU(cudaStreamWaitEvent(parts[h].s, c->ev_fork, 0));
  } else {
    parts[0] = {0, R, 0, c->stream};
  }
  const int ring_kb = overlap ? c->overlap_ring_kb : 0;
  const int prio = overlap ? c->prio_hi : 0;
  // programmatic dependent launch inside a micro-batch's projection chain (not for attention)
  const bool chain_pdl = overlap ? c->chain_pdl : c->use_pdl;
  t_use_pdl = overlap ? false : c->use_pdl;
  auto bytes = [](const void* base, size_t off) -> void* {
    return const_cast<uint8_t*>(static_cast<const uint8_t*>(base)) + off;
  };
  // timeline record of the next launch (llm_trace_step), nullptr when not tracing
  auto tr = [&](const char* name, int l, const Part& P) -> TraceRec* {
    if (!c->tracing || c->trace_labels.size() >= kTraceCap) return nullptr;
    char buf[64];
    snprintf(buf, sizeof buf, "%s L%d %c", name, l, np > 1 ? "ABCD"[P.idx] : '-');
    c->trace_labels.emplace_back(buf);
    return c->d_trace + (c->trace_labels.size() - 1);
  };

  auto norm = [&](const Part& P, const float* x, const float* w, bool embed, void* out_act, int8_t* q, float* sc,
                  TraceRec* trace) -> int {
    NormParams np_{};
    np_.trace = trace;
    np_.x = x ? x + static_cast<size_t>(P.r0) * D : nullptr;
    np_.row_index = nullptr;
    np_.embed = embed ? c->embed : nullptr;
    np_.tokens = c->d_tok + P.r0;
    np_.x_out = c->x + static_cast<size_t>(P.r0) * D;
    np_.w = w;
    np_.D = D;
    np_.rows = P.n;
    np_.eps = k.norm_eps;
    np_.out = out_act ? bytes(out_act, static_cast<size_t>(P.r0) * D * ab) : nullptr;
    np_.q = q ? q + static_cast<size_t>(P.r0) * D : nullptr;
    np_.scale = sc ? sc + P.r0 : nullptr;
    t_prio = prio;
    t_use_pdl = chain_pdl;
    CU(norm_any(c->act, q != nullptr, np_, P.s));
    return LLM_OK;
  };
  // attention-side norm input of layer l for part P (the residual stream x)
  auto norm_in = [&](const Part& P, const float* w, bool embed, int l) -> int {
    return norm(P, embed ? nullptr : c->x, w, embed, i8 ? nullptr : c->xn, i8 ? c->xq : nullptr, c->xs,
                tr(embed ? "embed+norm" : "norm(att)", l, P));
  };

  auto qkv = [&](const Part& P, int l) -> int {
    const LayerW& L = c->layers[l];
    GemmParams p{};
    p.A = i8 ? bytes(c->xq, static_cast<size_t>(P.r0) * D) : bytes(c->xn, static_cast<size_t>(P.r0) * D * ab);
    p.B = L.wqkv;
    p.M = P.n;
    p.N = Q + 2 * KV;
    p.K = D;
    p.a_scale = c->xs + P.r0;
    p.b_scale = L.sqkv;
    p.q_out = bytes(c->qbuf, static_cast<size_t>(P.r0) * Q * ab);
    p.kv_pool = c->kv_pool;
    p.block_table = c->d_block_table;
    p.seq_ids = c->d_seq + P.r0;
    p.positions = c->d_pos + P.r0;
    p.q_norm = L.q_norm;
    p.k_norm = L.k_norm;
    p.rope_cos = c->rope_cos;
    p.rope_sin = c->rope_sin;
    p.layer = l;
    p.n_pages = c->n_pages;
    p.max_pages_per_seq = c->max_pages_per_seq;
    p.n_heads = k.n_heads;
    p.n_kv_heads = k.n_kv_heads;
    p.head_dim = k.head_dim;
    p.qk_norm = k.qk_norm;
    p.eps = k.norm_eps;
    p.trace = tr("qkv", l, P);
    t_prio = prio;
    t_use_pdl = chain_pdl;
    return gemm(c, i8, EPI_QKV, p, P.s, ring_kb);
  };

  auto attention = [&](const Part& P, int l) -> int {
    if (rs.prefill_tiles) {  // prefill: query tiles over the paged cache, then the int8 quantiser
      PrefillAttnParams pp{};
      pp.q = c->qbuf;
      pp.kv_pool = c->kv_pool;
      pp.block_table = c->d_block_table;
      pp.max_pages_per_seq = c->max_pages_per_seq;
      pp.seq_ids = c->d_seq;
      pp.positions = c->d_pos;
      pp.tile_row0 = rs.d_blk_row0;
      pp.tile_nq = rs.d_blk_nq;
      pp.n_tiles = rs.n_blocks;
      pp.n_heads = k.n_heads;
      pp.n_kv_heads = k.n_kv_heads;
      pp.layer = l;
      pp.n_pages = c->n_pages;
      pp.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(k.head_dim)));
      pp.out = c->attn;
      pp.out_f32 = i8 ? 1 : 0;
      pp.err = c->d_err;
      pp.trace = tr("attention", l, P);
      t_prio = 0;
      if (c->prefill_tc) CU(attn_prefill_tc_any(c->act, k.head_dim, pp, P.s, false));
      else CU(attn_prefill_any(c->act, k.head_dim, pp, P.s, false));
      if (i8) {
        NormParams np_{};
        np_.x = static_cast<const float*>(c->attn);
        np_.w = nullptr;
        np_.D = Q;
        np_.rows = R;
        np_.q = c->aq;
        np_.scale = c->as;
        np_.trace = tr("quant(attn)", l, P);
        CU(norm_any(c->act, true, np_, P.s));
      }
      return LLM_OK;
    }
    AttnParams ap{};
    ap.q = bytes(c->qbuf, static_cast<size_t>(P.r0) * Q * ab);
    ap.kv_pool = c->kv_pool;
    ap.block_table = c->d_block_table;
    ap.max_pages_per_seq = c->max_pages_per_seq;
    ap.seq_ids = c->d_seq + P.r0;
    ap.positions = c->d_pos + P.r0;
    ap.blk_row0 = rs.d_blk_row0;
    ap.blk_nq = rs.d_blk_nq;
    ap.n_blocks = overlap ? P.n : rs.n_blocks;
    ap.n_heads = k.n_heads;
    ap.n_kv_heads = k.n_kv_heads;
    ap.layer = l;
    ap.n_pages = c->n_pages;
    ap.splits = rs.attn_splits;
    ap.early_kv = rs.early_kv ? 1 : 0;
    ap.ws_segs = attn_ws_segs(c);
    ap.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(k.head_dim)));
    ap.out = bytes(c->attn, static_cast<size_t>(P.r0) * Q * (i8 ? 4 : ab));
    ap.out_f32 = i8 ? 1 : 0;
    ap.ws = c->ws + P.idx * (c->ws_floats / kMaxParts);
    ap.counters = c->counters + P.idx * (kCounters / kMaxParts);
    ap.err = c->d_err;
    ap.trace = tr("attention", l, P);
    if (i8) {  // per-token quantisation of the output fused into the attention kernel
      ap.q8 = c->aq + static_cast<size_t>(P.r0) * Q;
      ap.q8_scale = c->as + P.r0;
      ap.row_counters = c->row_counters + P.r0;
    }
    t_prio = 0;
    t_use_pdl = overlap ? false : c->use_pdl;
    // overlapped schedule: this launch's "all CTAs started" event gates the other micro-batch's
    // next attention launch, which then fills the tail wave of this one
    t_lc_event = overlap && c->attn_chain == 1 ? c->ev_att[P.idx] : nullptr;
    const cudaError_t e = attn_any(c->act, k.head_dim, ap, P.s, false);
    t_lc_event = nullptr;
    CU(e);
    return LLM_OK;
  };

  // Wo + residual, FFN norm, W1/W3 + SiLU gate (+ quantiser), W2 + residual, next layer's norm
  auto post_attention = [&](const Part& P, int l) -> int {
    const LayerW& L = c->layers[l];
    {  // Wo + residual
      GemmParams p{};
      p.A = i8 ? bytes(c->aq, static_cast<size_t>(P.r0) * Q) : bytes(c->attn, static_cast<size_t>(P.r0) * Q * ab);
      p.B = L.wo;
      p.M = P.n;
      p.N = D;
      p.K = Q;
      p.a_scale = c->as + P.r0;
      p.b_scale = L.so;
      p.out = c->x + static_cast<size_t>(P.r0) * D;
      p.resid = c->x + static_cast<size_t>(P.r0) * D;
      p.ldo = D;
      p.resid_scale = c->resid_scale;
      p.trace = tr("wo", l, P);
      t_prio = prio;
      t_use_pdl = chain_pdl;
      p.k_splits = decode_rows ? decode_splits(c, EPI_RESID, p.N, p.K, overlap) : 1;
      RC(gemm(c, i8, EPI_RESID, p, P.s, ring_kb));
      RC(mark("wo_gemm+resid"));
    }
    RC(norm(P, c->x, L.rms_ffn, false, i8 ? nullptr : c->xn, i8 ? c->xq : nullptr, c->xs, tr("norm(ffn)", l, P)));
    RC(mark("norm"));
    {  // W1/W3 + SiLU gate
      GemmParams p{};
      p.A = i8 ? bytes(c->xq, static_cast<size_t>(P.r0) * D) : bytes(c->xn, static_cast<size_t>(P.r0) * D * ab);
      p.B = L.w13;
      p.M = P.n;
      p.N = 2 * F;
      p.K = D;
      p.a_scale = c->xs + P.r0;
      p.b_scale = L.s13;
      p.out = bytes(c->gbuf, static_cast<size_t>(P.r0) * F * (i8 ? 4 : ab));
      p.swiglu_f32 = i8 ? 1 : 0;
      p.silu_form = c->silu_form;
      p.trace = tr("w13", l, P);
      t_prio = prio;
      t_use_pdl = chain_pdl;
      RC(gemm(c, i8, EPI_SWIGLU, p, P.s, ring_kb));
      RC(mark("w13_gemm+swiglu"));
    }
    if (i8) {  // per-token quantisation of the SwiGLU output
      NormParams np_{};
      np_.x = static_cast<const float*>(c->gbuf) + static_cast<size_t>(P.r0) * F;
      np_.w = nullptr;
      np_.D = F;
      np_.rows = P.n;
      np_.q = c->gq + static_cast<size_t>(P.r0) * F;
      np_.scale = c->gs + P.r0;
      np_.trace = tr("quant(g)", l, P);
      t_prio = prio;
      t_use_pdl = chain_pdl;
      CU(norm_any(c->act, true, np_, P.s));
      RC(mark("quant(g)"));
    }
    {  // W2 + residual
      GemmParams p{};
      p.A = i8 ? bytes(c->gq, static_cast<size_t>(P.r0) * F) : bytes(c->gbuf, static_cast<size_t>(P.r0) * F * ab);
      p.B = L.w2;
      p.M = P.n;
      p.N = D;
      p.K = F;
      p.a_scale = c->gs + P.r0;
      p.b_scale = L.s2;
      p.out = c->x + static_cast<size_t>(P.r0) * D;
      p.resid = c->x + static_cast<size_t>(P.r0) * D;
      p.ldo = D;
      p.resid_scale = c->resid_scale;
      p.trace = tr("w2", l, P);
      t_prio = prio;
      t_use_pdl = chain_pdl;
      p.k_splits = decode_rows ? decode_splits(c, EPI_RESID, p.N, p.K, overlap) : 1;
      RC(gemm(c, i8, EPI_RESID, p, P.s, ring_kb));
      RC(mark("w2_gemm+resid"));
    }
    if (l + 1 < k.n_layers) {
      RC(norm_in(P, c->layers[l + 1].rms_att, false, l + 1));
      RC(mark("norm"));
    }
    return LLM_OK;
  };

  // layer 0 attention norm fused with the embedding gather
  for (int h = 0; h < np; ++h) RC(norm_in(parts[h], c->layers[0].rms_att, true, 0));
  RC(mark("embed+norm"));
  for (int l = 0; l < k.n_layers; ++l) {
    for (int h = 0; h < np; ++h) {
      const Part& P = parts[h];
      if (l == 0 || !overlap) RC(qkv(P, l));  // later layers: enqueued by post_attention's tail below
      RC(mark("qkv_gemm+rope+kv_write"));
      if (overlap && (h > 0 || l > 0))  // chain: after the previous part's attention launch
        CU(cudaStreamWaitEvent(P.s, c->ev_att[(h + np - 1) % np], 0));
      RC(attention(P, l));
      RC(mark(i8 ? "attention+quant" : "attention"));
      if (overlap && c->attn_chain == 0) CU(cudaEventRecord(c->ev_att[h], P.s));
    }
    for (int h = 0; h < np; ++h) {
      RC(post_attention(parts[h], l));
      if (overlap && l + 1 < k.n_layers) RC(qkv(parts[h], l + 1));
    }
  }
  t_prio = 0;
  t_use_pdl = overlap ? false : c->use_pdl;
  for (int h = 1; h < np; ++h) {
    CU(cudaEventRecord(c->ev_join, parts[h].s));
    CU(cudaStreamWaitEvent(c->stream, c->ev_join, 0));
  }
  // final norm on the rows whose next token is wanted, tied/untied lm_head + argmax
  const int NF = rs.d_final ? rs.n_final : R;
  {
    NormParams np_{};
    np_.x = c->x;
    np_.row_index = rs.d_final;
    np_.tokens = c->d_tok;
    np_.x_out = c->x;
    np_.w = c->rms_final;
    np_.D = D;
    np_.rows = NF;
    np_.eps = k.norm_eps;
    np_.out = c->xf;
    np_.trace = tr("final_norm", k.n_layers, parts[0]);
    CU(norm_any(c->act, false, np_, s));
  }
  RC(mark("final_norm"));
  {
    GemmParams p{};
    p.A = c->xf;
    p.B = c->lm_head;
    p.M = NF;
    p.N = k.vocab;
    p.K = D;
    p.argmax_part = c->argmax_part;
    p.logits = rs.d_logits ? rs.d_logits : (rs.sample ? c->logits : nullptr);
    p.ld_logits = k.vocab;
    p.trace = tr("lm_head", k.n_layers, parts[0]);
    RC(gemm(c, false, EPI_ARGMAX, p));
    RC(mark("lm_head+argmax"));
  }
  if (rs.sample) {
    SampleParams sp{};
    sp.logits = rs.d_logits ? rs.d_logits : c->logits;
    sp.rows = NF;
    sp.V = k.vocab;
    sp.ld = k.vocab;
    sp.inv_t = c->sample_inv_t;
    sp.row_index = rs.d_final;
    sp.seq_ids = c->d_seq;
    sp.seed = c->sample_seed;
    sp.draws = c->d_draws;
    sp.out = c->d_sampled;
    CU(launch_pdl(sample_kernel, dim3(NF), dim3(kSampleThreads), 0, s, sp));
    RC(mark("sample"));
  }
  {
    FinishParams f{};
    f.part = c->argmax_part;
    f.M = NF;
    f.n_tiles = (k.vocab + argmax_tile_width(c->use_umma) - 1) / argmax_tile_width(c->use_umma);
    f.next = c->d_next;
    f.tok_io = rs.tok_io;
    f.pos_io = rs.pos_io;
    f.gen_start = rs.gen_start;
    f.gen_out = rs.gen_out;
    f.gen_cap = rs.gen_cap;
    f.sampled = rs.sample ? c->d_sampled : nullptr;
    CU(launch_pdl(finish_kernel, dim3((NF + 7) / 8), dim3(256), 0, s, f));
    RC(mark("finish"));
  }
  return LLM_OK;
}

int ensure_logits(llm_ctx* c, int rows) {
  if (c->logits && c->logits_rows >= static_cast<size_t>(rows)) return LLM_OK;
  if (c->logits) {
    CU(cudaStreamSynchronize(c->stream));
    cudaFree(c->logits);
    c->allocs.erase(std::find(c->allocs.begin(), c->allocs.end(), static_cast<void*>(c->logits)));
    c->logits = nullptr;
  }
  RC(dalloc_t(c, &c->logits, static_cast<size_t>(rows) * c->cfg.vocab * 4, &c->bytes_other));
  c->logits_rows = rows;
  return LLM_OK;
}

// Decode step over rows 0..n-1 of d_seq/d_tok/d_pos, via a cached CUDA graph.
int run_step(llm_ctx* c, int n, int splits, int mode) {
  RowsSpec rs;
  rs.R = n;
  rs.n_blocks = n;
  rs.attn_splits = splits;
  rs.sample = sampling_on(c);
  if (mode == 1) rs.d_logits = c->logits;
  if (mode == 2) {
    rs.tok_io = c->d_tok;
    rs.pos_io = c->d_pos;
    rs.gen_start = c->d_gen_start;
    rs.gen_out = c->d_gen_out;
    rs.gen_cap = c->gen_max_steps;
  }
  // overlapped micro-batch steps launch eagerly unless LLM_OPT_OVERLAP_GRAPHS: their
  // cross-stream schedule measured faster from eager launches than from a replayed graph
  if (!c->use_graphs || c->tracing || (overlap_applies(c, n, true) && !c->overlap_graphs)) {
    // A host-driven step's inputs arrive by stream-ordered copies before its first launch.  An
    // eager device-resident step (mode 2) may start its first launches while the previous
    // step's last kernel (which advances the positions) still runs, so it keeps the wait first.
    rs.early_kv = mode != 2 && !c->tracing;
    return enqueue_forward(c, rs);
  }
  // successive graph launches are stream-ordered as a whole
  rs.early_kv = true;
  GraphKey key{n, splits, mode | (rs.sample ? 8 : 0)};
  auto it = c->graphs.find(key);
  if (it == c->graphs.end()) {
    cudaGraph_t g = nullptr;
    CU(cudaStreamBeginCapture(c->stream, cudaStreamCaptureModeThreadLocal));
    int rc = enqueue_forward(c, rs);
    cudaError_t e = cudaStreamEndCapture(c->stream, &g);
    if (rc) {
      if (g) cudaGraphDestroy(g);
      return rc;
    }
    if (e != cudaSuccess) return fail(LLM_ERR_CUDA, "graph capture failed: %s", cudaGetErrorString(e));
    cudaGraphExec_t ge = nullptr;
    e = cudaGraphInstantiate(&ge, g, 0);
    cudaGraphDestroy(g);
    if (e != cudaSuccess) return fail(LLM_ERR_CUDA, "graph instantiate failed: %s", cudaGetErrorString(e));
    it = c->graphs.emplace(key, ge).first;
  }
  CU(cudaGraphLaunch(it->second, c->stream));
  return LLM_OK;
}

}  // namespace

// ============================================================================ token loop API
extern "C" int llm_decode_step(llm_ctx* c, const int32_t* seq_ids, const int32_t* tokens, const int32_t* positions,
                               int n, int32_t* next_tokens, float* logits) {
  RC(check_ready(c));
  if (!seq_ids || !tokens || !positions || !next_tokens) return fail(LLM_ERR_INVALID, "nil buffer");
  if (n <= 0 || n > c->max_seqs) return fail(LLM_ERR_INVALID, "batch %d out of range (1..%d)", n, c->max_seqs);
  RC(set_device(c));
  int max_ctx = 0;
  double kv_positions = 0;
  start_stamp(c);
  // every row is checked before any page is reserved
  for (int i = 0; i < n; ++i) {
    RC(validate_row(c, seq_ids[i], tokens[i], positions[i]));
    if (seen_before(c, seq_ids[i])) return fail(LLM_ERR_INVALID, "sequence %d appears twice in one step", seq_ids[i]);
    max_ctx = std::max(max_ctx, positions[i] + 1);
    kv_positions += positions[i] + 1.0;
  }
  RC(reserve_rows(c, n, seq_ids, positions));
  c->step_kv_positions = kv_positions;
  int32_t* h = c->h_pin;
  memcpy(h, seq_ids, n * 4);
  memcpy(h + n, tokens, n * 4);
  memcpy(h + 2 * n, positions, n * 4);
  CU(cudaMemcpyAsync(c->d_seq, h, n * 4, cudaMemcpyHostToDevice, c->stream));
  CU(cudaMemcpyAsync(c->d_tok, h + n, n * 4, cudaMemcpyHostToDevice, c->stream));
  CU(cudaMemcpyAsync(c->d_pos, h + 2 * n, n * 4, cudaMemcpyHostToDevice, c->stream));
  if (logits || sampling_on(c)) RC(ensure_logits(c, n));
  // splits sized for the largest context this graph shape is likely to see: round up to a
  // power-of-two page count so graphs are reused across steps
  int pages = (max_ctx + 15) / 16, p2 = 1;
  while (p2 < pages) p2 <<= 1;
  const int splits = attn_splits_for(c, n, p2 * 16);
  RC(run_step(c, n, splits, logits ? 1 : 0));
  CU(cudaMemcpyAsync(h + 3 * n, c->d_next, n * 4, cudaMemcpyDeviceToHost, c->stream));
  if (logits)
    CU(cudaMemcpyAsync(logits, c->logits, static_cast<size_t>(n) * c->cfg.vocab * 4, cudaMemcpyDeviceToHost, c->stream));
  CU(cudaStreamSynchronize(c->stream));
  memcpy(next_tokens, h + 3 * n, n * 4);
  return check_device_error(c);
}

namespace {
// llm_prefill; with all_rows, every row's logits stay in c->logits ([rows][vocab], one chunk
// only) and every row's greedy token in c->d_next, without sampling (llm_eval_window).
int prefill_impl(llm_ctx* c, const int32_t* seq_ids, const int32_t* tokens, const int32_t* lens,
                 const int32_t* start_pos, int nseq, int32_t* next_tokens, float* logits, bool all_rows);
}  // namespace

extern "C" int llm_prefill(llm_ctx* c, const int32_t* seq_ids, const int32_t* tokens, const int32_t* lens,
                           const int32_t* start_pos, int nseq, int32_t* next_tokens, float* logits) {
  return prefill_impl(c, seq_ids, tokens, lens, start_pos, nseq, next_tokens, logits, false);
}

namespace {
int prefill_impl(llm_ctx* c, const int32_t* seq_ids, const int32_t* tokens, const int32_t* lens,
                 const int32_t* start_pos, int nseq, int32_t* next_tokens, float* logits, bool all_rows) {
  RC(check_ready(c));
  if (!seq_ids || !tokens || !lens || !next_tokens) return fail(LLM_ERR_INVALID, "nil buffer");
  if (nseq <= 0 || nseq > c->max_seqs) return fail(LLM_ERR_INVALID, "nseq %d out of range", nseq);
  RC(set_device(c));
  // attention blocks: query tiles of 128/group rows for attn_prefill_kernel (groups dividing
  // 8), else blocks of 8/group rows for the decode kernel's block-causal mode
  const bool tiles = c->prefill_tiles && 8 % c->group == 0;
  const int qpos = tiles ? kPrefillRows / c->group : std::max(1, 8 / c->group);
  // rows (seq, tok, pos, owner)
  struct Row { int seq, tok, pos, owner; };
  std::vector<Row> rows;
  size_t off = 0;
  start_stamp(c);
  for (int i = 0; i < nseq; ++i) {
    if (lens[i] <= 0) return fail(LLM_ERR_INVALID, "prompt %d is empty", i);
    const int p0 = start_pos ? start_pos[i] : 0;
    if (seq_ids[i] >= 0 && seq_ids[i] < c->max_seqs && seen_before(c, seq_ids[i]))
      return fail(LLM_ERR_INVALID, "sequence %d appears twice", seq_ids[i]);
    for (int j = 0; j < lens[i]; ++j) {
      RC(validate_row(c, seq_ids[i], tokens[off + j], p0 + j));
      rows.push_back({seq_ids[i], tokens[off + j], p0 + j, i});
    }
    off += lens[i];
  }
  {  // every row is checked before any page is reserved
    std::vector<int> upto(nseq);
    for (int i = 0; i < nseq; ++i) upto[i] = (start_pos ? start_pos[i] : 0) + lens[i] - 1;
    RC(reserve_rows(c, nseq, seq_ids, upto.data()));
  }
  if (all_rows && rows.size() > static_cast<size_t>(c->max_rows))
    return fail(LLM_ERR_INVALID, "%zu rows exceed one chunk of %d", rows.size(), c->max_rows);
  if (all_rows) RC(ensure_logits(c, static_cast<int>(rows.size())));
  else if (logits || sampling_on(c)) RC(ensure_logits(c, nseq));
  const int Rmax = c->max_rows;
  size_t r = 0;
  while (r < rows.size()) {
    const size_t r1 = std::min(rows.size(), r + Rmax);
    const int R = static_cast<int>(r1 - r);
    int32_t* h = c->h_pin;  // [seq R][tok R][pos R][row0 R][nq R][final R] and owners on host
    std::vector<int> final_owner;
    int nb = 0, nf = 0;
    for (int i = 0; i < R; ++i) {
      const Row& w = rows[r + i];
      h[i] = w.seq;
      h[R + i] = w.tok;
      h[2 * R + i] = w.pos;
    }
    // query blocks: runs of consecutive rows of one sequence, up to qpos rows each
    for (int i = 0; i < R;) {
      int j = i + 1;
      while (j < R && j - i < qpos && rows[r + j].owner == rows[r + i].owner) ++j;
      h[3 * R + nb] = i;
      h[4 * R + nb] = j - i;
      ++nb;
      i = j;
    }
    if (tiles) {
      // query tiles longest context first (the prefill kernels start them in list order)
      std::vector<std::pair<int, int>> blk(nb);
      for (int b = 0; b < nb; ++b) blk[b] = {h[3 * R + b], h[4 * R + b]};
      std::stable_sort(blk.begin(), blk.end(), [&](const std::pair<int, int>& a, const std::pair<int, int>& b) {
        return rows[r + a.first].pos + a.second > rows[r + b.first].pos + b.second;
      });
      for (int b = 0; b < nb; ++b) {
        h[3 * R + b] = blk[b].first;
        h[4 * R + b] = blk[b].second;
      }
    }
    for (int i = 0; i < R; ++i) {
      const Row& w = rows[r + i];
      const bool last = all_rows || (r + i + 1 == rows.size()) || rows[r + i + 1].owner != w.owner;
      if (last) {
        h[5 * R + nf++] = i;
        final_owner.push_back(w.owner);
      }
    }
    CU(cudaMemcpyAsync(c->d_seq, h, R * 4, cudaMemcpyHostToDevice, c->stream));
    CU(cudaMemcpyAsync(c->d_tok, h + R, R * 4, cudaMemcpyHostToDevice, c->stream));
    CU(cudaMemcpyAsync(c->d_pos, h + 2 * R, R * 4, cudaMemcpyHostToDevice, c->stream));
    CU(cudaMemcpyAsync(c->d_blk_row0, h + 3 * R, nb * 4, cudaMemcpyHostToDevice, c->stream));
    CU(cudaMemcpyAsync(c->d_blk_nq, h + 4 * R, nb * 4, cudaMemcpyHostToDevice, c->stream));
    if (nf) CU(cudaMemcpyAsync(c->d_final, h + 5 * R, nf * 4, cudaMemcpyHostToDevice, c->stream));
    int max_ctx = 0;
    for (int i = 0; i < R; ++i) max_ctx = std::max(max_ctx, rows[r + i].pos + 1);
    RowsSpec rs;
    rs.R = R;
    rs.d_blk_row0 = c->d_blk_row0;
    rs.d_blk_nq = c->d_blk_nq;
    rs.n_blocks = nb;
    rs.prefill_tiles = tiles;
    rs.attn_splits = tiles ? 1 : attn_splits_for(c, nb, max_ctx);
    rs.d_final = c->d_final;
    rs.n_final = nf;
    rs.d_logits = logits || all_rows ? c->logits : nullptr;
    rs.sample = sampling_on(c) && nf > 0 && !all_rows;
    if (all_rows) {
      RC(enqueue_forward(c, rs));
      CU(cudaStreamSynchronize(c->stream));
    } else if (nf > 0) {
      RC(enqueue_forward(c, rs));
      std::vector<int> nxt(nf);
      CU(cudaMemcpyAsync(nxt.data(), c->d_next, nf * 4, cudaMemcpyDeviceToHost, c->stream));
      if (logits)
        for (int i = 0; i < nf; ++i)
          CU(cudaMemcpyAsync(logits + static_cast<size_t>(final_owner[i]) * c->cfg.vocab,
                             c->logits + static_cast<size_t>(i) * c->cfg.vocab, c->cfg.vocab * 4,
                             cudaMemcpyDeviceToHost, c->stream));
      CU(cudaStreamSynchronize(c->stream));
      for (int i = 0; i < nf; ++i) next_tokens[final_owner[i]] = nxt[i];
    } else {
      // every row continues in the next chunk; the lm_head is still run on one row so the
      // launch sequence stays uniform (its result is discarded)
      h[5 * R] = R - 1;
      CU(cudaMemcpyAsync(c->d_final, h + 5 * R, 4, cudaMemcpyHostToDevice, c->stream));
      rs.n_final = 1;
      rs.d_logits = nullptr;
      RC(enqueue_forward(c, rs));
      CU(cudaStreamSynchronize(c->stream));
    }
    r = r1;
  }
  return check_device_error(c);
}
}  // namespace

// Channel-first copy of row-major logits: out[v][r] = in[r][v] (32x32 tiles through shared memory).
__global__ void __launch_bounds__(256) transpose_rows_kernel(const float* in, int rows, int V, float* out) {
  __shared__ float tile[32][33];
  const int v0 = blockIdx.x * 32, r0 = blockIdx.y * 32, tx = threadIdx.x, ty = threadIdx.y;
  for (int j = ty; j < 32; j += 8)
    if (r0 + j < rows && v0 + tx < V) tile[j][tx] = in[static_cast<size_t>(r0 + j) * V + v0 + tx];
  __syncthreads();
  for (int j = ty; j < 32; j += 8)
    if (v0 + j < V && r0 + tx < rows) out[static_cast<size_t>(v0 + j) * rows + r0 + tx] = tile[tx][j];
}

extern "C" int llm_eval_window(llm_ctx* c, int slot, const int32_t* tokens, int seq, int arithmetic,
                               int32_t* next_token, float* logits_cf) {
  RC(check_ready(c));
  if (!tokens || !next_token) return fail(LLM_ERR_INVALID, "nil buffer");
  if (slot < 0 || slot >= c->max_seqs) return fail(LLM_ERR_INVALID, "sequence %d out of range", slot);
  if (seq <= 0 || seq > c->max_pos || seq > c->max_rows)
    return fail(LLM_ERR_INVALID, "window length %d out of range (1..%d)", seq, std::min(c->max_pos, c->max_rows));
  if (arithmetic != LLM_ARITH_STORIES && arithmetic != LLM_ARITH_STORIESANE)
    return fail(LLM_ERR_INVALID, "unknown arithmetic %d", arithmetic);
  RC(set_device(c));
  struct ArithScope {
    llm_ctx* c;
    float r;
    int f;
    ~ArithScope() {
      c->resid_scale = r;
      c->silu_form = f;
    }
  } scope{c, c->resid_scale, c->silu_form};
  if (arithmetic == LLM_ARITH_STORIESANE) {
    // ane/storiesane/residual.go:9: float32(1 / sqrt(2 * layers))
    c->resid_scale = static_cast<float>(1.0 / std::sqrt(2.0 * static_cast<double>(c->cfg.n_layers)));
    c->silu_form = 1;
  }
  RC(llm_seq_release(c, slot));
  // a token outside [0, vocab) gives its position a zero embedding column, as EmbedLookup
  // (ane/stories/cpu.go:41-72) does for the storiesane forward (engine.go:818)
  std::vector<int32_t> toks(tokens, tokens + seq);
  for (int32_t& t : toks)
    if (t < 0 || t >= c->cfg.vocab) t = -1;
  struct NullScope {
    llm_ctx* c;
    ~NullScope() { c->null_tokens = false; }
  } nscope{c};
  c->null_tokens = true;
  int32_t len = seq, nt = 0;
  int rc = prefill_impl(c, &slot, toks.data(), &len, nullptr, 1, &nt, nullptr, true);
  if (!rc) {
    const int V = c->cfg.vocab;
    int32_t* h = c->h_pin;
    if (sampling_on(c)) {  // the last position's token, drawn from the slot's stream
      SampleParams sp{};
      sp.logits = c->logits + static_cast<size_t>(seq - 1) * V;
      sp.rows = 1;
      sp.V = V;
      sp.ld = V;
      sp.inv_t = c->sample_inv_t;
      sp.row_index = c->d_final + (seq - 1);
      sp.seq_ids = c->d_seq;
      sp.seed = c->sample_seed;
      sp.draws = c->d_draws;
      sp.out = c->d_sampled;
      sample_kernel<<<1, kSampleThreads, 0, c->stream>>>(sp);
      if (cudaGetLastError() != cudaSuccess) rc = fail(LLM_ERR_CUDA, "sample launch failed");
      else if (cudaMemcpyAsync(h, c->d_sampled, 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess)
        rc = fail(LLM_ERR_CUDA, "copy failed");
    } else if (cudaMemcpyAsync(h, c->d_next + (seq - 1), 4, cudaMemcpyDeviceToHost, c->stream) != cudaSuccess) {
      rc = fail(LLM_ERR_CUDA, "copy failed");
    }
    if (!rc && logits_cf) {
      if (!c->logits_t || c->logits_t_rows < static_cast<size_t>(seq)) {
        if (c->logits_t) {
          cudaStreamSynchronize(c->stream);
          cudaFree(c->logits_t);
          c->allocs.erase(std::find(c->allocs.begin(), c->allocs.end(), static_cast<void*>(c->logits_t)));
          c->logits_t = nullptr;
        }
        rc = dalloc_t(c, &c->logits_t, static_cast<size_t>(seq) * V * 4, &c->bytes_other);
        c->logits_t_rows = rc ? 0 : seq;
      }
      if (!rc) {
        transpose_rows_kernel<<<dim3((V + 31) / 32, (seq + 31) / 32), dim3(32, 8), 0, c->stream>>>(c->logits, seq, V,
                                                                                                 c->logits_t);
        if (cudaGetLastError() != cudaSuccess ||
            cudaMemcpyAsync(logits_cf, c->logits_t, static_cast<size_t>(seq) * V * 4, cudaMemcpyDeviceToHost,
                            c->stream) != cudaSuccess)
          rc = fail(LLM_ERR_CUDA, "channel-first logits copy failed");
      }
    }
    if (!rc && cudaStreamSynchronize(c->stream) != cudaSuccess) rc = fail(LLM_ERR_CUDA, "stream sync failed");
    if (!rc) *next_token = h[0];
  }
  const int rc2 = llm_seq_release(c, slot);
  if (rc) return rc;
  RC(rc2);
  return check_device_error(c);
}

extern "C" int llm_generate_begin(llm_ctx* c, const int32_t* seq_ids, const int32_t* tokens, const int32_t* positions,
                                  int n, int max_steps) {
  RC(check_ready(c));
  if (!seq_ids || !tokens || !positions) return fail(LLM_ERR_INVALID, "nil buffer");
  if (n <= 0 || n > c->max_seqs) return fail(LLM_ERR_INVALID, "batch %d out of range", n);
  if (max_steps <= 0) return fail(LLM_ERR_INVALID, "max_steps must be positive");
  RC(set_device(c));
  int max_ctx = 0;
  double kv_positions = 0;
  start_stamp(c);
  for (int i = 0; i < n; ++i) {
    RC(validate_row(c, seq_ids[i], tokens[i], positions[i]));
    if (positions[i] + max_steps - 1 >= c->max_pos)
      return fail(LLM_ERR_POS_RANGE, "position out of range: %d", positions[i] + max_steps - 1);
    if (seen_before(c, seq_ids[i])) return fail(LLM_ERR_INVALID, "sequence %d appears twice", seq_ids[i]);
    max_ctx = std::max(max_ctx, positions[i] + max_steps);
    kv_positions += positions[i] + 0.5 * max_steps + 0.5;
  }
  {
    std::vector<int> upto(n);
    for (int i = 0; i < n; ++i) upto[i] = positions[i] + max_steps - 1;
    RC(reserve_rows(c, n, seq_ids, upto.data()));
  }
  if (sampling_on(c)) RC(ensure_logits(c, n));
  const size_t need = static_cast<size_t>(max_steps) * n;
  if (need > c->gen_out_cap) {
    if (c->d_gen_out) {
      CU(cudaStreamSynchronize(c->stream));
      cudaFree(c->d_gen_out);
      c->allocs.erase(std::find(c->allocs.begin(), c->allocs.end(), static_cast<void*>(c->d_gen_out)));
      c->d_gen_out = nullptr;
      // graphs captured with the old buffer are stale
      for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second);
      c->graphs.clear();
    }
    RC(dalloc_t(c, &c->d_gen_out, need * 4, &c->bytes_other));
    c->gen_out_cap = need;
  }
  if (c->gen_max_steps != max_steps) {
    // the step capacity is baked into captured generate graphs
    for (auto it = c->graphs.begin(); it != c->graphs.end();) {
      if (it->first.mode == 2) {
        cudaGraphExecDestroy(it->second);
        it = c->graphs.erase(it);
      } else {
        ++it;
      }
    }
  }
  int32_t* h = c->h_pin;
  memcpy(h, seq_ids, n * 4);
  memcpy(h + n, tokens, n * 4);
  memcpy(h + 2 * n, positions, n * 4);
  CU(cudaMemcpyAsync(c->d_seq, h, n * 4, cudaMemcpyHostToDevice, c->stream));
  CU(cudaMemcpyAsync(c->d_tok, h + n, n * 4, cudaMemcpyHostToDevice, c->stream));
  CU(cudaMemcpyAsync(c->d_pos, h + 2 * n, n * 4, cudaMemcpyHostToDevice, c->stream));
  CU(cudaMemcpyAsync(c->d_gen_start, h + 2 * n, n * 4, cudaMemcpyHostToDevice, c->stream));
  CU(cudaStreamSynchronize(c->stream));
  c->gen_n = n;
  c->gen_steps_done = 0;
  c->gen_max_steps = max_steps;
  c->gen_splits = attn_splits_for(c, n, max_ctx);
  c->step_kv_positions = kv_positions;
  c->gen_seq.assign(seq_ids, seq_ids + n);
  c->gen_pos0.assign(positions, positions + n);
  return LLM_OK;
}

extern "C" int llm_generate_steps(llm_ctx* c, int steps) {
  RC(check_ready(c));
  if (c->gen_n <= 0) return fail(LLM_ERR_STATE, "llm_generate_begin not called");
  if (steps < 0 || c->gen_steps_done + steps > c->gen_max_steps)
    return fail(LLM_ERR_INVALID, "steps %d exceed the reserved %d", c->gen_steps_done + steps, c->gen_max_steps);
  RC(set_device(c));
  for (int i = 0; i < steps; ++i) RC(run_step(c, c->gen_n, c->gen_splits, 2));
  c->gen_steps_done += steps;
  return LLM_OK;
}

extern "C" int llm_generate_end(llm_ctx* c, int32_t* out_tokens, int32_t* steps_done) {
  RC(check_ready(c));
  RC(set_device(c));
  CU(cudaStreamSynchronize(c->stream));
  if (out_tokens && c->gen_steps_done > 0)
    CU(cudaMemcpy(out_tokens, c->d_gen_out, static_cast<size_t>(c->gen_steps_done) * c->gen_n * 4, cudaMemcpyDeviceToHost));
  if (steps_done) *steps_done = c->gen_steps_done;
  return check_device_error(c);
}

extern "C" int llm_generate(llm_ctx* c, const int32_t* seq_ids, const int32_t* tokens, const int32_t* positions, int n,
                            int steps, int32_t* out_tokens) {
  RC(llm_generate_begin(c, seq_ids, tokens, positions, n, steps));
  RC(llm_generate_steps(c, steps));
  int32_t done = 0;
  return llm_generate_end(c, out_tokens, &done);
}

// ============================================================================ stories.Decoder mirror
extern "C" int llm_stories_decode_batch(llm_ctx* c, const int32_t* prompts, const int32_t* prompt_lens, int nseq,
                                        int max_new, float temperature, int32_t* out_tokens, int32_t* n_tokens,
                                        int32_t* prompt_len, int32_t* stopped_on_eos) {
  RC(check_ready(c));
  if (!out_tokens || !n_tokens || !prompt_len || !stopped_on_eos || (!prompts && nseq > 0) || !prompt_lens)
    return fail(LLM_ERR_INVALID, "nil buffer");
  if (nseq <= 0 || nseq > c->max_seqs) return fail(LLM_ERR_INVALID, "nseq %d out of range", nseq);
  // infer.go:144-146: negative temperature -> 0 (greedy); the call samples with `temperature`
  // from the context's generator state (llm_set_sampling's seed and per-slot draw counts)
  if (!(temperature > 0.f)) temperature = 0.f;
  struct TempScope {
    llm_ctx* c;
    float saved;
    ~TempScope() { c->sample_temp = saved; }
  } scope{c, c->sample_temp};
  c->sample_temp = temperature;
  c->sample_inv_t = static_cast<double>(1.0f / temperature);
  const int max_seq = c->max_pos;  // Decoder.maxSeq
  if (max_new <= 0) max_new = 64;  // infer.go:147-149
  std::vector<std::vector<int>> toks(nseq);
  size_t off = 0;
  for (int i = 0; i < nseq; ++i) {
    const int L = prompt_lens[i];
    std::vector<int> p(prompts + off, prompts + off + std::max(0, L));
    off += std::max(0, L);
    if (p.empty()) p.push_back(1);                                                     // :153-155
    if (static_cast<int>(p.size()) > max_seq) p.erase(p.begin(), p.end() - max_seq);  // :156-158
    for (size_t j = 0; j < p.size(); ++j)
      if (p[j] < 0 || p[j] >= c->cfg.vocab)
        return fail(LLM_ERR_TOKEN_RANGE, "prompt token[%zu]=%d out of range", j, p[j]);
    toks[i] = std::move(p);
    prompt_len[i] = static_cast<int32_t>(toks[i].size());
    stopped_on_eos[i] = 0;
  }
  for (int i = 0; i < nseq; ++i) RC(llm_seq_release(c, i));
  // prefill every prompt; the next token of a prompt that already fills max_seq is unused
  std::vector<int> seq(nseq), lens(nseq), flat;
  for (int i = 0; i < nseq; ++i) {
    seq[i] = i;
    lens[i] = static_cast<int>(toks[i].size());
    flat.insert(flat.end(), toks[i].begin(), toks[i].end());
  }
  std::vector<int> next(nseq);
  RC(llm_prefill(c, seq.data(), flat.data(), lens.data(), nullptr, nseq, next.data(), nullptr));
  std::vector<int> active(nseq, 1), steps(nseq, 0);
  auto accept = [&](int i, int tok) {
    toks[i].push_back(tok);
    ++steps[i];
    if (tok == 2) {  // EOS, infer.go:190-193
      stopped_on_eos[i] = 1;
      active[i] = 0;
    }
    if (steps[i] >= max_new || static_cast<int>(toks[i].size()) >= max_seq) active[i] = 0;
  };
  for (int i = 0; i < nseq; ++i) {
    if (max_new > 0 && static_cast<int>(toks[i].size()) < max_seq) accept(i, next[i]);
    else active[i] = 0;
  }
  // constant batch: finished rows re-run their last position and their outputs are ignored
  std::vector<int> tk(nseq), ps(nseq), nx(nseq);
  for (;;) {
    bool any = false;
    for (int i = 0; i < nseq; ++i) any |= active[i] != 0;
    if (!any) break;
    for (int i = 0; i < nseq; ++i) {
      tk[i] = toks[i].back();
      ps[i] = static_cast<int>(toks[i].size()) - 1;
    }
    RC(llm_decode_step(c, seq.data(), tk.data(), ps.data(), nseq, nx.data(), nullptr));
    for (int i = 0; i < nseq; ++i)
      if (active[i]) accept(i, nx[i]);
  }
  for (int i = 0; i < nseq; ++i) {
    n_tokens[i] = static_cast<int32_t>(toks[i].size());
    std::copy(toks[i].begin(), toks[i].end(), out_tokens + static_cast<size_t>(i) * max_seq);
  }
  return LLM_OK;
}

extern "C" int llm_stories_decode(llm_ctx* c, int seq, const int32_t* prompt, int n_prompt, int max_new,
                                  float temperature, int32_t* out_tokens, int32_t* n_tokens, int32_t* prompt_len,
                                  int32_t* stopped_on_eos) {
  if (seq != 0) return fail(LLM_ERR_INVALID, "llm_stories_decode uses sequence slot 0");
  int32_t lens = n_prompt;
  static const int32_t empty = 0;
  return llm_stories_decode_batch(c, prompt ? prompt : &empty, &lens, 1, max_new, temperature, out_tokens, n_tokens,
                                  prompt_len, stopped_on_eos);
}

// ============================================================================ options
extern "C" double llm_sample_uniform(uint64_t seed, int32_t slot, uint64_t counter) {
  return sample_uniform(seed, kSampleStreamBase + static_cast<uint64_t>(slot), counter);
}

extern "C" int llm_set_sampling(llm_ctx* c, float temperature, uint64_t seed, int reset_draws) {
  if (!c) return fail(LLM_ERR_INVALID, "nil context");
  if (std::isnan(temperature)) return fail(LLM_ERR_INVALID, "temperature is NaN");
  RC(set_device(c));
  CU(cudaStreamSynchronize(c->stream));
  c->sample_temp = temperature > 0.f ? temperature : 0.f;
  c->sample_inv_t = c->sample_temp > 0.f ? static_cast<double>(1.0f / c->sample_temp) : 0.0;
  c->sample_seed = seed;
  if (reset_draws && c->d_draws) CU(cudaMemsetAsync(c->d_draws, 0, static_cast<size_t>(c->max_seqs) * 8, c->stream));
  // the temperature and seed are kernel arguments baked into captured steps
  for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second);
  c->graphs.clear();
  return LLM_OK;
}

extern "C" int llm_set_option(llm_ctx* c, int option, int value) {
  if (!c) return fail(LLM_ERR_INVALID, "nil context");
  bool* flag = nullptr;
  switch (option) {
    case LLM_OPT_CUDA_GRAPHS: flag = &c->use_graphs; break;
    case LLM_OPT_TCGEN05_GEMM: flag = &c->use_umma; break;
    case LLM_OPT_PDL: flag = &c->use_pdl; break;
    case LLM_OPT_OVERLAP:
      if (value < 0 || value > 2) return fail(LLM_ERR_INVALID, "overlap mode %d out of range [0, 2]", value);
      if (c->overlap != value) {
        RC(set_device(c));
        CU(cudaStreamSynchronize(c->stream));
        for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second);
        c->graphs.clear();
        c->overlap = value;
      }
      return LLM_OK;
    case LLM_OPT_OVERLAP_GRAPHS: flag = &c->overlap_graphs; break;
    case LLM_OPT_CHAIN_PDL: flag = &c->chain_pdl; break;
    case LLM_OPT_PREFILL_TILES: flag = &c->prefill_tiles; break;
    case LLM_OPT_PREFILL_TC: flag = &c->prefill_tc; break;
    case LLM_OPT_PREFILL_PERSIST: flag = &c->prefill_persist; break;
    case LLM_OPT_DECODE_SPLITK: flag = &c->decode_splitk; break;
    case LLM_OPT_ATTN_CHAIN:
      if (value < 0 || value > 1) return fail(LLM_ERR_INVALID, "attention chain mode %d out of range [0, 1]", value);
      if (c->attn_chain != value) {
        RC(set_device(c));
        CU(cudaStreamSynchronize(c->stream));
        for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second);
        c->graphs.clear();
        c->attn_chain = value;
      }
      return LLM_OK;
    case LLM_OPT_MICRO_BATCHES:
      if (value < 2 || value > kMaxParts) return fail(LLM_ERR_INVALID, "micro-batches %d out of range [2, %d]", value, kMaxParts);
      if (c->micro_batches != value) {
        RC(set_device(c));
        CU(cudaStreamSynchronize(c->stream));
        for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second);
        c->graphs.clear();
        c->micro_batches = value;
      }
      return LLM_OK;
    case LLM_OPT_PREFILL_RING_KB:
    case LLM_OPT_PREFILL_BN:
      if (value < 0 || (option == LLM_OPT_PREFILL_RING_KB && value > 200) ||
          (option == LLM_OPT_PREFILL_BN && value != 0 && value != 64 && value != 128 && value != 256))
        return fail(LLM_ERR_INVALID, "option %d value %d out of range", option, value);
      (option == LLM_OPT_PREFILL_RING_KB ? c->prefill_ring_kb : c->prefill_bn) = value;
      return LLM_OK;
    case LLM_OPT_ATTN_SPLITS:
      if (value < 0 || value > 64) return fail(LLM_ERR_INVALID, "attention splits %d out of range [0, 64]", value);
      c->attn_splits = value;  // applies from the next llm_generate_begin / step
      return LLM_OK;
    case LLM_OPT_OVERLAP_RING_KB:
      if (value < 16 || value > 200) return fail(LLM_ERR_INVALID, "ring size %d KB out of range [16, 200]", value);
      if (c->overlap_ring_kb != value) {
        RC(set_device(c));
        CU(cudaStreamSynchronize(c->stream));
        for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second);
        c->graphs.clear();
        c->overlap_ring_kb = value;
      }
      return LLM_OK;
    default: return fail(LLM_ERR_INVALID, "unknown option %d", option);
  }
  if (*flag != (value != 0)) {
    RC(set_device(c));
    CU(cudaStreamSynchronize(c->stream));
    for (auto& kv : c->graphs) cudaGraphExecDestroy(kv.second);
    c->graphs.clear();
    *flag = value != 0;
  }
  return LLM_OK;
}

// ============================================================================ introspection
extern "C" int llm_ctx_stream(llm_ctx* c, void** stream) {
  if (!c || !stream) return fail(LLM_ERR_INVALID, "nil argument");
  *stream = c->stream;
  return LLM_OK;
}

extern "C" int llm_synchronize(llm_ctx* c) {
  if (!c) return fail(LLM_ERR_INVALID, "nil context");
  RC(set_device(c));
  CU(cudaStreamSynchronize(c->stream));
  return check_device_error(c);
}

extern "C" int llm_step_parts(llm_ctx* c, int n, int* parts) {
  if (!c || !parts) return fail(LLM_ERR_INVALID, "nil argument");
  *parts = overlap_parts(c, n, true);
  return LLM_OK;
}

extern "C" int llm_step_kernel_count(llm_ctx* c, int n, int* count) {
  if (!c || !count) return fail(LLM_ERR_INVALID, "nil argument");
  // embed+norm, per layer: qkv, attention, wo, norm, w13, w2 (+ the SwiGLU quant kernel for int8)
  // + the next layer's norm, then final norm, lm_head, finish
  // + the next layer's norm, then final norm, lm_head, finish; the overlapped schedule runs the
  // per-row part once per micro-batch
  const int per_layer = 6 + (c->in8 ? 1 : 0);
  const int parts = overlap_parts(c, n, true);
  *count = parts * (1 + c->cfg.n_layers * per_layer + (c->cfg.n_layers - 1)) + 3;
  return LLM_OK;
}

extern "C" int llm_memory_bytes(llm_ctx* c, uint64_t* weights, uint64_t* kv_pool, uint64_t* other) {
  if (!c) return fail(LLM_ERR_INVALID, "nil context");
  if (weights) *weights = c->bytes_weights;
  if (kv_pool) *kv_pool = c->bytes_kv;
  if (other) *other = c->bytes_other;
  return LLM_OK;
}

// Writes gen_pos0[i] + offset into d_pos (the generate loop's position state) and waits.
int set_gen_positions(llm_ctx* c, int offset) {
  int32_t* h = c->h_pin;
  for (int i = 0; i < c->gen_n; ++i) h[i] = c->gen_pos0[i] + offset;
  CU(cudaMemcpyAsync(c->d_pos, h, c->gen_n * 4, cudaMemcpyHostToDevice, c->stream));
  CU(cudaStreamSynchronize(c->stream));
  return LLM_OK;
}

extern "C" int llm_time_attention(llm_ctx* c, int iters, double* us_per_launch, double* bytes_per_launch) {
  RC(check_ready(c));
  if (c->gen_n <= 0) return fail(LLM_ERR_STATE, "llm_generate_begin not called");
  if (c->gen_steps_done <= 0) return fail(LLM_ERR_STATE, "no generate step has run yet");
  if (iters <= 0) return fail(LLM_ERR_INVALID, "iters must be positive");
  RC(set_device(c));
  // Time the attention of the last executed step: its positions (pos0 + done - 1) have their
  // K/V written and their pages reserved.  d_pos (the next position) is restored afterwards.
  CU(cudaStreamSynchronize(c->stream));
  RC(set_gen_positions(c, c->gen_steps_done - 1));
  const llm_model_config& k = c->cfg;
  AttnParams ap{};
  ap.q = c->qbuf;
  ap.kv_pool = c->kv_pool;
  ap.block_table = c->d_block_table;
  ap.max_pages_per_seq = c->max_pages_per_seq;
  ap.seq_ids = c->d_seq;
  ap.positions = c->d_pos;
  ap.n_blocks = c->gen_n;
  ap.n_heads = k.n_heads;
  ap.n_kv_heads = k.n_kv_heads;
  ap.n_pages = c->n_pages;
  ap.splits = c->gen_splits;
  ap.ws_segs = attn_ws_segs(c);
  ap.scale_log2 = static_cast<float>(1.4426950408889634 / std::sqrt(static_cast<double>(k.head_dim)));
  ap.out = c->attn;
  ap.out_f32 = c->in8 ? 1 : 0;
  ap.ws = c->ws;
  ap.counters = c->counters;
  ap.err = c->d_err;
  cudaEvent_t e0, e1;
  CU(cudaEventCreate(&e0));
  CU(cudaEventCreate(&e1));
  // warm-up pass over every layer
  for (int l = 0; l < k.n_layers; ++l) {
    ap.layer = l;
    CU(attn_any(c->act, k.head_dim, ap, c->stream, false));
  }
  CU(cudaEventRecord(e0, c->stream));
  for (int i = 0; i < iters; ++i)
    for (int l = 0; l < k.n_layers; ++l) {
      ap.layer = l;
      CU(attn_any(c->act, k.head_dim, ap, c->stream, false));
    }
  CU(cudaEventRecord(e1, c->stream));
  CU(cudaEventSynchronize(e1));
  float ms = 0.f;
  CU(cudaEventElapsedTime(&ms, e0, e1));
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  RC(set_gen_positions(c, c->gen_steps_done));
  const double launches = static_cast<double>(iters) * k.n_layers;
  if (us_per_launch) *us_per_launch = ms * 1e3 / launches;
  if (bytes_per_launch) {
    // K and V of every cached position of the context (positions 0 .. pos0 + done - 1,
    // inclusive), the q rows read and the attention rows written
    double b = 0;
    const double per_tok = 2.0 * c->kv_dim * act_bytes(c);
    for (int i = 0; i < c->gen_n; ++i) b += per_tok * (c->gen_pos0[i] + c->gen_steps_done);
    b += static_cast<double>(c->gen_n) * c->q_dim * act_bytes(c);
    b += static_cast<double>(c->gen_n) * c->q_dim * (c->in8 ? 4.0 : static_cast<double>(act_bytes(c)));
    *bytes_per_launch = b;
  }
  return check_device_error(c);
}

extern "C" int llm_profile_step(llm_ctx* c, int iters, char* report, size_t report_len, double* step_us) {
  RC(check_ready(c));
  if (c->gen_n <= 0) return fail(LLM_ERR_STATE, "llm_generate_begin not called");
  if (c->gen_steps_done >= c->gen_max_steps)
    return fail(LLM_ERR_STATE, "no reserved generate step left to profile (reserve one more in llm_generate_begin)");
  if (iters <= 0) return fail(LLM_ERR_INVALID, "iters must be positive");
  RC(set_device(c));
  // Eager launches of the next step (its position is reserved; the K/V it writes there are
  // rewritten by the real step), with an event after each one; tokens/positions are not advanced.
  RowsSpec rs;
  rs.R = c->gen_n;
  rs.n_blocks = c->gen_n;
  rs.attn_splits = c->gen_splits;
  std::map<std::string, std::pair<int, double>> acc;
  std::vector<std::string> order;
  double total = 0;
  for (int it = 0; it <= iters; ++it) {
    std::vector<std::pair<const char*, cudaEvent_t>> tr;
    c->trace = &tr;
    int rc = enqueue_forward(c, rs);
    c->trace = nullptr;
    cudaError_t e = cudaStreamSynchronize(c->stream);
    if (!rc && e == cudaSuccess && it > 0) {  // iteration 0 warms up
      for (size_t i = 1; i < tr.size(); ++i) {
        float ms = 0.f;
        cudaEventElapsedTime(&ms, tr[i - 1].second, tr[i].second);
        auto& a = acc[tr[i].first];
        if (a.first == 0 && it == 1) order.push_back(tr[i].first);
        a.first += 1;
        a.second += ms * 1e3;
        total += ms * 1e3;
      }
    }
    for (auto& x : tr) cudaEventDestroy(x.second);
    if (rc) return rc;
    if (e != cudaSuccess) return fail(LLM_ERR_CUDA, "profile step: %s", cudaGetErrorString(e));
  }
  std::string out;
  char line[256];
  snprintf(line, sizeof line, "%-26s %7s %11s %11s %7s\n", "kernel", "count", "us/launch", "us/step", "share");
  out += line;
  for (auto& name : order) {
    auto& a = acc[name];
    snprintf(line, sizeof line, "%-26s %7d %11.2f %11.2f %6.1f%%\n", name.c_str(), a.first / iters, a.second / a.first,
             a.second / iters, 100.0 * a.second / total);
    out += line;
  }
  snprintf(line, sizeof line, "%-26s %7s %11s %11.2f\n", "total (eager)", "", "", total / iters);
  out += line;
  if (report && report_len) {
    size_t n = std::min(report_len - 1, out.size());
    memcpy(report, out.data(), n);
    report[n] = 0;
  }
  if (step_us) *step_us = total / iters;
  return check_device_error(c);
}

namespace {
// Start recording launch timelines: every following enqueue_forward appends its launches
// (up to kTraceCap) until trace_finish.
int trace_begin(llm_ctx* c) {
  RC(set_device(c));
  if (!c->d_trace) RC(dalloc_t(c, &c->d_trace, kTraceCap * sizeof(TraceRec), &c->bytes_other));
  std::vector<TraceRec> h(kTraceCap, TraceRec{~0ull, 0ull, 0ull, 0ull});
  CU(cudaMemcpyAsync(c->d_trace, h.data(), kTraceCap * sizeof(TraceRec), cudaMemcpyHostToDevice, c->stream));
  CU(cudaStreamSynchronize(c->stream));
  c->trace_labels.clear();
  c->tracing = true;
  return LLM_OK;
}

// Stop recording and format one line per recorded launch.
int trace_finish(llm_ctx* c, char* report, size_t report_len, double* span_us) {
  c->tracing = false;
  RC(set_device(c));
  CU(cudaStreamSynchronize(c->stream));
  if (!c->d_trace) return fail(LLM_ERR_STATE, "no trace recorded");
  std::vector<TraceRec> h(kTraceCap);
  CU(cudaMemcpy(h.data(), c->d_trace, kTraceCap * sizeof(TraceRec), cudaMemcpyDeviceToHost));
  unsigned long long t0 = ~0ull, t1 = 0;
  for (size_t i = 0; i < c->trace_labels.size(); ++i)
    if (h[i].ctas) {
      t0 = std::min(t0, h[i].first_start);
      t1 = std::max(t1, h[i].last_end);
    }
  std::string out;
  char line[160];
  snprintf(line, sizeof line, "%-22s %10s %10s %10s %10s %6s\n", "launch", "start_us", "spread_us", "end_us", "dur_us", "ctas");
  out += line;
  for (size_t i = 0; i < c->trace_labels.size(); ++i) {
    const TraceRec& r = h[i];
    if (!r.ctas) continue;
    snprintf(line, sizeof line, "%-22s %10.2f %10.2f %10.2f %10.2f %6llu\n", c->trace_labels[i].c_str(),
             (r.first_start - t0) * 1e-3, (r.last_start - r.first_start) * 1e-3, (r.last_end - t0) * 1e-3,
             (r.last_end - r.first_start) * 1e-3, r.ctas);
    out += line;
  }
  if (report && report_len) {
    const size_t n = std::min(report_len - 1, out.size());
    memcpy(report, out.data(), n);
    report[n] = 0;
  }
  if (span_us) *span_us = t1 > t0 ? (t1 - t0) * 1e-3 : 0.0;
  return check_device_error(c);
}
}  // namespace

extern "C" int llm_trace_step(llm_ctx* c, char* report, size_t report_len, double* step_us) {
  RC(check_ready(c));
  if (c->gen_n <= 0) return fail(LLM_ERR_STATE, "llm_generate_begin not called");
  if (c->gen_steps_done >= c->gen_max_steps)
    return fail(LLM_ERR_STATE, "no reserved generate step left to trace (reserve one more in llm_generate_begin)");
  RC(trace_begin(c));
  // The next step of the generate batch (its position is reserved), launched eagerly in the
  // current schedule; tokens and positions are not advanced.
  RowsSpec rs;
  rs.R = c->gen_n;
  rs.n_blocks = c->gen_n;
  rs.attn_splits = c->gen_splits;
  const int rc = enqueue_forward(c, rs);
  if (rc) {
    c->tracing = false;
    return rc;
  }
  return trace_finish(c, report, report_len, step_us);
}

extern "C" int llm_trace_begin(llm_ctx* c) {
  RC(check_ready(c));
  return trace_begin(c);
}

extern "C" int llm_trace_end(llm_ctx* c, char* report, size_t report_len, double* span_us) {
  if (!c) return fail(LLM_ERR_INVALID, "nil context");
  return trace_finish(c, report, report_len, span_us);
}

extern "C" int llm_debug_read_kv(llm_ctx* c, int layer, int seq, int pos, float* kout, float* vout) {
  RC(check_ready(c));
  if (layer < 0 || layer >= c->cfg.n_layers) return fail(LLM_ERR_INVALID, "layer %d out of range", layer);
  if (seq < 0 || seq >= c->max_seqs) return fail(LLM_ERR_INVALID, "sequence %d out of range", seq);
  if (pos < 0 || pos / 16 >= c->seq_npages[seq]) return fail(LLM_ERR_POS_RANGE, "position out of range: %d", pos);
  RC(set_device(c));
  const int page = c->h_block_table[static_cast<size_t>(seq) * c->max_pages_per_seq + pos / 16];
  float* d = nullptr;
  CU(cudaMalloc(&d, 2 * c->kv_dim * 4));
  const int n = 2 * c->kv_dim;
  if (c->act == 1)
    read_kv_kernel<__half><<<(n + 255) / 256, 256, 0, c->stream>>>(static_cast<const __half*>(c->kv_pool), layer, c->n_pages,
                                                                  c->cfg.n_kv_heads, c->cfg.head_dim, page, pos & 15, d, d + c->kv_dim);
  else
    read_kv_kernel<__nv_bfloat16><<<(n + 255) / 256, 256, 0, c->stream>>>(static_cast<const __nv_bfloat16*>(c->kv_pool), layer,
                                                                          c->n_pages, c->cfg.n_kv_heads, c->cfg.head_dim, page,
                                                                          pos & 15, d, d + c->kv_dim);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  if (e == cudaSuccess) e = cudaMemcpy(kout, d, c->kv_dim * 4, cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemcpy(vout, d + c->kv_dim, c->kv_dim * 4, cudaMemcpyDeviceToHost);
  cudaFree(d);
  if (e != cudaSuccess) return fail(LLM_ERR_CUDA, "read kv: %s", cudaGetErrorString(e));
  return LLM_OK;
}

// ============================================================================ debug hooks
namespace {
struct DevBuf {
  void* p = nullptr;
  ~DevBuf() {
    if (p) cudaFree(p);
  }
};
}  // namespace

extern "C" int llm_debug_norm_quant(int device, const float* x, const float* w, int rows, int cols, double eps, int8_t* q,
                                    float* scales) {
  if (!x || !q || !scales || rows <= 0 || cols <= 0 || cols % 4) return fail(LLM_ERR_INVALID, "bad arguments");
  CU(cudaSetDevice(device));
  DevBuf dx, dw, dq, ds;
  CU(cudaMalloc(&dx.p, static_cast<size_t>(rows) * cols * 4));
  CU(cudaMalloc(&dq.p, static_cast<size_t>(rows) * cols));
  CU(cudaMalloc(&ds.p, rows * 4));
  CU(cudaMemcpy(dx.p, x, static_cast<size_t>(rows) * cols * 4, cudaMemcpyHostToDevice));
  if (w) {
    CU(cudaMalloc(&dw.p, cols * 4));
    CU(cudaMemcpy(dw.p, w, cols * 4, cudaMemcpyHostToDevice));
  }
  NormParams np{};
  np.x = static_cast<const float*>(dx.p);
  np.w = static_cast<const float*>(dw.p);
  np.D = cols;
  np.rows = rows;
  np.eps = eps;
  np.q = static_cast<int8_t*>(dq.p);
  np.scale = static_cast<float*>(ds.p);
  CU(norm_any(2, true, np, 0));
  CU(cudaDeviceSynchronize());
  CU(cudaMemcpy(q, dq.p, static_cast<size_t>(rows) * cols, cudaMemcpyDeviceToHost));
  CU(cudaMemcpy(scales, ds.p, rows * 4, cudaMemcpyDeviceToHost));
  return LLM_OK;
}

namespace {
int debug_gemm(int device, bool in8, int act, const void* hA, const void* hB, size_t esz, int M, int N, int K, int splits,
               int epi, void* hC, bool umma_path) {
  CU(cudaSetDevice(device));
  cudaDeviceProp prop{};
  CU(cudaGetDeviceProperties(&prop, device));
  DevBuf dA, dB, dC, dws, dcnt, dsa, dsb;
  CU(cudaMalloc(&dA.p, static_cast<size_t>(M) * K * esz));
  CU(cudaMalloc(&dB.p, static_cast<size_t>(N) * K * esz));
  CU(cudaMalloc(&dC.p, static_cast<size_t>(M) * N * 4));
  CU(cudaMemcpy(dA.p, hA, static_cast<size_t>(M) * K * esz, cudaMemcpyHostToDevice));
  CU(cudaMemcpy(dB.p, hB, static_cast<size_t>(N) * K * esz, cudaMemcpyHostToDevice));
  const size_t ws_cap = 32u << 20;
  CU(cudaMalloc(&dws.p, ws_cap * 4));
  CU(cudaMalloc(&dcnt.p, 65536 * 4));
  CU(cudaMemset(dcnt.p, 0, 65536 * 4));
  GemmPlan pl = plan_gemm(M, N, K, in8 ? 1 : 2, prop.multiProcessorCount, umma_path ? 0 : splits, ws_cap);
  GemmParams p{};
  p.A = dA.p;
  p.B = dB.p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.k_splits = pl.splits;
  p.k_tiles_per_split = pl.kts;
  p.ws = static_cast<float*>(dws.p);
  p.counters = static_cast<int*>(dcnt.p);
  p.out = dC.p;
  p.ldo = N;
  if (umma_path) {
    // splits: -1 = the model's channel tile, -bn = that tile width, -(1000 + S) = split-K over
    // clusters of S = 2, 4 or 8 CTAs (the decode projections' form)
    const int ks = splits <= -1000 ? -splits - 1000 : 1;
    if (ks != 1 && ks != 2 && ks != 4 && ks != 8) return fail(LLM_ERR_INVALID, "split-K %d not in {2, 4, 8}", ks);
    if (ks > 1 && (N % 4 || (K * static_cast<int>(esz) / 128) < ks))
      return fail(LLM_ERR_INVALID, "split-K %d needs channels in fours and a K slice per split", ks);
    const int bn = splits <= -2 && splits > -1000 ? -splits
                                                  : umma_bn_for(M, N, epi, 0, std::max(1, prop.multiProcessorCount / ks),
                                                                ks == 2 ? 128 : 256);
    if (!umma_bn_supported(epi, bn)) return fail(LLM_ERR_INVALID, "unsupported tcgen05 channel tile %d", bn);
    CUtensorMap tw{}, tx{};
    RC(make_kmajor_map(&tx, dA.p, static_cast<int>(esz), act == 2, K, M, kUmmaTokens));
    RC(make_kmajor_map(&tw, dB.p, static_cast<int>(esz), act == 2, K, N, bn));
    DevBuf derr;
    CU(cudaMalloc(&derr.p, 4));
    CU(cudaMemset(derr.p, 0, 4));
    p.k_splits = ks;
    p.k_tiles_per_split = K * static_cast<int>(esz) / 128 / ks;
    p.err = static_cast<int*>(derr.p);
    dim3 grid((M + kUmmaTokens - 1) / kUmmaTokens, (N + bn - 1) / bn, ks);
    CU(umma_any(act, in8, tx, tw, p, epi, bn, grid, 0, true));
    t_cluster_z = ks;
    const cudaError_t le = umma_any(act, in8, tx, tw, p, epi, bn, grid, 0, false);
    t_cluster_z = 1;
    CU(le);
    CU(cudaDeviceSynchronize());
    int herr = 0;
    CU(cudaMemcpy(&herr, derr.p, 4, cudaMemcpyDeviceToHost));
    if (herr) return fail(LLM_ERR_DEVICE, "tcgen05 GEMM reported device error %d", herr);
    CU(cudaMemcpy(hC, dC.p, static_cast<size_t>(M) * N * 4, cudaMemcpyDeviceToHost));
    return LLM_OK;
  }
  CU(gemm_any(act, in8, p, epi, pl.bm, pl.grid, 0, true));
  CU(gemm_any(act, in8, p, epi, pl.bm, pl.grid, 0, false));
  CU(cudaDeviceSynchronize());
  CU(cudaMemcpy(hC, dC.p, static_cast<size_t>(M) * N * 4, cudaMemcpyDeviceToHost));
  return LLM_OK;
}
}  // namespace

// A wait that nothing completes: one mbarrier expecting an arrival that never comes, polled at
// most `polls` times, then the kernel records kDevWaitTimeout and returns (the failure path of
// every bounded wait in the token loop's kernels).
__global__ void wait_probe_kernel(uint32_t polls, int* err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
  }
  __syncthreads();
  bool done = false;
  for (uint32_t i = 0; i < polls && !done; ++i) done = mbar_try_wait(smem_u32(&bar), 0);
  if (!done && threadIdx.x == 0) atomicExch(err, kDevWaitTimeout);
}

extern "C" int llm_debug_wait_timeout(int device, uint32_t polls) {
  if (cudaSetDevice(device) != cudaSuccess) return fail(LLM_ERR_CUDA, "cudaSetDevice(%d) failed", device);
  DevBuf derr;
  CU(cudaMalloc(&derr.p, 4));
  CU(cudaMemset(derr.p, 0, 4));
  wait_probe_kernel<<<1, 32>>>(polls, static_cast<int*>(derr.p));
  CU(cudaGetLastError());
  CU(cudaDeviceSynchronize());
  int h = 0;
  CU(cudaMemcpy(&h, derr.p, 4, cudaMemcpyDeviceToHost));
  if (h) return fail(LLM_ERR_DEVICE, "kernel reported device error %d (%s)", h,
                     h == kDevWaitTimeout ? "bounded wait expired" : "unknown");
  return LLM_OK;
}

extern "C" int llm_debug_sample(int device, const float* logits, int rows, int vocab, float temperature,
                                const double* u, int32_t* out) {
  if (!logits || !u || !out || rows <= 0 || vocab <= 0) return fail(LLM_ERR_INVALID, "bad arguments");
  if (!(temperature > 1e-6f)) return fail(LLM_ERR_INVALID, "temperature %g takes the greedy path", static_cast<double>(temperature));
  if (cudaSetDevice(device) != cudaSuccess) return fail(LLM_ERR_CUDA, "cudaSetDevice(%d) failed", device);
  DevBuf dl, du, dout;
  CU(cudaMalloc(&dl.p, static_cast<size_t>(rows) * vocab * 4));
  CU(cudaMalloc(&du.p, static_cast<size_t>(rows) * 8));
  CU(cudaMalloc(&dout.p, static_cast<size_t>(rows) * 4));
  CU(cudaMemcpy(dl.p, logits, static_cast<size_t>(rows) * vocab * 4, cudaMemcpyHostToDevice));
  CU(cudaMemcpy(du.p, u, static_cast<size_t>(rows) * 8, cudaMemcpyHostToDevice));
  SampleParams sp{};
  sp.logits = static_cast<const float*>(dl.p);
  sp.rows = rows;
  sp.V = vocab;
  sp.ld = vocab;
  sp.inv_t = static_cast<double>(1.0f / temperature);
  sp.u = static_cast<const double*>(du.p);
  sp.out = static_cast<int*>(dout.p);
  sample_kernel<<<rows, kSampleThreads>>>(sp);
  CU(cudaGetLastError());
  CU(cudaDeviceSynchronize());
  CU(cudaMemcpy(out, dout.p, static_cast<size_t>(rows) * 4, cudaMemcpyDeviceToHost));
  return LLM_OK;
}

__global__ void exp2_probe_kernel(const float* x, float* y, int n) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) y[i] = exp2_det(x[i]);
}

extern "C" int llm_debug_exp2(int device, const float* x, int n, float* out) {
  if (!x || !out || n <= 0) return fail(LLM_ERR_INVALID, "bad arguments");
  if (cudaSetDevice(device) != cudaSuccess) return fail(LLM_ERR_CUDA, "cudaSetDevice(%d) failed", device);
  DevBuf dx, dy;
  CU(cudaMalloc(&dx.p, static_cast<size_t>(n) * 4));
  CU(cudaMalloc(&dy.p, static_cast<size_t>(n) * 4));
  CU(cudaMemcpy(dx.p, x, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice));
  exp2_probe_kernel<<<(n + 255) / 256, 256>>>(static_cast<const float*>(dx.p), static_cast<float*>(dy.p), n);
  CU(cudaGetLastError());
  CU(cudaDeviceSynchronize());
  CU(cudaMemcpy(out, dy.p, static_cast<size_t>(n) * 4, cudaMemcpyDeviceToHost));
  return LLM_OK;
}

extern "C" int llm_debug_gemm_i8(int device, const int8_t* A, const int8_t* B, int M, int N, int K, int splits, int32_t* C) {
  if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0 || K % 128) return fail(LLM_ERR_INVALID, "bad arguments (K %% 128 == 0)");
  // splits < 0 selects the tcgen05 kernel (-1: the model's channel tile, -bn: tile width bn,
  // -(1000 + S): split-K over clusters of S CTAs), otherwise the warp-level kernel with that
  // split (0: its automatic plan)
  return debug_gemm(device, true, 2, A, B, 1, M, N, K, splits, EPI_S32, C, splits < 0);
}

extern "C" int llm_debug_gemm_f16(int device, int dtype, const float* A, const float* B, int M, int N, int K, int splits,
                                  float* C) {
  if (!A || !B || !C || M <= 0 || N <= 0 || K <= 0 || K % 64 || N % 2) return fail(LLM_ERR_INVALID, "bad arguments");
  if (dtype != LLM_DTYPE_F16 && dtype != LLM_DTYPE_BF16) return fail(LLM_ERR_INVALID, "dtype must be F16 or BF16");
  const int act = dtype == LLM_DTYPE_F16 ? 1 : 2;
  // round on the device with the model's conversion
  CU(cudaSetDevice(device));
  DevBuf fA, fB, hA, hB;
  const size_t na = static_cast<size_t>(M) * K, nb = static_cast<size_t>(N) * K;
  CU(cudaMalloc(&fA.p, na * 4));
  CU(cudaMalloc(&fB.p, nb * 4));
  CU(cudaMalloc(&hA.p, na * 2));
  CU(cudaMalloc(&hB.p, nb * 2));
  CU(cudaMemcpy(fA.p, A, na * 4, cudaMemcpyHostToDevice));
  CU(cudaMemcpy(fB.p, B, nb * 4, cudaMemcpyHostToDevice));
  if (act == 1) {
    f32_to_act_kernel<__half><<<(na + 255) / 256, 256>>>(static_cast<float*>(fA.p), static_cast<__half*>(hA.p), na);
    f32_to_act_kernel<__half><<<(nb + 255) / 256, 256>>>(static_cast<float*>(fB.p), static_cast<__half*>(hB.p), nb);
  } else {
    f32_to_act_kernel<__nv_bfloat16><<<(na + 255) / 256, 256>>>(static_cast<float*>(fA.p), static_cast<__nv_bfloat16*>(hA.p), na);
    f32_to_act_kernel<__nv_bfloat16><<<(nb + 255) / 256, 256>>>(static_cast<float*>(fB.p), static_cast<__nv_bfloat16*>(hB.p), nb);
  }
  CU(cudaGetLastError());
  std::vector<uint16_t> ha(na), hb(nb);
  CU(cudaMemcpy(ha.data(), hA.p, na * 2, cudaMemcpyDeviceToHost));
  CU(cudaMemcpy(hb.data(), hB.p, nb * 2, cudaMemcpyDeviceToHost));
  return debug_gemm(device, false, act, ha.data(), hb.data(), 2, M, N, K, splits, EPI_F32, C, splits < 0);
}

// ============================================================================ linear kernels
// model.Compile / Kernel.WriteInputF32 / EvalWithStats / ReadOutputF32 of a 1x1 convolution
// (ane/model/model_darwin.go:138-414, ane/forward/conv.go:11-48): y[out][t] = sum_i W[out][i] x[i][t]
// on channel-first fp32 tensors, run as one tcgen05 GEMM with the token loop's arithmetic
// (16-bit: inputs and weights rounded, f32 accumulate; W8A8: per-row int8 weights, per-token int8
// inputs, int32 accumulate, (acc * s_x) * s_w).
struct llm_linear {
  int device = 0, act = 2, in8 = 0, out_dim = 0, in_dim = 0, bn = 16;
  void* w = nullptr;
  float* w_scale = nullptr;
  CUtensorMap tw{};
  int cap = 0;  // tokens the buffers below hold
  float *x_cf = nullptr, *x_t = nullptr, *y = nullptr, *y_cf = nullptr, *xs = nullptr;
  void* xa = nullptr;
  int* err = nullptr;
  cudaStream_t stream = nullptr;
  cudaEvent_t e0 = nullptr, e1 = nullptr;
};

namespace {
void linear_free_bufs(llm_linear* k) {
  for (void* p : {static_cast<void*>(k->x_cf), static_cast<void*>(k->x_t), static_cast<void*>(k->y),
                  static_cast<void*>(k->y_cf), static_cast<void*>(k->xs), k->xa})
    if (p) cudaFree(p);
  k->x_cf = k->x_t = k->y = k->y_cf = k->xs = nullptr;
  k->xa = nullptr;
  k->cap = 0;
}
}  // namespace

extern "C" int llm_linear_destroy(llm_linear* k) {
  if (!k) return LLM_OK;
  cudaSetDevice(k->device);
  if (k->stream) cudaStreamSynchronize(k->stream);
  linear_free_bufs(k);
  if (k->w) cudaFree(k->w);
  if (k->w_scale) cudaFree(k->w_scale);
  if (k->err) cudaFree(k->err);
  if (k->e0) cudaEventDestroy(k->e0);
  if (k->e1) cudaEventDestroy(k->e1);
  if (k->stream) cudaStreamDestroy(k->stream);
  delete k;
  return LLM_OK;
}

extern "C" int llm_linear_create(int device, int dtype, const float* w, int out_dim, int in_dim, llm_linear** out) {
  if (!w || !out) return fail(LLM_ERR_INVALID, "nil argument");
  if (dtype < LLM_DTYPE_F16 || dtype > LLM_DTYPE_W8A8_BF16) return fail(LLM_ERR_INVALID, "unknown dtype %d", dtype);
  if (out_dim <= 0 || in_dim <= 0 || out_dim % 16 || in_dim % 128)
    return fail(LLM_ERR_INVALID, "linear %dx%d: out_dim must be a multiple of 16 and in_dim of 128", out_dim, in_dim);
  if (cudaSetDevice(device) != cudaSuccess) return fail(LLM_ERR_CUDA, "cudaSetDevice(%d) failed", device);
  std::unique_ptr<llm_linear, int (*)(llm_linear*)> k(new llm_linear(), llm_linear_destroy);
  k->device = device;
  k->in8 = dtype == LLM_DTYPE_W8A8_F16 || dtype == LLM_DTYPE_W8A8_BF16;
  k->act = (dtype == LLM_DTYPE_F16 || dtype == LLM_DTYPE_W8A8_F16) ? 1 : 2;
  k->out_dim = out_dim;
  k->in_dim = in_dim;
  CU(cudaStreamCreateWithFlags(&k->stream, cudaStreamNonBlocking));
  CU(cudaEventCreate(&k->e0));
  CU(cudaEventCreate(&k->e1));
  CU(cudaMalloc(&k->err, 4));
  CU(cudaMemsetAsync(k->err, 0, 4, k->stream));
  const size_t n = static_cast<size_t>(out_dim) * in_dim;
  CU(cudaMalloc(&k->w, n * (k->in8 ? 1 : 2)));
  if (k->in8) CU(cudaMalloc(&k->w_scale, static_cast<size_t>(out_dim) * 4));
  DevBuf tmp;
  CU(cudaMalloc(&tmp.p, n * 4));
  // on the kernel's own (non-blocking) stream: a synchronous copy from pageable memory may
  // return before its DMA lands, and that stream does not wait for the legacy stream
  CU(cudaMemcpyAsync(tmp.p, w, n * 4, cudaMemcpyHostToDevice, k->stream));
  ConvertParams cp{static_cast<const float*>(tmp.p), out_dim, in_dim, 1, 0, k->w, k->w_scale};
  const dim3 grid((out_dim + 7) / 8);
  if (k->in8) convert_rows_kernel<int8_t><<<grid, 256, 0, k->stream>>>(cp);
  else if (k->act == 1) convert_rows_kernel<__half><<<grid, 256, 0, k->stream>>>(cp);
  else convert_rows_kernel<__nv_bfloat16><<<grid, 256, 0, k->stream>>>(cp);
  CU(cudaGetLastError());
  CU(cudaStreamSynchronize(k->stream));
  *out = k.release();
  return LLM_OK;
}

extern "C" int llm_linear_eval_cf(llm_linear* k, const float* x_cf, int s, float* y_cf, uint64_t* hw_ns) {
  if (!k || !x_cf || !y_cf) return fail(LLM_ERR_INVALID, "nil argument");
  if (s <= 0) return fail(LLM_ERR_INVALID, "sequence length %d must be positive", s);
  CU(cudaSetDevice(k->device));
  const int I = k->in_dim, O = k->out_dim;
  if (s > k->cap) {
    CU(cudaStreamSynchronize(k->stream));
    linear_free_bufs(k);
    const size_t si = static_cast<size_t>(s) * I, so = static_cast<size_t>(s) * O;
    CU(cudaMalloc(&k->x_cf, si * 4));
    CU(cudaMalloc(&k->x_t, si * 4));
    CU(cudaMalloc(&k->xa, si * (k->in8 ? 1 : 2)));
    CU(cudaMalloc(&k->xs, static_cast<size_t>(s) * 4));
    CU(cudaMalloc(&k->y, so * 4));
    CU(cudaMalloc(&k->y_cf, so * 4));
    k->cap = s;
  }
  cudaDeviceProp prop{};
  CU(cudaGetDeviceProperties(&prop, k->device));
  const int esz = k->in8 ? 1 : 2;
  const int bn = umma_bn_for(s, O, EPI_F32, 0, prop.multiProcessorCount);
  CUtensorMap tx{}, tw{};
  RC(make_kmajor_map(&tx, k->xa, esz, k->act == 2, I, s, kUmmaTokens));
  RC(make_kmajor_map(&tw, k->w, esz, k->act == 2, I, O, bn));
  GemmParams p{};
  p.A = k->xa;
  p.B = k->w;
  p.M = s;
  p.N = O;
  p.K = I;
  p.a_scale = k->xs;
  p.b_scale = k->w_scale;
  p.out = k->y;
  p.ldo = O;
  p.k_splits = 1;
  p.k_tiles_per_split = I * esz / 128;
  p.err = k->err;
  CU(umma_any(k->act, k->in8, tx, tw, p, EPI_F32, bn, dim3(1), k->stream, true));
  CU(cudaMemcpyAsync(k->x_cf, x_cf, static_cast<size_t>(s) * I * 4, cudaMemcpyHostToDevice, k->stream));
  CU(cudaEventRecord(k->e0, k->stream));
  // channel-first [I][s] -> token rows [s][I]
  transpose_rows_kernel<<<dim3((s + 31) / 32, (I + 31) / 32), dim3(32, 8), 0, k->stream>>>(k->x_cf, I, s, k->x_t);
  CU(cudaGetLastError());
  if (k->in8) {
    NormParams np_{};
    np_.x = k->x_t;
    np_.w = nullptr;  // the per-token quantiser alone
    np_.D = I;
    np_.rows = s;
    np_.q = static_cast<int8_t*>(k->xa);
    np_.scale = k->xs;
    CU(norm_any(k->act, true, np_, k->stream));
  } else if (k->act == 1) {
    f32_to_act_kernel<__half><<<(static_cast<size_t>(s) * I + 255) / 256, 256, 0, k->stream>>>(
        k->x_t, static_cast<__half*>(k->xa), static_cast<size_t>(s) * I);
  } else {
    f32_to_act_kernel<__nv_bfloat16><<<(static_cast<size_t>(s) * I + 255) / 256, 256, 0, k->stream>>>(
        k->x_t, static_cast<__nv_bfloat16*>(k->xa), static_cast<size_t>(s) * I);
  }
  CU(cudaGetLastError());
  const dim3 grid((s + kUmmaTokens - 1) / kUmmaTokens, (O + bn - 1) / bn, 1);
  CU(umma_any(k->act, k->in8, tx, tw, p, EPI_F32, bn, grid, k->stream, false));
  // token rows [s][O] -> channel-first [O][s]
  transpose_rows_kernel<<<dim3((O + 31) / 32, (s + 31) / 32), dim3(32, 8), 0, k->stream>>>(k->y, s, O, k->y_cf);
  CU(cudaGetLastError());
  CU(cudaEventRecord(k->e1, k->stream));
  CU(cudaMemcpyAsync(y_cf, k->y_cf, static_cast<size_t>(s) * O * 4, cudaMemcpyDeviceToHost, k->stream));
  int herr = 0;
  CU(cudaMemcpyAsync(&herr, k->err, 4, cudaMemcpyDeviceToHost, k->stream));
  CU(cudaStreamSynchronize(k->stream));
  if (herr) {
    cudaMemsetAsync(k->err, 0, 4, k->stream);
    return fail(LLM_ERR_DEVICE, "linear kernel reported device error %d", herr);
  }
  if (hw_ns) {
    float ms = 0.f;
    CU(cudaEventElapsedTime(&ms, k->e0, k->e1));
    *hw_ns = static_cast<uint64_t>(static_cast<double>(ms) * 1e6);
  }
  return LLM_OK;
}
