// noalloc.cu -- an allocation-free variant of the split-K int8 GEMM.
//
// Some callers cannot allocate device memory while they run.  A serving loop that reserved
// nearly all of HBM for its KV page pool at start-up has nothing left for a new cudaMalloc;
// a decode loop cannot afford the device-wide synchronisation that cudaFree implies in the
// middle of a step; and a host that embeds this library behind an FFI (a Go program through
// cgo, for example) may own the memory policy and forbid the library from allocating on its
// own.  For them, llm_gemm_i8_splitk_noalloc takes caller-owned device buffers for its
// inputs and output and keeps the split-K scratch (per-split partial tiles and the per-tile
// arrival counters) in one file-scope device array of fixed size, so a call allocates
// nothing.
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <mutex>

#include "../../include/llm_cuda.h"
#include "gemm.cuh"

using namespace llm;

// Sets the thread's last error (defined in llm_cuda.cu) and returns `code`.
int llm_detail_fail(int code, const char* msg);

namespace {

constexpr size_t kNoAllocPartialFloats = size_t{1} << 20;  // 4 MiB of split partials
constexpr int kNoAllocCounters = 1024;                     // per-tile arrival counters
constexpr int kNoAllocMaxDevices = 64;

// The scratch every call shares.  Partials first, then the counters (as int bit patterns).
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocPartialFloats + kNoAllocCounters];

std::mutex g_setup_mu;
void* g_scratch_addr[kNoAllocMaxDevices] = {};

int fail_fmt(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  return llm_detail_fail(code, buf);
}

template <int BM>
cudaError_t launch(const GemmParams& p, dim3 grid, cudaStream_t s) {
  constexpr int smem = gemm_smem_bytes<BM, 128, 4>();
  gemm_kernel<int8_t, __nv_bfloat16, BM, 128, 4, EPI_S32><<<grid, kGemmThreads, smem, s>>>(p);
  return cudaGetLastError();
}

// One-time set-up on `device` (the caller made it current): resolve the device address of
// the scratch array (its host-side name is only a stand-in) and raise the kernels' dynamic
// shared-memory limit.
int setup(int device, void** addr) {
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (g_scratch_addr[device]) {
    *addr = g_scratch_addr[device];
    return LLM_OK;
  }
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
  if (e != cudaSuccess) return fail_fmt(LLM_ERR_CUDA, "cudaGetSymbolAddress(scratch) failed: %s", cudaGetErrorString(e));
  e = cudaFuncSetAttribute(gemm_kernel<int8_t, __nv_bfloat16, 64, 128, 4, EPI_S32>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize, gemm_smem_bytes<64, 128, 4>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(gemm_kernel<int8_t, __nv_bfloat16, 128, 128, 4, EPI_S32>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, gemm_smem_bytes<128, 128, 4>());
  if (e != cudaSuccess) return fail_fmt(LLM_ERR_CUDA, "kernel set-up failed: %s", cudaGetErrorString(e));
  g_scratch_addr[device] = p;
  *addr = p;
  return LLM_OK;
}

}  // namespace

extern "C" int llm_gemm_i8_splitk_noalloc(int device, const int8_t* A, const int8_t* B, int M, int N, int K,
                                          int splits, int32_t* C, void* stream) {
  if (!A || !B || !C) return fail_fmt(LLM_ERR_INVALID, "nil device buffer");
  // the kernel reads A and B with 16-byte copies and stores C as int32: a misaligned pointer
  // (an FFI slice at an odd offset) would fault on the device instead of failing here
  if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(C) % 4 != 0)
    return fail_fmt(LLM_ERR_INVALID, "misaligned device buffer (A and B need 16-byte, C 4-byte alignment)");
  if (M <= 0 || N <= 0 || K <= 0 || K % 128)
    return fail_fmt(LLM_ERR_INVALID, "bad shape M=%d N=%d K=%d (K must be a positive multiple of 128)", M, N, K);
  if (device < 0 || device >= kNoAllocMaxDevices) return fail_fmt(LLM_ERR_INVALID, "device %d out of range", device);
  // the split plan of the warp-level GEMM: BM x 128 tiles, K in 128-byte slices
  const int bm = M <= 64 ? 64 : 128;
  const int tiles_m = (M + bm - 1) / bm, tiles_n = (N + 127) / 128;
  const int tiles = tiles_m * tiles_n;
  const int k_tiles = K / 128;
  if (splits < 1) splits = 1;
  if (splits > k_tiles) splits = k_tiles;
  const int kts = (k_tiles + splits - 1) / splits;
  const int eff = (k_tiles + kts - 1) / kts;
  const size_t need = eff > 1 ? static_cast<size_t>(eff) * tiles * bm * 128 : 0;
  if (need > kNoAllocPartialFloats || (eff > 1 && tiles > kNoAllocCounters))
    return fail_fmt(LLM_ERR_INVALID,
                    "split-K scratch for M=%d N=%d splits=%d needs %zu partial floats and %d counters; the fixed "
                    "array holds %zu and %d (use fewer splits or a smaller GEMM)",
                    M, N, eff, need, tiles, kNoAllocPartialFloats, kNoAllocCounters);

  int prev = 0;
  if (cudaGetDevice(&prev) != cudaSuccess) return fail_fmt(LLM_ERR_CUDA, "cudaGetDevice failed");
  if (cudaSetDevice(device) != cudaSuccess) return fail_fmt(LLM_ERR_CUDA, "cudaSetDevice(%d) failed", device);
  void* scratch = nullptr;
  int rc = setup(device, &scratch);
  if (rc == LLM_OK) {
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float* ws = static_cast<float*>(scratch);
    int* counters = reinterpret_cast<int*>(ws + kNoAllocPartialFloats);
    // counters must start at zero; the previous call's last CTAs reset theirs, but a call
    // that did not complete could have left some behind
    cudaError_t e = eff > 1 ? cudaMemsetAsync(counters, 0, sizeof(int) * tiles, s) : cudaSuccess;
    if (e == cudaSuccess) {
      GemmParams p{};
      p.A = A;
      p.B = B;
      p.M = M;
      p.N = N;
      p.K = K;
      p.k_splits = eff;
      p.k_tiles_per_split = kts;
      p.ws = ws;
      p.counters = counters;
      p.out = C;
      p.ldo = N;
      dim3 grid(tiles_m, tiles_n, eff);
      e = bm == 64 ? launch<64>(p, grid, s) : launch<128>(p, grid, s);
    }
    if (e != cudaSuccess) rc = fail_fmt(LLM_ERR_CUDA, "split-K launch failed: %s", cudaGetErrorString(e));
  }
  cudaSetDevice(prev);
  return rc;
}
