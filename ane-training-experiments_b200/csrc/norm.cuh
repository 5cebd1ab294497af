// norm.cuh -- row kernels: embedding gather, RMSNorm, per-token int8 quantisation.
//
// One CTA per row (see norm_rows_kernel for the thread layout and the fixed float64
// summation order); explicit round-to-nearest intrinsics keep fused multiply-adds out, and
// the CPU oracle restates the same order for its bit-exact quantiser check.
//
// Reference arithmetic: ane/stories/infer.go:301-311 (rmsNormVec: float64 sum, f32 rrms,
// x*rrms*w), bridge/ane_bridge.m:374-398 (quantiser, applied per row).
#pragma once
#include "common.cuh"

namespace llm {

struct NormParams {
  const float* x;          // [rows][D] residual stream (ignored when embed != nullptr)
  const int* row_index;    // optional: row r reads x row row_index[r]
  const void* embed;       // optional [vocab][D] act-type table: gather tokens[r] into x_out
  const int* tokens;       // [rows] (with embed)
  float* x_out;            // [rows][D] gathered rows (with embed)
  const float* w;          // [D] norm weight; nullptr = quantise only (no norm)
  int D;
  int rows;
  double eps;
  void* out;               // [rows][D] act type (when !QUANT)
  int8_t* q;               // [rows][D] (QUANT)
  float* scale;            // [rows]    (QUANT)
  TraceRec* trace;         // llm_trace_step
};

// Convert 4 activation-type values to float.
template <typename T>
__device__ __forceinline__ float4 load4_act(const T* p) {
  uint2 raw = *reinterpret_cast<const uint2*>(p);
  const T* h = reinterpret_cast<const T*>(&raw);
  return make_float4(ActTraits<T>::to_f(h[0]), ActTraits<T>::to_f(h[1]), ActTraits<T>::to_f(h[2]),
                     ActTraits<T>::to_f(h[3]));
}

// One CTA per row: thread t of the row's nt = D/(4*NV) threads holds the float4 groups
// starting at elements 4*t + 4*nt*j (j = 0..NV-1), so loads are coalesced and every thread's
// dependent chain is NV groups long.  The float64 sum of squares is taken in a fixed order:
// each thread j-major / component-minor, an xor butterfly inside each warp, then thread 0
// adds the warp totals in warp order.  oracle_norm_quant_rows restates exactly this order.
constexpr int kNormMaxD = 8192;

__host__ __device__ constexpr int norm_groups_per_thread(int D) { return D >= 512 ? 2 : 1; }
__host__ __device__ constexpr int norm_threads(int D) { return D / (4 * norm_groups_per_thread(D)); }

template <typename T, bool QUANT, int NV>
__global__ void __launch_bounds__(1024) norm_rows_kernel(NormParams p) {
  griddep_launch_dependents();
  trace_start(p.trace);
  griddep_wait();
  __shared__ double s_ss[32];
  __shared__ float s_mx[32];
  __shared__ float s_bc[2];
  const int row = blockIdx.x;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const int nt = blockDim.x, nwarps = (nt + 31) >> 5;
  const int D = p.D;

  float4 v[NV];
  if (p.embed != nullptr) {
    // a negative token id (a window's out-of-range token, ane/stories/cpu.go:59-64) gathers a
    // zero row
    const int tok = p.tokens[row];
    const T* e = reinterpret_cast<const T*>(p.embed) + static_cast<size_t>(tok < 0 ? 0 : tok) * D;
    float* xo = p.x_out + static_cast<size_t>(row) * D;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      v[j] = tok < 0 ? make_float4(0.f, 0.f, 0.f, 0.f) : load4_act<T>(e + 4 * t + 4 * nt * j);
      *reinterpret_cast<float4*>(xo + 4 * t + 4 * nt * j) = v[j];
    }
  } else {
    const int src = p.row_index ? p.row_index[row] : row;
    const float* xr = p.x + static_cast<size_t>(src) * D;
#pragma unroll
    for (int j = 0; j < NV; ++j) v[j] = *reinterpret_cast<const float4*>(xr + 4 * t + 4 * nt * j);
  }

  if (p.w != nullptr) {
    double acc = 0.0;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      acc = __dadd_rn(acc, __dmul_rn((double)v[j].x, (double)v[j].x));
      acc = __dadd_rn(acc, __dmul_rn((double)v[j].y, (double)v[j].y));
      acc = __dadd_rn(acc, __dmul_rn((double)v[j].z, (double)v[j].z));
      acc = __dadd_rn(acc, __dmul_rn((double)v[j].w, (double)v[j].w));
    }
    // threads of a partial last warp contribute 0.0 to the butterfly
    acc = warp_sum_f64(acc);
    if (lane == 0) s_ss[warp] = acc;
    __syncthreads();
    if (t == 0) {
      double tot = s_ss[0];
      for (int w = 1; w < nwarps; ++w) tot = __dadd_rn(tot, s_ss[w]);
      const double mean = __dadd_rn(__ddiv_rn(tot, (double)D), p.eps);
      s_bc[0] = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(mean)));
    }
    __syncthreads();
    const float rrms = s_bc[0];
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      const float4 w = *reinterpret_cast<const float4*>(p.w + 4 * t + 4 * nt * j);
      v[j].x = __fmul_rn(__fmul_rn(v[j].x, rrms), w.x);
      v[j].y = __fmul_rn(__fmul_rn(v[j].y, rrms), w.y);
      v[j].z = __fmul_rn(__fmul_rn(v[j].z, rrms), w.z);
      v[j].w = __fmul_rn(__fmul_rn(v[j].w, rrms), w.w);
    }
  }

  if constexpr (!QUANT) {
    T* o = reinterpret_cast<T*>(p.out) + static_cast<size_t>(row) * D;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      uint2 packed;
      packed.x = ActTraits<T>::pack2(v[j].x, v[j].y);
      packed.y = ActTraits<T>::pack2(v[j].z, v[j].w);
      *reinterpret_cast<uint2*>(o + 4 * t + 4 * nt * j) = packed;
    }
  } else {
    float mx = 0.0f;
#pragma unroll
    for (int j = 0; j < NV; ++j)
      mx = fmaxf(fmaxf(fmaxf(mx, fabsf(v[j].x)), fmaxf(fabsf(v[j].y), fabsf(v[j].z))), fabsf(v[j].w));
    mx = warp_max(mx);
    if (lane == 0) s_mx[warp] = mx;
    __syncthreads();
    if (t == 0) {
      float m = s_mx[0];
      for (int w = 1; w < nwarps; ++w) m = fmaxf(m, s_mx[w]);
      float sc = __fdiv_rn(m, 127.0f);
      if (sc == 0.0f) sc = 1.0f;
      s_bc[1] = sc;
      p.scale[row] = sc;
    }
    __syncthreads();
    const float sc = s_bc[1];
    const float inv = __fdiv_rn(1.0f, sc);
    int8_t* qo = p.q + static_cast<size_t>(row) * D;
#pragma unroll
    for (int j = 0; j < NV; ++j) {
      char4 c;
      c.x = quant_bridge_fast(v[j].x, sc, inv);
      c.y = quant_bridge_fast(v[j].y, sc, inv);
      c.z = quant_bridge_fast(v[j].z, sc, inv);
      c.w = quant_bridge_fast(v[j].w, sc, inv);
      *reinterpret_cast<char4*>(qo + 4 * t + 4 * nt * j) = c;
    }
  }
  trace_end(p.trace);
}

// The same row computation with one warp per row and no block-wide barriers (the decode-sized
// launches are latency-bound: the CTA-per-row kernel spends most of its time in dependent
// loads and __syncthreads).  Lane l plays the virtual threads t = l + 32 v (v < W) of the
// CTA-per-row layout above, so every float64 partial, the butterfly of each virtual warp and
// the in-order sum of the virtual warps' totals are the same operations in the same order:
// bit-identical results.  kNormWarpRows rows per CTA.
constexpr int kNormWarpRows = 4;

template <typename T, bool QUANT, int G, int W>
__global__ void __launch_bounds__(kNormWarpRows * 32) norm_rows_warp_kernel(NormParams p) {
  griddep_launch_dependents();
  trace_start(p.trace);
  griddep_wait();
  constexpr int TT = 32 * W;  // virtual threads per row
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * kNormWarpRows + (threadIdx.x >> 5);
  const int D = p.D;
  if (row < p.rows) {
    float4 v[W][G];
    if (p.embed != nullptr) {
      const int tok = p.tokens[row];  // negative: a zero row (ane/stories/cpu.go:59-64)
      const T* e = reinterpret_cast<const T*>(p.embed) + static_cast<size_t>(tok < 0 ? 0 : tok) * D;
      float* xo = p.x_out + static_cast<size_t>(row) * D;
#pragma unroll
      for (int vw = 0; vw < W; ++vw)
#pragma unroll
        for (int j = 0; j < G; ++j) {
          const int i = 4 * (32 * vw + lane) + 4 * TT * j;
          v[vw][j] = tok < 0 ? make_float4(0.f, 0.f, 0.f, 0.f) : load4_act<T>(e + i);
          *reinterpret_cast<float4*>(xo + i) = v[vw][j];
        }
    } else {
      const int src = p.row_index ? p.row_index[row] : row;
      const float* xr = p.x + static_cast<size_t>(src) * D;
#pragma unroll
      for (int vw = 0; vw < W; ++vw)
#pragma unroll
        for (int j = 0; j < G; ++j) v[vw][j] = *reinterpret_cast<const float4*>(xr + 4 * (32 * vw + lane) + 4 * TT * j);
    }
    if (p.w != nullptr) {
      double tot = 0.0;
#pragma unroll
      for (int vw = 0; vw < W; ++vw) {
        double acc = 0.0;
#pragma unroll
        for (int j = 0; j < G; ++j) {
          acc = __dadd_rn(acc, __dmul_rn((double)v[vw][j].x, (double)v[vw][j].x));
          acc = __dadd_rn(acc, __dmul_rn((double)v[vw][j].y, (double)v[vw][j].y));
          acc = __dadd_rn(acc, __dmul_rn((double)v[vw][j].z, (double)v[vw][j].z));
          acc = __dadd_rn(acc, __dmul_rn((double)v[vw][j].w, (double)v[vw][j].w));
        }
        acc = warp_sum_f64(acc);
        tot = vw == 0 ? acc : __dadd_rn(tot, acc);
      }
      const double mean = __dadd_rn(__ddiv_rn(tot, (double)D), p.eps);
      const float rrms = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(mean)));
#pragma unroll
      for (int vw = 0; vw < W; ++vw)
#pragma unroll
        for (int j = 0; j < G; ++j) {
          const float4 w = *reinterpret_cast<const float4*>(p.w + 4 * (32 * vw + lane) + 4 * TT * j);
          v[vw][j].x = __fmul_rn(__fmul_rn(v[vw][j].x, rrms), w.x);
          v[vw][j].y = __fmul_rn(__fmul_rn(v[vw][j].y, rrms), w.y);
          v[vw][j].z = __fmul_rn(__fmul_rn(v[vw][j].z, rrms), w.z);
          v[vw][j].w = __fmul_rn(__fmul_rn(v[vw][j].w, rrms), w.w);
        }
    }
    if constexpr (!QUANT) {
      T* o = reinterpret_cast<T*>(p.out) + static_cast<size_t>(row) * D;
#pragma unroll
      for (int vw = 0; vw < W; ++vw)
#pragma unroll
        for (int j = 0; j < G; ++j) {
          uint2 packed;
          packed.x = ActTraits<T>::pack2(v[vw][j].x, v[vw][j].y);
          packed.y = ActTraits<T>::pack2(v[vw][j].z, v[vw][j].w);
          *reinterpret_cast<uint2*>(o + 4 * (32 * vw + lane) + 4 * TT * j) = packed;
        }
    } else {
      float mx = 0.0f;
#pragma unroll
      for (int vw = 0; vw < W; ++vw)
#pragma unroll
        for (int j = 0; j < G; ++j)
          mx = fmaxf(fmaxf(fmaxf(mx, fabsf(v[vw][j].x)), fmaxf(fabsf(v[vw][j].y), fabsf(v[vw][j].z))),
                     fabsf(v[vw][j].w));
      mx = warp_max(mx);
      float sc = __fdiv_rn(mx, 127.0f);
      if (sc == 0.0f) sc = 1.0f;
      const float inv = __fdiv_rn(1.0f, sc);
      if (lane == 0) p.scale[row] = sc;
      int8_t* qo = p.q + static_cast<size_t>(row) * D;
#pragma unroll
      for (int vw = 0; vw < W; ++vw)
#pragma unroll
        for (int j = 0; j < G; ++j) {
          char4 c;
          c.x = quant_bridge_fast(v[vw][j].x, sc, inv);
          c.y = quant_bridge_fast(v[vw][j].y, sc, inv);
          c.z = quant_bridge_fast(v[vw][j].z, sc, inv);
          c.w = quant_bridge_fast(v[vw][j].w, sc, inv);
          *reinterpret_cast<char4*>(qo + 4 * (32 * vw + lane) + 4 * TT * j) = c;
        }
    }
  }
  trace_end(p.trace);
}

// Weight conversion: fp32 rows -> act type (rounded) or int8 with per-row scales.
// dst_row(r) maps source row r to its destination row (used to interleave W1/W3).
struct ConvertParams {
  const float* src;  // [rows][cols]
  int rows, cols;
  int dst_row_mul, dst_row_add;  // destination row = r * mul + add
  void* dst;                     // act type or int8
  float* dst_scale;              // int8 only, indexed like dst rows
};

template <typename T>
__global__ void __launch_bounds__(256) convert_rows_kernel(ConvertParams p) {
  const int row = blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= p.rows) return;
  const float* s = p.src + static_cast<size_t>(row) * p.cols;
  const size_t drow = static_cast<size_t>(row) * p.dst_row_mul + p.dst_row_add;
  if constexpr (sizeof(T) == 1) {
    float mx = 0.0f;
    for (int i = lane; i < p.cols; i += 32) mx = fmaxf(mx, fabsf(s[i]));
    mx = warp_max(mx);
    float sc = __fdiv_rn(mx, 127.0f);
    if (sc == 0.0f) sc = 1.0f;
    int8_t* d = reinterpret_cast<int8_t*>(p.dst) + drow * p.cols;
    for (int i = lane; i < p.cols; i += 32) d[i] = quant_bridge(s[i], sc);
    if (lane == 0) p.dst_scale[drow] = sc;
  } else {
    T* d = reinterpret_cast<T*>(p.dst) + drow * p.cols;
    for (int i = lane; i < p.cols; i += 32) d[i] = ActTraits<T>::from_f(s[i]);
  }
}

}  // namespace llm
