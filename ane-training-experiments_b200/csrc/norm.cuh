// norm.cuh -- row kernels: embedding gather, RMSNorm, per-token int8 quantisation.
//
// One warp per row (4 rows per 128-thread block).  Lane l owns the float4 groups starting
// at 4*l + 128*j, so every access is a coalesced 512-byte warp transaction.  The float64 sum of squares is taken
// in that fixed order (lane partials j-major / component-minor, then an xor butterfly),
// with explicit round-to-nearest intrinsics so no fused multiply-add can change it; the
// CPU oracle restates exactly this order for its bit-exact quantiser check.
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
};

// Convert 4 activation-type values to float.
template <typename T>
__device__ __forceinline__ float4 load4_act(const T* p) {
  uint2 raw = *reinterpret_cast<const uint2*>(p);
  const T* h = reinterpret_cast<const T*>(&raw);
  return make_float4(ActTraits<T>::to_f(h[0]), ActTraits<T>::to_f(h[1]), ActTraits<T>::to_f(h[2]),
                     ActTraits<T>::to_f(h[3]));
}

// Rows are held in registers: lane l keeps float4 groups j = 0..NV-1 (element 4*l + 128*j),
// so a row of 128*NV elements is read from global memory exactly once.  NV is a template
// parameter so the code is exactly as long as the row needs (a generic NV = 0 variant loops
// over any multiple of 4 up to 128*kNormMaxV).
constexpr int kNormMaxV = 32;  // rows up to 4096 elements

template <typename T, bool QUANT, int NV>
__global__ void __launch_bounds__(128) norm_rows_kernel(NormParams p) {
  constexpr int CAP = NV > 0 ? NV : kNormMaxV;
  const int warps = blockDim.x / 32;
  const int row = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= p.rows) return;
  const int D = p.D;
  const int nv = NV > 0 ? NV : (D + 127) / 128;
  auto live = [&](int j) { return NV > 0 ? true : (j < nv && 4 * lane + 128 * j < D); };

  float4 v[CAP];
  if (p.embed != nullptr) {
    const T* e = reinterpret_cast<const T*>(p.embed) + static_cast<size_t>(p.tokens[row]) * D;
    float* xo = p.x_out + static_cast<size_t>(row) * D;
#pragma unroll
    for (int j = 0; j < CAP; ++j)
      if (live(j)) {
        v[j] = load4_act<T>(e + 4 * lane + 128 * j);
        *reinterpret_cast<float4*>(xo + 4 * lane + 128 * j) = v[j];
      }
  } else {
    const int src = p.row_index ? p.row_index[row] : row;
    const float* xr = p.x + static_cast<size_t>(src) * D;
#pragma unroll
    for (int j = 0; j < CAP; ++j)
      if (live(j)) v[j] = *reinterpret_cast<const float4*>(xr + 4 * lane + 128 * j);
  }

  if (p.w != nullptr) {
    double acc = 0.0;
#pragma unroll
    for (int j = 0; j < CAP; ++j)
      if (live(j)) {
        acc = __dadd_rn(acc, __dmul_rn((double)v[j].x, (double)v[j].x));
        acc = __dadd_rn(acc, __dmul_rn((double)v[j].y, (double)v[j].y));
        acc = __dadd_rn(acc, __dmul_rn((double)v[j].z, (double)v[j].z));
        acc = __dadd_rn(acc, __dmul_rn((double)v[j].w, (double)v[j].w));
      }
    const double tot = warp_sum_f64(acc);
    const double mean = __dadd_rn(__ddiv_rn(tot, (double)D), p.eps);
    const float rrms = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(mean)));
#pragma unroll
    for (int j = 0; j < CAP; ++j)
      if (live(j)) {
        const float4 w = *reinterpret_cast<const float4*>(p.w + 4 * lane + 128 * j);
        v[j].x = __fmul_rn(__fmul_rn(v[j].x, rrms), w.x);
        v[j].y = __fmul_rn(__fmul_rn(v[j].y, rrms), w.y);
        v[j].z = __fmul_rn(__fmul_rn(v[j].z, rrms), w.z);
        v[j].w = __fmul_rn(__fmul_rn(v[j].w, rrms), w.w);
      }
  }

  if constexpr (!QUANT) {
    T* o = reinterpret_cast<T*>(p.out) + static_cast<size_t>(row) * D;
#pragma unroll
    for (int j = 0; j < CAP; ++j)
      if (live(j)) {
        uint2 packed;
        packed.x = ActTraits<T>::pack2(v[j].x, v[j].y);
        packed.y = ActTraits<T>::pack2(v[j].z, v[j].w);
        *reinterpret_cast<uint2*>(o + 4 * lane + 128 * j) = packed;
      }
  } else {
    float mx = 0.0f;
#pragma unroll
    for (int j = 0; j < CAP; ++j)
      if (live(j)) mx = fmaxf(fmaxf(fmaxf(mx, fabsf(v[j].x)), fmaxf(fabsf(v[j].y), fabsf(v[j].z))), fabsf(v[j].w));
    mx = warp_max(mx);
    float sc = __fdiv_rn(mx, 127.0f);
    if (sc == 0.0f) sc = 1.0f;
    const float inv = __fdiv_rn(1.0f, sc);
    int8_t* qo = p.q + static_cast<size_t>(row) * D;
#pragma unroll
    for (int j = 0; j < CAP; ++j)
      if (live(j)) {
        char4 c;
        c.x = quant_bridge_fast(v[j].x, sc, inv);
        c.y = quant_bridge_fast(v[j].y, sc, inv);
        c.z = quant_bridge_fast(v[j].z, sc, inv);
        c.w = quant_bridge_fast(v[j].w, sc, inv);
        *reinterpret_cast<char4*>(qo + 4 * lane + 128 * j) = c;
      }
    if (lane == 0) p.scale[row] = sc;
  }
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
