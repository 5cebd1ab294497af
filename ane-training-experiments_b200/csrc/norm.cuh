// norm.cuh -- row kernels: embedding gather, RMSNorm, per-token int8 quantisation.
//
// One warp per row.  Lane l owns the float4 groups starting at 4*l + 128*j, so every
// access is a coalesced 512-byte warp transaction.  The float64 sum of squares is taken
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

template <typename T, bool QUANT>
__global__ void __launch_bounds__(256) norm_rows_kernel(NormParams p) {
  const int warps = blockDim.x / 32;
  const int row = blockIdx.x * warps + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= p.rows) return;
  const int D = p.D;

  const float* xr;
  if (p.embed != nullptr) {
    const T* e = reinterpret_cast<const T*>(p.embed) + static_cast<size_t>(p.tokens[row]) * D;
    float* xo = p.x_out + static_cast<size_t>(row) * D;
    for (int i = 4 * lane; i < D; i += 128) *reinterpret_cast<float4*>(xo + i) = load4_act<T>(e + i);
    __syncwarp();
    xr = xo;
  } else {
    const int src = p.row_index ? p.row_index[row] : row;
    xr = p.x + static_cast<size_t>(src) * D;
  }

  float rrms = 1.0f;
  if (p.w != nullptr) {
    double acc = 0.0;
    for (int i = 4 * lane; i < D; i += 128) {
      float4 v = *reinterpret_cast<const float4*>(xr + i);
      acc = __dadd_rn(acc, __dmul_rn((double)v.x, (double)v.x));
      acc = __dadd_rn(acc, __dmul_rn((double)v.y, (double)v.y));
      acc = __dadd_rn(acc, __dmul_rn((double)v.z, (double)v.z));
      acc = __dadd_rn(acc, __dmul_rn((double)v.w, (double)v.w));
    }
    double tot = warp_sum_f64(acc);
    double mean = __dadd_rn(__ddiv_rn(tot, (double)D), p.eps);
    rrms = __double2float_rn(__ddiv_rn(1.0, __dsqrt_rn(mean)));
  }

  auto normed = [&](float xv, float wv) -> float {
    return p.w != nullptr ? __fmul_rn(__fmul_rn(xv, rrms), wv) : xv;
  };

  if constexpr (!QUANT) {
    T* o = reinterpret_cast<T*>(p.out) + static_cast<size_t>(row) * D;
    for (int i = 4 * lane; i < D; i += 128) {
      float4 v = *reinterpret_cast<const float4*>(xr + i);
      float4 w = *reinterpret_cast<const float4*>(p.w + i);
      uint2 packed;
      packed.x = ActTraits<T>::pack2(normed(v.x, w.x), normed(v.y, w.y));
      packed.y = ActTraits<T>::pack2(normed(v.z, w.z), normed(v.w, w.w));
      *reinterpret_cast<uint2*>(o + i) = packed;
    }
  } else {
    float mx = 0.0f;
    for (int i = 4 * lane; i < D; i += 128) {
      float4 v = *reinterpret_cast<const float4*>(xr + i);
      float4 w = p.w ? *reinterpret_cast<const float4*>(p.w + i) : make_float4(1.f, 1.f, 1.f, 1.f);
      mx = fmaxf(mx, fabsf(normed(v.x, w.x)));
      mx = fmaxf(mx, fabsf(normed(v.y, w.y)));
      mx = fmaxf(mx, fabsf(normed(v.z, w.z)));
      mx = fmaxf(mx, fabsf(normed(v.w, w.w)));
    }
    mx = warp_max(mx);
    float sc = __fdiv_rn(mx, 127.0f);
    if (sc == 0.0f) sc = 1.0f;
    int8_t* qo = p.q + static_cast<size_t>(row) * D;
    for (int i = 4 * lane; i < D; i += 128) {
      float4 v = *reinterpret_cast<const float4*>(xr + i);
      float4 w = p.w ? *reinterpret_cast<const float4*>(p.w + i) : make_float4(1.f, 1.f, 1.f, 1.f);
      char4 c;
      c.x = quant_bridge(normed(v.x, w.x), sc);
      c.y = quant_bridge(normed(v.y, w.y), sc);
      c.z = quant_bridge(normed(v.z, w.z), sc);
      c.w = quant_bridge(normed(v.w, w.w), sc);
      *reinterpret_cast<char4*>(qo + i) = c;
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
