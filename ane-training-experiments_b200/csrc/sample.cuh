// sample.cuh -- temperature sampling of the next token from materialised logits.
//
// Reference: ane/stories/infer.go:347-371 (sampleFromLogits).  For temperature > 1e-6:
//   mx    = max_i logits[i]                      (f32)
//   invT  = float64(1 / temperature)             (f32 division, widened)
//   total = sum_i exp((f64(logits[i]) - f64(mx)) * invT)
//   target = u * total,  u uniform in [0, 1)
//   return the first i whose running sum of the same terms reaches target (>=), else V - 1.
// The reference draws u from Go's math/rand stream of the decoder's seed; that stream cannot
// be reproduced here, so u comes from a documented counter-based generator instead:
//   key = splitmix64(seed ^ splitmix64(stream * 0xD1B54A32D192ED03 + 0x8CB92BA72F3D8DD7))
//   u   = (splitmix64(key + counter) >> 11) * 2^-53
// with stream = kSampleStreamBase + sequence slot and counter = that slot's number of draws
// so far.  The CPU oracle restates the same generator and sampler.
//
// One CTA per row.  Thread t owns the contiguous index range [t*chunk, (t+1)*chunk) and sums
// its terms in index order; an inclusive scan of the per-thread sums in thread order gives
// every range's starting running sum; the first thread whose range end reaches target rescans
// its range term by term.  The running sums therefore group the terms by range instead of
// strictly left to right: the chosen index can differ from a sequential scan only when target
// lies within the rounding of the float64 sums (~1e-16 relative) of a range boundary.
#pragma once
#include "common.cuh"

namespace llm {

__host__ __device__ inline uint64_t splitmix64_hd(uint64_t x) {
  x += 0x9E3779B97F4A7C15ull;
  x = (x ^ (x >> 30)) * 0xBF58476D1CE4E5B9ull;
  x = (x ^ (x >> 27)) * 0x94D049BB133111EBull;
  return x ^ (x >> 31);
}

constexpr uint64_t kSampleStreamBase = 0x5A4D000000000000ull;

__host__ __device__ inline double sample_uniform(uint64_t seed, uint64_t stream, uint64_t counter) {
  const uint64_t key = splitmix64_hd(seed ^ splitmix64_hd(stream * 0xD1B54A32D192ED03ull + 0x8CB92BA72F3D8DD7ull));
  return static_cast<double>(splitmix64_hd(key + counter) >> 11) * (1.0 / 9007199254740992.0);
}

struct SampleParams {
  const float* logits;             // [rows][ld]
  int rows, V, ld;
  double inv_t;                    // float64(1 / temperature), the division in f32
  const int* row_index;            // optional: logits row i is activation row row_index[i]
  const int* seq_ids;              // activation row -> sequence slot (the generator's stream)
  uint64_t seed;
  unsigned long long* draws;       // [slots] draws so far per slot; advanced by one per sample
  const double* u;                 // optional explicit uniforms per row (then draws is unused)
  int* out;                        // [rows]
};

constexpr int kSampleThreads = 1024;

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(SampleParams p) {
  griddep_launch_dependents();
  griddep_wait();
  __shared__ float s_mx[32];
  __shared__ double s_w[32];
  __shared__ double s_total;
  __shared__ int s_first;
  const int row = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
  constexpr int NW = kSampleThreads / 32;
  const float* lg = p.logits + static_cast<size_t>(row) * p.ld;

  float mx = -INFINITY;
  for (int i = t; i < p.V; i += kSampleThreads) mx = fmaxf(mx, lg[i]);
  mx = warp_max(mx);
  if (lane == 0) s_mx[warp] = mx;
  if (t == 0) s_first = kSampleThreads;
  __syncthreads();
  mx = s_mx[0];
#pragma unroll
  for (int w = 1; w < NW; ++w) mx = fmaxf(mx, s_mx[w]);
  const double dmx = static_cast<double>(mx);

  const int chunk = (p.V + kSampleThreads - 1) / kSampleThreads;
  const int b = min(p.V, t * chunk), e = min(p.V, b + chunk);
  double s = 0.0;
  for (int i = b; i < e; ++i) s += exp((static_cast<double>(lg[i]) - dmx) * p.inv_t);

  // exclusive running sum of the per-thread sums in thread order
  double inc = s;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const double y = __shfl_up_sync(0xffffffffu, inc, off);
    if (lane >= off) inc += y;
  }
  double wexcl = __shfl_up_sync(0xffffffffu, inc, 1);
  if (lane == 0) wexcl = 0.0;
  if (lane == 31) s_w[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    double w = s_w[lane];
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const double y = __shfl_up_sync(0xffffffffu, w, off);
      if (lane >= off) w += y;
    }
    s_w[lane] = w;  // inclusive warp totals
    if (lane == 31) s_total = w;
  }
  __syncthreads();
  const double excl = (warp > 0 ? s_w[warp - 1] : 0.0) + wexcl;
  const double incl = excl + s;

  const int ai = p.row_index ? p.row_index[row] : row;
  const int seq = p.seq_ids ? p.seq_ids[ai] : ai;
  double u;
  if (p.u) u = p.u[row];
  else u = sample_uniform(p.seed, kSampleStreamBase + static_cast<uint64_t>(seq), p.draws[seq]);
  const double target = u * s_total;
  if (e > b && incl >= target) atomicMin(&s_first, t);
  __syncthreads();
  if (t == s_first) {
    double acc = excl;
    int res = e - 1;  // the range end reached target as a whole: rounding left the scan short
    for (int i = b; i < e; ++i) {
      acc += exp((static_cast<double>(lg[i]) - dmx) * p.inv_t);
      if (acc >= target) {
        res = i;
        break;
      }
    }
    p.out[row] = res;
  }
  if (t == 0) {
    if (s_first == kSampleThreads) p.out[row] = p.V - 1;  // infer.go:370
    if (!p.u) p.draws[seq] += 1;
  }
}

}  // namespace llm
