// common.cuh -- device helpers shared by the token-loop kernels (sm_100a).
//
// Inline PTX wrappers for the instructions the kernels are built from: warp-level
// tensor-core MMA (bf16/fp16 -> f32, s8 -> s32), ldmatrix, 16-byte cp.async with zero
// fill, mbarrier waits with an iteration bound, and the bulk (TMA) global->shared copy.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <math.h>
#include <stdint.h>
#include <string.h>

namespace llm {

// Error words a kernel writes into the context's device error flag.
enum DeviceError : int {
  kDevOk = 0,
  kDevWaitTimeout = 1,  // an mbarrier wait exceeded its iteration bound
  kDevBadPage = 2,      // a block-table entry pointed outside the page pool
};

// Bound on mbarrier polls (each try_wait sleeps up to ~64 ns): about a second, far longer
// than any legitimate wait.
constexpr uint32_t kMaxWaitPolls = 1u << 24;

// ----------------------------------------------------------------------------- types
template <typename T> struct ActTraits;
template <> struct ActTraits<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float2 unpack2(uint32_t v) {
    __half2 h = *reinterpret_cast<__half2*>(&v);
    return __half22float2(h);
  }
};
template <> struct ActTraits<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  static __device__ __forceinline__ float2 unpack2(uint32_t v) {
    return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
  }
};

// ----------------------------------------------------------------------------- mma.sync
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                          __half) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void mma_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1,
                                          __nv_bfloat16) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// s8 x s8 -> s32, k = 32 bytes per instruction.
__device__ __forceinline__ void mma_16832_s8(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], uint32_t saddr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t saddr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(saddr));
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ----------------------------------------------------------------------------- cp.async
// 16-byte async copy; src_bytes == 0 zero-fills the destination (out-of-range rows).
__device__ __forceinline__ void cp_async_16(uint32_t dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(src_bytes));
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> __device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

// ----------------------------------------------------------------------------- mbarrier + bulk copy
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}
// Returns true once the phase with parity `parity` has completed.  The suspend-time hint
// (nanoseconds) bounds how long a waiting thread sleeps before re-checking: without it the
// system default applies, and a wait that spans a whole GEMM main loop was observed to round
// kernel durations up to multiples of ~2 us.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(64u)
      : "memory");
  return ok != 0;
}
// 2^x built only from IEEE round-to-nearest operations, so that a CPU restatement with the same
// operations (C99 fmaf) gives the same bits.  x is clamped to [-127, 127.49999]; n = rint(x)
// by the 1.5 * 2^23 addition (t = x + 1.5*2^23 holds n in its low mantissa bits); f = x - n in
// [-0.5, 0.5]; 2^f by a degree-5 polynomial with constant term 1 (coefficients fitted to 2^f on
// [-0.5, 0.5] by weighted least squares iterated toward the minimax relative error, then rounded
// to f32; 1.6e-7 relative) in Horner form with fused multiply-adds; then one multiplication by
// 2^n built from its exponent bits, which are 0 for n = -127, so x < -126.5 (and -inf, NaN)
// gives 0.  Within 2.5e-7 relative of 2^x for x in [-125, 127.4]; results in [2^-126.5, 2^-125)
// are rounded subnormals; x >= 127.5 gives 2^127.49999; exp2_det(0) = 1 exactly.  Runs on the FMA
// and integer pipes only (no MUFU, no conversion instructions), 13 instructions.
constexpr float kExp2Magic = 12582912.0f;  // 1.5 * 2^23
__host__ __device__ __forceinline__ float exp2_poly(float f) {
#ifdef __CUDA_ARCH__
  float p = __fmaf_rn(0x1.5bb9e2p-10f, f, 0x1.3cea80p-7f);
  p = __fmaf_rn(p, f, 0x1.c6b754p-5f);
  p = __fmaf_rn(p, f, 0x1.ebf9bcp-3f);
  p = __fmaf_rn(p, f, 0x1.62e42ap-1f);
  return __fmaf_rn(p, f, 1.0f);
#else
  float p = fmaf(0x1.5bb9e2p-10f, f, 0x1.3cea80p-7f);
  p = fmaf(p, f, 0x1.c6b754p-5f);
  p = fmaf(p, f, 0x1.ebf9bcp-3f);
  p = fmaf(p, f, 0x1.62e42ap-1f);
  return fmaf(p, f, 1.0f);
#endif
}
// x already at most 127.49999 (e.g. a softmax exponent s - max <= 0): the same result as
// exp2_det without the upper clamp.
__device__ __forceinline__ float exp2_det_lo(float x) {
  const float xc = fmaxf(x, -127.0f);
  const float t = __fadd_rn(xc, kExp2Magic);
  const float f = __fsub_rn(xc, __fsub_rn(t, kExp2Magic));
  const float p = exp2_poly(f);
  return __fmul_rn(p, __int_as_float((__float_as_int(t) + (127 - 0x4B400000)) << 23));
}
__host__ __device__ __forceinline__ float exp2_det(float x) {
#ifdef __CUDA_ARCH__
  return exp2_det_lo(fminf(x, 127.49999f));
#else
  const float xc = fminf(fmaxf(x, -127.0f), 127.49999f);
  const float t = xc + kExp2Magic;
  const float f = xc - (t - kExp2Magic);
  const float p = exp2_poly(f);
  int32_t ti;
  memcpy(&ti, &t, 4);
  const uint32_t bits = static_cast<uint32_t>(ti + (127 - 0x4B400000)) << 23;
  float sc;
  memcpy(&sc, &bits, 4);
  return p * sc;
#endif
}

// Packed pairs of f32 operations (sm_100: one instruction for two lanes' worth of f32 work).
__device__ __forceinline__ uint64_t f2_bits(float2 v) {
  return static_cast<uint64_t>(__float_as_uint(v.x)) | (static_cast<uint64_t>(__float_as_uint(v.y)) << 32);
}
__device__ __forceinline__ float2 bits_f2(uint64_t b) {
  return make_float2(__uint_as_float(static_cast<uint32_t>(b)), __uint_as_float(static_cast<uint32_t>(b >> 32)));
}
__device__ __forceinline__ float2 fma2_rn(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;\n" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
  return bits_f2(d);
}
__device__ __forceinline__ float2 add2_rn(float2 a, float2 b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;\n" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}
__device__ __forceinline__ float2 sub2_rn(float2 a, float2 b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;\n" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}
__device__ __forceinline__ float2 mul2_rn(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;\n" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return bits_f2(d);
}
// exp2_det_lo of two values with packed f32 pairs: each lane's result is bit-identical to the
// scalar function (the same round-to-nearest operations per element).
__device__ __forceinline__ float2 exp2_det_lo2(float2 x) {
  const float2 xc = make_float2(fmaxf(x.x, -127.0f), fmaxf(x.y, -127.0f));
  const float2 mg = make_float2(kExp2Magic, kExp2Magic);
  const float2 t = add2_rn(xc, mg);
  const float2 f = sub2_rn(xc, sub2_rn(t, mg));
  float2 p = fma2_rn(make_float2(0x1.5bb9e2p-10f, 0x1.5bb9e2p-10f), f, make_float2(0x1.3cea80p-7f, 0x1.3cea80p-7f));
  p = fma2_rn(p, f, make_float2(0x1.c6b754p-5f, 0x1.c6b754p-5f));
  p = fma2_rn(p, f, make_float2(0x1.ebf9bcp-3f, 0x1.ebf9bcp-3f));
  p = fma2_rn(p, f, make_float2(0x1.62e42ap-1f, 0x1.62e42ap-1f));
  p = fma2_rn(p, f, make_float2(1.0f, 1.0f));
  const float2 sc = make_float2(__int_as_float((__float_as_int(t.x) + (127 - 0x4B400000)) << 23),
                                __int_as_float((__float_as_int(t.y) + (127 - 0x4B400000)) << 23));
  return mul2_rn(p, sc);
}
// Bounded wait: false when the bound ran out (the caller reports kDevWaitTimeout).
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity) {
  for (uint32_t i = 0; i < kMaxWaitPolls; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  return false;
}
// Order this thread's generic-proxy shared-memory accesses before later async-proxy ones
// (a bulk copy refilling a buffer that was just read or written).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}
// Bulk (TMA engine) copy of `bytes` contiguous bytes from global to this CTA's shared
// memory, completing `bytes` of transaction count on mbarrier `bar`.  Both addresses
// 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar)
      : "memory");
}

// ----------------------------------------------------------------------------- programmatic dependent launch
// Kernels of the token loop are launched with programmatic stream serialisation: a kernel
// may start while its predecessor drains.  Every kernel signals its dependents as soon as all
// of its CTAs are resident (deadlock-free: the dependent grid starts only after every CTA of
// this grid has executed the signal) and waits for its predecessor's completion and memory
// before it reads anything the predecessor produced.  Outside such launches both are no-ops.
__device__ __forceinline__ void griddep_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }

// Launch timeline record (llm_trace_step): globaltimer nanoseconds of the first and the last
// CTA start and of the last CTA end, and the number of CTAs that finished.  Thread 0 of each
// CTA records; a null pointer records nothing.
struct TraceRec {
  unsigned long long first_start, last_start, last_end, ctas;
};
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}
__device__ __forceinline__ void trace_start(TraceRec* r) {
  if (r != nullptr && threadIdx.x == 0) {
    const unsigned long long t = global_ns();
    atomicMin(&r->first_start, t);
    atomicMax(&r->last_start, t);
  }
}
__device__ __forceinline__ void trace_end(TraceRec* r) {
  if (r != nullptr && threadIdx.x == 0) {
    atomicMax(&r->last_end, global_ns());
    atomicAdd(&r->ctas, 1ull);
  }
}

// ----------------------------------------------------------------------------- misc
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
// float64 xor-butterfly sum: every lane ends with the bitwise-identical total because
// each level adds the same two operands (IEEE addition is commutative).
__device__ __forceinline__ double warp_sum_f64(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = __dadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Order-preserving map of a float to uint32 (larger float -> larger key).
__device__ __forceinline__ uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
// (value desc, index asc) packed so that the unsigned max picks the first maximum.
__device__ __forceinline__ unsigned long long argmax_key(float v, int idx) {
  return (static_cast<unsigned long long>(float_key(v)) << 32) | (0xffffffffu - static_cast<uint32_t>(idx));
}
__device__ __forceinline__ int argmax_key_index(unsigned long long k) {
  return static_cast<int>(0xffffffffu - static_cast<uint32_t>(k & 0xffffffffu));
}

// The bridge quantiser (bridge/ane_bridge.m:389-392) on one value given its row scale:
// IEEE division, clamp to [-128,127], add +-0.5 in f32, truncate toward zero.
__device__ __forceinline__ int8_t quant_bridge(float x, float scale) {
  float v = __fdiv_rn(x, scale);
  v = fminf(v, 127.0f);
  v = fmaxf(v, -128.0f);
  float r = __fadd_rn(v, v >= 0.0f ? 0.5f : -0.5f);
  return static_cast<int8_t>(__float2int_rz(r));
}

// The same result as quant_bridge(x, scale) without a division in the common case:
// y = x * inv (inv = 1/scale rounded) is within 2 ulps of fl(x / scale), and the bridge rule
// only depends on where the quotient falls relative to the k + 0.5 rounding points and the
// clamp, so when y is more than 4 ulps from every such point it decides the same integer;
// otherwise the exact IEEE quotient is computed.
__device__ __forceinline__ int8_t quant_bridge_fast(float x, float scale, float inv) {
  const float y = __fmul_rn(x, inv);
  const float a = fabsf(y);
  const float frac = a - floorf(a);
  const bool near = fabsf(frac - 0.5f) <= __fmul_rn(a, 4.76837158203125e-7f) + 1e-30f || a >= 126.0f;
  const float v0 = near ? __fdiv_rn(x, scale) : y;
  float v = fminf(v0, 127.0f);
  v = fmaxf(v, -128.0f);
  const float r = __fadd_rn(v, v >= 0.0f ? 0.5f : -0.5f);
  return static_cast<int8_t>(__float2int_rz(r));
}

// Byte offset of 16-byte chunk `chunk` of row `row` in a tile whose rows are `row_bytes`
// long, XOR-swizzled within each 128-byte group so that 8 consecutive rows reading the
// same logical chunk hit 8 different bank groups.
// Byte offset of 16-byte chunk `chunk` (8 elements) of row `row` (0..15) inside the K or the V
// block of a KV-cache page (16 rows x head_dim 2-byte elements).  Each 64-element half of a row
// is a 128-byte row of its own 16 x 128 B sub-block (sub-blocks 2 KB apart), with chunk c of
// row r at position c ^ (r & 7): the 128-byte-swizzle layout of a K-major tcgen05 operand, and
// bank-conflict free for ldmatrix.  For head_dim 64 this is one sub-block.
__host__ __device__ __forceinline__ uint32_t kv_off(int row, int chunk) {
  return static_cast<uint32_t>((chunk >> 3) * 2048 + row * 128 + (((chunk & 7) ^ (row & 7)) << 4));
}
__device__ __forceinline__ uint32_t swz(int row, int chunk, int row_bytes) {
  return static_cast<uint32_t>(row * row_bytes + ((chunk ^ (row & 7)) << 4));
}

}  // namespace llm
