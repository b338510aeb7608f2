// Shared device helpers for the maple-b200 decode kernels (sm_100a).
//
// Every kernel here follows one "canonical numerics" contract so that a CPU
// restatement can reproduce its output bit for bit:
//   * bf16 <-> fp32 conversions are explicit; fp32 -> bf16 is round-to-nearest-
//     even with NaN mapped to 0x7FC0.
//   * The library is compiled with --fmad=false: a multiply followed by an add
//     is two roundings unless the source says fmaf().
//   * Sums over a vector use the "R128 order": partial p_j (j = 0..127)
//     accumulates elements j, j+128, j+256, ... sequentially from 0.0f (a
//     product term x*y is added as fmaf(x, y, p_j)); then for lane l < 32,
//     q_l = ((p_l + p_{l+32}) + p_{l+64}) + p_{l+96}; then the 32 q_l are
//     combined by an xor butterfly (16, 8, 4, 2, 1).
//   * exp() is mexp() below (Cody-Waite reduction + degree-7 Taylor series),
//     division and sqrt are IEEE round-to-nearest.
//   * Packed-code contractions (ternary / RTN-4 rows against an activation
//     vector) are exact integer sums over a fixed-point encoding of the
//     activation (FXA, see fxa_* below), so their result does not depend on the
//     order, tiling or split of the reduction.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mb {

enum Status : int {
  kOk = 0,
  kErrShape = 1,      // bad shape / size argument (Python: ValueError)
  kErrDtype = 2,      // unsupported dtype (Python: TypeError)
  kErrBounds = 3,     // an index or length outside its buffer (Python: ValueError)
  kErrTimeout = 4,    // a bounded device wait gave up (Python: RuntimeError)
  kErrCuda = 5,       // CUDA launch / runtime error (Python: RuntimeError)
  kErrWorkspace = 6,  // caller workspace too small (Python: ValueError)
  kErrAlign = 7,      // pointer or stride misaligned for vector loads (Python: ValueError)
  kErrScratchLimit = 8,  // request exceeds a fixed internal scratch (Python: ValueError)
};

enum DType : int { kF32 = 0, kBF16 = 1 };

// ---------------------------------------------------------------- bf16 ----
__device__ __forceinline__ float bf16_to_f32(uint16_t h) {
  return __uint_as_float(static_cast<uint32_t>(h) << 16);
}

__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;  // NaN
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

template <int DT>
__device__ __forceinline__ float load_f(const void* p, int64_t i) {
  if constexpr (DT == kBF16) {
    return bf16_to_f32(static_cast<const uint16_t*>(p)[i]);
  } else {
    return static_cast<const float*>(p)[i];
  }
}

template <int DT>
__device__ __forceinline__ void store_f(void* p, int64_t i, float v) {
  if constexpr (DT == kBF16) {
    static_cast<uint16_t*>(p)[i] = f32_to_bf16(v);
  } else {
    static_cast<float*>(p)[i] = v;
  }
}

// ---------------------------------------------------------------- exp -----
// exp(x) by Cody-Waite range reduction (x = n*ln2 + r, |r| <= ln2/2) and the
// Taylor series of e^r to degree 7 in Horner form, then an exact scaling by
// 2^n split in two factors so that subnormal results round once.  The CPU
// oracle runs the same sequence of IEEE operations.
__device__ __forceinline__ float mexp(float x) {
  if (x != x) return x;
  if (x < -104.0f) return 0.0f;
  if (x > 88.7228393554688f) return __int_as_float(0x7f800000);
  const float n = rintf(__fmul_rn(x, 1.44269504088896341f));
  float r = __fmaf_rn(-n, 0.693145751953125f, x);
  r = __fmaf_rn(-n, 1.42860676533018704e-06f, r);
  float p = 1.98412698412698413e-04f;               // 1/7!
  p = __fmaf_rn(p, r, 1.38888888888888889e-03f);    // 1/6!
  p = __fmaf_rn(p, r, 8.33333333333333333e-03f);    // 1/5!
  p = __fmaf_rn(p, r, 4.16666666666666667e-02f);    // 1/4!
  p = __fmaf_rn(p, r, 1.66666666666666667e-01f);    // 1/3!
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  const int ni = static_cast<int>(n);
  const int n1 = ni / 2;
  const int n2 = ni - n1;
  p = __fmul_rn(p, __int_as_float((n1 + 127) << 23));
  return __fmul_rn(p, __int_as_float((n2 + 127) << 23));
}

__device__ __forceinline__ float msigmoid(float x) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, mexp(-x)));
}

// rstd = 1 / sqrt(sumsq / n + eps), every step IEEE round-to-nearest.
__device__ __forceinline__ float rstd_of(float sumsq, int n, float eps) {
  const float var = __fdiv_rn(sumsq, static_cast<float>(n));
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
}

// ---------------------------------------------------------------- warp ----
__device__ __forceinline__ float warp_butterfly_sum(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}

// R128 combine of four lane partials (p_l, p_{l+32}, p_{l+64}, p_{l+96}).
__device__ __forceinline__ float r128_lane_finish(float p0, float p1, float p2, float p3) {
  return warp_butterfly_sum(__fadd_rn(__fadd_rn(__fadd_rn(p0, p1), p2), p3));
}

// R128 combine of 128 partials held in shared memory; called by one full warp.
__device__ __forceinline__ float r128_smem_finish(const float* p, int lane) {
  return r128_lane_finish(p[lane], p[lane + 32], p[lane + 64], p[lane + 96]);
}

// ---------------------------------------------------------------- FXA -----
// Fixed-point activation encoding.  For a vector v (fp32) with amax =
// max|v_k| and e = unbiased exponent field of amax, the shift is s = 25 - e and
// X_k = rint(v_k * 2^s) (exact in double), so |X_k| < 2^26.  X_k is split into
// four balanced base-128 digits d_j in [-64, 63]: X = sum_j d_j * 128^j.
// A packed contraction sum_k c_k * v_k is evaluated as the exact integer
// S = sum_k c_k X_k and returned as fp32(double(S) * 2^-s): one rounding.
__device__ __forceinline__ double pow2d(int s) {
  return __longlong_as_double(static_cast<long long>(s + 1023) << 52);
}

// Returns the FXA shift for an amax given as fp32 bits (sign cleared).
// Non-finite amax -> kFxaNonFinite (callers emit NaN rows).
constexpr int kFxaNonFinite = 1 << 20;
__device__ __forceinline__ int fxa_shift(uint32_t amax_bits) {
  if (amax_bits == 0) return 0;
  const int ef = static_cast<int>(amax_bits >> 23);
  if (ef == 0xff) return kFxaNonFinite;
  return 25 - (ef - 127);
}

__device__ __forceinline__ int fxa_encode(float v, int s) {
  return static_cast<int>(rint(static_cast<double>(v) * pow2d(s)));
}

__device__ __forceinline__ int fxa_digit(int X, int j) {
  int d = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    d = ((X + 64) & 127) - 64;
    if (i == j) break;
    X = (X - d) >> 7;
  }
  return d;
}

// fp32 value of an exact contraction S at FXA shift s.
__device__ __forceinline__ float fxa_value(long long S, int s) {
  return __double2float_rn(static_cast<double>(S) * pow2d(-s));
}

// ---------------------------------------------------------------- mma -----
// D(16x8 s32) += A(16x32 u8, row) * B(32x8 s8, col).
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Streaming 16-byte load of packed weights: bypass L1, weights are read once.
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Plain 16-byte load (activations written by the previous kernel).
__device__ __forceinline__ uint4 ld_u4(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}

// Widen the 16 bytes of a vector load to fp32 values (8 bf16 or 4 fp32).
template <int XT>
__device__ __forceinline__ void widen_u4(const uint4& r, float* out) {
  if constexpr (XT == kBF16) {
    const uint32_t w[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      out[2 * i] = __uint_as_float(w[i] << 16);
      out[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  } else {
    out[0] = __uint_as_float(r.x); out[1] = __uint_as_float(r.y);
    out[2] = __uint_as_float(r.z); out[3] = __uint_as_float(r.w);
  }
}

// Copy src[0:n) (dtype XT) into dst[0:n) as fp32 with 16-byte loads that
// are all issued before any is used (one memory round trip for rows of up to
// NT * MAXC vectors).  Threads 0..NT-1 of the block take part (the caller
// synchronises).  Falls back to element loads when src is not 16-byte
// aligned or n is not a whole number of vectors.
// stage_row in two halves: each thread's first 16-byte chunk is loaded into a
// register early (stage_row_issue), so that the load goes out ahead of later
// traffic, and written out with the remaining chunks by stage_row_finish.
template <int XT, int NT>
__device__ __forceinline__ uint4 stage_row_issue(const void* src, int n, int tid) {
  constexpr int EPC = XT == kBF16 ? 8 : 4;
  uint4 r = make_uint4(0u, 0u, 0u, 0u);
  if ((reinterpret_cast<uintptr_t>(src) & 15) == 0 && n % EPC == 0 && tid < n / EPC)
    r = ld_u4(static_cast<const char*>(src) + (size_t)tid * 16);
  return r;
}

template <int XT, int NT>
__device__ __forceinline__ void stage_row_finish(const void* src, int n, float* dst, int tid, const uint4& r) {
  constexpr int EPC = XT == kBF16 ? 8 : 4;
  if ((reinterpret_cast<uintptr_t>(src) & 15) == 0 && n % EPC == 0) {
    const int nch = n / EPC;
    const char* s8 = static_cast<const char*>(src);
    if (tid < nch) widen_u4<XT>(r, dst + (size_t)tid * EPC);
    for (int c = tid + NT; c < nch; c += NT) widen_u4<XT>(ld_u4(s8 + (size_t)c * 16), dst + (size_t)c * EPC);
  } else {
    for (int k = tid; k < n; k += NT) dst[k] = load_f<XT>(src, k);
  }
}

template <int XT, int NT, int MAXC>
__device__ __forceinline__ void stage_row(const void* src, int n, float* dst, int tid) {
  constexpr int EPC = XT == kBF16 ? 8 : 4;
  if ((reinterpret_cast<uintptr_t>(src) & 15) == 0 && n % EPC == 0) {
    const int nch = n / EPC;
    const char* s8 = static_cast<const char*>(src);
    uint4 r[MAXC];
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = tid + i * NT;
      if (c < nch) r[i] = ld_u4(s8 + (size_t)c * 16);
    }
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = tid + i * NT;
      if (c < nch) widen_u4<XT>(r[i], dst + (size_t)c * EPC);
    }
    for (int c = tid + MAXC * NT; c < nch; c += NT) widen_u4<XT>(ld_u4(s8 + (size_t)c * 16), dst + (size_t)c * EPC);
  } else {
    for (int k = tid; k < n; k += NT) dst[k] = load_f<XT>(src, k);
  }
}

}  // namespace mb
