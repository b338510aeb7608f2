// FXA prologues: turn an activation vector into the int8 digit fragments that
// the u8 x s8 tensor-core contraction of packed codes consumes.
//
// Fragment layout (per K iteration of 256 codes): entry (it, m, lane) is a
// uint2 holding the 8 digits that lane (g = lane/4, t = lane%4) feeds to
// mma.m16n8k32 number m (0..7) as its B fragment; column g of B is digit g of
// the activation (g < 4; columns 4..7 are zero).  A lane holding row words
// [4t, 4t+4) of an iteration masks word q with (w >> 2j) & 0x03030303, so byte
// b of A register j carries the code for k = 16*(4t+q) + 4b + j; the entry's
// bytes are laid out to match (frag_byte below).
#pragma once

#include "common.cuh"

namespace mb {

constexpr int kIterK = 256;  // 2-bit codes per row per warp iteration (16 words)

// Codes per row per warp iteration and fragment entries per iteration for a
// packed width of BITS (2: ternary, 4: RTN-4).  A warp iteration always
// covers 16 words per row (4 lanes x 16 bytes).
template <int BITS> struct Pack;
template <> struct Pack<2> { static constexpr int kIter = 256; static constexpr int kMmas = 8; };
template <> struct Pack<4> { static constexpr int kIter = 128; static constexpr int kMmas = 4; };

// Byte offset inside the fragment array of digit j of local code index kk.
// 2-bit: byte b of A register j (j = 0..3) of word q holds code 4b + j;
// MMA m = 2q + j/2 takes registers j = 2(m&1), 2(m&1)+1.
// 4-bit: byte b of A register j (j = 0..1) of word q holds code 2b + j;
// MMA m = q takes registers j = 0, 1.
template <int BITS>
__device__ __forceinline__ int frag_byte(int kk, int j) {
  if constexpr (BITS == 2) {
    const int it = kk >> 8, r = kk & 255, w = r >> 4, i = r & 15;
    const int t = w >> 2, q = w & 3, b = i >> 2, jj = i & 3;
    const int m = 2 * q + (jj >> 1);
    const int entry = (it * 8 + m) * 32 + 4 * j + t;
    return entry * 8 + (jj & 1) * 4 + b;
  } else {
    const int it = kk >> 7, r = kk & 127, w = r >> 3, i = r & 7;
    const int t = w >> 2, m = w & 3, b = i >> 1;
    const int entry = (it * 4 + m) * 32 + 4 * j + t;
    return entry * 8 + (i & 1) * 4 + b;
  }
}

struct FxaShared {
  unsigned amax[4];
  float part[128];
  int dsum[4][4];
  int s;
  float rstd;
  int tot[4];  // digit sums over the fragment's K slice
};

// Block prologue (blockDim.x == 128).  Reads x[0:K) once (times rms_w when
// RMS), computes the FXA shift over all K, the R128 rstd of the raw x (RMS),
// and the digit fragments for local codes [0, iters*Pack::kIter) starting at
// k_lo.  xsm must hold K floats and wsm (RMS only) K floats.  Ends with
// __syncthreads().
template <int XT, int RT, bool RMS, int BITS = 2>
__device__ __forceinline__ void fxa_block_prologue(const void* xr, const void* rms_w, int K, float eps,
                                                   int k_lo, int iters, float* xsm, uint2* frag,
                                                   FxaShared& sh, float* wsm = nullptr) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  stage_row<XT, 128, 4>(xr, K, xsm, tid);
  if constexpr (RMS) stage_row<RT, 128, 4>(rms_w, K, wsm, tid);
  for (int e = tid; e < iters * Pack<BITS>::kMmas * 32; e += 128) frag[e] = make_uint2(0u, 0u);
  __syncthreads();
  float ss = 0.0f;
  unsigned amax = 0;
  for (int k = tid; k < K; k += 128) {
    float v = xsm[k];
    if constexpr (RMS) {
      ss = __fmaf_rn(v, v, ss);
      v = __fmul_rn(v, wsm[k]);
      xsm[k] = v;
    }
    amax = max(amax, __float_as_uint(v) & 0x7fffffffu);
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, m));
  if (lane == 0) sh.amax[warp] = amax;
  if constexpr (RMS) sh.part[tid] = ss;
  __syncthreads();
  if (warp == 0) {
    const unsigned a = max(max(sh.amax[0], sh.amax[1]), max(sh.amax[2], sh.amax[3]));
    float rs = 1.0f;
    if constexpr (RMS) rs = rstd_of(r128_smem_finish(sh.part, lane), K, eps);
    if (lane == 0) {
      sh.s = fxa_shift(a);
      sh.rstd = rs;
    }
  }
  __syncthreads();
  const int s = sh.s;
  const bool bad = (s == kFxaNonFinite);
  unsigned char* fb = reinterpret_cast<unsigned char*>(frag);
  int dsum[4] = {0, 0, 0, 0};
  for (int kk = tid; kk < iters * Pack<BITS>::kIter; kk += 128) {
    const int k = k_lo + kk;
    int X = (k < K && !bad) ? fxa_encode(xsm[k], s) : 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int d = ((X + 64) & 127) - 64;
      dsum[j] += d;
      fb[frag_byte<BITS>(kk, j)] = static_cast<unsigned char>(d & 0xff);
      X = (X - d) >> 7;
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) dsum[j] += __shfl_xor_sync(0xffffffffu, dsum[j], m);
    if (lane == 0) sh.dsum[warp][j] = dsum[j];
  }
  __syncthreads();
  if (tid < 4) sh.tot[tid] = sh.dsum[0][tid] + sh.dsum[1][tid] + sh.dsum[2][tid] + sh.dsum[3][tid];
  __syncthreads();
}

// Warp prologue: the same for one warp and one activation row (no RMSNorm),
// K codes starting at 0.  xsm holds K floats, frag iters*256 entries; both are
// private to the warp.  Returns the FXA shift; tot[] gets the digit sums.
template <int XT>
__device__ __forceinline__ int fxa_warp_prologue(const void* xr, int K, int iters, float* xsm,
                                                 uint2* frag, int (&tot)[4]) {
  const int lane = threadIdx.x & 31;
  stage_row<XT, 32, 4>(xr, K, xsm, lane);
  for (int e = lane; e < iters * 256; e += 32) frag[e] = make_uint2(0u, 0u);
  __syncwarp();
  unsigned amax = 0;
  for (int k = lane; k < K; k += 32) amax = max(amax, __float_as_uint(xsm[k]) & 0x7fffffffu);
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, m));
  const int s = fxa_shift(amax);
  const bool bad = (s == kFxaNonFinite);
  __syncwarp();
  unsigned char* fb = reinterpret_cast<unsigned char*>(frag);
  int dsum[4] = {0, 0, 0, 0};
  for (int kk = lane; kk < iters * kIterK; kk += 32) {
    int X = (kk < K && !bad) ? fxa_encode(xsm[kk], s) : 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int d = ((X + 64) & 127) - 64;
      dsum[j] += d;
      fb[frag_byte<2>(kk, j)] = static_cast<unsigned char>(d & 0xff);
      X = (X - d) >> 7;
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) dsum[j] += __shfl_xor_sync(0xffffffffu, dsum[j], m);
    tot[j] = dsum[j];
  }
  __syncwarp();
  return s;
}

// ------------------------------------------------------------------ fast --
// Offset that turns the balanced base-128 digits of X (|X| < 2^26) into the
// plain digits of u = X + kFxaOffset: d_j = ((u >> 7j) & 127) - 64.
constexpr int kFxaOffset = 135274560;  // 64 * (1 + 128 + 128^2 + 128^3)

__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }

// X = rint(v * 2^s) in fp32: the scaling by a power of two is exact and
// |v * 2^s| < 2^26, so this equals the double-precision definition.
__device__ __forceinline__ int fxa_enc(float v, int s) {
  const float f = (s <= 127) ? __fmul_rn(v, pow2f(s)) : __fmul_rn(__fmul_rn(v, pow2f(s - 76)), pow2f(76));
  return __float2int_rn(f);
}

// Four 7-bit plain digits (digit j of u0..u3) packed in bytes, and the same
// as signed balanced digits (raw - 64 per byte, two's complement).
__device__ __forceinline__ uint32_t raw_digits(uint32_t u0, uint32_t u1, uint32_t u2, uint32_t u3, int j) {
  const int sh = 7 * j;
  return ((u0 >> sh) & 127u) | (((u1 >> sh) & 127u) << 8) | (((u2 >> sh) & 127u) << 16) |
         (((u3 >> sh) & 127u) << 24);
}
__device__ __forceinline__ uint32_t signed_digits(uint32_t raw) {
  return ((raw | 0x80808080u) - 0x40404040u) ^ 0x80808080u;
}

// Shift, rstd and digit totals shared by a block (up to 16 warps).
struct FxaBlock {
  unsigned amax[16];
  int rawsum[16][4];
  int s;
  float rstd;
  int tot[4];  // sum over the fragment's codes of digit j (balanced)
};

// Fragment builder for codes [0, iters*Pack::kIter) of the activation xs
// (fp32 values in shared memory, zero beyond n): each thread owns whole
// fragment entries ("combos": 8 codes x 4 digits), writes them with 64-bit
// stores (digits 4..7 as zeros) and accumulates the raw digit sums.  For
// RTN-4 (BITS=4) it also adds each combo's sum of X into xg[group]
// (64-bit shared atomics) when xg != nullptr.
template <int BITS>
__device__ __forceinline__ void fxa_build(const float* xs, int n, int s, bool bad, int iters, uint2* frag,
                                          int tid, int nt, int (&raws)[4], long long* xg = nullptr,
                                          int group = 0) {
  constexpr int kCombosPerIter = Pack<BITS>::kMmas * 4;
  for (int c = tid; c < iters * kCombosPerIter; c += nt) {
    const int it = c / kCombosPerIter, r = c - it * kCombosPerIter;
    int m, t, k0;
    int off[8];
    if constexpr (BITS == 2) {
      m = r >> 2; t = r & 3;
      k0 = it * 256 + 16 * (4 * t + (m >> 1)) + 2 * (m & 1);
      off[0] = 0; off[1] = 4; off[2] = 8; off[3] = 12; off[4] = 1; off[5] = 5; off[6] = 9; off[7] = 13;
    } else {
      m = r >> 2; t = r & 3;
      k0 = it * 128 + 8 * (4 * t + m);
      off[0] = 0; off[1] = 2; off[2] = 4; off[3] = 6; off[4] = 1; off[5] = 3; off[6] = 5; off[7] = 7;
    }
    uint32_t u[8];
    long long xsum = 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int k = k0 + off[e];
      const int X = (k < n && !bad) ? fxa_enc(xs[k], s) : 0;
      xsum += X;
      u[e] = static_cast<uint32_t>(X + kFxaOffset);
    }
    uint2* dst = frag + (it * Pack<BITS>::kMmas + m) * 32 + t;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t w0 = raw_digits(u[0], u[1], u[2], u[3], j);
      const uint32_t w1 = raw_digits(u[4], u[5], u[6], u[7], j);
      raws[j] = static_cast<int>(__dp4a(w0, 0x01010101u, static_cast<unsigned>(raws[j])));
      raws[j] = static_cast<int>(__dp4a(w1, 0x01010101u, static_cast<unsigned>(raws[j])));
      dst[4 * j] = make_uint2(signed_digits(w0), signed_digits(w1));
      dst[4 * j + 16] = make_uint2(0u, 0u);
    }
    if constexpr (BITS == 4) {
      if (xg != nullptr) atomicAdd(reinterpret_cast<unsigned long long*>(&xg[k0 / group]),
                                   static_cast<unsigned long long>(xsum));
    }
  }
}

// Block prologue for NT threads: stage x (and the RMS weights), FXA shift over
// all K, R128 rstd of the raw x (RMS), fragments of codes [k_lo, k_lo +
// iters*Pack::kIter).  xsm and wsm hold K floats each.  Ends synchronised.
template <int XT, int RT, bool RMS, int BITS, int NT>
__device__ __forceinline__ void fxa_prologue(const void* xr, const void* rms_w, int K, float eps, int k_lo,
                                             int iters, float* xsm, float* wsm, uint2* frag, FxaBlock& fb,
                                             long long* xg = nullptr, int group = 0, bool w_staged = false,
                                             bool x_staged = false) {
  constexpr int NW = NT / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  // x_staged: the caller already wrote x into xsm
  if (!x_staged) stage_row<XT, NT, (8192 * 2 / 16 + NT - 1) / NT>(xr, K, xsm, tid);
  // w_staged: the caller already copied the norm weight into wsm (before its
  // dependency wait, since the weight is static)
  if constexpr (RMS) {
    if (!w_staged) stage_row<RT, NT, (8192 * 4 / 16 + NT - 1) / NT>(rms_w, K, wsm, tid);
  }
  if (xg != nullptr)
    for (int g = tid; g < K / group; g += NT) xg[g] = 0;
  __syncthreads();
  unsigned amax = 0;
  for (int k = tid; k < K; k += NT) {
    float v = xsm[k];
    if constexpr (RMS) {
      v = __fmul_rn(v, wsm[k]);
      wsm[k] = v;
    }
    amax = max(amax, __float_as_uint(v) & 0x7fffffffu);
  }
  float ss = 0.0f;
  if constexpr (RMS) {
    if (tid < 128)
      for (int k = tid; k < K; k += 128) ss = __fmaf_rn(xsm[k], xsm[k], ss);
  }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, m));
  __shared__ float part[128];
  if (lane == 0) fb.amax[warp] = amax;
  if constexpr (RMS) {
    if (tid < 128) part[tid] = ss;
  }
  __syncthreads();
  if (warp == 0) {
    unsigned a = 0;
    for (int w = 0; w < NW; ++w) a = max(a, fb.amax[w]);
    float rs = 1.0f;
    if constexpr (RMS) rs = rstd_of(r128_smem_finish(part, lane), K, eps);
    if (lane == 0) {
      fb.s = fxa_shift(a);
      fb.rstd = rs;
    }
  }
  __syncthreads();
  const int s = fb.s;
  const bool bad = (s == kFxaNonFinite);
  int raws[4] = {0, 0, 0, 0};
  const float* xh = RMS ? wsm : xsm;
  fxa_build<BITS>(xh + k_lo, K - k_lo, s, bad, iters, frag, tid, NT, raws, xg, group);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) raws[j] += __shfl_xor_sync(0xffffffffu, raws[j], m);
    if (lane == 0) fb.rawsum[warp][j] = raws[j];
  }
  __syncthreads();
  if (tid < 4) {
    int t = 0;
    for (int w = 0; w < NW; ++w) t += fb.rawsum[w][tid];
    fb.tot[tid] = t - 64 * iters * Pack<BITS>::kIter;  // balanced digit sums (padding digits are 0)
  }
  __syncthreads();
}

// Warp version (one activation row per warp, no RMS, 2-bit layout).
template <int XT>
__device__ __forceinline__ int fxa_warp_prologue2(const void* xr, int K, int iters, float* xsm, uint2* frag,
                                                  int (&tot)[4]) {
  const int lane = threadIdx.x & 31;
  stage_row<XT, 32, 8>(xr, K, xsm, lane);
  __syncwarp();
  unsigned amax = 0;
  for (int k = lane; k < K; k += 32) amax = max(amax, __float_as_uint(xsm[k]) & 0x7fffffffu);
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, m));
  const int s = fxa_shift(amax);
  int raws[4] = {0, 0, 0, 0};
  fxa_build<2>(xsm, K, s, s == kFxaNonFinite, iters, frag, lane, 32, raws);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) raws[j] += __shfl_xor_sync(0xffffffffu, raws[j], m);
    tot[j] = raws[j] - 64 * iters * 256;
  }
  __syncwarp();
  return s;
}

// ----------------------------------------------------------- direct --
// Direct prologue pieces: a thread owns whole 16-value blocks of the
// activation row, loads them straight into registers (no shared-memory
// staging), and once the row's shift is known writes the digit fragments of
// its blocks into a COMPACT fragment array: 16 entries per (iteration, MMA),
// entry 4j + t = digit j for lane (g = j, t).  Only lanes 0-15 (columns 0-3,
// the four digits) read it; lanes 16-31 feed the zero columns 4-7 from a
// register.  Block b (values 16b .. 16b+15) of iteration it = b / 16 is
// exactly the pair of fragment entries (it, 2q, t) and (it, 2q+1, t) with
// t = (b / 4) % 4 and q = b % 4, so the digits equal fxa_build's.
template <int XT> struct XBlk { static constexpr int kChunks = XT == kBF16 ? 2 : 4; };

// Load activation blocks tid, tid + NT, ... (b < K/16) into raw registers in
// the 16-byte-vector layout widen_u4 expects.  Unaligned rows use element
// loads packed into the same layout.
template <int XT, int NT, int MAXB>
__device__ __forceinline__ void xblk_issue(const void* src, int K, int tid, uint4 (&r)[MAXB][XBlk<XT>::kChunks]) {
  constexpr int C = XBlk<XT>::kChunks;
  const char* s8 = static_cast<const char*>(src);
  const bool aligned = (reinterpret_cast<uintptr_t>(src) & 15) == 0;
#pragma unroll
  for (int i = 0; i < MAXB; ++i) {
    const int b = tid + i * NT;
#pragma unroll
    for (int c = 0; c < C; ++c) r[i][c] = make_uint4(0u, 0u, 0u, 0u);
    if (b < (K >> 4)) {
      if (aligned) {
#pragma unroll
        for (int c = 0; c < C; ++c) r[i][c] = ld_u4(s8 + (size_t)b * 16 * C + 16 * c);
      } else {
#pragma unroll
        for (int c = 0; c < C; ++c) {
          uint32_t w[4];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            if constexpr (XT == kBF16) {
              const uint16_t* h = reinterpret_cast<const uint16_t*>(s8) + (size_t)b * 16 + 8 * c + 2 * q;
              w[q] = static_cast<uint32_t>(h[0]) | (static_cast<uint32_t>(h[1]) << 16);
            } else {
              w[q] = reinterpret_cast<const uint32_t*>(s8)[(size_t)b * 16 + 4 * c + q];
            }
          }
          r[i][c] = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
  }
}

// The 16 fp32 values of one raw block.
template <int XT>
__device__ __forceinline__ void xblk_values(const uint4 (&r)[XBlk<XT>::kChunks], float (&v)[16]) {
  constexpr int C = XBlk<XT>::kChunks;
#pragma unroll
  for (int c = 0; c < C; ++c) widen_u4<XT>(r[c], v + c * (16 / C));
}

// Write the compact fragment entries of block b (values v, already scaled
// like the contraction's input) at shift s; adds its plain digits to raws.
__device__ __forceinline__ void fxa_block_encode(const float (&v)[16], int b, int s, bool bad, uint2* frag,
                                                 int (&raws)[4]) {
  const int it = b >> 4, t = (b >> 2) & 3, q = b & 3;
  uint32_t u[16];
#pragma unroll
  for (int e = 0; e < 16; ++e) u[e] = static_cast<uint32_t>((bad ? 0 : fxa_enc(v[e], s)) + kFxaOffset);
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    // entry (it, 2q + h, t): values 2h + {0, 4, 8, 12} (low word), 2h + 1 + {0, 4, 8, 12} (high word)
    uint2* dst = frag + (it * 8 + 2 * q + h) * 16 + t;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t w0 = raw_digits(u[2 * h], u[2 * h + 4], u[2 * h + 8], u[2 * h + 12], j);
      const uint32_t w1 = raw_digits(u[2 * h + 1], u[2 * h + 5], u[2 * h + 9], u[2 * h + 13], j);
      raws[j] = static_cast<int>(__dp4a(w0, 0x01010101u, static_cast<unsigned>(raws[j])));
      raws[j] = static_cast<int>(__dp4a(w1, 0x01010101u, static_cast<unsigned>(raws[j])));
      dst[4 * j] = make_uint2(signed_digits(w0), signed_digits(w1));
    }
  }
}

// contract_tile2 over a compact fragment array (16 entries per MMA).
template <int NI>
__device__ __forceinline__ void contract_tile2c(const uint4 (&wa)[NI], const uint4 (&wb)[NI], int iters,
                                                const uint2* frag, int lane, int (&acc)[4]) {
  int a2[4] = {0, 0, 0, 0};
  const bool rd = lane < 16;
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    if (i < iters) {
      const uint32_t ga[4] = {wa[i].x, wa[i].y, wa[i].z, wa[i].w};
      const uint32_t gb[4] = {wb[i].x, wb[i].y, wb[i].z, wb[i].w};
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const int q = m >> 1, sh = 4 * (m & 1);
        const uint32_t a0 = (ga[q] >> sh) & 0x03030303u;
        const uint32_t a2r = (ga[q] >> (sh + 2)) & 0x03030303u;
        const uint32_t a1 = (gb[q] >> sh) & 0x03030303u;
        const uint32_t a3 = (gb[q] >> (sh + 2)) & 0x03030303u;
        const uint2 bf = rd ? frag[(i * 8 + m) * 16 + lane] : make_uint2(0u, 0u);
        if (m & 1) mma_u8s8(a2, a0, a1, a2r, a3, bf.x, bf.y);
        else mma_u8s8(acc, a0, a1, a2r, a3, bf.x, bf.y);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) acc[j] += a2[j];
}

// Contraction with two independent accumulator chains (even / odd MMAs),
// summed at the end (exact integers).  Same tile semantics as contract_tile.
template <int NI>
__device__ __forceinline__ void contract_tile2(const uint4 (&wa)[NI], const uint4 (&wb)[NI], int iters,
                                               const uint2* frag, int lane, int (&acc)[4]) {
  int a2[4] = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    if (i < iters) {
      const uint32_t ga[4] = {wa[i].x, wa[i].y, wa[i].z, wa[i].w};
      const uint32_t gb[4] = {wb[i].x, wb[i].y, wb[i].z, wb[i].w};
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const int q = m >> 1, sh = 4 * (m & 1);
        const uint32_t a0 = (ga[q] >> sh) & 0x03030303u;
        const uint32_t a2r = (ga[q] >> (sh + 2)) & 0x03030303u;
        const uint32_t a1 = (gb[q] >> sh) & 0x03030303u;
        const uint32_t a3 = (gb[q] >> (sh + 2)) & 0x03030303u;
        const uint2 bf = frag[(i * 8 + m) * 32 + lane];
        if (m & 1) mma_u8s8(a2, a0, a1, a2r, a3, bf.x, bf.y);
        else mma_u8s8(acc, a0, a1, a2r, a3, bf.x, bf.y);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) acc[j] += a2[j];
}

// Contract one warp's 16-row tile: rows g and g+8 supply words via wa/wb
// (already loaded), frag holds the digit fragments of the matching K range.
// acc: lanes t<2 end with digits 2t, 2t+1 for rows g (acc0,1) and g+8 (acc2,3).
template <int NI>
__device__ __forceinline__ void contract_tile(const uint4 (&wa)[NI], const uint4 (&wb)[NI], int iters,
                                              const uint2* frag, int lane, int (&acc)[4]) {
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    if (i < iters) {
      const uint32_t ga[4] = {wa[i].x, wa[i].y, wa[i].z, wa[i].w};
      const uint32_t gb[4] = {wb[i].x, wb[i].y, wb[i].z, wb[i].w};
#pragma unroll
      for (int m = 0; m < 8; ++m) {
        const int q = m >> 1, sh = 4 * (m & 1);
        const uint32_t a0 = (ga[q] >> sh) & 0x03030303u;
        const uint32_t a2 = (ga[q] >> (sh + 2)) & 0x03030303u;
        const uint32_t a1 = (gb[q] >> sh) & 0x03030303u;
        const uint32_t a3 = (gb[q] >> (sh + 2)) & 0x03030303u;
        const uint2 bf = frag[(i * 8 + m) * 32 + lane];
        mma_u8s8(acc, a0, a1, a2, a3, bf.x, bf.y);
      }
    }
  }
}

// Combine the four digit sums of rows g / g+8 (spread over lanes t=0,1) into
// exact int64 contractions, valid on lanes with t == 0.
__device__ __forceinline__ void combine_digits(const int (&acc)[4], const int (&tot)[4], int t,
                                               long long& Sg, long long& Sh) {
  int a0 = acc[0], a1 = acc[1], a2 = acc[2], a3 = acc[3];
  if (t < 2) {
    a0 -= tot[2 * t]; a1 -= tot[2 * t + 1];
    a2 -= tot[2 * t]; a3 -= tot[2 * t + 1];
  }
  const long long pg = (long long)a0 + 128LL * a1;
  const long long ph = (long long)a2 + 128LL * a3;
  const long long ug = __shfl_down_sync(0xffffffffu, pg, 1);
  const long long uh = __shfl_down_sync(0xffffffffu, ph, 1);
  Sg = pg + 16384LL * ug;
  Sh = ph + 16384LL * uh;
}

}  // namespace mb
