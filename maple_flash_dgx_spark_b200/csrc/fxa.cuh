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
