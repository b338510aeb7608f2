// Packed ternary GEMV (dense and selected-expert) with optional fused input
// RMSNorm or fused SwiGLU epilogue.
//
// Reference: maple_run/kernels/ternary_gemv.py:261-388 (ternary_gemv; kernels
// :76-153 batch 1, :156-258 batched), kernels/ternary_expert.py:125-234
// (ternary_expert_gemv) and :403-468 (ternary_expert_swiglu, kernel
// :240-319).  Codes are the reference layout: uint32 [N, K/16] (experts
// stacked [E, N, K/16]), 16 LSB-first 2-bit codes per word, code c meaning c-1.
//
// B200 design.  A batch-1 2-bit GEMV at HBM speed leaves ~1.4 issue slots per
// code on CUDA cores, which an unpack + fp32 add cannot meet.  Here the codes
// go straight into the int8 tensor pipe: a lane's 16-byte load of one row is
// masked into u8 code registers ((w >> 2j) & 0x03030303) and mma.m16n8k32
// (u8 x s8 -> s32) contracts them with the FXA digits of the activation
// (fxa.cuh).  The sum is an exact integer, so it does not depend on tiling or
// K split, and is rounded once to fp32.  t = c - 1 enters as
// sum_k c_k d_k - sum_k d_k per digit.
//
// Work split: CTA = 4 warps, each a 16-row tile.  MODE 0: 64 output rows per
// CTA.  MODE 1 (SwiGLU): 32 outputs per CTA, warps 0-1 take up rows n and
// warps 2-3 the gate rows I+n.  grid.y splits K only when K > 2048; split
// partials are exact int32 and the last CTA of a row group (atomic ticket)
// finishes the rows.  grid.z = activation row (token, or token x top-k slot).
#include "bulk.cuh"
#include "fxa.cuh"
#include "launch.cuh"

namespace mb {

constexpr int kMaxIters = 8;                 // K iterations held in registers (K <= 2048)

enum GemvMode : int { kPlain = 0, kSwiglu = 1 };

struct TGemvParams {
  const void* x;            // activation rows, row stride x_stride elements
  const uint32_t* codes;    // [E?, rows, nwords]
  const int* ids;           // [Z] expert per z, or nullptr (dense)
  const void* alpha;        // [E?, rows]
  const void* rms_w;        // [K] or nullptr
  void* y;                  // [Z, n_out], row stride y_stride elements
  int* ws;                  // split-K partials [Z, ks, rows, 4]
  unsigned* tickets;        // [Z, gridDim.x]
  int64_t x_stride, y_stride;
  int64_t expert_words;     // rows * nwords
  int64_t alpha_estride;    // alpha stride between experts
  int x_div;                // activation row of z is z / x_div
  int rows;                 // code rows per expert (MODE 1: 2*I)
  int n_out;                // outputs per z (MODE 0: rows; MODE 1: I)
  int n_experts;
  int K, nwords, ks, iters;
  float eps;
  int* err;                 // device error word (bounded waits), or nullptr
  int bulk_w;               // SwiGLU expert rows staged by bulk copies (K <= 2048, WM = 4)
};

template <int XT, int AT, int RT, bool RMS, int MODE>
__global__ void __launch_bounds__(128) ternary_gemv_kernel(TGemvParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ FxaShared sh;
  __shared__ float s_val[64];
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int z = blockIdx.z, ksi = blockIdx.y;
  const int it0 = ksi * p.iters;
  const int iters = min(p.iters, (p.nwords + 15) / 16 - it0);

  uint2* frag = reinterpret_cast<uint2*>(smem);
  float* xsm = reinterpret_cast<float*>(smem + (size_t)p.iters * 256 * sizeof(uint2));

  // Expert selection (out-of-range ids produce NaN rows rather than a fault).
  // The ids come from the previous launch, so expert GEMVs wait first; dense
  // GEMVs load their weights before waiting.
  const bool dense = p.ids == nullptr;
  if (!dense) {
    pdl_wait();
    pdl_trigger();
  }
  int e = 0;
  bool bad_id = false;
  if (!dense) {
    e = p.ids[z];
    if (e < 0 || e >= p.n_experts) { bad_id = true; e = 0; }
  }
  const uint32_t* codes = p.codes + (int64_t)e * p.expert_words;

  // Code rows of this warp's tile.
  int tile0;
  if constexpr (MODE == kSwiglu) {
    const int n0 = blockIdx.x * 32;
    tile0 = (warp < 2) ? n0 + 16 * warp : (p.rows >> 1) + n0 + 16 * (warp - 2);
  } else {
    tile0 = blockIdx.x * 64 + 16 * warp;
  }
  const int row_g = tile0 + g, row_h = tile0 + g + 8;
  const int lim = (MODE == kSwiglu) ? ((warp < 2) ? (p.rows >> 1) : p.rows) : p.rows;
  const bool ok_g = row_g < lim && (MODE != kSwiglu || (row_g - ((warp < 2) ? 0 : (p.rows >> 1))) < p.n_out);
  const bool ok_h = row_h < lim && (MODE != kSwiglu || (row_h - ((warp < 2) ? 0 : (p.rows >> 1))) < p.n_out);

  // 1) Weight loads first: they do not depend on the activation.
  uint4 wa[kMaxIters], wb[kMaxIters];
#pragma unroll
  for (int i = 0; i < kMaxIters; ++i) {
    wa[i] = make_uint4(0, 0, 0, 0);
    wb[i] = make_uint4(0, 0, 0, 0);
    if (i < iters) {
      const int word = (it0 + i) * 16 + 4 * t;
      if (word < p.nwords) {
        if (ok_g) wa[i] = ld_stream_u4(codes + (int64_t)row_g * p.nwords + word);
        if (ok_h) wb[i] = ld_stream_u4(codes + (int64_t)row_h * p.nwords + word);
      }
    }
  }

  if (dense) {
    pdl_wait();
    pdl_trigger();
  }
  // 2) Activation prologue (shift over all K, fragments for this split).
  const int xrow = z / p.x_div;
  const void* xr = static_cast<const char*>(p.x) + xrow * p.x_stride * (XT == kBF16 ? 2 : 4);
  fxa_block_prologue<XT, RT, RMS>(xr, p.rms_w, p.K, p.eps, it0 * kIterK, p.iters, xsm, frag, sh, xsm + p.K);
  const int s = sh.s;
  const bool nan_out = (s == kFxaNonFinite) || bad_id;

  // 3) Tensor-core contraction.
  int acc[4] = {0, 0, 0, 0};
  contract_tile<kMaxIters>(wa, wb, iters, frag, lane, acc);

  const void* alpha = static_cast<const char*>(p.alpha) + (int64_t)e * p.alpha_estride * (AT == kBF16 ? 2 : 4);
  auto value = [&](int row, long long S) -> float {
    float v = nan_out ? __int_as_float(0x7fc00000) : fxa_value(S, s);
    if constexpr (RMS) v = __fmul_rn(v, sh.rstd);
    return __fmul_rn(v, load_f<AT>(alpha, row));
  };
  char* yz = static_cast<char*>(p.y) + (int64_t)z * p.y_stride * (XT == kBF16 ? 2 : 4);
  auto swiglu_finish = [&]() {
    __syncthreads();
    if (tid < 32) {
      const int n = blockIdx.x * 32 + tid;
      if (n < p.n_out) {
        float up = s_val[tid], gate = s_val[32 + tid];
        up = fminf(fmaxf(up, -7.0f), 7.0f);
        gate = fminf(gate, 7.0f);
        store_f<XT>(yz, n, __fmul_rn(__fmul_rn(up, gate), msigmoid(gate)));
      }
    }
  };

  if (p.ks == 1) {
    long long Sg, Sh;
    combine_digits(acc, sh.tot, t, Sg, Sh);
    if (t == 0) {
      if constexpr (MODE == kSwiglu) {
        s_val[16 * warp + g] = ok_g ? value(row_g, Sg) : 0.0f;
        s_val[16 * warp + g + 8] = ok_h ? value(row_h, Sh) : 0.0f;
      } else {
        if (ok_g) store_f<XT>(yz, row_g, value(row_g, Sg));
        if (ok_h) store_f<XT>(yz, row_h, value(row_h, Sh));
      }
    }
    if constexpr (MODE == kSwiglu) swiglu_finish();
    return;
  }

  // Split-K: publish exact partials (digit correction of this split applied),
  // the last CTA of the row group finishes.
  if (t < 2) {
    acc[0] -= sh.tot[2 * t]; acc[1] -= sh.tot[2 * t + 1];
    acc[2] -= sh.tot[2 * t]; acc[3] -= sh.tot[2 * t + 1];
  }
  int* wsz = p.ws + ((int64_t)z * p.ks + ksi) * (int64_t)p.rows * 4;
  if (t < 2) {
    if (ok_g) *reinterpret_cast<int2*>(wsz + (int64_t)row_g * 4 + 2 * t) = make_int2(acc[0], acc[1]);
    if (ok_h) *reinterpret_cast<int2*>(wsz + (int64_t)row_h * 4 + 2 * t) = make_int2(acc[2], acc[3]);
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    unsigned* tk = p.tickets + (int64_t)z * gridDim.x + blockIdx.x;
    const unsigned old = atomicAdd(tk, 1u);
    s_last = (old == static_cast<unsigned>(p.ks - 1));
    if (s_last) atomicExch(tk, 0u);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  if (tid < 64) {
    const int w2 = tid >> 4, r2 = tid & 15;
    int row;
    bool ok;
    if constexpr (MODE == kSwiglu) {
      const int n0 = blockIdx.x * 32;
      const int nn = n0 + 16 * (w2 & 1) + r2;
      row = (w2 < 2) ? nn : (p.rows >> 1) + nn;
      ok = nn < p.n_out;
    } else {
      row = blockIdx.x * 64 + tid;
      ok = row < p.rows;
    }
    float v = 0.0f;
    if (ok) {
      long long L[4] = {0, 0, 0, 0};
      for (int k2 = 0; k2 < p.ks; ++k2) {
        const int4 q = __ldcg(reinterpret_cast<const int4*>(
            p.ws + (((int64_t)z * p.ks + k2) * p.rows + row) * 4));
        L[0] += q.x; L[1] += q.y; L[2] += q.z; L[3] += q.w;
      }
      v = value(row, L[0] + 128LL * L[1] + 16384LL * L[2] + 2097152LL * L[3]);
      if constexpr (MODE != kSwiglu) store_f<XT>(yz, row, v);
    }
    if constexpr (MODE == kSwiglu) s_val[tid] = v;
  }
  if constexpr (MODE == kSwiglu) swiglu_finish();
}


// ---------------------------------------------------------------------------
// v2: one CTA covers all of K.  8 warps = WM row tiles x WK K-slices; the
// K-slices' exact int32 partials are summed in shared memory, so no
// workspace is needed.
//
// Activation prologue (the direct form, fxa.cuh): each thread loads whole
// 16-value blocks of the row into registers right after the dependency wait,
// one block-wide max gives the FXA shift, and each thread writes the compact
// digit fragments of its own blocks; a second barrier publishes them.  The
// digits, shift, digit totals and the R128 sum of squares (fused RMSNorm) are
// the same values fxa_prologue computes, so the results are bit-identical.
template <int XT, int AT, int RT, bool RMS, int MODE, int WM, int WK, int NI>
__global__ void __launch_bounds__(32 * WM * WK) tgemv2_kernel(TGemvParams p) {
  constexpr int NT = 32 * WM * WK, NW = NT / 32;
  constexpr int MAXB = (8192 / 16 + NT - 1) / NT;  // activation blocks per thread (K <= 8192)
  constexpr int C = XBlk<XT>::kChunks;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ unsigned s_amax[NW];
  __shared__ int s_raw[NW][4];
  __shared__ float s_part[RMS ? 128 : 1];
  __shared__ int red[WK > 1 ? WK - 1 : 1][WM][32][4];
  __shared__ float s_val[16 * WM];
  __shared__ uint64_t wbar;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = warp % WM, wk = warp / WM;
  const int g = lane >> 2, t = lane & 3;
  const int z = blockIdx.z;
  const int iters_total = (p.nwords + 15) / 16;
  const int ipw = (iters_total + WK - 1) / WK;
  const int it0 = wk * ipw;
  const int my_iters = max(0, min(ipw, iters_total - it0));
  uint2* frag = reinterpret_cast<uint2*>(smem);  // compact: iters_total * 128 entries
  float* wsm = reinterpret_cast<float*>(smem + (size_t)iters_total * 128 * sizeof(uint2));
  // Bulk-staged expert rows (SwiGLU, bulk_w): the CTA's 8*WM up rows, then its
  // 8*WM gate rows, each row nwords words.  The rows depend on the routing ids
  // of the previous launch, so they are fetched after the dependency wait; two
  // bulk copies put the whole 32 KB tile in flight at once, where per-thread
  // 16-byte loads stall at issue once the SM's outstanding requests fill up.
  unsigned char* wtile = smem + (size_t)iters_total * 128 * sizeof(uint2) + (RMS ? (size_t)p.K * sizeof(float) : 0);
  const bool bulkw = MODE == kSwiglu && p.bulk_w != 0;
  const unsigned rowb = (unsigned)p.nwords * 4u;

  const bool dense = p.ids == nullptr;
  const void* xr = static_cast<const char*>(p.x) + (z / p.x_div) * p.x_stride * (XT == kBF16 ? 2 : 4);
  uint4 xb[MAXB][C];
  if (!dense) {
    pdl_wait();
    pdl_trigger();
    // The activation row comes from the previous launch like the ids: its
    // loads go out before the expert rows', so they do not queue behind them.
    xblk_issue<XT, NT, MAXB>(xr, p.K, tid, xb);
  }
  int e = 0;
  bool bad_id = false;
  if (!dense) {
    e = p.ids[z];
    if (e < 0 || e >= p.n_experts) { bad_id = true; e = 0; }
  }
  const uint32_t* codes = p.codes + (int64_t)e * p.expert_words;
  int tile0;
  if constexpr (MODE == kSwiglu) {
    const int n0 = blockIdx.x * (8 * WM);
    tile0 = (wm < WM / 2) ? n0 + 16 * wm : (p.rows >> 1) + n0 + 16 * (wm - WM / 2);
  } else {
    tile0 = blockIdx.x * (16 * WM) + 16 * wm;
  }
  const int row_g = tile0 + g, row_h = tile0 + g + 8;
  const int base = (MODE == kSwiglu && wm >= WM / 2) ? (p.rows >> 1) : 0;
  const int lim = (MODE == kSwiglu) ? base + p.n_out : p.rows;
  const bool ok_g = row_g < lim, ok_h = row_h < lim;

  if (bulkw && tid == 0) {
    const int n0 = blockIdx.x * (8 * WM), nrows = min(8 * WM, p.n_out - n0);
    mbar_init(&wbar, 1);
    mbar_expect_tx(&wbar, 2u * (unsigned)nrows * rowb);
    bulk_g2s(wtile, codes + (int64_t)n0 * p.nwords, (unsigned)nrows * rowb, &wbar);
    bulk_g2s(wtile + (size_t)(8 * WM) * rowb, codes + (int64_t)((p.rows >> 1) + n0) * p.nwords,
             (unsigned)nrows * rowb, &wbar);
  }
  uint4 wa[NI], wb[NI];
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    wa[i] = make_uint4(0, 0, 0, 0);
    wb[i] = make_uint4(0, 0, 0, 0);
    if (i < my_iters && !bulkw) {
      const int word = (it0 + i) * 16 + 4 * t;
      if (word < p.nwords) {
        if (ok_g) wa[i] = ld_stream_u4(codes + (int64_t)row_g * p.nwords + word);
        if (ok_h) wb[i] = ld_stream_u4(codes + (int64_t)row_h * p.nwords + word);
      }
    }
  }
  // Row scales and the norm weight are static: they load with the codes,
  // not after the contraction (each is a DRAM round trip of its own).
  const void* alpha = static_cast<const char*>(p.alpha) + (int64_t)e * p.alpha_estride * (AT == kBF16 ? 2 : 4);
  float al_g = 0.0f, al_h = 0.0f;
  if (wk == 0 && t == 0) {
    if (ok_g) al_g = load_f<AT>(alpha, row_g);
    if (ok_h) al_h = load_f<AT>(alpha, row_h);
  }
  if constexpr (RMS) {
    stage_row<RT, NT, (8192 * 4 / 16 + NT - 1) / NT>(p.rms_w, p.K, wsm, tid);
    __syncthreads();
  }
  if (dense) {
    pdl_wait();
    pdl_trigger();
    xblk_issue<XT, NT, MAXB>(xr, p.K, tid, xb);
  }
  // Fused RMSNorm: the R128 partial sums of squares of the raw row (thread
  // tid < 128 sums k = tid, tid + 128, ... in order), loaded beside the blocks.
  float ss = 0.0f;
  if constexpr (RMS) {
    if (tid < 128)
      for (int k = tid; k < p.K; k += 128) {
        const float xv = load_f<XT>(xr, k);
        ss = __fmaf_rn(xv, xv, ss);
      }
  }
  unsigned am = 0;
#pragma unroll
  for (int i = 0; i < MAXB; ++i) {
    const int b = tid + i * NT;
    if (b < (p.K >> 4)) {
      float v[16];
      xblk_values<XT>(xb[i], v);
#pragma unroll
      for (int q = 0; q < 16; ++q) {
        if constexpr (RMS) v[q] = __fmul_rn(v[q], wsm[16 * b + q]);
        am = max(am, __float_as_uint(v[q]) & 0x7fffffffu);
      }
    }
  }
  am = __reduce_max_sync(0xffffffffu, am);
  if (lane == 0) s_amax[warp] = am;
  if constexpr (RMS) {
    if (tid < 128) s_part[tid] = ss;
  }
  __syncthreads();
  unsigned amax = 0;
#pragma unroll
  for (int w = 0; w < NW; ++w) amax = max(amax, s_amax[w]);
  const int s = fxa_shift(amax);
  const bool bad = (s == kFxaNonFinite);
  int raws[4] = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < MAXB; ++i) {
    const int b = tid + i * NT;
    if (b < (p.K >> 4)) {
      float v[16];
      xblk_values<XT>(xb[i], v);
      if constexpr (RMS) {
#pragma unroll
        for (int q = 0; q < 16; ++q) v[q] = __fmul_rn(v[q], wsm[16 * b + q]);
      }
      fxa_block_encode(v, b, s, bad, frag, raws);
    }
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    raws[j] = __reduce_add_sync(0xffffffffu, raws[j]);
    if (lane == 0) s_raw[warp][j] = raws[j];
  }
  __syncthreads();
  const bool nan_out = bad || bad_id;
  if (bulkw) {
    // the staged rows: a wait that runs out is reported, lets the copies
    // land (bounded) and ends the CTA before anything is read
    const bool ready = mbar_wait_bounded(&wbar, 0);
    if (__syncthreads_or(!ready)) {
      if (tid == 0 && p.err != nullptr) atomicOr(p.err, kErrFlagTimeout);
      mbar_wait_bounded(&wbar, 0);
      return;
    }
    const int lr = (wm < WM / 2 ? 0 : 8 * WM) + 16 * (wm % (WM / 2)) + g;  // local row of row_g
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      if (i < my_iters) {
        const int word = (it0 + i) * 16 + 4 * t;
        if (word < p.nwords) {
          if (ok_g) wa[i] = *reinterpret_cast<const uint4*>(wtile + (size_t)lr * rowb + 4 * word);
          if (ok_h) wb[i] = *reinterpret_cast<const uint4*>(wtile + (size_t)(lr + 8) * rowb + 4 * word);
        }
      }
    }
  }

  int acc[4] = {0, 0, 0, 0};
  contract_tile2c<NI>(wa, wb, my_iters, frag + (size_t)it0 * 128, lane, acc);
  if (wk > 0) {
#pragma unroll
    for (int j = 0; j < 4; ++j) red[wk - 1][wm][lane][j] = acc[j];
  }
  __syncthreads();
  char* yz = static_cast<char*>(p.y) + (int64_t)z * p.y_stride * (XT == kBF16 ? 2 : 4);
  if (wk == 0) {
#pragma unroll
    for (int w2 = 0; w2 < WK - 1; ++w2)
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] += red[w2][wm][lane][j];
    int tot[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      int r = 0;
#pragma unroll
      for (int w = 0; w < NW; ++w) r += s_raw[w][j];
      tot[j] = r - 64 * p.K;  // balanced digit sums over the row's K values
    }
    float rstd = 1.0f;
    if constexpr (RMS) rstd = rstd_of(r128_smem_finish(s_part, lane), p.K, p.eps);
    long long Sg, Sh;
    combine_digits(acc, tot, t, Sg, Sh);
    if (t == 0) {
      auto value = [&](float a, long long S) -> float {
        float v = nan_out ? __int_as_float(0x7fc00000) : fxa_value(S, s);
        if constexpr (RMS) v = __fmul_rn(v, rstd);
        return __fmul_rn(v, a);
      };
      if constexpr (MODE == kSwiglu) {
        s_val[16 * wm + g] = ok_g ? value(al_g, Sg) : 0.0f;
        s_val[16 * wm + g + 8] = ok_h ? value(al_h, Sh) : 0.0f;
      } else {
        if (ok_g) store_f<XT>(yz, row_g, value(al_g, Sg));
        if (ok_h) store_f<XT>(yz, row_h, value(al_h, Sh));
      }
    }
  }
  if constexpr (MODE == kSwiglu) {
    __syncthreads();
    constexpr int H = 8 * WM;  // outputs per CTA
    if (tid < H) {
      const int n = blockIdx.x * H + tid;
      if (n < p.n_out) {
        float up = s_val[tid], gate = s_val[H + tid];
        up = fminf(fmaxf(up, -7.0f), 7.0f);
        gate = fminf(gate, 7.0f);
        store_f<XT>(yz, n, __fmul_rn(__fmul_rn(up, gate), msigmoid(gate)));
      }
    }
  }
}

}  // namespace mb

using namespace mb;

namespace {

int gemv_splits(int64_t nwords) {
  const int64_t iters_total = (nwords + 15) / 16;
  int ks = 1;
  while ((iters_total + ks - 1) / ks > kMaxIters) ++ks;
  return ks;
}

size_t gemv_smem(int iters, int K) {
  return (size_t)iters * 256 * sizeof(uint2) + 2 * (size_t)K * sizeof(float);
}

template <int XT, int AT, int RT, bool RMS, int MODE>
cudaError_t launch_tgemv(const TGemvParams& p, int Z, cudaStream_t st) {
  const int per_cta = (MODE == kSwiglu) ? 32 : 64;
  dim3 grid((p.n_out + per_cta - 1) / per_cta, p.ks, Z);
  const size_t smem = gemv_smem(p.iters, p.K);
  auto kern = ternary_gemv_kernel<XT, AT, RT, RMS, MODE>;
  if (smem > 32 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  launch_k(kern, dim3(grid), dim3(128), smem, st, p);
  return cudaGetLastError();
}

template <int XT, int AT, int MODE>
cudaError_t dispatch_rms(const TGemvParams& p, int rms_dtype, int Z, cudaStream_t st) {
  if (p.rms_w == nullptr) return launch_tgemv<XT, AT, kF32, false, MODE>(p, Z, st);
  if (rms_dtype == kF32) return launch_tgemv<XT, AT, kF32, true, MODE>(p, Z, st);
  return launch_tgemv<XT, AT, kBF16, true, MODE>(p, Z, st);
}

template <int MODE>
cudaError_t dispatch(const TGemvParams& p, int x_dtype, int alpha_dtype, int rms_dtype, int Z,
                     cudaStream_t st) {
  if (x_dtype == kBF16)
    return alpha_dtype == kBF16 ? dispatch_rms<kBF16, kBF16, MODE>(p, rms_dtype, Z, st)
                                : dispatch_rms<kBF16, kF32, MODE>(p, rms_dtype, Z, st);
  return alpha_dtype == kBF16 ? dispatch_rms<kF32, kBF16, MODE>(p, rms_dtype, Z, st)
                              : dispatch_rms<kF32, kF32, MODE>(p, rms_dtype, Z, st);
}

template <int XT, int AT, int RT, bool RMS, int MODE, int WM, int WK, int NI>
cudaError_t launch_v2(const TGemvParams& p, int Z, cudaStream_t st) {
  const int iters_total = (p.nwords + 15) / 16;
  const size_t smem = (size_t)iters_total * 128 * sizeof(uint2) + (RMS ? (size_t)p.K * sizeof(float) : 0) +
                      (p.bulk_w ? (size_t)(16 * WM) * p.nwords * 4 : 0);
  const int per_cta = (MODE == kSwiglu) ? 8 * WM : 16 * WM;
  dim3 grid((p.n_out + per_cta - 1) / per_cta, 1, Z);
  auto kern = tgemv2_kernel<XT, AT, RT, RMS, MODE, WM, WK, NI>;
  if (smem > 32 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  // The whole shared-memory carveout, so the next launch's CTAs (which start
  // early under PDL) find room beside these.
  static const cudaError_t carve =
      cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout, cudaSharedmemCarveoutMaxShared);
  if (carve != cudaSuccess) return carve;
  return launch_k(kern, grid, dim3(32 * WM * WK), smem, st, p);
}

template <int XT, int AT, int RT, bool RMS, int MODE>
cudaError_t pick_v2(const TGemvParams& p, int Z, cudaStream_t st) {
  const int iters_total = (p.nwords + 15) / 16;
  if (iters_total <= 8) {
    // SwiGLU expert rows by bulk copies when the error word is there for the wait
    TGemvParams q = p;
    q.bulk_w = (MODE == kSwiglu && p.ids != nullptr && p.err != nullptr) ? 1 : 0;
    return launch_v2<XT, AT, RT, RMS, MODE, 4, 2, 4>(q, Z, st);
  }
  if (iters_total <= 16) return launch_v2<XT, AT, RT, RMS, MODE, 2, 4, 4>(p, Z, st);
  return launch_v2<XT, AT, RT, RMS, MODE, 2, 4, 8>(p, Z, st);
}

template <int XT, int AT, int MODE>
cudaError_t dispatch_v2(const TGemvParams& p, int rms_dtype, int Z, cudaStream_t st) {
  if (p.rms_w == nullptr) return pick_v2<XT, AT, kF32, false, MODE>(p, Z, st);
  if (rms_dtype == kF32) return pick_v2<XT, AT, kF32, true, MODE>(p, Z, st);
  return pick_v2<XT, AT, kBF16, true, MODE>(p, Z, st);
}

template <int MODE>
cudaError_t dispatch2(const TGemvParams& p, int x_dtype, int alpha_dtype, int rms_dtype, int Z, cudaStream_t st) {
  if (x_dtype == kBF16)
    return alpha_dtype == kBF16 ? dispatch_v2<kBF16, kBF16, MODE>(p, rms_dtype, Z, st)
                                : dispatch_v2<kBF16, kF32, MODE>(p, rms_dtype, Z, st);
  return alpha_dtype == kBF16 ? dispatch_v2<kF32, kBF16, MODE>(p, rms_dtype, Z, st)
                              : dispatch_v2<kF32, kF32, MODE>(p, rms_dtype, Z, st);
}


int common_checks(int x_dtype, int alpha_dtype, const void* rms_w, int rms_dtype, int64_t k) {
  if ((x_dtype != kF32 && x_dtype != kBF16) || (alpha_dtype != kF32 && alpha_dtype != kBF16) ||
      (rms_w && rms_dtype != kF32 && rms_dtype != kBF16))
    return kErrDtype;
  if (k % 64 != 0 || k > 8192) return kErrShape;
  return kOk;
}


}  // namespace

extern "C" int64_t maple_ternary_gemv_workspace_bytes(int64_t batch, int64_t n, int64_t k) {
  (void)batch; (void)n; (void)k;
  return 0;  // one CTA covers all of K (k <= 8192): no split-K scratch
}

extern "C" int maple_ternary_gemv(const void* x, int x_dtype, int64_t batch, int64_t k,
                                  int64_t x_row_stride, const uint32_t* codes, int64_t n,
                                  const void* alpha, int alpha_dtype, const void* rms_w,
                                  int rms_dtype, float eps, void* y, int64_t y_row_stride,
                                  void* workspace, int64_t workspace_bytes, void* stream) {
  if (batch < 0 || n < 0 || k < 0) return kErrShape;
  if (batch == 0 || n == 0) return kOk;
  if (int rc = common_checks(x_dtype, alpha_dtype, rms_w, rms_dtype, k)) return rc;
  if (!x || !codes || !alpha || !y) return kErrShape;
  if ((reinterpret_cast<uintptr_t>(codes) & 15) != 0) return kErrAlign;
  if (batch > 65535 || n > (1LL << 30)) return kErrShape;
  TGemvParams p{};
  p.x = x; p.codes = codes; p.alpha = alpha; p.rms_w = rms_w; p.y = y;
  p.x_stride = x_row_stride; p.y_stride = y_row_stride; p.x_div = 1;
  p.rows = (int)n; p.n_out = (int)n; p.n_experts = 1;
  p.K = (int)k; p.nwords = (int)(k / 16); p.eps = eps;
  (void)workspace; (void)workspace_bytes;
  const cudaError_t e = dispatch2<kPlain>(p, x_dtype, alpha_dtype, rms_dtype, (int)batch,
                                          static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int64_t maple_ternary_expert_gemv_workspace_bytes(int64_t slots, int64_t n, int64_t k) {
  (void)slots; (void)n; (void)k;
  return 0;
}

extern "C" int maple_ternary_expert_gemv(const void* x, int x_dtype, int64_t x_row_stride,
                                         int64_t x_rows_per_token, const int32_t* expert_ids,
                                         int64_t slots, int64_t k, const uint32_t* codes,
                                         int64_t n_experts, int64_t n, const void* alpha,
                                         int alpha_dtype, void* y, int64_t y_row_stride,
                                         void* workspace, int64_t workspace_bytes, void* stream) {
  if (slots < 0 || n < 0 || k < 0 || n_experts <= 0) return kErrShape;
  if (slots == 0 || n == 0) return kOk;
  if (int rc = common_checks(x_dtype, alpha_dtype, nullptr, 0, k)) return rc;
  if (!x || !codes || !alpha || !y || !expert_ids) return kErrShape;
  if ((reinterpret_cast<uintptr_t>(codes) & 15) != 0) return kErrAlign;
  if (slots > 65535 || x_rows_per_token < 1) return kErrShape;
  TGemvParams p{};
  p.x = x; p.codes = codes; p.ids = expert_ids; p.alpha = alpha; p.y = y;
  p.x_stride = x_row_stride; p.y_stride = y_row_stride; p.x_div = (int)x_rows_per_token;
  p.rows = (int)n; p.n_out = (int)n; p.n_experts = (int)n_experts;
  p.expert_words = n * (k / 16); p.alpha_estride = n;
  p.K = (int)k; p.nwords = (int)(k / 16);
  (void)workspace; (void)workspace_bytes;
  const cudaError_t e = dispatch2<kPlain>(p, x_dtype, alpha_dtype, 0, (int)slots,
                                          static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int64_t maple_ternary_expert_swiglu_workspace_bytes(int64_t slots, int64_t inter,
                                                                int64_t k) {
  (void)slots; (void)inter; (void)k;
  return 0;
}

extern "C" int maple_ternary_expert_swiglu(const void* x, int x_dtype, int64_t x_row_stride,
                                           const int32_t* expert_ids, int64_t tokens, int64_t topk,
                                           int64_t k, const uint32_t* codes, int64_t n_experts,
                                           int64_t inter, const void* alpha, int alpha_dtype,
                                           void* y, int64_t y_row_stride, void* workspace,
                                           int64_t workspace_bytes, int* err, void* stream) {
  if (tokens < 0 || topk <= 0 || k < 0 || inter < 0 || n_experts <= 0) return kErrShape;
  if (tokens == 0 || inter == 0) return kOk;
  if (int rc = common_checks(x_dtype, alpha_dtype, nullptr, 0, k)) return rc;
  if (!x || !codes || !alpha || !y || !expert_ids) return kErrShape;
  if ((reinterpret_cast<uintptr_t>(codes) & 15) != 0) return kErrAlign;
  const int64_t slots = tokens * topk;
  if (slots > 65535) return kErrShape;
  TGemvParams p{};
  p.x = x; p.codes = codes; p.ids = expert_ids; p.alpha = alpha; p.y = y;
  p.x_stride = x_row_stride; p.y_stride = y_row_stride; p.x_div = (int)topk;
  p.rows = (int)(2 * inter); p.n_out = (int)inter; p.n_experts = (int)n_experts;
  p.expert_words = 2 * inter * (k / 16); p.alpha_estride = 2 * inter;
  p.K = (int)k; p.nwords = (int)(k / 16); p.err = err;
  (void)workspace; (void)workspace_bytes;
  const cudaError_t e = dispatch2<kSwiglu>(p, x_dtype, alpha_dtype, 0, (int)slots,
                                           static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? kOk : kErrCuda;
}

// ---------------------------------------------------------------------------
// Ternary GEMV for callers that cannot allocate device memory.
//
// Some callers of this library own no CUDA allocator: a host that binds the
// library through a thin foreign-function layer (cgo, JNI, ctypes) and is
// handed only the input and output buffers, or a serving loop whose device
// memory is fully reserved up front by its KV-cache pool.  They cannot size,
// allocate and zero the workspace that maple_ternary_gemv wants for its
// split-K partials.  This entry point takes no workspace: its scratch is the
// file-scope array below, a fixed 2 MiB on every GPU that loads the library,
// held until the process exits.  It never calls cudaMalloc or cudaFree.
//
// * The first call on a device looks up the array's device address there
//   (cudaGetSymbolAddress) and remembers it; make that first call before any
//   stream capture.
// * All calls share the one array, which keeps the last call's contents.
//   The completion tickets are cleared at the start of every call; the split
//   partials are fully rewritten before they are read.  Two calls that can
//   run at the same time on the GPU (different streams, no ordering) race on
//   the array and give wrong results: serialise them.
// * Requests whose split-K scratch does not fit (see kNoAllocPartialBytes)
//   return MAPLE_ERR_SCRATCH_LIMIT without launching anything.
#include <mutex>

namespace {

constexpr int64_t kNoAllocScratchBytes = 2 * 1024 * 1024;
constexpr int64_t kNoAllocTicketBytes = 16 * 1024;  // 4096 completion tickets
constexpr int64_t kNoAllocPartialBytes = kNoAllocScratchBytes - kNoAllocTicketBytes;
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void* g_noalloc_address[kNoAllocMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device, looked up once.
cudaError_t noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kNoAllocMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_address[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return e;
    g_noalloc_address[dev] = p;
  }
  *out = g_noalloc_address[dev];
  return cudaSuccess;
}

}  // namespace

extern "C" int maple_ternary_gemv_noalloc(const void* x, int x_dtype, int64_t batch, int64_t k,
                                          int64_t x_row_stride, const uint32_t* codes, int64_t n,
                                          const void* alpha, int alpha_dtype, const void* rms_w,
                                          int rms_dtype, float eps, void* y, int64_t y_row_stride,
                                          void* stream) {
  if (batch < 0 || n < 0 || k < 0) return kErrShape;
  if (batch == 0 || n == 0) return kOk;
  if (int rc = common_checks(x_dtype, alpha_dtype, rms_w, rms_dtype, k)) return rc;
  if (!x || !codes || !alpha || !y) return kErrShape;
  if ((reinterpret_cast<uintptr_t>(codes) & 15) != 0) return kErrAlign;
  if (batch > 65535 || n > (1LL << 30)) return kErrShape;
  TGemvParams p{};
  p.x = x; p.codes = codes; p.alpha = alpha; p.rms_w = rms_w; p.y = y;
  p.x_stride = x_row_stride; p.y_stride = y_row_stride; p.x_div = 1;
  p.rows = (int)n; p.n_out = (int)n; p.n_experts = 1;
  p.K = (int)k; p.nwords = (int)(k / 16); p.eps = eps;
  p.ks = gemv_splits(p.nwords);
  const int iters_total = (p.nwords + 15) / 16;
  p.iters = (iters_total + p.ks - 1) / p.ks;
  p.ks = (iters_total + p.iters - 1) / p.iters;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (p.ks > 1) {
    const int64_t tickets = batch * ((n + 63) / 64);
    const int64_t partials = batch * p.ks * n * 4 * (int64_t)sizeof(int);
    if (tickets * (int64_t)sizeof(unsigned) > kNoAllocTicketBytes || partials > kNoAllocPartialBytes)
      return kErrScratchLimit;
    void* base = nullptr;
    if (noalloc_scratch(&base) != cudaSuccess) return kErrCuda;
    if (cudaMemsetAsync(base, 0, tickets * sizeof(unsigned), st) != cudaSuccess) return kErrCuda;
    p.tickets = static_cast<unsigned*>(base);
    p.ws = reinterpret_cast<int*>(static_cast<char*>(base) + kNoAllocTicketBytes);
  }
  const cudaError_t e = dispatch<kPlain>(p, x_dtype, alpha_dtype, rms_dtype, (int)batch, st);
  return e == cudaSuccess ? kOk : kErrCuda;
}
