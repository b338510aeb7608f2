// Batched packed-ternary GEMM (dense and expert-grouped) with the weights read
// once per batch.
//
// Reference: maple_run/kernels/ternary_gemv.py:156-258, 355-388 (batched
// _ternary_gemm_kernel), kernels/ternary_expert.py:125-234 and :403-468 (the
// expert paths, which the reference runs per (token, slot)).
//
// B200 design.  The arithmetic is the batch-1 GEMV's (exact integer
// contraction of codes with the FXA digits of each activation row, rounded
// once), so every output row is bit-identical to the batch-1 result:
//   1. fxa_encode_kernel encodes each activation row once (optionally with the
//      fused input RMSNorm) into a compact digit buffer: for row r, entry
//      ((it*8 + m)*16 + l) holds the s8 digit quad that lane l (< 16) of the
//      m16n8k32 B fragment needs, plus 32 bytes of row metadata
//      (shift, rstd, balanced digit totals).
//   2. tgemm_kernel: each warp keeps a 16-row weight tile in registers for its
//      K slice and contracts it with a chunk of activation rows staged in
//      shared memory by cp.async.bulk (double-buffered).  One MMA covers two
//      activation rows: B columns 0-3 are row a's four digits, columns 4-7
//      row b's, so lanes 0-15 read row a's compact entries and lanes 16-31
//      row b's.  K-slices of a CTA meet in shared memory.
//   3. Grouped mode: moe_plan_kernel sorts the (token, slot) pairs by expert
//      on the device; grid.y = expert, and a CTA runs all of its expert's
//      slots against one register-resident tile, so each selected expert's
//      bytes are read once per batch.
#include "bulk.cuh"
#include "fxa.cuh"
#include "launch.cuh"

namespace mb {

enum GemmMode : int { kGPlain = 0, kGSwiglu = 1 };
constexpr int kMetaInts = 8;  // s, rstd bits, tot[0..3], 0, 0
constexpr unsigned kBadSlot = 0x80000000u;

__host__ __device__ constexpr int fxa_iters(int K) { return (K + 255) / 256; }

// ------------------------------------------------------------- encode ----
template <int XT, int RT, bool RMS>
__global__ void __launch_bounds__(256) fxa_encode_kernel(const void* x, int64_t x_stride, const void* rms_w, int K,
                                                         float eps, uint2* out, int* meta) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ FxaBlock fb;
  const int iters = fxa_iters(K);
  uint2* frag = reinterpret_cast<uint2*>(smem);
  float* xsm = reinterpret_cast<float*>(smem + (size_t)iters * 256 * sizeof(uint2));
  float* wsm = xsm + K;
  const int64_t r = blockIdx.x;
  pdl_wait();
  pdl_trigger();
  const void* xr = static_cast<const char*>(x) + r * x_stride * (XT == kBF16 ? 2 : 4);
  fxa_prologue<XT, RT, RMS, 2, 256>(xr, rms_w, K, eps, 0, iters, xsm, wsm, frag, fb);
  uint4* o = reinterpret_cast<uint4*>(out + r * iters * 128);
  const uint4* f4 = reinterpret_cast<const uint4*>(frag);
  // entry (i, l<16) of the full layout is frag[i*32 + l]; two entries per uint4
  for (int c = threadIdx.x; c < iters * 64; c += 256) o[c] = f4[(c >> 3) * 16 + (c & 7)];
  if (threadIdx.x < kMetaInts) {
    const int j = threadIdx.x;
    int v = 0;
    if (j == 0) v = fb.s;
    else if (j == 1) v = __float_as_int(fb.rstd);
    else if (j < 6) v = fb.tot[j - 2];
    meta[r * kMetaInts + j] = v;
  }
}

// --------------------------------------------------------------- plan ----
// Counting sort of slots (t*top_k + j) by expert, for the experts
// [e_first, e_first + n_local) held here (all of them on one GPU; a rank's
// share under expert parallelism).  offsets[e] .. offsets[e+1] index list[]
// by local expert.  An out-of-range id is listed under expert 0 with
// kBadSlot set (its output row becomes NaN, as in the batch-1 expert GEMV).
// The order inside an expert is irrelevant: every row's result is exact on
// its own.
__global__ void __launch_bounds__(1024) moe_plan_kernel(const int* ids, int n_slots, int E, int e_first, int n_local,
                                                        int* offsets, unsigned* list) {
  extern __shared__ int cnt[];  // [n_local] counts, then [n_local] cursors
  int* cur = cnt + n_local;
  pdl_wait();
  pdl_trigger();
  for (int e = threadIdx.x; e < n_local; e += blockDim.x) cnt[e] = 0;
  __syncthreads();
  for (int s = threadIdx.x; s < n_slots; s += blockDim.x) {
    int e = ids[s];
    if (e < 0 || e >= E) e = 0;
    e -= e_first;
    if (e >= 0 && e < n_local) atomicAdd(&cnt[e], 1);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    int acc = 0;
    for (int e = 0; e < n_local; ++e) {
      offsets[e] = acc;
      cur[e] = acc;
      acc += cnt[e];
    }
    offsets[n_local] = acc;
  }
  __syncthreads();
  for (int s = threadIdx.x; s < n_slots; s += blockDim.x) {
    const int e0 = ids[s];
    const bool bad = e0 < 0 || e0 >= E;
    const int e = (bad ? 0 : e0) - e_first;
    if (e >= 0 && e < n_local) {
      const int pos = atomicAdd(&cur[e], 1);
      list[pos] = static_cast<unsigned>(s) | (bad ? kBadSlot : 0u);
    }
  }
}

// --------------------------------------------------------------- GEMM ----
struct TGemmParams {
  const uint32_t* codes;   // [E?, rows, nwords]
  const void* alpha;       // [E?, rows]
  const uint2* frag;       // [R_in, iters*128] compact digits
  const int* meta;         // [R_in, 8]
  void* y;                 // output rows, stride y_stride elements
  const int* offsets;      // grouped: [E+1]; nullptr = dense
  const unsigned* list;    // grouped: slots sorted by expert
  int* err;
  int64_t y_stride;
  int64_t expert_words;    // rows * nwords
  int64_t alpha_estride;
  int rows;                // code rows (SwiGLU: 2*I)
  int n_out;               // outputs per activation row (SwiGLU: I)
  int K, nwords, iters;
  int R;                   // dense: activation rows
  int chunks_per_cta;      // dense: row chunks per CTA
  int in_div;              // grouped: input row = slot / in_div
  int use_rstd;            // multiply by the row's rstd (fused input RMSNorm)
  int plan_final;          // grouped: plan written before the previous launch
};

// Shared memory: 2 x [RC rows x iters*128 uint2] digits, 2 x [RC x 8] meta,
// then the K-slice reduction and the SwiGLU staging.
template <int WM, int WK, int RC>
__host__ __device__ constexpr size_t tgemm_red_bytes() {
  return (size_t)(WK > 1 ? WK - 1 : 1) * WM * (RC / 2) * 32 * 4 * sizeof(int);
}

// NBUF = 2 double-buffers the digit chunks (many rows per CTA); NBUF = 1
// halves the shared memory for decode-sized groups (one chunk per expert),
// so two CTAs share an SM.
template <int AT, int OT, int MODE, int WM, int WK, int NI, int RC, int NBUF>
__global__ void __launch_bounds__(32 * WM * WK, NBUF == 1 ? 2 : 1) tgemm_kernel(TGemmParams p) {
  constexpr int NT = 32 * WM * WK, NP = RC / 2;
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ uint64_t bar[2];
  __shared__ unsigned s_slot[2][RC];
  __shared__ float s_val[MODE == kGSwiglu ? RC : 1][16 * WM];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int wm = warp % WM, wk = warp / WM;
  const int g = lane >> 2, t = lane & 3;
  const int iters = p.iters;
  const int rowu2 = iters * 128;
  const size_t buf_bytes = (size_t)RC * rowu2 * sizeof(uint2);
  uint2* buf0 = reinterpret_cast<uint2*>(smem);
  int* meta_s = reinterpret_cast<int*>(smem + NBUF * buf_bytes);                          // [NBUF][RC][8]
  int* red = reinterpret_cast<int*>(smem + NBUF * buf_bytes + NBUF * RC * kMetaInts * 4);  // [WK-1][WM][NP][32][4]

  const bool grouped = p.offsets != nullptr;
  const int e = grouped ? blockIdx.y : 0;
  if (grouped && !p.plan_final) {
    pdl_wait();
    pdl_trigger();
  }
  int first = 0, count = 0;
  if (grouped) {
    first = p.offsets[e];
    count = p.offsets[e + 1] - first;
  } else {
    first = blockIdx.y * p.chunks_per_cta * RC;
    count = min(p.chunks_per_cta * RC, p.R - first);
  }
  if (count <= 0) {
    if (!grouped || p.plan_final) {
      pdl_wait();
      pdl_trigger();
    }
    return;
  }
  const int nchunks = (count + RC - 1) / RC;

  // This warp's 16-row weight tile over its K slice, loaded before the wait.
  const int ipw = (iters + WK - 1) / WK;
  const int it0 = wk * ipw;
  const int my_iters = max(0, min(ipw, iters - it0));
  const uint32_t* codes = p.codes + (int64_t)e * p.expert_words;
  int tile0;
  if constexpr (MODE == kGSwiglu) {
    const int n0 = blockIdx.x * (8 * WM);
    tile0 = (wm < WM / 2) ? n0 + 16 * wm : (p.rows >> 1) + n0 + 16 * (wm - WM / 2);
  } else {
    tile0 = blockIdx.x * (16 * WM) + 16 * wm;
  }
  const int row_g = tile0 + g, row_h = tile0 + g + 8;
  const int base = (MODE == kGSwiglu && wm >= WM / 2) ? (p.rows >> 1) : 0;
  const int lim = (MODE == kGSwiglu) ? base + p.n_out : p.rows;
  const bool ok_g = row_g < lim, ok_h = row_h < lim;
  uint4 wa[NI], wb[NI];
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    wa[i] = make_uint4(0, 0, 0, 0);
    wb[i] = make_uint4(0, 0, 0, 0);
    if (i < my_iters) {
      const int word = (it0 + i) * 16 + 4 * t;
      if (word < p.nwords) {
        if (ok_g) wa[i] = ld_stream_u4(codes + (int64_t)row_g * p.nwords + word);
        if (ok_h) wb[i] = ld_stream_u4(codes + (int64_t)row_h * p.nwords + word);
      }
    }
  }
  const void* alpha = static_cast<const char*>(p.alpha) + (int64_t)e * p.alpha_estride * (AT == kBF16 ? 2 : 4);
  const float a_g = ok_g ? load_f<AT>(alpha, row_g) : 0.0f;
  const float a_h = ok_h ? load_f<AT>(alpha, row_h) : 0.0f;
  if (!grouped || p.plan_final) {
    pdl_wait();
    pdl_trigger();
  }

  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
  }
  __syncthreads();
  // Stage chunk c into buffer c % NBUF (thread 0).  The chunk's slot ids are
  // loaded together (one L2 round trip, not one per slot) before the copies
  // that depend on them are issued.
  auto issue = [&](int c) {
    const int b = c % NBUF;
    const int n = min(RC, count - c * RC);
    unsigned sl[RC];
#pragma unroll
    for (int i = 0; i < RC; ++i)
      sl[i] = i < n ? (grouped ? p.list[first + c * RC + i] : static_cast<unsigned>(first + c * RC + i))
                    : 0xffffffffu;
#pragma unroll
    for (int i = 0; i < RC; ++i) s_slot[b][i] = sl[i];
    mbar_expect_tx(&bar[b], (unsigned)n * ((unsigned)(rowu2 * sizeof(uint2)) + kMetaInts * 4));
#pragma unroll
    for (int i = 0; i < RC; ++i) {
      if (i >= n) break;
      const unsigned slot = sl[i];
      const int64_t in_row = grouped ? (int64_t)(slot & ~kBadSlot) / p.in_div : (int64_t)slot;
      bulk_g2s(buf0 + ((size_t)b * RC + i) * rowu2, p.frag + in_row * rowu2, (unsigned)(rowu2 * sizeof(uint2)),
               &bar[b]);
      bulk_g2s(meta_s + (b * RC + i) * kMetaInts, p.meta + in_row * kMetaInts, kMetaInts * 4, &bar[b]);
    }
  };
  if (tid == 0) issue(0);

  for (int c = 0; c < nchunks; ++c) {
    const int b = c % NBUF;
    const unsigned par = (unsigned)(c / NBUF) & 1u;
    if (tid == 0) {
      if (NBUF == 2 && c + 1 < nchunks) {
        fence_proxy_async_smem();
        issue(c + 1);
      } else if (NBUF == 1 && c > 0) {
        fence_proxy_async_smem();
        issue(c);
      }
    }
    const bool ready = mbar_wait_bounded(&bar[b], par);
    if (__syncthreads_or(!ready)) {
      if (tid == 0) atomicOr(p.err, kErrFlagTimeout);
      // let copies still in flight land before the block exits
      mbar_wait_bounded(&bar[b], par);
      if (NBUF == 2 && c + 1 < nchunks) mbar_wait_bounded(&bar[b ^ 1], (unsigned)((c + 1) / NBUF) & 1u);
      return;
    }
    const uint2* fr = buf0 + (size_t)b * RC * rowu2;
    int acc[NP][4];
#pragma unroll
    for (int q = 0; q < NP; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0;
    const int half = lane >> 4, l16 = lane & 15;
    // One code word of each row (q4) per pass: with two CTAs per SM (NBUF 1,
    // 128 registers) a fully unrolled pass hoists every fragment load and
    // spills; a rolled q4 loop keeps 8 fragment registers live.
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      if (i < my_iters) {
#pragma unroll(NBUF == 1 ? 1 : 4)
        for (int q4 = 0; q4 < 4; ++q4) {
          const uint32_t wga = q4 == 0 ? wa[i].x : q4 == 1 ? wa[i].y : q4 == 2 ? wa[i].z : wa[i].w;
          const uint32_t wgb = q4 == 0 ? wb[i].x : q4 == 1 ? wb[i].y : q4 == 2 ? wb[i].z : wb[i].w;
#pragma unroll
          for (int hm = 0; hm < 2; ++hm) {
            const int sh = 4 * hm;
            const uint32_t a0 = (wga >> sh) & 0x03030303u;
            const uint32_t a2 = (wga >> (sh + 2)) & 0x03030303u;
            const uint32_t a1 = (wgb >> sh) & 0x03030303u;
            const uint32_t a3 = (wgb >> (sh + 2)) & 0x03030303u;
            const int ent = ((it0 + i) * 8 + 2 * q4 + hm) * 16 + l16;
#pragma unroll
            for (int q = 0; q < NP; ++q) {
              const uint2 bv = fr[(size_t)(2 * q + half) * rowu2 + ent];
              mma_u8s8(acc[q], a0, a1, a2, a3, bv.x, bv.y);
            }
          }
        }
      }
    }
    if (WK > 1 && wk > 0) {
#pragma unroll
      for (int q = 0; q < NP; ++q)
#pragma unroll
        for (int j = 0; j < 4; ++j) red[((((wk - 1) * WM + wm) * NP + q) * 32 + lane) * 4 + j] = acc[q][j];
    }
    __syncthreads();
    char* y = static_cast<char*>(p.y);
    if (wk == 0) {
#pragma unroll
      for (int q = 0; q < NP; ++q) {
#pragma unroll
        for (int w2 = 0; w2 < WK - 1; ++w2)
#pragma unroll
          for (int j = 0; j < 4; ++j) acc[q][j] += red[(((w2 * WM + wm) * NP + q) * 32 + lane) * 4 + j];
        const int tok = 2 * q + (t >> 1);  // lanes t<2 hold row a's digits, t>=2 row b's
        const int* ms = meta_s + (b * RC + tok) * kMetaInts;
        const int tt = t & 1;
        int a0 = acc[q][0] - ms[2 + 2 * tt], a1 = acc[q][1] - ms[3 + 2 * tt];
        int a2 = acc[q][2] - ms[2 + 2 * tt], a3 = acc[q][3] - ms[3 + 2 * tt];
        const long long pg = (long long)a0 + 128LL * a1;
        const long long ph = (long long)a2 + 128LL * a3;
        const long long ug = __shfl_down_sync(0xffffffffu, pg, 1);
        const long long uh = __shfl_down_sync(0xffffffffu, ph, 1);
        const unsigned slot = s_slot[b][tok];
        if (tt == 0 && slot != 0xffffffffu) {
          const int s = ms[0];
          const bool nan_out = (s == kFxaNonFinite) || (slot & kBadSlot);
          const float rstd = __int_as_float(ms[1]);
          auto value = [&](long long S, float a) -> float {
            float v = nan_out ? __int_as_float(0x7fc00000) : fxa_value(S, s);
            if (p.use_rstd) v = __fmul_rn(v, rstd);
            return __fmul_rn(v, a);
          };
          const long long Sg = pg + 16384LL * ug, Sh = ph + 16384LL * uh;
          if constexpr (MODE == kGSwiglu) {
            s_val[tok][16 * wm + g] = ok_g ? value(Sg, a_g) : 0.0f;
            s_val[tok][16 * wm + g + 8] = ok_h ? value(Sh, a_h) : 0.0f;
          } else {
            const int64_t orow = grouped ? (int64_t)(slot & ~kBadSlot) : (int64_t)slot;
            char* yr = y + orow * p.y_stride * (OT == kBF16 ? 2 : 4);
            if (ok_g) store_f<OT>(yr, row_g, value(Sg, a_g));
            if (ok_h) store_f<OT>(yr, row_h, value(Sh, a_h));
          }
        }
      }
    }
    if constexpr (MODE == kGSwiglu) {
      __syncthreads();
      constexpr int H = 8 * WM;
      for (int idx = tid; idx < RC * H; idx += NT) {
        const int tok = idx / H, nn = idx - tok * H;
        const unsigned slot = s_slot[b][tok];
        const int n = blockIdx.x * H + nn;
        if (slot != 0xffffffffu && n < p.n_out) {
          float up = s_val[tok][nn], gate = s_val[tok][H + nn];
          up = fminf(fmaxf(up, -7.0f), 7.0f);
          gate = fminf(gate, 7.0f);
          const int64_t orow = grouped ? (int64_t)(slot & ~kBadSlot) : (int64_t)slot;
          // an out-of-range expert id gives a NaN row (the clamps would turn NaN into -49)
          const bool bad = grouped && (slot & kBadSlot);
          store_f<OT>(y + orow * p.y_stride * (OT == kBF16 ? 2 : 4), n,
                      bad ? __int_as_float(0x7fc00000) : __fmul_rn(__fmul_rn(up, gate), msigmoid(gate)));
        }
      }
    }
    __syncthreads();  // buffer b, s_slot[b], red and s_val free for reuse
  }
}

template <int AT, int OT, int MODE, int WM, int WK, int NI, int RC, int NBUF>
cudaError_t launch_tgemm(const TGemmParams& p, dim3 grid, cudaStream_t st) {
  const size_t smem = NBUF * (size_t)RC * p.iters * 128 * sizeof(uint2) + NBUF * RC * kMetaInts * 4 +
                      tgemm_red_bytes<WM, WK, RC>();
  auto kern = tgemm_kernel<AT, OT, MODE, WM, WK, NI, RC, NBUF>;
  if (smem > 32 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  return launch_k(kern, grid, dim3(32 * WM * WK), smem, st, p);
}

// Tile shapes by K: RC rows per chunk keep two chunks of digits within
// 128 KB; NI K-iterations per warp stay in registers (<= 255 per thread).
inline int tgemm_wm(int iters) { return iters <= 8 ? 4 : 2; }
inline int tile_rows(int mode, int iters) { return (mode == kGSwiglu ? 8 : 16) * tgemm_wm(iters); }

// Single-buffer expert groups (decode-sized: about 8 routed slots per expert
// at configs[3]) take 8 slots per chunk also for K <= 1024, so fewer MMAs and
// digit bytes go to empty slots (measured with the weights streaming from
// HBM: grouped down GEMM 61.1 -> 55.4 us; 4-slot chunks: 57.9 us, and the
// SwiGLU 98.8 -> 101.6 us).  Dense launches keep their chunks: the host sizes
// their grid by them.
template <int AT, int OT, int MODE, int NBUF>
cudaError_t dispatch_tgemm_buf(const TGemmParams& p, dim3 grid, cudaStream_t st) {
  const bool small_groups = NBUF == 1 && p.offsets != nullptr;
  if (p.iters <= 4)  // K <= 1024
    return small_groups ? launch_tgemm<AT, OT, MODE, 4, 2, 2, 8, NBUF>(p, grid, st)
                        : launch_tgemm<AT, OT, MODE, 4, 2, 2, 16, NBUF>(p, grid, st);
  if (p.iters <= 8)  // K <= 2048
    return launch_tgemm<AT, OT, MODE, 4, 2, 4, 8, NBUF>(p, grid, st);
  if (p.iters <= 16) return launch_tgemm<AT, OT, MODE, 2, 4, 4, 4, NBUF>(p, grid, st);   // K <= 4096
  return cudaErrorInvalidValue;
}

// One buffer when a CTA sees at most about one chunk of rows.
template <int AT, int OT, int MODE>
cudaError_t dispatch_tgemm(const TGemmParams& p, dim3 grid, cudaStream_t st, bool single_chunk) {
  return single_chunk ? dispatch_tgemm_buf<AT, OT, MODE, 1>(p, grid, st) : dispatch_tgemm_buf<AT, OT, MODE, 2>(p, grid, st);
}

template <int MODE>
cudaError_t dispatch_tgemm_types(const TGemmParams& p, int a_dtype, int y_dtype, dim3 grid, cudaStream_t st,
                                 bool single_chunk) {
  if (a_dtype == kBF16) {
    return y_dtype == kBF16 ? dispatch_tgemm<kBF16, kBF16, MODE>(p, grid, st, single_chunk)
                            : dispatch_tgemm<kBF16, kF32, MODE>(p, grid, st, single_chunk);
  }
  return y_dtype == kBF16 ? dispatch_tgemm<kF32, kBF16, MODE>(p, grid, st, single_chunk)
                          : dispatch_tgemm<kF32, kF32, MODE>(p, grid, st, single_chunk);
}

}  // namespace mb

using namespace mb;

extern "C" int64_t maple_fxa_frag_bytes(int64_t rows, int64_t k) {
  if (rows < 0 || k <= 0) return -1;
  return rows * (int64_t)fxa_iters((int)k) * 128 * 8;
}

extern "C" int64_t maple_fxa_meta_bytes(int64_t rows) { return rows < 0 ? -1 : rows * kMetaInts * 4; }

extern "C" int maple_fxa_encode(const void* x, int x_dtype, int64_t rows, int64_t k, int64_t x_row_stride,
                                const void* rms_w, int rms_dtype, float eps, void* frag, void* meta,
                                void* stream) {
  if (rows < 0 || k <= 0 || k > 8192 || k % 64 != 0) return kErrShape;
  if (rows == 0) return kOk;
  if (!x || !frag || !meta || rows > (1LL << 31) - 1) return kErrShape;
  if (x_dtype != kBF16 && x_dtype != kF32) return kErrDtype;
  if (rms_w && rms_dtype != kBF16 && rms_dtype != kF32) return kErrDtype;
  if ((reinterpret_cast<uintptr_t>(frag) | reinterpret_cast<uintptr_t>(meta)) & 15) return kErrAlign;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || ((x_row_stride * (x_dtype == kBF16 ? 2 : 4)) & 15))
    return kErrAlign;
  const int K = (int)k, iters = fxa_iters(K);
  const size_t smem = (size_t)iters * 256 * sizeof(uint2) + 2 * (size_t)K * sizeof(float);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
#define MB_ENC(XT, RT, RMS)                                                                          \
  do {                                                                                               \
    auto kern = fxa_encode_kernel<XT, RT, RMS>;                                                      \
    if (smem > 32 * 1024)                                                                            \
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);        \
    if (e == cudaSuccess)                                                                            \
      e = launch_k(kern, dim3((unsigned)rows), dim3(256), smem, st, x, x_row_stride, rms_w, K, eps,  \
                   static_cast<uint2*>(frag), static_cast<int*>(meta));                              \
  } while (0)
  if (x_dtype == kBF16) {
    if (!rms_w) MB_ENC(kBF16, kF32, false);
    else if (rms_dtype == kBF16) MB_ENC(kBF16, kBF16, true);
    else MB_ENC(kBF16, kF32, true);
  } else {
    if (!rms_w) MB_ENC(kF32, kF32, false);
    else if (rms_dtype == kBF16) MB_ENC(kF32, kBF16, true);
    else MB_ENC(kF32, kF32, true);
  }
#undef MB_ENC
  return e == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_ternary_gemm(const void* frag, const void* meta, int64_t rows, int64_t k, const uint32_t* codes,
                                  int64_t n, const void* alpha, int alpha_dtype, int use_rstd, void* y, int y_dtype,
                                  int64_t y_row_stride, int* err, void* stream) {
  if (rows < 0 || n < 0 || k <= 0 || k > 4096 || k % 64 != 0) return kErrShape;
  if (rows == 0 || n == 0) return kOk;
  if (!frag || !meta || !codes || !alpha || !y || !err) return kErrShape;
  if ((alpha_dtype != kBF16 && alpha_dtype != kF32) || (y_dtype != kBF16 && y_dtype != kF32)) return kErrDtype;
  if ((reinterpret_cast<uintptr_t>(codes) | reinterpret_cast<uintptr_t>(frag) | reinterpret_cast<uintptr_t>(meta)) &
      15)
    return kErrAlign;
  if (rows > (1LL << 31) - 1 || n > (1LL << 30)) return kErrShape;
  TGemmParams p = {};
  p.codes = codes; p.alpha = alpha; p.frag = static_cast<const uint2*>(frag); p.meta = static_cast<const int*>(meta);
  p.y = y; p.err = err; p.y_stride = y_row_stride;
  p.rows = (int)n; p.n_out = (int)n; p.K = (int)k; p.nwords = (int)(k / 16); p.iters = fxa_iters((int)k);
  p.R = (int)rows; p.use_rstd = use_rstd; p.in_div = 1;
  const int rc = p.iters <= 4 ? 16 : p.iters <= 8 ? 8 : 4;
  const int per = tile_rows(kGPlain, p.iters);
  const int tiles = (int)((n + per - 1) / per);
  const int chunks = (int)((rows + rc - 1) / rc);
  const int want_y = tiles >= 296 ? 1 : (296 + tiles - 1) / tiles;
  const int ctas_y = chunks < want_y ? chunks : want_y;
  p.chunks_per_cta = (chunks + ctas_y - 1) / ctas_y;
  const int gy = (chunks + p.chunks_per_cta - 1) / p.chunks_per_cta;
  if (gy > 65535) return kErrShape;
  cudaError_t e = dispatch_tgemm_types<kGPlain>(p, alpha_dtype, y_dtype, dim3((unsigned)tiles, (unsigned)gy),
                                                static_cast<cudaStream_t>(stream), p.chunks_per_cta <= 1);
  return e == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_moe_plan_range(const int32_t* ids, int64_t n_slots, int64_t n_experts, int64_t e_first,
                                    int64_t n_local, int32_t* offsets, uint32_t* list, void* stream) {
  if (n_slots < 0 || n_experts <= 0 || n_local <= 0 || n_local > 8192 || e_first < 0 ||
      e_first + n_local > n_experts)
    return kErrShape;
  if (!offsets || (n_slots > 0 && (!ids || !list)) || n_slots > (1LL << 31) - 1) return kErrShape;
  const size_t smem = 2 * (size_t)n_local * sizeof(int);
  auto kern = moe_plan_kernel;
  cudaError_t e = cudaSuccess;
  if (smem > 32 * 1024) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e == cudaSuccess)
    e = launch_k(kern, dim3(1), dim3(1024), smem, static_cast<cudaStream_t>(stream), ids, (int)n_slots,
                 (int)n_experts, (int)e_first, (int)n_local, offsets, list);
  return e == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_moe_plan(const int32_t* ids, int64_t n_slots, int64_t n_experts, int32_t* offsets,
                              uint32_t* list, void* stream) {
  return maple_moe_plan_range(ids, n_slots, n_experts, 0, n_experts, offsets, list, stream);
}

extern "C" int maple_ternary_grouped_gemm(const void* frag, const void* meta, int64_t in_rows, int64_t k,
                                          const uint32_t* codes, int64_t n_experts, int64_t code_rows,
                                          const void* alpha, int alpha_dtype, const int32_t* offsets,
                                          const uint32_t* list, int64_t n_slots, int64_t in_div, int swiglu,
                                          int plan_final, void* y, int y_dtype, int64_t y_row_stride, int* err,
                                          void* stream) {
  if (in_rows < 0 || n_slots < 0 || n_experts <= 0 || code_rows <= 0 || k <= 0 || k > 4096 || k % 64 != 0 ||
      in_div <= 0)
    return kErrShape;
  if (n_slots == 0) return kOk;
  if (swiglu && code_rows % 2 != 0) return kErrShape;
  if (!frag || !meta || !codes || !alpha || !offsets || !list || !y || !err) return kErrShape;
  if ((n_slots - 1) / in_div >= in_rows) return kErrBounds;
  if ((alpha_dtype != kBF16 && alpha_dtype != kF32) || (y_dtype != kBF16 && y_dtype != kF32)) return kErrDtype;
  if ((reinterpret_cast<uintptr_t>(codes) | reinterpret_cast<uintptr_t>(frag) | reinterpret_cast<uintptr_t>(meta)) &
      15)
    return kErrAlign;
  if (n_experts > 65535 || code_rows > (1LL << 30)) return kErrShape;
  TGemmParams p = {};
  p.codes = codes; p.alpha = alpha; p.frag = static_cast<const uint2*>(frag); p.meta = static_cast<const int*>(meta);
  p.y = y; p.err = err; p.y_stride = y_row_stride; p.offsets = offsets; p.list = list;
  p.rows = (int)code_rows; p.n_out = swiglu ? (int)(code_rows / 2) : (int)code_rows;
  p.K = (int)k; p.nwords = (int)(k / 16); p.iters = fxa_iters((int)k);
  p.expert_words = code_rows * (k / 16); p.alpha_estride = code_rows;
  p.in_div = (int)in_div; p.plan_final = plan_final; p.use_rstd = 0;
  const int per = tile_rows(swiglu ? kGSwiglu : kGPlain, p.iters);
  dim3 grid((unsigned)((p.n_out + per - 1) / per), (unsigned)n_experts);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // decode-sized routing (about one chunk of slots per expert): one buffer, two CTAs per SM
  const int rc = p.iters <= 4 ? 16 : p.iters <= 8 ? 8 : 4;
  const bool single = n_slots <= (int64_t)rc * n_experts;
  cudaError_t e = swiglu ? dispatch_tgemm_types<kGSwiglu>(p, alpha_dtype, y_dtype, grid, st, single)
                         : dispatch_tgemm_types<kGPlain>(p, alpha_dtype, y_dtype, grid, st, single);
  return e == cudaSuccess ? kOk : kErrCuda;
}
