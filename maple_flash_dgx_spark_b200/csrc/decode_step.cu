// Batch-1 decode of every decoder layer in ONE persistent launch.
//
// Reference: the per-token layer loop of model.py:848-886 (MapleForCausalLM.
// forward) through MapleDecoderLayer :490-506, MapleAttention's decode branch
// :368-414 and MapleSparseMoeBlock :465-474, i.e. per layer
//   ternary_gemv(RMSNorm -> QKV)   kernels/ternary_gemv.py:261-353
//   apply_qkv_decode               kernels/decode_attn.py:362-439
//   decode_gqa_attn                kernels/decode_attn.py:470-592
//   ternary_gemv(O)                kernels/ternary_gemv.py:261-353
//   add_rms_norm + router_topk     kernels/fused_norm.py:128-161, kernels/router.py:141-217
//   ternary_expert_swiglu          kernels/ternary_expert.py:403-468
//   ternary_expert_gemv(down) + moe_reduce_add
//                                  kernels/ternary_expert.py:125-234, kernels/fused_norm.py:164-202
//
// Why one launch.  At batch 1 a layer moves ~18 MB (2.7 us of HBM time on a
// B200) but as eight dependent launches it costs ~45 us: every launch pays
// its start, the wait for its predecessor and a first memory round trip.
// Here one CTA per SM (256 threads) stays resident for all layers; the six
// dependent phases of a layer are separated by a grid barrier (one atomic
// arrival per CTA on a count that grows through the launch, bounded wait), and the weights a
// phase needs are already on chip or in L2 when its barrier opens:
//   * the dense weights of layer l+1 (QKV, O, router, norms) are pulled into
//     L2 with bulk prefetches spread over all CTAs while layer l runs;
//   * the K/V rows of a CTA's attention split that were final before this
//     step are bulk-copied into shared memory while the QKV phase runs;
//   * the down-projection rows of the selected experts are prefetched into
//     L2 as soon as the top-k is known, while the SwiGLU phase runs.
//
// Phases of a layer (each CTA takes items blockIdx.x, +gridDim.x, ...):
//   1 QKV     RMSNorm folded GEMV, 16*WM rows per item
//   2 ATTN    per (kv head, split): q/k RMSNorm + RoPE of its heads, the new
//             K/V row stored by the split that holds it, scores, softmax,
//             P.V; the last split of a head merges (ticket)
//   3 O       GEMV, 16*WM rows per item
//   4 ROUTER  residual add + RMSNorm (CTA 0 stores both rows), logits of 4
//             experts per item
//   5 SWIGLU  every CTA: softmax + top-k of the logits; then the fused
//             up|gate GEMV + SwiGLU, 8*WM outputs of one slot per item
//   6 DOWN    16 rows per item, all slots: down GEMV, weighted combine,
//             residual add -> the layer output (next layer's input)
//
// Arithmetic is exactly that of the per-operator kernels (ternary_gemv.cu
// tgemv2_kernel, attn.cu qk_norm_rope_store_kernel / gqa_cluster_kernel /
// gqa_decode_kernel, moe.cu router_kernel / down_sum_kernel): the packed
// contractions are exact FXA integer sums, every other reduction keeps its
// order, and the rounding points are the same, so the output is bit for bit
// the output of the operator-by-operator path.
#include "bulk.cuh"
#include "fxa.cuh"
#include "launch.cuh"

#include "maple_b200.h"

namespace mb {

constexpr int kStepThreads = 256;
constexpr int kStepWarps = kStepThreads / 32;
constexpr int kStepNI = 8;         // K iterations per warp held in registers (down phase)
constexpr int kQkvTpw = 1, kOTpw = 1, kSwTpw = 2;  // 16-row tiles per warp in the split-K phases
constexpr int kStepMaxTopk = 8;
constexpr int kStepMaxG = 8;       // query heads per KV head
constexpr int kStepMaxE = 256;
constexpr int kRouterExpertsPerItem = 2;

struct StepParams {
  const maple_decode_layer* layers;
  int n_layers;
  uint16_t* x;                 // [H] bf16 residual stream: layer-0 input in, last layer output out
  const int64_t* seqlen;       // [1] position of the new token
  const int32_t* row_map;      // [1] cache row, or nullptr (row 0)
  const void* cos;             // [cs_len, R] rope tables
  const void* sin;
  int64_t cs_stride, cs_len;
  int cs_f32, alpha_f32, norm_f32, gate_f32;
  int H, Hq, Hkv, D, R, E, topk, I, T, Bc, P, NS;
  int64_t kc_sb, kc_sh;        // cache strides (elements), identical for K and V
  float eps, scale;
  int qkv_nks, qkv_ipw, o_nks, o_ipw, sw_nks, sw_ipw;  // split-K slices and iterations per slice
  // scratch
  unsigned long long* qkv_sum; // [(Hq + 2 Hkv) D] exact int64 row sums, zero between uses
  unsigned long long* o_sum;   // [H]
  unsigned long long* sw_sum;  // [topk, 2 I]
  uint16_t* ybuf;              // [topk, H] expert outputs of the down projection
  float* meta;                 // [0] QKV shift (int), [1] rstd, [2] O shift (int), [3] SwiGLU shift (int)
  uint16_t* attn;              // [Hq D]
  uint16_t* resid;             // [H]
  uint16_t* normed;            // [H]
  float* logits;               // [E]
  float* att_acc;              // [Hq, NS, D]
  float* att_ml;               // [Hq, NS, 2]
  unsigned* sync;              // [0] barrier arrivals, [1] CTAs retired, [2] trace switch
  int64_t* trace;              // [n_layers * 6 + 1][2][grid] barrier arrival / release times (ns), then checkpoints
  int64_t trace_bytes;
  unsigned* att_tickets;       // [Hkv]
  int* err;
  // dynamic shared memory carve-up (bytes)
  int off_frag, off_xs, off_xr, off_att, off_layers, off_in, off_post, off_qn, off_kn, off_cos, off_sin, off_gate;
  int frag_entries;
};

__device__ __forceinline__ float ldf(const void* p, int64_t i, int f32) {
  return f32 ? static_cast<const float*>(p)[i] : bf16_to_f32(static_cast<const uint16_t*>(p)[i]);
}

__device__ __forceinline__ float bf16_round(float v) { return bf16_to_f32(f32_to_bf16(v)); }

// mexp / msigmoid (common.cuh) as single shared copies for the persistent kernel.
__device__ __noinline__ float mexp_call(float x) { return mexp(x); }
__device__ __noinline__ float msigmoid_call(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, mexp(-x))); }

__device__ __forceinline__ unsigned ld_acquire_u32(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void prefetch_l2(const void* p) {
  asm volatile("prefetch.global.L2 [%0];\n" ::"l"(p));
}

// Every thread of the CTA prefetches 128-byte lines of this CTA's share of
// [base, base + bytes) into L2 (ordinary prefetch instructions: no TMA queue).
__device__ __forceinline__ void l2_prefetch_share(const void* base, int64_t bytes) {
  if (base == nullptr || bytes <= 0) return;
  const int64_t lines = (bytes + 127) / 128;
  const int64_t per = (lines + gridDim.x - 1) / gridDim.x;
  const int64_t l0 = per * blockIdx.x, l1 = min(l0 + per, lines);
  const char* b = static_cast<const char*>(base);
  for (int64_t l = l0 + threadIdx.x; l < l1; l += blockDim.x) prefetch_l2(b + l * 128);
}

__device__ __forceinline__ int64_t global_ns() {
  int64_t t;
  asm volatile("mov.u64 %0, %globaltimer;\n" : "=l"(t));
  return t;
}

// Grid barrier on a count that only grows within a launch: barrier k of the
// launch opens when the count reaches k * gridDim.x.  Thread 0 of each CTA
// arrives with a release reduction (no return trip) and polls with acquire
// loads (bounded).  The last CTA to leave the kernel -- every CTA leaves only
// after its last barrier -- resets the count for the next launch.  Returns
// false, with the timeout bit set in the error word, when a wait gave up.
__device__ __forceinline__ void red_release_add(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ bool grid_barrier(const StepParams& p, unsigned& epoch, int* s_ok, int64_t* trace) {
  __syncthreads();
  ++epoch;
  if (threadIdx.x == 0 && *s_ok) {
    if (trace != nullptr) trace[blockIdx.x] = global_ns();
    // the CTA's writes and reductions before the barrier are visible to every
    // CTA after it (the fence after bar.sync covers the whole CTA)
    __threadfence();
    red_release_add(&p.sync[0], 1u);
    const unsigned target = epoch * gridDim.x;
    bool done = false;
    for (int i = 0; i < kWaitSpins && !done; ++i) done = ld_acquire_u32(&p.sync[0]) >= target;
    if (!done) {
      atomicOr(p.err, kErrFlagTimeout);
      *s_ok = 0;
    }
    if (trace != nullptr) trace[gridDim.x + blockIdx.x] = global_ns();
  }
  __syncthreads();
  return *s_ok != 0;
}

// Called once by every CTA after its last barrier.
__device__ __forceinline__ void grid_barrier_retire(const StepParams& p) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned old = atomicAdd(&p.sync[1], 1u);
    if (old == gridDim.x - 1) {
      atomicExch(&p.sync[0], 0u);
      atomicExch(&p.sync[1], 0u);
    }
  }
}

struct StepShared {
  FxaBlock fb;
  int red[kStepWarps - 1][32][4];
  float s_val[16 * kStepWarps];
  int ids[kStepMaxTopk];
  float wts[kStepMaxTopk];
  float y[kStepMaxTopk][16];
  float part[4][128];
  float tk_p[kStepMaxE];
  float tk_sel_p[kStepMaxTopk];
  int tk_sel_i[kStepMaxTopk];
  int last, ok, tracing;
  long long* mk;  // clock64 checkpoints of the current (layer, phase), or nullptr
  uint64_t bar_kv, bar_st, bar_in, bar_rope;
};

// Checkpoint k (0..7) of the current phase: thread 0's clock64.
__device__ __forceinline__ void tmark(const StepShared& S, int k) {
  if (threadIdx.x == 0 && S.mk != nullptr) S.mk[k * gridDim.x + blockIdx.x] = clock64();
}

// Bulk copy of n bytes into shared memory on bar; returns n.  A misaligned
// request is not issued: its transaction bytes never arrive, the bounded
// wait gives up and the timeout bit reports it.
__device__ __forceinline__ unsigned stage_bytes(void* dst, const void* src, unsigned n, uint64_t* bar) {
  if (n == 0) return 0;
  if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | n) & 15) != 0) return 0;
  bulk_g2s(dst, src, n, bar);
  return n;
}

// Shared-memory regions (byte offsets into the dynamic shared memory).
struct StepSmem {
  uint2* frag;
  float* xs;          // encoded activation (fp32)
  float* xr;          // raw activation / residual sum (fp32)
  unsigned char* att; // attention tiles
  unsigned char* layers;  // all layer descriptors
  const void* in_norm;    // staged static vectors, source dtypes
  const void* post_norm;
  const void* q_norm;
  const void* k_norm;
  const void* cos;
  const void* sin;
  const void* gate;       // this CTA's router rows
};

// ------------------------------------------------- FXA prologue pieces ----
// Block-wide maximum of the threads' |x| bits -> FXA shift (one barrier; the
// caller has written its x values to shared memory before calling).
__device__ __forceinline__ int amax_exchange(StepShared& S, unsigned amax) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, m));
  if (lane == 0) S.fb.amax[warp] = amax;
  __syncthreads();
  unsigned a = 0;
#pragma unroll
  for (int w = 0; w < kStepWarps; ++w) a = max(a, S.fb.amax[w]);
  return fxa_shift(a);
}

// Staged activations live in shared memory at pidx(k) = k + k/32: the
// fragment builder's reads (8 codes at stride 4 from 16-code groups 64
// apart) and the stagers' 8-consecutive-value writes then meet at most two
// accesses per bank.
__device__ __forceinline__ int pidx(int k) { return k + (k >> 5); }
__host__ __device__ constexpr int padded_len(int n) { return n + (n >> 5) + 1; }

// fxa_build's fragment entries (2-bit layout) from xs stored at pidx(k).
// Each thread owns whole combos (8 codes x 4 digits); it writes the digits
// in an order rotated by m & 3 so a warp's 8-byte stores spread over the
// banks.  Only the digit half of an entry is written: the zero half (B
// columns 4-7) is cleared once per launch and never written again.
__device__ __noinline__ int4 build_frag2_call(const float* xs, int n, int s, bool bad, int iters, uint2* frag,
                                              int t_local, int nt);

__device__ __forceinline__ void build_frag2(const float* xs, int n, int s, bool bad, int iters, uint2* frag,
                                            int t_local, int nt, int (&raws)[4]) {
  const int4 r = build_frag2_call(xs, n, s, bad, iters, frag, t_local, nt);
  raws[0] += r.x; raws[1] += r.y; raws[2] += r.z; raws[3] += r.w;
}

// One shared copy of the builder: the persistent kernel runs it in four
// phases of every layer, and inlined copies crowd the instruction cache.
__device__ __noinline__ int4 build_frag2_call(const float* xs, int n, int s, bool bad, int iters, uint2* frag,
                                              int t_local, int nt) {
  int raws[4] = {0, 0, 0, 0};
  constexpr int off[8] = {0, 4, 8, 12, 1, 5, 9, 13};
  for (int c = t_local; c < iters * 32; c += nt) {
    const int it = c >> 5, r = c & 31;
    const int m = r >> 2, t = r & 3;
    const int k0 = it * 256 + 16 * (4 * t + (m >> 1)) + 2 * (m & 1);
    uint32_t u[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int k = k0 + off[e];
      const int X = (k < n && !bad) ? fxa_enc(xs[pidx(k)], s) : 0;
      u[e] = static_cast<uint32_t>(X + kFxaOffset);
    }
    uint2* dst = frag + (it * 8 + m) * 32 + t;
    const int rot = m & 3;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int j = (jj + rot) & 3;
      const uint32_t w0 = raw_digits(u[0], u[1], u[2], u[3], j);
      const uint32_t w1 = raw_digits(u[4], u[5], u[6], u[7], j);
      const int add = static_cast<int>(__dp4a(w0, 0x01010101u, __dp4a(w1, 0x01010101u, 0u)));
      raws[0] += j == 0 ? add : 0;
      raws[1] += j == 1 ? add : 0;
      raws[2] += j == 2 ? add : 0;
      raws[3] += j == 3 ? add : 0;
      dst[4 * j] = make_uint2(signed_digits(w0), signed_digits(w1));
    }
  }
  return make_int4(raws[0], raws[1], raws[2], raws[3]);
}

// Fragments of codes [0, iters*256) of xs (n values at pidx) by threads
// t_local of nt (a multiple of 32) and each warp's raw digit sums in
// S.fb.rawsum.
__device__ __forceinline__ void build_frags(StepShared& S, const float* xs, int n, int s, int iters, uint2* frag,
                                            int t_local, int nt) {
  int raws[4] = {0, 0, 0, 0};
  build_frag2(xs, n, s, s == kFxaNonFinite, iters, frag, t_local, nt, raws);
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) raws[j] += __shfl_xor_sync(0xffffffffu, raws[j], m);
    if (lane == 0) S.fb.rawsum[warp][j] = raws[j];
  }
}

// Balanced digit sums of the fragments built by all warps.
__device__ __forceinline__ void digit_totals(const StepShared& S, int iters, int (&tot)[4]) {
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    int t = 0;
#pragma unroll
    for (int w = 0; w < kStepWarps; ++w) t += S.fb.rawsum[w][j];
    tot[j] = t - 64 * iters * 256;
  }
}

// Load one row tile's packed words for this warp's K slice into registers.
template <int NI>
__device__ __forceinline__ void load_tile(const uint32_t* codes, int row_g, int row_h, bool ok_g, bool ok_h,
                                          int nwords, int it0, int my_iters, int t, uint4 (&wa)[NI],
                                          uint4 (&wb)[NI]) {
#pragma unroll
  for (int i = 0; i < NI; ++i) {
    wa[i] = make_uint4(0, 0, 0, 0);
    wb[i] = make_uint4(0, 0, 0, 0);
    if (i < my_iters) {
      const int word = (it0 + i) * 16 + 4 * t;
      if (word < nwords) {
        if (ok_g) wa[i] = ld_stream_u4(codes + (int64_t)row_g * nwords + word);
        if (ok_h) wb[i] = ld_stream_u4(codes + (int64_t)row_h * nwords + word);
      }
    }
  }
}

// ------------------------------------------------------- split-K GEMV ----
// The packed GEMVs of a layer run split-K over CTAs: an item is a block of
// rows and a K slice of `ipw` iterations (256 codes each).  A CTA reads the
// whole activation row (the FXA shift needs max|x| over all of K) but
// encodes only its slice, contracts its rows against it, and adds the exact
// partial sums S_slice = sum_j 128^j (acc_j - tot_j) to an int64 accumulator
// per row with atomics: the total is the exact integer contraction whatever
// the split, so the phase that reads a row finishes it exactly as the
// single-CTA kernels do (fxa_value(S, s) [* rstd] * alpha).  The producer's
// CTA 0 publishes the shift (and rstd) in p.meta.
struct SplitGeom {
  int tpw, nks, ipw;  // tiles of 16 rows per warp, K slices, iterations per slice
  __device__ int rows_per_item() const { return kStepWarps * tpw * 16; }
};

// Stage this thread's chunks of the activation (8 values per chunk): values
// of the slice [k0, k0 + n_slice) go to M.xs at pidx(k - k0); returns the
// thread's max |x|.  fetch(c, v) fills chunk c's 8 values.
template <typename Fetch>
__device__ __forceinline__ unsigned stage_slice(const StepSmem& M, int K, int k0, int n_slice, Fetch fetch) {
  unsigned amax = 0;
  for (int c = threadIdx.x; c < K / 8; c += kStepThreads) {
    float v[8];
    fetch(c, v);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int k = c * 8 + e;
      amax = max(amax, __float_as_uint(v[e]) & 0x7fffffffu);
      if (k >= k0 && k < k0 + n_slice) M.xs[pidx(k - k0)] = v[e];
    }
  }
  return amax;
}

// This warp's TPW row tiles (code rows row_of(j) + g, + 8) of the slice,
// loaded into registers (issued before the activation is staged).
template <int TPW, int NI>
struct SplitTiles {
  uint4 wa[TPW][NI], wb[TPW][NI];
};

template <int TPW, int NI, typename RowOf>
__device__ __forceinline__ void splitk_load(SplitTiles<TPW, NI>& T, const uint32_t* codes, int nwords, int it0,
                                            int n_it, RowOf row_of) {
  const int t = threadIdx.x & 3, g = (threadIdx.x & 31) >> 2;
#pragma unroll
  for (int j = 0; j < TPW; ++j) {
    const int r = row_of(j);
    load_tile<NI>(codes, r + g, r + g + 8, r >= 0, r >= 0, nwords, it0, n_it, t, T.wa[j], T.wb[j]);
  }
}

// Contract the loaded tiles against the slice's fragments and add the exact
// partial sums to sums[out_of(j) + g (+ 8)].
template <int TPW, int NI, typename RowOf, typename OutOf>
__device__ __forceinline__ void splitk_finish(const SplitTiles<TPW, NI>& T, const StepSmem& M, int n_it,
                                              const int (&tot)[4], RowOf row_of, OutOf out_of,
                                              unsigned long long* sums) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int j = 0; j < TPW; ++j) {
    int acc[4] = {0, 0, 0, 0};
    contract_tile2<NI>(T.wa[j], T.wb[j], n_it, M.frag, lane, acc);
    long long Sg, Sh;
    combine_digits(acc, tot, t, Sg, Sh);
    const int o = out_of(j);
    if (t == 0 && o >= 0 && row_of(j) >= 0) {
      atomicAdd(&sums[o + g], static_cast<unsigned long long>(Sg));
      atomicAdd(&sums[o + g + 8], static_cast<unsigned long long>(Sh));
    }
  }
}

// Exact value of a finished row: fxa_value(S, s) (NaN when the activation
// was not finite) -- the value tgemv2_kernel computes before its scalings.
__device__ __forceinline__ float fxa_row(long long S, int s) {
  return s == kFxaNonFinite ? __int_as_float(0x7fc00000) : fxa_value(S, s);
}

__device__ __forceinline__ void zero_share(unsigned long long* p, int64_t n) {
  for (int64_t i = (int64_t)blockIdx.x * kStepThreads + threadIdx.x; i < n; i += (int64_t)gridDim.x * kStepThreads)
    p[i] = 0ull;
}

// -------------------------------------------------------------- QKV ----
// x = this layer's input: the previous layer's down outputs combined in slot
// order with the residual, x[k] = bf16(fmaf-chain_s(w_s, y_s[k]) +
// resid[k]) (down_sum_kernel MODE 0 / moe_reduce_add), or the embedded token
// for layer 0.  Every CTA forms x (CTA 0 stores it); then the RMSNorm-folded
// QKV GEMV, split-K, into p.qkv_sum; CTA 0 publishes the shift and rstd.
template <int TPW>
__device__ __forceinline__ void qkv_phase(StepShared& S, const StepSmem& M, const StepParams& p,
                                          const maple_decode_layer& w, bool first_layer) {
  const int tid = threadIdx.x, warp = tid >> 5;
  const int K = p.H, N = (p.Hq + 2 * p.Hkv) * p.D;
  const SplitGeom G{TPW, p.qkv_nks, p.qkv_ipw};
  const int nwords = K / 16, iters_total = (nwords + 15) / 16;
  const int n_rb = (N + G.rows_per_item() - 1) / G.rows_per_item();
  const int n_items = n_rb * G.nks;
  const int item = blockIdx.x;
  const bool has_item = item < n_items;
  const int rb = item / G.nks, ks = item % G.nks;
  const int it0 = ks * G.ipw, n_it = max(0, min(G.ipw, iters_total - it0));
  const int k0 = it0 * 256, n_slice = min(K, (it0 + n_it) * 256) - k0;
  if (!has_item && blockIdx.x != 0) return;
  const int base = rb * G.rows_per_item() + warp * TPW * 16;
  auto row_of = [&](int j) { const int r = base + 16 * j; return (has_item && r < N) ? r : -1; };
  SplitTiles<TPW, 4> T;
  splitk_load(T, w.qkv_codes, nwords, it0, n_it, row_of);
  // x, x_hat = x * w_in; raw x to xr for the RMS partials
  auto fetch = [&](int c, float (&v)[8]) {
    float xv[8];
    if (first_layer) {
      widen_u4<kBF16>(ld_u4(reinterpret_cast<const char*>(p.x) + (size_t)c * 16), xv);
    } else {
      uint4 yr[kStepMaxTopk];
#pragma unroll
      for (int s = 0; s < kStepMaxTopk; ++s)
        if (s < p.topk) yr[s] = ld_u4(reinterpret_cast<const char*>(p.ybuf + (int64_t)s * p.H) + (size_t)c * 16);
      float rv[8];
      widen_u4<kBF16>(ld_u4(reinterpret_cast<const char*>(p.resid) + (size_t)c * 16), rv);
      float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int s = 0; s < kStepMaxTopk; ++s) {
        if (s < p.topk) {
          float yv[8];
          widen_u4<kBF16>(yr[s], yv);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] = __fmaf_rn(S.wts[s], yv[e], acc[e]);
        }
      }
      uint32_t q[4];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const uint16_t b = f32_to_bf16(__fadd_rn(acc[e], rv[e]));
        xv[e] = bf16_to_f32(b);
        if (e & 1) q[e >> 1] |= static_cast<uint32_t>(b) << 16;
        else q[e >> 1] = b;
      }
      if (blockIdx.x == 0)
        *reinterpret_cast<uint4*>(reinterpret_cast<char*>(p.x) + (size_t)c * 16) = make_uint4(q[0], q[1], q[2], q[3]);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int k = c * 8 + e;
      M.xr[k] = xv[e];
      v[e] = __fmul_rn(xv[e], ldf(M.in_norm, k, p.norm_f32));
    }
  };
  const unsigned amax = stage_slice(M, K, k0, n_slice, fetch);
  if (!has_item) return;  // CTA 0 without an item has stored x
  const int s = amax_exchange(S, amax);
  if (tid < 128) {
    float ss = 0.0f;
    for (int k = tid; k < K; k += 128) ss = __fmaf_rn(M.xr[k], M.xr[k], ss);
    S.part[0][tid] = ss;
  }
  build_frags(S, M.xs, n_slice, s, n_it, M.frag, tid, kStepThreads);
  __syncthreads();
  int tot[4];
  digit_totals(S, n_it, tot);
  if (blockIdx.x == 0 && warp == 0) {
    const float rstd = rstd_of(r128_smem_finish(S.part[0], tid & 31), K, p.eps);
    if (tid == 0) {
      reinterpret_cast<int*>(p.meta)[0] = s;
      p.meta[1] = rstd;
    }
  }
  tmark(S, 2);
  splitk_finish(T, M, n_it, tot, row_of, [&](int j) { return base + 16 * j; }, p.qkv_sum);
}

// ---------------------------------------------------------------- O ----
// The attention output (bf16 [Hq D]) against the O rows, split-K into
// p.o_sum; CTA 0 publishes the shift.  Also clears the QKV accumulators the
// attention phase has finished reading.
template <int TPW>
__device__ __forceinline__ void o_phase(StepShared& S, const StepSmem& M, const StepParams& p,
                                        const maple_decode_layer& w) {
  const int tid = threadIdx.x, warp = tid >> 5;
  zero_share(p.qkv_sum, (int64_t)(p.Hq + 2 * p.Hkv) * p.D);
  const int K = p.Hq * p.D, N = p.H;
  const SplitGeom G{TPW, p.o_nks, p.o_ipw};
  const int nwords = K / 16, iters_total = (nwords + 15) / 16;
  const int n_rb = (N + G.rows_per_item() - 1) / G.rows_per_item();
  const int item = blockIdx.x;
  if (item >= n_rb * G.nks) return;
  const int rb = item / G.nks, ks = item % G.nks;
  const int it0 = ks * G.ipw, n_it = max(0, min(G.ipw, iters_total - it0));
  const int k0 = it0 * 256, n_slice = min(K, (it0 + n_it) * 256) - k0;
  const int base = rb * G.rows_per_item() + warp * TPW * 16;
  auto row_of = [&](int j) { const int r = base + 16 * j; return r < N ? r : -1; };
  SplitTiles<TPW, 4> T;
  splitk_load(T, w.o_codes, nwords, it0, n_it, row_of);
  const unsigned amax = stage_slice(M, K, k0, n_slice, [&](int c, float (&v)[8]) {
    widen_u4<kBF16>(ld_u4(reinterpret_cast<const char*>(p.attn) + (size_t)c * 16), v);
  });
  const int s = amax_exchange(S, amax);
  build_frags(S, M.xs, n_slice, s, n_it, M.frag, tid, kStepThreads);
  __syncthreads();
  int tot[4];
  digit_totals(S, n_it, tot);
  if (blockIdx.x == 0 && tid == 0) reinterpret_cast<int*>(p.meta)[2] = s;
  tmark(S, 2);
  splitk_finish(T, M, n_it, tot, row_of, [&](int j) { return base + 16 * j; }, p.o_sum);
}

// ----------------------------------------------------------- router ----
// o[k] = bf16(fxa_value(S_o[k], s_o) * alpha_o[k]); v = x + o; CTA 0 stores
// resid = bf16(v) and normed = bf16(v * rstd * w); logits[e] = R128
// dot(bf16(normed), gate[e]) (router_kernel<FUSE>).  One item per CTA: 2
// experts; warp (e_local = w / 4, q = w % 4) owns R128 partials 32q + lane.
// The norm weights and this CTA's gate rows were staged before the barrier.
__device__ __forceinline__ void router_phase(StepShared& S, const StepSmem& M, const StepParams& p,
                                             const maple_decode_layer& w) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = p.H;
  const int n_items = (p.E + kRouterExpertsPerItem - 1) / kRouterExpertsPerItem;
  if ((int)blockIdx.x >= n_items) return;
  float* vs = M.xr;  // x + o, fp32
  float* xs = M.xs;  // bf16(normed), fp32 at pidx
  const int s_o = __ldcg(reinterpret_cast<const int*>(p.meta) + 2);
  for (int c = tid; c < K / 8; c += kStepThreads) {
    float a[8];
    widen_u4<kBF16>(ld_u4(reinterpret_cast<const char*>(p.x) + (size_t)c * 16), a);
    long long so[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) so[e] = static_cast<long long>(__ldcg(p.o_sum + c * 8 + e));
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int k = c * 8 + e;
      const float ov = bf16_round(__fmul_rn(fxa_row(so[e], s_o), ldf(w.o_alpha, k, p.alpha_f32)));
      vs[k] = __fadd_rn(a[e], ov);
    }
  }
  __syncthreads();
  tmark(S, 1);
  if (tid < 128) {
    float ss = 0.0f;
    for (int k = tid; k < K; k += 128) ss = __fmaf_rn(vs[k], vs[k], ss);
    S.part[0][tid] = ss;
  }
  __syncthreads();
  const float rstd = rstd_of(r128_smem_finish(S.part[0], lane), K, p.eps);
  tmark(S, 2);
  for (int c = tid; c < K / 8; c += kStepThreads) {
    uint32_t rq[4], nq[4];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int k = c * 8 + e;
      const float v = vs[k];
      const float nv = __fmul_rn(__fmul_rn(v, rstd), ldf(M.post_norm, k, p.norm_f32));
      const uint16_t nb = f32_to_bf16(nv);
      xs[pidx(k)] = bf16_to_f32(nb);
      const uint16_t vb = f32_to_bf16(v);
      if (e & 1) {
        rq[e >> 1] |= static_cast<uint32_t>(vb) << 16;
        nq[e >> 1] |= static_cast<uint32_t>(nb) << 16;
      } else {
        rq[e >> 1] = vb;
        nq[e >> 1] = nb;
      }
    }
    if (blockIdx.x == 0) {
      *reinterpret_cast<uint4*>(reinterpret_cast<char*>(p.resid) + (size_t)c * 16) = make_uint4(rq[0], rq[1], rq[2], rq[3]);
      *reinterpret_cast<uint4*>(reinterpret_cast<char*>(p.normed) + (size_t)c * 16) = make_uint4(nq[0], nq[1], nq[2], nq[3]);
    }
  }
  __syncthreads();
  tmark(S, 3);
  const int el = warp / 4, q = warp % 4;
  const int e = blockIdx.x * kRouterExpertsPerItem + el;
  if (e < p.E) {
    const int j = 32 * q + lane;
    float pj = 0.0f;
#pragma unroll 4
    for (int k = j; k < K; k += 128) pj = __fmaf_rn(xs[pidx(k)], ldf(M.gate, (int64_t)el * K + k, p.gate_f32), pj);
    S.part[el][j] = pj;
  }
  __syncthreads();
  if (q == 0 && e < p.E) {
    const float logit = r128_smem_finish(S.part[el], lane);
    if (lane == 0) p.logits[e] = logit;
  }
  tmark(S, 4);
}

// ------------------------------------------------------------ SwiGLU ----
// Every CTA: softmax + top-k + renorm of the E logits (router_kernel's
// last-CTA part; the order of its repeated argmax, largest first and ties to
// the lowest index, is each expert's rank, one thread per expert).  Then the
// up|gate rows of the selected experts against bf16(normed), split-K into
// p.sw_sum[slot][2I]; CTA 0 publishes the shift.  The down rows of this CTA's
// down item go to L2 once the experts are known; the O accumulators are
// cleared.
template <int TPW>
__device__ __forceinline__ void swiglu_phase(StepShared& S, const StepSmem& M, const StepParams& p,
                                             const maple_decode_layer& w) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = p.H, I = p.I, E = p.E;
  const float ninf = __int_as_float(0xff800000);
  zero_share(p.o_sum, p.H);
  // 1. the logits (warp 0) -> probabilities
  if (warp == 0) {
    float v[kStepMaxE / 32];
    float m = ninf;
#pragma unroll
    for (int i = 0; i < kStepMaxE / 32; ++i) {
      const int ee = lane + 32 * i;
      v[i] = ee < E ? __ldcg(&p.logits[ee]) : ninf;
      m = fmaxf(m, v[i]);
    }
    m = warp_max(m);
    float q0 = 0.f, q1 = 0.f, q2 = 0.f, q3 = 0.f;
#pragma unroll
    for (int i = 0; i < kStepMaxE / 32; ++i) {
      const int ee = lane + 32 * i;
      v[i] = ee < E ? mexp_call(__fsub_rn(v[i], m)) : 0.0f;
      const int j = (i & 3);
      if (j == 0) q0 = __fadd_rn(q0, v[i]);
      if (j == 1) q1 = __fadd_rn(q1, v[i]);
      if (j == 2) q2 = __fadd_rn(q2, v[i]);
      if (j == 3) q3 = __fadd_rn(q3, v[i]);
    }
    const float sum = r128_lane_finish(q0, q1, q2, q3);
#pragma unroll
    for (int i = 0; i < kStepMaxE / 32; ++i) {
      const int ee = lane + 32 * i;
      if (ee < E) S.tk_p[ee] = __fdiv_rn(v[i], sum);
    }
    if (lane < kStepMaxTopk) {
      S.tk_sel_p[lane] = ninf;
      S.tk_sel_i[lane] = 0x7fffffff;
    }
  }
  // 2. this CTA's slice of bf16(normed) while warp 0 works
  const SplitGeom G{TPW, p.sw_nks, p.sw_ipw};
  const int nwords = K / 16, iters_total = (nwords + 15) / 16;
  const int rpi = G.rows_per_item();       // code rows per item: rpi/2 up rows + rpi/2 gate rows
  const int outs = rpi / 2;
  const int n_ob = (I + outs - 1) / outs;
  const int n_items = p.topk * n_ob * G.nks;
  const int item = blockIdx.x;
  const bool has_item = item < n_items;
  const int slot = item / (n_ob * G.nks), ob = (item / G.nks) % n_ob, ks = item % G.nks;
  const int it0 = ks * G.ipw, n_it = max(0, min(G.ipw, iters_total - it0));
  const int k0 = it0 * 256, n_slice = min(K, (it0 + n_it) * 256) - k0;
  unsigned amax = 0;
  if (has_item)
    amax = stage_slice(M, K, k0, n_slice, [&](int c, float (&v)[8]) {
      widen_u4<kBF16>(ld_u4(reinterpret_cast<const char*>(p.normed) + (size_t)c * 16), v);
    });
  const int s = amax_exchange(S, amax);  // also publishes the probabilities
  // 3. rank of expert tid (NaN is never picked by the argmax rounds)
  if (tid < E) {
    const float pi = S.tk_p[tid];
    if (pi == pi) {
      int rank = 0;
#pragma unroll 8
      for (int j = 0; j < E; ++j) {
        const float pj = S.tk_p[j];
        rank += (pj > pi || (pj == pi && j < tid)) ? 1 : 0;
      }
      if (rank < p.topk) {
        S.tk_sel_p[rank] = pi;
        S.tk_sel_i[rank] = tid;
      }
    }
  }
  __syncthreads();
  // 4. the selected expert's rows of this item, then the fragments while they arrive
  int e_item = has_item ? S.tk_sel_i[slot] : 0;
  if (e_item < 0 || e_item >= E) e_item = 0;  // a bad id finishes as NaN in the down phase
  const uint32_t* codes = w.ug_codes + (int64_t)e_item * 2 * I * nwords;
  const int lbase = warp * TPW * 16;
  auto code_row = [&](int j) {
    const int lr = lbase + 16 * j;
    const int r = lr < outs ? ob * outs + lr : I + ob * outs + (lr - outs);
    const int lim = lr < outs ? I : 2 * I;
    return (has_item && r < lim) ? r : -1;
  };
  SplitTiles<TPW, 4> T;
  splitk_load(T, codes, nwords, it0, n_it, code_row);
  if (has_item) build_frags(S, M.xs, n_slice, s, n_it, M.frag, tid, kStepThreads);
  float total = 0.0f;
  for (int rr = 0; rr < p.topk; ++rr) total = __fadd_rn(total, S.tk_sel_p[rr]);
  const float inv = __fdiv_rn(1.0f, __fadd_rn(total, 1e-20f));
  if (tid < p.topk) {
    S.ids[tid] = S.tk_sel_i[tid];
    S.wts[tid] = __fmul_rn(S.tk_sel_p[tid], inv);
  }
  if (blockIdx.x == 0 && tid == 0) reinterpret_cast<int*>(p.meta)[3] = s;
  tmark(S, 1);
  // 4. this CTA's down rows into L2: down item = (slot, 128 rows)
  {
    const int n_db = (p.H + 127) / 128;
    const int ditem = blockIdx.x;
    if (ditem < p.topk * n_db) {
      const int dslot = ditem / n_db, r0 = (ditem % n_db) * 128;
      const int e = S.tk_sel_i[dslot];
      if (e >= 0 && e < E) {
        const int64_t row_bytes = (int64_t)I / 4;
        const int64_t bytes = min(128, p.H - r0) * row_bytes;
        const char* base = reinterpret_cast<const char*>(w.dn_codes) + ((int64_t)e * p.H + r0) * row_bytes;
        for (int64_t off = (int64_t)tid * 128; off < bytes; off += (int64_t)kStepThreads * 128) prefetch_l2(base + off);
      }
    }
  }
  __syncthreads();
  if (!has_item) return;
  int tot[4];
  digit_totals(S, n_it, tot);
  tmark(S, 2);
  // warp's local rows [warp * TPW * 16, +TPW*16): the first half of the item's rows are up rows, the rest gate rows
  splitk_finish(T, M, n_it, tot, code_row, [&](int j) { return slot * 2 * I + code_row(j); }, p.sw_sum);
}

// -------------------------------------------------------------- down ----
// Item (slot, 128 rows): h = bf16(clamp(u, +-7) * min(g, 7) * sigmoid(min(g,
// 7))) with u, g the finished up / gate rows of the slot's expert
// (tgemv2_kernel<kSwiglu>'s epilogue), encoded whole; the item's down rows
// against it; y[slot][row] = bf16(fxa_value(S, s_h) * alpha) (the expert
// output the combine reads in the next layer's QKV phase).
__device__ __forceinline__ void down_phase(StepShared& S, const StepSmem& M, const StepParams& p,
                                           const maple_decode_layer& w) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const int K = p.I, N = p.H;
  const int nwords = K / 16, iters_total = (nwords + 15) / 16;
  const int n_db = (N + 127) / 128;
  const int item = blockIdx.x;
  if (item >= p.topk * n_db) return;
  const int slot = item / n_db, r0 = (item % n_db) * 128;
  int e = S.ids[slot];
  const bool bad = (e < 0 || e >= p.E);
  if (bad) e = 0;
  const int row_g = r0 + warp * 16 + g, row_h = row_g + 8;
  uint4 wa[kStepNI], wb[kStepNI];
  load_tile<kStepNI>(w.dn_codes + (int64_t)e * N * nwords, row_g, row_h, row_g < N, row_h < N, nwords, 0,
                     iters_total, t, wa, wb);
  const void* al = static_cast<const char*>(w.dn_alpha) + (int64_t)e * N * (p.alpha_f32 ? 4 : 2);
  const float ag = row_g < N ? ldf(al, row_g, p.alpha_f32) : 0.f;
  const float ah = row_h < N ? ldf(al, row_h, p.alpha_f32) : 0.f;
  tmark(S, 1);
  const int s_sw = __ldcg(reinterpret_cast<const int*>(p.meta) + 3);
  const unsigned long long* su = p.sw_sum + (int64_t)slot * 2 * K;
  const void* ua = static_cast<const char*>(w.ug_alpha) + (int64_t)e * 2 * K * (p.alpha_f32 ? 4 : 2);
  const unsigned amax = stage_slice(M, K, 0, K, [&](int c, float (&v)[8]) {
    long long Su[8], Sg[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      Su[q] = static_cast<long long>(__ldcg(su + c * 8 + q));
      Sg[q] = static_cast<long long>(__ldcg(su + K + c * 8 + q));
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int k = c * 8 + q;
      const float nanv = __int_as_float(0x7fc00000);
      float up = bad ? nanv : __fmul_rn(fxa_row(Su[q], s_sw), ldf(ua, k, p.alpha_f32));
      float gate = bad ? nanv : __fmul_rn(fxa_row(Sg[q], s_sw), ldf(ua, K + k, p.alpha_f32));
      up = fminf(fmaxf(up, -7.0f), 7.0f);
      gate = fminf(gate, 7.0f);
      v[q] = bf16_round(__fmul_rn(__fmul_rn(up, gate), msigmoid_call(gate)));
    }
  });
  const int sh = amax_exchange(S, amax);
  build_frags(S, M.xs, K, sh, iters_total, M.frag, tid, kStepThreads);
  __syncthreads();
  int tot[4];
  digit_totals(S, iters_total, tot);
  tmark(S, 2);
  int acc[4] = {0, 0, 0, 0};
  contract_tile2<kStepNI>(wa, wb, iters_total, M.frag, lane, acc);
  long long Sg, Sh;
  combine_digits(acc, tot, t, Sg, Sh);
  if (t == 0) {
    const bool nan_out = bad || sh == kFxaNonFinite;
    const float nanv = __int_as_float(0x7fc00000);
    uint16_t* y = p.ybuf + (int64_t)slot * N;
    if (row_g < N) y[row_g] = f32_to_bf16(__fmul_rn(nan_out ? nanv : fxa_value(Sg, sh), ag));
    if (row_h < N) y[row_h] = f32_to_bf16(__fmul_rn(nan_out ? nanv : fxa_value(Sh, sh), ah));
  }
  tmark(S, 3);
}

// Final combine after the last layer: x = bf16(fmaf-chain_s(w_s, y_s) +
// resid) into p.x (CTA 0), and the SwiGLU accumulators cleared.
__device__ __forceinline__ void final_phase(StepShared& S, const StepParams& p) {
  zero_share(p.sw_sum, (int64_t)p.topk * 2 * p.I);
  if (blockIdx.x != 0) return;
  for (int c = threadIdx.x; c < p.H / 8; c += kStepThreads) {
    float rv[8], acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    widen_u4<kBF16>(ld_u4(reinterpret_cast<const char*>(p.resid) + (size_t)c * 16), rv);
    for (int s = 0; s < p.topk; ++s) {
      float yv[8];
      widen_u4<kBF16>(ld_u4(reinterpret_cast<const char*>(p.ybuf + (int64_t)s * p.H) + (size_t)c * 16), yv);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = __fmaf_rn(S.wts[s], yv[e], acc[e]);
    }
    uint32_t q[4];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint16_t b = f32_to_bf16(__fadd_rn(acc[e], rv[e]));
      if (e & 1) q[e >> 1] |= static_cast<uint32_t>(b) << 16;
      else q[e >> 1] = b;
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<char*>(p.x) + (size_t)c * 16) = make_uint4(q[0], q[1], q[2], q[3]);
  }
}

// ----------------------------------------------------------- attention ----
struct AttnGeom {
  int64_t pos;
  int kv_len, start, ns, cb;
  bool cb_ok;
};

__device__ __forceinline__ AttnGeom attn_geom(const StepParams& p, int window) {
  AttnGeom a;
  a.pos = p.seqlen[0];
  a.kv_len = (int)min(a.pos + 1, (int64_t)p.T);
  a.start = window > 0 ? max(0, a.kv_len - window) : 0;
  a.ns = a.kv_len > a.start ? (a.kv_len - a.start + p.P - 1) / p.P : 0;
  a.cb = p.row_map != nullptr ? p.row_map[0] : 0;
  a.cb_ok = a.cb >= 0 && a.cb < p.Bc;
  if (!a.cb_ok) a.cb = 0;
  return a;
}

// Bulk-copy (one thread) the K/V rows of item `item` that were final before
// this step, positions [t0, min(t0 + n, pos)); returns the bytes per tensor.
template <int D>
__device__ __forceinline__ int attn_issue(const StepParams& p, const AttnGeom& a, const maple_decode_layer& w,
                                          int item, unsigned char* att, uint64_t* bar) {
  const int h = item / a.ns, s = item % a.ns;
  const int t0 = a.start + s * p.P;
  const int n = min(p.P, a.kv_len - t0);
  const int n_pre = max(0, (int)min((int64_t)n, a.pos - t0));
  if (n_pre <= 0) return 0;
  const unsigned bytes = (unsigned)(n_pre * D * 2);
  const char* ksrc = static_cast<const char*>(w.k_cache) + (a.cb * p.kc_sb + h * p.kc_sh + (int64_t)t0 * D) * 2;
  const char* vsrc = static_cast<const char*>(w.v_cache) + (a.cb * p.kc_sb + h * p.kc_sh + (int64_t)t0 * D) * 2;
  fence_proxy_async_smem();
  mbar_expect_tx(bar, 2 * bytes);
  stage_bytes(att, ksrc, bytes, bar);
  stage_bytes(att + (size_t)p.P * D * 2, vsrc, bytes, bar);
  return (int)bytes;
}

// RMSNorm (R128 over D) * w, RoPE, bf16 of one head by one warp
// (qk_norm_rope_store_kernel); dst (D floats, shared) ends with the bf16
// values as fp32.
template <int D>
__device__ __noinline__ void norm_rope_head_call(uint2 packed, const void* nw, int norm_f32, const void* cs,
                                                 const void* sn, int cs_f32, int use_rope, int R, float eps,
                                                 float* dst);

template <int D>
__device__ __forceinline__ void norm_rope_head(const uint16_t (&raw)[D / 32], const void* nw, int norm_f32,
                                               const void* cs, const void* sn, int cs_f32, int use_rope, int R,
                                               float eps, float* dst) {
  constexpr int U = D / 32;
  uint32_t w4[2] = {0u, 0u};
#pragma unroll
  for (int u = 0; u < U; ++u) w4[u >> 1] |= static_cast<uint32_t>(raw[u]) << (16 * (u & 1));
  norm_rope_head_call<D>(make_uint2(w4[0], w4[1]), nw, norm_f32, cs, sn, cs_f32, use_rope, R, eps, dst);
}

// One shared copy (q heads and the new K row of every layer).
template <int D>
__device__ __noinline__ void norm_rope_head_call(uint2 packed, const void* nw, int norm_f32, const void* cs,
                                                 const void* sn, int cs_f32, int use_rope, int R, float eps,
                                                 float* dst) {
  constexpr int U = D / 32;
  uint16_t raw[U];
  const uint32_t w4[2] = {packed.x, packed.y};
#pragma unroll
  for (int u = 0; u < U; ++u) raw[u] = static_cast<uint16_t>(w4[u >> 1] >> (16 * (u & 1)));
  const int lane = threadIdx.x & 31;
  const int half = R / 2;
  float xv[U];
  float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int u = 0; u < U; ++u) {
    xv[u] = bf16_to_f32(raw[u]);
    part[u & 3] = __fmaf_rn(xv[u], xv[u], part[u & 3]);
  }
  const float rstd = rstd_of(r128_lane_finish(part[0], part[1], part[2], part[3]), D, eps);
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int d = lane + 32 * u;
    dst[d] = __fmul_rn(__fmul_rn(xv[u], rstd), ldf(nw, d, norm_f32));
  }
  __syncwarp();
  float o[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int d = lane + 32 * u;
    float v = dst[d];
    if (use_rope && d < R) {
      const float c = ldf(cs, d, cs_f32), s = ldf(sn, d, cs_f32);
      if (d < half) v = __fadd_rn(__fmul_rn(dst[d], c), __fmul_rn(-dst[d + half], s));
      else v = __fadd_rn(__fmul_rn(dst[d], c), __fmul_rn(dst[d - half], s));
    }
    o[u] = bf16_round(v);
  }
  __syncwarp();
#pragma unroll
  for (int u = 0; u < U; ++u) dst[lane + 32 * u] = o[u];
}

// Per (kv head h, split s): RMSNorm + RoPE of the group's q heads (and of the
// new K row, which the split holding position pos stores together with the
// new V row), scores, split softmax, P.V; the last split of a head merges
// (qk_norm_rope_store_kernel + gqa_decode_kernel arithmetic).  Norm weights
// and the RoPE row were staged in shared memory before the barrier; the first
// item's final K/V rows were bulk-copied during the QKV phase.
template <int D>
__device__ __forceinline__ void attention_phase(StepShared& S, const StepSmem& M, const StepParams& p,
                                                const maple_decode_layer& w, const AttnGeom& a, unsigned& ph_kv) {
  constexpr int U = D / 32;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int P = p.P, G = p.Hq / p.Hkv;
  unsigned char* ktile = M.att;
  unsigned char* vtile = M.att + (size_t)P * D * 2;
  const uint16_t* kt16 = reinterpret_cast<const uint16_t*>(ktile);
  float* scores = reinterpret_cast<float*>(M.att + 2 * (size_t)P * D * 2);  // [8][P]
  float* pb = scores + 8 * P;                                                 // [8][P]
  float* qs = pb + 8 * P;                                                     // [8][D]
  float* ks = qs + 8 * D;                                                     // [D]
  const int n_items = p.Hkv * a.ns;
  const float ninf = __int_as_float(0xff800000);
  const int use_rope = (int)w.use_rope;
  const bool store_ok = a.pos >= 0 && a.pos < p.T && a.cb_ok;
  const int s_qkv = __ldcg(reinterpret_cast<const int*>(p.meta));
  const float rstd_qkv = __ldcg(p.meta + 1);
  bool first = true;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int h = item / a.ns, s = item % a.ns;
    const int t0 = a.start + s * P;
    const int n = min(P, a.kv_len - t0);
    const int n_pre = max(0, (int)min((int64_t)n, a.pos - t0));
    if (!first && tid == 0) attn_issue<D>(p, a, w, item, M.att, &S.bar_kv);
    first = false;
    const bool has_new = a.pos >= t0 && a.pos < (int64_t)t0 + n && store_ok;
    // q head of warp g < G, the new K (warp 0) and V (warp 1) rows, finished
    // from the QKV sums as ternary_gemv does: bf16((fxa(S) * rstd) * alpha)
    uint16_t rq[U], rk[U], rv[U];
    {
      long long sq[U], sk[U], sv[U];
      float aq[U], ak[U], av[U];
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int rq_ = (h * G + warp) * D + lane + 32 * u;
        const int rk_ = (p.Hq + h) * D + lane + 32 * u;
        const int rv_ = (p.Hq + p.Hkv + h) * D + lane + 32 * u;
        const bool wq = warp < G, wk = warp == 0 && has_new, wv = warp == 1 && has_new;
        sq[u] = wq ? static_cast<long long>(__ldcg(p.qkv_sum + rq_)) : 0;
        sk[u] = wk ? static_cast<long long>(__ldcg(p.qkv_sum + rk_)) : 0;
        sv[u] = wv ? static_cast<long long>(__ldcg(p.qkv_sum + rv_)) : 0;
        aq[u] = wq ? ldf(w.qkv_alpha, rq_, p.alpha_f32) : 0.f;
        ak[u] = wk ? ldf(w.qkv_alpha, rk_, p.alpha_f32) : 0.f;
        av[u] = wv ? ldf(w.qkv_alpha, rv_, p.alpha_f32) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < U; ++u) {
        rq[u] = f32_to_bf16(__fmul_rn(__fmul_rn(fxa_row(sq[u], s_qkv), rstd_qkv), aq[u]));
        rk[u] = f32_to_bf16(__fmul_rn(__fmul_rn(fxa_row(sk[u], s_qkv), rstd_qkv), ak[u]));
        rv[u] = f32_to_bf16(__fmul_rn(__fmul_rn(fxa_row(sv[u], s_qkv), rstd_qkv), av[u]));
      }
    }
    if (warp < G) {
      norm_rope_head<D>(rq, M.q_norm, p.norm_f32, M.cos, M.sin, p.cs_f32, use_rope, p.R, p.eps, qs + warp * D);
    } else {
#pragma unroll
      for (int u = 0; u < U; ++u) qs[warp * D + lane + 32 * u] = 0.0f;
    }
    if (warp == 0 && has_new) {
      norm_rope_head<D>(rk, M.k_norm, p.norm_f32, M.cos, M.sin, p.cs_f32, use_rope, p.R, p.eps, ks);
      uint16_t* kdst = static_cast<uint16_t*>(w.k_cache) + (a.cb * p.kc_sb + h * p.kc_sh + a.pos * D);
      uint16_t* kt = reinterpret_cast<uint16_t*>(ktile) + (size_t)(a.pos - t0) * D;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint16_t b = f32_to_bf16(ks[lane + 32 * u]);
        kdst[lane + 32 * u] = b;
        kt[lane + 32 * u] = b;
      }
    } else if (warp == 1 && has_new) {
      uint16_t* vdst = static_cast<uint16_t*>(w.v_cache) + (a.cb * p.kc_sb + h * p.kc_sh + a.pos * D);
      uint16_t* vt = reinterpret_cast<uint16_t*>(vtile) + (size_t)(a.pos - t0) * D;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        vdst[lane + 32 * u] = rv[u];
        vt[lane + 32 * u] = rv[u];
      }
    }
    __syncthreads();
    tmark(S, 1);
    bool ok = true;
    if (n_pre > 0) {
      bool ready = mbar_wait_bounded(&S.bar_kv, ph_kv);
      if (!ready) {
        ok = false;
        if (tid == 0) atomicOr(p.err, kErrFlagTimeout);
        mbar_wait_bounded(&S.bar_kv, ph_kv);
      }
      ph_kv ^= 1u;
    }
    tmark(S, 2);
    // scores: warp w takes position groups of 4 (gqa_cluster_kernel); the
    // group's q values stay in registers
    float qv[8][U];
#pragma unroll
    for (int gg = 0; gg < 8; ++gg)
#pragma unroll
      for (int u = 0; u < U; ++u) qv[gg][u] = qs[gg * D + lane + 32 * u];
    if (ok) {
      for (int grp = warp; grp * 4 < n; grp += kStepWarps) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int tt = grp * 4 + i;
          float kk[U];
#pragma unroll
          for (int u = 0; u < U; ++u) kk[u] = tt < n ? bf16_to_f32(kt16[(size_t)tt * D + lane + 32 * u]) : 0.0f;
#pragma unroll
          for (int gg = 0; gg < 8; ++gg) {
            float pj[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int u = 0; u < U; ++u) pj[u & 3] = __fmaf_rn(qv[gg][u], kk[u], pj[u & 3]);
            v[i * 8 + gg] = __fadd_rn(__fadd_rn(__fadd_rn(pj[0], pj[1]), pj[2]), pj[3]);
          }
        }
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) {
          const bool upper = (lane & m) != 0;
#pragma unroll
          for (int i = 0; i < m; ++i) {
            const float keep = upper ? v[i + m] : v[i];
            const float send = upper ? v[i] : v[i + m];
            v[i] = __fadd_rn(keep, __shfl_xor_sync(0xffffffffu, send, m));
          }
        }
        const int tt = grp * 4 + (lane >> 3), gg = lane & 7;
        if (tt < n && gg < G) scores[gg * P + tt] = __fmul_rn(v[0], p.scale);
      }
    }
    __syncthreads();
    tmark(S, 3);
    if (ok && warp < G) {
      const int gg = warp;
      float sv[4];
      float m = ninf;
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int tt = lane + 32 * u;
        sv[u] = (tt < n) ? scores[gg * P + tt] : ninf;
        m = fmaxf(m, sv[u]);
      }
      m = warp_max(m);
      float pp[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int tt = lane + 32 * u;
        pp[u] = (tt < n) ? mexp_call(__fsub_rn(sv[u], m)) : 0.0f;
        if (tt < P) pb[gg * P + tt] = (tt < n) ? bf16_round(pp[u]) : 0.0f;
      }
      const float l = r128_lane_finish(pp[0], pp[1], pp[2], pp[3]);
      __syncwarp();
      // P.V: lane owns dims dv(u) = 64 (u / 2) + 2 lane + u % 2 (bf16 pairs);
      // each dim is a sequential fmaf chain over the positions
      float acc[U];
#pragma unroll
      for (int u = 0; u < U; ++u) acc[u] = 0.0f;
      const uint32_t* vt32 = reinterpret_cast<const uint32_t*>(vtile);
      int tt = 0;
      for (; tt + 4 <= n; tt += 4) {
        float pq[4];
        uint32_t vv[4][U / 2];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          pq[i] = pb[gg * P + tt + i];
#pragma unroll
          for (int h2 = 0; h2 < U / 2; ++h2) vv[i][h2] = vt32[((size_t)(tt + i) * D + 64 * h2 + 2 * lane) >> 1];
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int h2 = 0; h2 < U / 2; ++h2) {
            acc[2 * h2] = __fmaf_rn(pq[i], __uint_as_float(vv[i][h2] << 16), acc[2 * h2]);
            acc[2 * h2 + 1] = __fmaf_rn(pq[i], __uint_as_float(vv[i][h2] & 0xffff0000u), acc[2 * h2 + 1]);
          }
      }
      for (; tt < n; ++tt) {
        const float pt = pb[gg * P + tt];
#pragma unroll
        for (int h2 = 0; h2 < U / 2; ++h2) {
          const uint32_t vv = vt32[((size_t)tt * D + 64 * h2 + 2 * lane) >> 1];
          acc[2 * h2] = __fmaf_rn(pt, __uint_as_float(vv << 16), acc[2 * h2]);
          acc[2 * h2 + 1] = __fmaf_rn(pt, __uint_as_float(vv & 0xffff0000u), acc[2 * h2 + 1]);
        }
      }
      const int hq = h * G + gg;
      if (a.ns == 1) {
#pragma unroll
        for (int h2 = 0; h2 < U / 2; ++h2) {
          const uint32_t lo = f32_to_bf16(__fdiv_rn(acc[2 * h2], l)), hi = f32_to_bf16(__fdiv_rn(acc[2 * h2 + 1], l));
          reinterpret_cast<uint32_t*>(p.attn + hq * D + 64 * h2)[lane] = lo | (hi << 16);
        }
      } else {
        float* wa = p.att_acc + ((int64_t)hq * p.NS + s) * D;
#pragma unroll
        for (int h2 = 0; h2 < U / 2; ++h2)
          reinterpret_cast<float2*>(wa + 64 * h2)[lane] = make_float2(acc[2 * h2], acc[2 * h2 + 1]);
        if (lane == 0) {
          float* wml = p.att_ml + ((int64_t)hq * p.NS + s) * 2;
          wml[0] = m;
          wml[1] = l;
        }
      }
    }
    tmark(S, 4);
    if (a.ns > 1) {
      // the last split of head h merges all splits in split order
      __syncthreads();
      if (tid == 0) {
        __threadfence();
        const unsigned old = atomicAdd(&p.att_tickets[h], 1u);
        S.last = (old == static_cast<unsigned>(a.ns - 1));
        if (S.last) atomicExch(&p.att_tickets[h], 0u);
        __threadfence();
      }
      __syncthreads();
      tmark(S, 5);
      if (S.last && warp < G) {
        // M = max_j m_j, w_j = exp(m_j - M), den / num as fmaf chains in split
        // order (the workspace merge of gqa_decode_kernel), 8 splits per
        // round of loads
        const int hq = h * G + warp;
        const float* ml = p.att_ml + (int64_t)hq * p.NS * 2;
        const float* ac = p.att_acc + (int64_t)hq * p.NS * D;
        float M2 = ninf;
        for (int j = lane; j < a.ns; j += 32) M2 = fmaxf(M2, __ldcg(ml + 2 * j));
        M2 = warp_max(M2);
        float num[U];
#pragma unroll
        for (int u = 0; u < U; ++u) num[u] = 0.0f;
        float den = 0.0f;
        for (int j0 = 0; j0 < a.ns; j0 += 8) {
          float mj[8], lj[8];
          float2 aj[8][U / 2];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int j = j0 + i;
            if (j < a.ns) {
              mj[i] = __ldcg(ml + 2 * j);
              lj[i] = __ldcg(ml + 2 * j + 1);
#pragma unroll
              for (int h2 = 0; h2 < U / 2; ++h2)
                aj[i][h2] = __ldcg(reinterpret_cast<const float2*>(ac + (int64_t)j * D + 64 * h2) + lane);
            }
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (j0 + i < a.ns) {
              const float wgt = mexp_call(__fsub_rn(mj[i], M2));
              den = __fmaf_rn(wgt, lj[i], den);
#pragma unroll
              for (int h2 = 0; h2 < U / 2; ++h2) {
                num[2 * h2] = __fmaf_rn(wgt, aj[i][h2].x, num[2 * h2]);
                num[2 * h2 + 1] = __fmaf_rn(wgt, aj[i][h2].y, num[2 * h2 + 1]);
              }
            }
          }
        }
#pragma unroll
        for (int h2 = 0; h2 < U / 2; ++h2) {
          const uint32_t lo = f32_to_bf16(__fdiv_rn(num[2 * h2], den)), hi = f32_to_bf16(__fdiv_rn(num[2 * h2 + 1], den));
          reinterpret_cast<uint32_t*>(p.attn + hq * D + 64 * h2)[lane] = lo | (hi << 16);
        }
      }
    }
    __syncthreads();
    tmark(S, 6);
  }
}

// Dense weights of layer w into L2, this CTA's share (all threads).
__device__ __forceinline__ void prefetch_layer_dense(const StepParams& p, const maple_decode_layer& w) {
  const int qkv_n = (p.Hq + 2 * p.Hkv) * p.D;
  const int ab = p.alpha_f32 ? 4 : 2;
  l2_prefetch_share(w.qkv_codes, (int64_t)qkv_n * p.H / 4);
  l2_prefetch_share(w.o_codes, (int64_t)p.H * p.Hq * p.D / 4);
  l2_prefetch_share(w.qkv_alpha, (int64_t)qkv_n * ab);
  l2_prefetch_share(w.o_alpha, (int64_t)p.H * ab);
}

// One thread: stage layer w's static vectors (q/k norm weights, post-
// attention norm weights, this CTA's gate rows) on bar_st, its input norm
// weights on bar_in, and the final K/V rows of this CTA's first attention
// item on bar_kv.  Issued at the end of the previous layer (or at launch), so
// the copies run during that layer's barrier and this layer's QKV phase.
template <int D>
__device__ __forceinline__ void stage_layer(StepShared& S, const StepParams& p, const StepSmem& M,
                                            const maple_decode_layer& w, const AttnGeom& ag) {
  const unsigned nb = p.norm_f32 ? 4 : 2, gb = p.gate_f32 ? 4 : 2;
  const int e0 = blockIdx.x * kRouterExpertsPerItem;
  const int ne = max(0, min(kRouterExpertsPerItem, p.E - e0));
  fence_proxy_async_smem();
  mbar_expect_tx(&S.bar_in, (unsigned)p.H * nb);
  stage_bytes(const_cast<void*>(M.in_norm), w.in_norm, (unsigned)p.H * nb, &S.bar_in);
  if (ag.ns > 0 && (int)blockIdx.x < p.Hkv * ag.ns) attn_issue<D>(p, ag, w, blockIdx.x, M.att, &S.bar_kv);
  const unsigned total = 2 * (unsigned)p.D * nb + (unsigned)p.H * nb + (unsigned)(ne * p.H) * gb;
  mbar_expect_tx(&S.bar_st, total);
  stage_bytes(const_cast<void*>(M.q_norm), w.q_norm, (unsigned)p.D * nb, &S.bar_st);
  stage_bytes(const_cast<void*>(M.k_norm), w.k_norm, (unsigned)p.D * nb, &S.bar_st);
  stage_bytes(const_cast<void*>(M.post_norm), w.post_norm, (unsigned)p.H * nb, &S.bar_st);
  if (ne > 0)
    stage_bytes(const_cast<void*>(M.gate), static_cast<const char*>(w.gate) + (size_t)e0 * p.H * gb,
                (unsigned)(ne * p.H) * gb, &S.bar_st);
}

__device__ __forceinline__ bool wait_stage(const StepParams& p, uint64_t* bar, unsigned& ph) {
  const bool ready = mbar_wait_bounded(bar, ph);
  if (!ready && threadIdx.x == 0) atomicOr(p.err, kErrFlagTimeout);
  ph ^= 1u;
  return ready;
}

template <int D>
__global__ void __launch_bounds__(kStepThreads, 1) decode_layers_kernel(StepParams p) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ StepShared S;
  const int tid = threadIdx.x;
  StepSmem M;
  M.frag = reinterpret_cast<uint2*>(smem + p.off_frag);
  M.xs = reinterpret_cast<float*>(smem + p.off_xs);
  M.xr = reinterpret_cast<float*>(smem + p.off_xr);
  M.att = smem + p.off_att;
  M.layers = smem + p.off_layers;
  M.in_norm = smem + p.off_in;
  M.post_norm = smem + p.off_post;
  M.q_norm = smem + p.off_qn;
  M.k_norm = smem + p.off_kn;
  M.cos = smem + p.off_cos;
  M.sin = smem + p.off_sin;
  M.gate = smem + p.off_gate;
  const maple_decode_layer* L = reinterpret_cast<const maple_decode_layer*>(M.layers);
  constexpr int kLast = kStepThreads - 1;  // the thread that issues the staging copies

  pdl_wait();
  unsigned epoch = 0;
  const int64_t pos0 = p.seqlen[0];
  if (tid == 0) {
    S.ok = 1;
    S.mk = nullptr;
    mbar_init(&S.bar_kv, 1);
    mbar_init(&S.bar_st, 1);
    mbar_init(&S.bar_in, 1);
    mbar_init(&S.bar_rope, 1);
    S.tracing = p.trace != nullptr && p.sync[2] != 0u;
    // the RoPE row of this step's position (every layer reads the same row)
    const unsigned cb = p.cs_f32 ? 4 : 2;
    const int64_t row = pos0 < 0 ? 0 : (pos0 >= p.cs_len ? p.cs_len - 1 : pos0);
    const unsigned rb = p.R > 0 ? (unsigned)p.R * cb : 0;
    mbar_expect_tx(&S.bar_rope, 2 * rb);
    stage_bytes(const_cast<void*>(M.cos), static_cast<const char*>(p.cos) + row * p.cs_stride * cb, rb, &S.bar_rope);
    stage_bytes(const_cast<void*>(M.sin), static_cast<const char*>(p.sin) + row * p.cs_stride * cb, rb, &S.bar_rope);
  }
  // every layer descriptor into shared memory (plain loads: a few KB)
  for (int i = tid; i < p.n_layers * (int)(sizeof(maple_decode_layer) / 8); i += kStepThreads)
    reinterpret_cast<uint64_t*>(M.layers)[i] = reinterpret_cast<const uint64_t*>(p.layers)[i];
  // the fragments' zero halves (B columns 4-7): written here only
  for (int i = tid; i < p.frag_entries; i += kStepThreads) M.frag[i] = make_uint2(0u, 0u);
  __syncthreads();
  unsigned ph_kv = 0, ph_st = 0, ph_in = 0, ph_rope = 0;
  if (tid == kLast) stage_layer<D>(S, p, M, L[0], attn_geom(p, (int)L[0].window));
  prefetch_layer_dense(p, L[0]);
  int64_t* tr = S.tracing ? p.trace : nullptr;  // advanced by 2 * grid per barrier
  auto next_tr = [&]() {
    int64_t* t = tr;
    if (tr != nullptr) tr += 2 * gridDim.x;
    return t;
  };
  // per-phase checkpoints: [layer][phase][8][grid] clock64 after the barrier timestamps, when they fit
  long long* marks = (S.tracing && p.n_layers * 6 * 8 * (int64_t)gridDim.x * 8 +
                                       p.n_layers * 6 * 2 * (int64_t)gridDim.x * 8 <= p.trace_bytes)
                         ? reinterpret_cast<long long*>(p.trace + p.n_layers * 6 * 2 * (int64_t)gridDim.x)
                         : nullptr;
  auto phase_marks = [&](int l, int ph) {
    if (tid == 0) S.mk = marks ? marks + ((int64_t)(l * 6 + ph) * 8) * gridDim.x : nullptr;
    tmark(S, 0);
  };
  wait_stage(p, &S.bar_rope, ph_rope);

  for (int l = 0; l < p.n_layers; ++l) {
    const maple_decode_layer& w = L[l];
    const AttnGeom ag = attn_geom(p, (int)w.window);
    // a position outside the cache (or a bad cache row) stores no K/V, as in qk_norm_rope_store_kernel
    if (blockIdx.x == 0 && tid == 0 && (ag.pos < 0 || ag.pos >= p.T || !ag.cb_ok)) atomicOr(p.err, kErrFlagBounds);
    // 1: combine the previous layer's experts -> x; RMSNorm -> QKV (split-K)
    phase_marks(l, 0);
    wait_stage(p, &S.bar_in, ph_in);
    if (l > 0) zero_share(p.sw_sum, (int64_t)p.topk * 2 * p.I);
    qkv_phase<kQkvTpw>(S, M, p, w, l == 0);
    tmark(S, 7);
    if (!grid_barrier(p, epoch, &S.ok, next_tr())) break;
    // 2: attention (first item's final rows are in flight since the previous layer)
    phase_marks(l, 1);
    wait_stage(p, &S.bar_st, ph_st);
    attention_phase<D>(S, M, p, w, ag, ph_kv);
    tmark(S, 7);
    if (!grid_barrier(p, epoch, &S.ok, next_tr())) break;
    // 3: O projection (split-K)
    phase_marks(l, 2);
    o_phase<kOTpw>(S, M, p, w);
    tmark(S, 7);
    if (!grid_barrier(p, epoch, &S.ok, next_tr())) break;
    // 4: residual add + RMSNorm + router logits; the next layer's dense
    // weights into L2 once this CTA is done
    phase_marks(l, 3);
    router_phase(S, M, p, w);
    if (l + 1 < p.n_layers) prefetch_layer_dense(p, L[l + 1]);
    tmark(S, 7);
    if (!grid_barrier(p, epoch, &S.ok, next_tr())) break;
    // 5: top-k (every CTA), up|gate of the selected experts (split-K)
    phase_marks(l, 4);
    swiglu_phase<kSwTpw>(S, M, p, w);
    tmark(S, 7);
    if (!grid_barrier(p, epoch, &S.ok, next_tr())) break;
    // 6: SwiGLU + down per (slot, rows); then the next layer's staging copies
    phase_marks(l, 5);
    down_phase(S, M, p, w);
    if (l + 1 < p.n_layers && tid == kLast) stage_layer<D>(S, p, M, L[l + 1], attn_geom(p, (int)L[l + 1].window));
    tmark(S, 7);
    if (!grid_barrier(p, epoch, &S.ok, next_tr())) break;
  }
  if (S.ok) final_phase(S, p);
  // a layer that stopped early (timeout) leaves no staging copy in flight
  if (tid == 0 && S.ok == 0) {
    mbar_wait_bounded(&S.bar_in, ph_in);
    mbar_wait_bounded(&S.bar_st, ph_st);
    mbar_wait_bounded(&S.bar_kv, ph_kv);
  }
  grid_barrier_retire(p);
}

}  // namespace mb

using namespace mb;

namespace {

constexpr int64_t kStepSyncBytes = 4096;
constexpr int64_t kStepTraceBytes = 1 << 20;  // barrier timestamps, written only when switched on

int64_t align256(int64_t v) { return (v + 255) & ~int64_t(255); }

struct StepLayout {
  int64_t qkv_sum, o_sum, sw_sum, ybuf, meta, attn, resid, normed, logits, acc, ml, trace, total;
  int off_frag, off_xs, off_xr, off_att, off_layers, off_in, off_post, off_qn, off_kn, off_cos, off_sin, off_gate, smem;
};

StepLayout step_layout(int64_t H, int64_t Hq, int64_t Hkv, int64_t D, int64_t E, int64_t topk, int64_t I,
                       int64_t NS, int64_t P, int64_t R, int64_t n_layers) {
  StepLayout L{};
  int64_t off = kStepSyncBytes;
  L.qkv_sum = off; off = align256(off + (Hq + 2 * Hkv) * D * 8);
  L.o_sum = off; off = align256(off + H * 8);
  L.sw_sum = off; off = align256(off + topk * 2 * I * 8);
  L.ybuf = off; off = align256(off + topk * H * 2);
  L.meta = off; off = align256(off + 64);
  L.attn = off; off = align256(off + Hq * D * 2);
  L.resid = off; off = align256(off + H * 2);
  L.normed = off; off = align256(off + H * 2);
  L.logits = off; off = align256(off + E * 4);
  L.acc = off; off = align256(off + Hq * NS * D * 4);
  L.ml = off; off = align256(off + Hq * NS * 2 * 4);
  L.trace = off; off = align256(off + kStepTraceBytes);
  L.total = off;
  auto iters = [](int64_t K) { return (K / 16 + 15) / 16; };
  auto a128 = [](int64_t v) { return (v + 127) & ~int64_t(127); };
  // fragments: a split-K slice (<= 4 iterations) or the down phase's whole K
  const int64_t frag = std::max<int64_t>(4, iters(I)) * 2048;
  // xs: a split-K slice (<= 4 iterations), the down phase's whole K, or the router's normed row
  const int64_t xs = std::max<int64_t>(std::max<int64_t>(padded_len(4 * 256), padded_len((int)I)), padded_len((int)H));
  const int64_t xr = H;
  int64_t s = 0;
  L.off_frag = (int)s; s += a128(frag);
  L.off_xs = (int)s; s += a128(xs * 4);
  L.off_xr = (int)s; s += a128(xr * 4);
  L.off_att = (int)s; s += a128(2 * P * D * 2 + 2 * 8 * P * 4 + 8 * D * 4 + D * 4);
  L.off_layers = (int)s; s += a128(n_layers * (int64_t)sizeof(maple_decode_layer));
  L.off_in = (int)s; s += a128(H * 4);
  L.off_post = (int)s; s += a128(H * 4);
  L.off_qn = (int)s; s += a128(D * 4);
  L.off_kn = (int)s; s += a128(D * 4);
  L.off_cos = (int)s; s += a128(std::max<int64_t>(R, 1) * 4);
  L.off_sin = (int)s; s += a128(std::max<int64_t>(R, 1) * 4);
  L.off_gate = (int)s; s += a128(kRouterExpertsPerItem * H * 4);
  L.smem = (int)s;
  return L;
}

// Split-K geometry: the fewest iterations per slice (<= 4) whose items
// (row blocks x slices) fit one wave of CTAs; -1 when none does.
int pick_ipw(int64_t row_blocks, int64_t K, int grid) {
  const int64_t it = (K / 16 + 15) / 16;
  for (int ipw = 1; ipw <= 4; ++ipw) {
    const int64_t nks = (it + ipw - 1) / ipw;
    if (row_blocks * nks <= grid) return ipw;
  }
  return -1;
}

}  // namespace

extern "C" int64_t maple_decode_layers_workspace_bytes(int64_t hidden, int64_t num_heads, int64_t num_kv_heads,
                                                       int64_t head_dim, int64_t n_experts, int64_t topk,
                                                       int64_t inter, int64_t max_len, int64_t split_len) {
  if (split_len <= 0 || max_len <= 0) return -1;
  const int64_t NS = (max_len + split_len - 1) / split_len;
  return step_layout(hidden, num_heads, num_kv_heads, head_dim, n_experts, topk, inter, NS, split_len, 0, 0).total;
}

extern "C" int maple_decode_layers(const maple_decode_layer* layers, int64_t n_layers, void* x,
                                   const int64_t* seqlen, const int32_t* row_map, const void* cos, const void* sin,
                                   int cs_dtype, int64_t cs_row_stride, int64_t cs_table_len, int64_t hidden,
                                   int64_t num_heads, int64_t num_kv_heads, int64_t head_dim, int64_t rotary_dim,
                                   int64_t n_experts, int64_t topk, int64_t inter, int64_t cache_batch,
                                   int64_t max_len, int64_t cache_sb, int64_t cache_sh, int64_t split_len,
                                   int alpha_dtype, int norm_dtype, int gate_dtype, float eps, float scale,
                                   void* workspace, int64_t workspace_bytes, int* err, void* stream) {
  if (n_layers < 0) return kErrShape;
  if (n_layers == 0) return kOk;
  if (!layers || !x || !seqlen || !err || !workspace) return kErrShape;
  if ((alpha_dtype != kF32 && alpha_dtype != kBF16) || (norm_dtype != kF32 && norm_dtype != kBF16) ||
      (gate_dtype != kF32 && gate_dtype != kBF16) || (cs_dtype != kF32 && cs_dtype != kBF16))
    return kErrDtype;
  if (head_dim != 64 && head_dim != 128) return kErrShape;
  if (num_kv_heads <= 0 || num_heads % num_kv_heads != 0 || num_heads / num_kv_heads > kStepMaxG) return kErrShape;
  if (topk <= 0 || topk > kStepMaxTopk || n_experts < topk || n_experts > kStepMaxE) return kErrShape;
  if (hidden % 64 || (num_heads * head_dim) % 64 || inter % 64 || hidden > 8192 || num_heads * head_dim > 8192)
    return kErrShape;
  if ((inter / 16 + 15) / 16 > kStepNI) return kErrShape;  // down: one warp holds a slot's K in registers
  if (split_len != 32 && split_len != 64 && split_len != 128) return kErrShape;
  if (rotary_dim < 0 || rotary_dim > head_dim || (rotary_dim & 1)) return kErrShape;
  if (rotary_dim > 0 && (!cos || !sin || cs_table_len <= 0)) return kErrShape;
  if (((cache_sb * 2) & 15) || ((cache_sh * 2) & 15)) return kErrAlign;
  // bulk-staged rows: the RoPE row, norm weights and router rows start on 16 bytes
  const int64_t cse = cs_dtype == kF32 ? 4 : 2;
  if (rotary_dim > 0 && (((rotary_dim * cse) & 15) || ((cs_row_stride * cse) & 15) ||
                         (reinterpret_cast<uintptr_t>(cos) & 15) || (reinterpret_cast<uintptr_t>(sin) & 15)))
    return kErrAlign;
  if (((head_dim * (norm_dtype == kF32 ? 4 : 2)) & 15) != 0) return kErrAlign;
  const int64_t NS = (max_len + split_len - 1) / split_len;
  const StepLayout L = step_layout(hidden, num_heads, num_kv_heads, head_dim, n_experts, topk, inter, NS, split_len,
                                   rotary_dim, n_layers);
  if (workspace_bytes < L.total) return kErrWorkspace;
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0) return kErrAlign;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kErrCuda;
  int n_sm = 0, max_smem = 0;
  if (cudaDeviceGetAttribute(&n_sm, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return kErrCuda;
  if (cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) return kErrCuda;
  const int static_smem = (int)sizeof(StepShared) + 1024;
  if (L.smem + static_smem > max_smem) return kErrShape;

  const int grid = n_sm;
  StepParams p{};
  p.layers = layers; p.n_layers = (int)n_layers;
  p.x = static_cast<uint16_t*>(x); p.seqlen = seqlen; p.row_map = row_map;
  p.cos = cos; p.sin = sin; p.cs_stride = cs_row_stride; p.cs_len = cs_table_len;
  p.cs_f32 = cs_dtype == kF32; p.alpha_f32 = alpha_dtype == kF32; p.norm_f32 = norm_dtype == kF32;
  p.gate_f32 = gate_dtype == kF32;
  p.H = (int)hidden; p.Hq = (int)num_heads; p.Hkv = (int)num_kv_heads; p.D = (int)head_dim; p.R = (int)rotary_dim;
  p.E = (int)n_experts; p.topk = (int)topk; p.I = (int)inter; p.T = (int)max_len; p.Bc = (int)cache_batch;
  p.P = (int)split_len; p.NS = (int)NS; p.kc_sb = cache_sb; p.kc_sh = cache_sh;
  p.eps = eps; p.scale = scale;
  auto iters = [](int64_t K) { return (int)((K / 16 + 15) / 16); };
  const int64_t qkv_rows = (num_heads + 2 * num_kv_heads) * head_dim;
  const int64_t qkv_rb = (qkv_rows + kStepWarps * kQkvTpw * 16 - 1) / (kStepWarps * kQkvTpw * 16);
  const int64_t o_rb = (hidden + kStepWarps * kOTpw * 16 - 1) / (kStepWarps * kOTpw * 16);
  const int64_t sw_outs = kStepWarps * kSwTpw * 16 / 2;
  const int64_t sw_rb = topk * ((inter + sw_outs - 1) / sw_outs);
  p.qkv_ipw = pick_ipw(qkv_rb, hidden, grid);
  p.o_ipw = pick_ipw(o_rb, num_heads * head_dim, grid);
  p.sw_ipw = pick_ipw(sw_rb, hidden, grid);
  if (p.qkv_ipw < 0 || p.o_ipw < 0 || p.sw_ipw < 0) return kErrShape;
  p.qkv_nks = (iters(hidden) + p.qkv_ipw - 1) / p.qkv_ipw;
  p.o_nks = (iters(num_heads * head_dim) + p.o_ipw - 1) / p.o_ipw;
  p.sw_nks = (iters(hidden) + p.sw_ipw - 1) / p.sw_ipw;
  if (topk * ((hidden + 127) / 128) > grid) return kErrShape;  // down items: (slot, 128 rows)
  char* ws = static_cast<char*>(workspace);
  p.qkv_sum = reinterpret_cast<unsigned long long*>(ws + L.qkv_sum);
  p.o_sum = reinterpret_cast<unsigned long long*>(ws + L.o_sum);
  p.sw_sum = reinterpret_cast<unsigned long long*>(ws + L.sw_sum);
  p.ybuf = reinterpret_cast<uint16_t*>(ws + L.ybuf);
  p.meta = reinterpret_cast<float*>(ws + L.meta);
  p.attn = reinterpret_cast<uint16_t*>(ws + L.attn);
  p.resid = reinterpret_cast<uint16_t*>(ws + L.resid);
  p.normed = reinterpret_cast<uint16_t*>(ws + L.normed);
  p.logits = reinterpret_cast<float*>(ws + L.logits);
  p.att_acc = reinterpret_cast<float*>(ws + L.acc);
  p.att_ml = reinterpret_cast<float*>(ws + L.ml);
  p.sync = reinterpret_cast<unsigned*>(ws);
  // timestamps of every barrier (opt-in through sync word 2) when they fit
  p.trace = ((n_layers * 6 + 1) * 2 * (int64_t)grid * 8 <= kStepTraceBytes) ? reinterpret_cast<int64_t*>(ws + L.trace)
                                                                      : nullptr;
  p.trace_bytes = kStepTraceBytes;
  p.att_tickets = reinterpret_cast<unsigned*>(ws + 256);
  p.err = err;
  p.off_frag = L.off_frag; p.off_xs = L.off_xs; p.off_xr = L.off_xr; p.off_att = L.off_att;
  p.off_layers = L.off_layers; p.off_in = L.off_in; p.off_post = L.off_post; p.off_qn = L.off_qn;
  p.off_kn = L.off_kn; p.off_cos = L.off_cos; p.off_sin = L.off_sin; p.off_gate = L.off_gate;
  p.frag_entries = (L.off_xs - L.off_frag) / (int)sizeof(uint2);
  if ((n_experts + kRouterExpertsPerItem - 1) / kRouterExpertsPerItem > grid) return kErrShape;
  if (num_kv_heads * 4 > kStepSyncBytes - 256) return kErrShape;

  auto kern = head_dim == 64 ? decode_layers_kernel<64> : decode_layers_kernel<128>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L.smem) != cudaSuccess) return kErrCuda;
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kStepThreads, L.smem) != cudaSuccess) return kErrCuda;
  if (occ < 1) return kErrShape;

  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)grid);
  cfg.blockDim = dim3(kStepThreads);
  cfg.dynamicSmemBytes = (size_t)L.smem;
  cfg.stream = static_cast<cudaStream_t>(stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, p);
  return e == cudaSuccess ? kOk : kErrCuda;
}
