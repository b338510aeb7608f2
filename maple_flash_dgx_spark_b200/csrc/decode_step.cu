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
constexpr int kStepNI = 8;         // K iterations per warp held in registers
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
  int wm_qkv, wm_o, wm_sw;     // row tiles per item of the QKV, O and SwiGLU phases
  // scratch
  uint16_t* qkv;               // [(Hq + 2 Hkv) D]
  uint16_t* attn;              // [Hq D]
  uint16_t* o;                 // [H]
  uint16_t* resid;             // [H]
  uint16_t* normed;            // [H]
  uint16_t* hact;              // [topk, I]
  float* logits;               // [E]
  float* att_acc;              // [Hq, NS, D]
  float* att_ml;               // [Hq, NS, 2]
  unsigned* sync;              // [0] barrier arrivals, [1] CTAs retired, [2] trace switch
  int64_t* trace;              // [n_layers * 6][2][grid] barrier arrival / release times (ns), then checkpoints
  int64_t trace_bytes;
  unsigned* att_tickets;       // [Hkv]
  int* err;
  // dynamic shared memory carve-up (bytes)
  int off_frag, off_xs, off_xr, off_att, off_layers, off_in, off_post, off_qn, off_kn, off_cos, off_sin, off_gate;
};

__device__ __forceinline__ float ldf(const void* p, int64_t i, int f32) {
  return f32 ? static_cast<const float*>(p)[i] : bf16_to_f32(static_cast<const uint16_t*>(p)[i]);
}

__device__ __forceinline__ float bf16_round(float v) { return bf16_to_f32(f32_to_bf16(v)); }

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

// Fragments of codes [0, iters*256) of xs (n values) by threads t_local of
// nt (a multiple of 32) and each warp's raw digit sums in S.fb.rawsum.
__device__ __forceinline__ void build_frags(StepShared& S, const float* xs, int n, int s, int iters, uint2* frag,
                                            int t_local, int nt) {
  int raws[4] = {0, 0, 0, 0};
  fxa_build<2>(xs, n, s, s == kFxaNonFinite, iters, frag, t_local, nt, raws);
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

// ------------------------------------------------------------ dense GEMV --
// y[n] = bf16(fxa(S_n) [* rstd] * alpha[n]) for n < N over the activation x
// (bf16, K elements), with the input RMSNorm folded in when rms_w (staged in
// shared memory) is given.  Same arithmetic as tgemv2_kernel.  Items: 16*WM
// rows; the 8 warps are WM row tiles x (8/WM) K slices whose exact int32
// partials add up in shared memory.  The activation is read once (one L2
// round trip); the RMS partial sums run between the two prologue barriers.
template <int NI>
__device__ __forceinline__ void dense_gemv(StepShared& S, const StepSmem& M, const void* x, const void* rms_w,
                                           int norm_f32, float eps, const uint32_t* codes, const void* alpha,
                                           int alpha_f32, uint16_t* y, int N, int K, int WM) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const int WK = kStepWarps / WM;
  const int wm = warp % WM, wk = warp / WM;
  const int nwords = K / 16, iters_total = (nwords + 15) / 16;
  const int ipw = (iters_total + WK - 1) / WK;
  const int it0 = wk * ipw, my_iters = max(0, min(ipw, iters_total - it0));
  const int per_item = 16 * WM, n_items = (N + per_item - 1) / per_item;
  const bool rms = rms_w != nullptr;
  bool first = true;
  int s = 0;
  int tot[4] = {0, 0, 0, 0};
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int row_g = item * per_item + 16 * wm + g, row_h = row_g + 8;
    const bool ok_g = row_g < N, ok_h = row_h < N;
    uint4 wa[NI], wb[NI];
    load_tile(codes, row_g, row_h, ok_g, ok_h, nwords, it0, my_iters, t, wa, wb);
    tmark(S, 1);
    if (first) {
      // stage x (8 values per 16-byte chunk), x_hat = x * w, local |x_hat| max
      const int nch = K / 8;
      uint4 r[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (tid + i * kStepThreads < nch) r[i] = ld_u4(static_cast<const char*>(x) + (size_t)(tid + i * kStepThreads) * 16);
      unsigned amax = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = tid + i * kStepThreads;
        if (c < nch) {
          float v[8];
          widen_u4<kBF16>(r[i], v);
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const int k = c * 8 + e;
            float h = v[e];
            if (rms) {
              M.xr[k] = v[e];
              h = __fmul_rn(v[e], ldf(rms_w, k, norm_f32));
            }
            M.xs[k] = h;
            amax = max(amax, __float_as_uint(h) & 0x7fffffffu);
          }
        }
      }
      s = amax_exchange(S, amax);
      if (rms && tid < 128) {
        float ss = 0.0f;
        for (int k = tid; k < K; k += 128) ss = __fmaf_rn(M.xr[k], M.xr[k], ss);
        S.part[0][tid] = ss;
      }
      build_frags(S, M.xs, K, s, iters_total, M.frag, tid, kStepThreads);
      __syncthreads();
      digit_totals(S, iters_total, tot);
      first = false;
    }
    tmark(S, 2);
    int acc[4] = {0, 0, 0, 0};
    contract_tile2<NI>(wa, wb, my_iters, M.frag + (size_t)it0 * 256, lane, acc);
    if (wk > 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j) S.red[(wk - 1) * WM + wm][lane][j] = acc[j];
    }
    __syncthreads();
    tmark(S, 3);
    if (wk == 0) {
      for (int w2 = 1; w2 < WK; ++w2)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[j] += S.red[(w2 - 1) * WM + wm][lane][j];
      long long Sg, Sh;
      combine_digits(acc, tot, t, Sg, Sh);
      const float rstd = rms ? rstd_of(r128_smem_finish(S.part[0], lane), K, eps) : 1.0f;
      if (t == 0) {
        const bool nan_out = (s == kFxaNonFinite);
        auto value = [&](int row, long long Sv) -> float {
          float v = nan_out ? __int_as_float(0x7fc00000) : fxa_value(Sv, s);
          if (rms) v = __fmul_rn(v, rstd);
          return __fmul_rn(v, ldf(alpha, row, alpha_f32));
        };
        if (ok_g) y[row_g] = f32_to_bf16(value(row_g, Sg));
        if (ok_h) y[row_h] = f32_to_bf16(value(row_h, Sh));
      }
    }
    __syncthreads();
    tmark(S, 4);
  }
}

// -------------------------------------------------------------- SwiGLU ----
// Every CTA: softmax + top-k + renorm of the E logits (router_kernel's
// last-CTA part).  The order of its repeated argmax (largest first, ties to
// the lowest index) is each expert's rank, one thread per expert.  Then
// h[slot, n] = bf16(clamp(u, +-7) * min(g, 7) * sigmoid(min(g, 7))) with u, g
// the up / gate rows of expert ids[slot] (tgemv2_kernel<kSwiglu>).  Items:
// (slot, 8*WM outputs); warps wm < WM/2 take up rows, the rest gate rows.
// The down rows of this CTA's down item go to L2 as soon as the experts are
// known.
__device__ __forceinline__ void swiglu_phase(StepShared& S, const StepSmem& M, const StepParams& p,
                                             const maple_decode_layer& w) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const int WM = p.wm_sw, WK = kStepWarps / WM;
  const int wm = warp % WM, wk = warp / WM;
  const int K = p.H, I = p.I, E = p.E;
  const int nwords = K / 16, iters_total = (nwords + 15) / 16;
  const int ipw = (iters_total + WK - 1) / WK;
  const int it0 = wk * ipw, my_iters = max(0, min(ipw, iters_total - it0));
  const int outs = 8 * WM, nblk = (I + outs - 1) / outs, n_items = p.topk * nblk;
  const int64_t expert_words = (int64_t)2 * I * nwords;
  const float ninf = __int_as_float(0xff800000);
  // 1. the normed row (all) and the logits (warp 0) in one round trip
  const int nch = K / 8;
  uint4 r[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (tid + i * kStepThreads < nch) r[i] = ld_u4(reinterpret_cast<const char*>(p.normed) + (size_t)(tid + i * kStepThreads) * 16);
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
      v[i] = ee < E ? mexp(__fsub_rn(v[i], m)) : 0.0f;
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
  unsigned amax = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = tid + i * kStepThreads;
    if (c < nch) {
      float v[8];
      widen_u4<kBF16>(r[i], v);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        M.xs[c * 8 + e] = v[e];
        amax = max(amax, __float_as_uint(v[e]) & 0x7fffffffu);
      }
    }
  }
  const int s = amax_exchange(S, amax);  // also publishes the probabilities
  // 2. rank of expert tid (NaN is never picked by the argmax rounds)
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
  float total = 0.0f;
  for (int rr = 0; rr < p.topk; ++rr) total = __fadd_rn(total, S.tk_sel_p[rr]);
  const float inv = __fdiv_rn(1.0f, __fadd_rn(total, 1e-20f));
  if (tid < p.topk) {
    S.ids[tid] = S.tk_sel_i[tid];
    S.wts[tid] = __fmul_rn(S.tk_sel_p[tid], inv);
  }
  tmark(S, 1);
  // 3. this CTA's down rows into L2 (slot = warp, one 128-byte line per lane)
  {
    const int64_t row_bytes = (int64_t)I / 4;
    const int n_down = (p.H + 15) / 16;
    if (warp < p.topk && (int)blockIdx.x < n_down) {
      const int e = S.tk_sel_i[warp];
      if (e >= 0 && e < E) {
        const int r0 = blockIdx.x * 16;
        const int64_t bytes = min(16, p.H - r0) * row_bytes;
        const char* base = reinterpret_cast<const char*>(w.dn_codes) + ((int64_t)e * p.H + r0) * row_bytes;
        for (int64_t off = (int64_t)lane * 128; off < bytes; off += 32 * 128) prefetch_l2(base + off);
      }
    }
  }
  // 4. expert rows, then the fragments while they arrive
  bool first = true;
  int tot[4] = {0, 0, 0, 0};
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int slot = item / nblk, n0 = (item % nblk) * outs;
    int e = S.tk_sel_i[slot];
    const bool bad_id = (e < 0 || e >= E);
    if (bad_id) e = 0;
    const uint32_t* codes = w.ug_codes + (int64_t)e * expert_words;
    const int base = (wm < WM / 2) ? 0 : I;
    const int tile0 = base + n0 + 16 * ((wm < WM / 2) ? wm : wm - WM / 2);
    const int row_g = tile0 + g, row_h = row_g + 8;
    const bool ok_g = row_g < base + I, ok_h = row_h < base + I;
    uint4 wa[kStepNI], wb[kStepNI];
    load_tile(codes, row_g, row_h, ok_g, ok_h, nwords, it0, my_iters, t, wa, wb);
    tmark(S, 2);
    if (first) {
      build_frags(S, M.xs, K, s, iters_total, M.frag, tid, kStepThreads);
      __syncthreads();
      digit_totals(S, iters_total, tot);
      first = false;
    }
    tmark(S, 3);
    int acc[4] = {0, 0, 0, 0};
    contract_tile2<kStepNI>(wa, wb, my_iters, M.frag + (size_t)it0 * 256, lane, acc);
    if (wk > 0) {
#pragma unroll
      for (int j = 0; j < 4; ++j) S.red[(wk - 1) * WM + wm][lane][j] = acc[j];
    }
    if (WK > 1) __syncthreads();
    tmark(S, 4);
    if (wk == 0) {
      for (int w2 = 1; w2 < WK; ++w2)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[j] += S.red[(w2 - 1) * WM + wm][lane][j];
      long long Sg, Sh;
      combine_digits(acc, tot, t, Sg, Sh);
      if (t == 0) {
        const bool nan_out = (s == kFxaNonFinite) || bad_id;
        const void* al = static_cast<const char*>(w.ug_alpha) + (int64_t)e * 2 * I * (p.alpha_f32 ? 4 : 2);
        auto value = [&](int row, long long Sv) -> float {
          const float v = nan_out ? __int_as_float(0x7fc00000) : fxa_value(Sv, s);
          return __fmul_rn(v, ldf(al, row, p.alpha_f32));
        };
        S.s_val[16 * wm + g] = ok_g ? value(row_g, Sg) : 0.0f;
        S.s_val[16 * wm + g + 8] = ok_h ? value(row_h, Sh) : 0.0f;
      }
    }
    __syncthreads();
    if (tid < outs) {
      const int n = n0 + tid;
      if (n < I) {
        float up = S.s_val[tid], gate = S.s_val[outs + tid];
        up = fminf(fmaxf(up, -7.0f), 7.0f);
        gate = fminf(gate, 7.0f);
        p.hact[(int64_t)slot * I + n] = f32_to_bf16(__fmul_rn(__fmul_rn(up, gate), msigmoid(gate)));
      }
    }
    __syncthreads();
    tmark(S, 5);
  }
}

// ---------------------------------------------------------------- down ----
// out[n] = bf16(fmaf-chain_slot(w_slot, bf16(alpha_e[n] * S_slot[n])) +
// residual[n]) (down_sum_kernel MODE 0).  Warp `slot` encodes that slot's
// activation row itself (no block barrier) and contracts the item's 16 rows
// of expert ids[slot] against it; the weighted combine adds the slots in
// order.
__device__ __forceinline__ void down_phase(StepShared& S, const StepSmem& M, const StepParams& p,
                                           const maple_decode_layer& w) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, g = lane >> 2, t = lane & 3;
  const int K = p.I, N = p.H;
  const int nwords = K / 16, iters_total = (nwords + 15) / 16;
  const int slot = warp;
  const int n_items = (N + 15) / 16;
  const size_t frag_stride = (size_t)iters_total * 256;
  const bool active = slot < p.topk;
  int e = active ? S.ids[slot] : 0;
  const bool bad = (e < 0 || e >= p.E);
  if (bad) e = 0;
  const uint32_t* codes = w.dn_codes + (int64_t)e * N * nwords;
  const void* al = static_cast<const char*>(w.dn_alpha) + (int64_t)e * N * (p.alpha_f32 ? 4 : 2);
  bool first = true;
  int sh = 0;
  int tot[4] = {0, 0, 0, 0};
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int row_g = item * 16 + g, row_h = row_g + 8;
    uint4 wa[kStepNI], wb[kStepNI];
    load_tile(codes, row_g, row_h, active && row_g < N, active && row_h < N, nwords, 0, active ? iters_total : 0, t,
              wa, wb);
    tmark(S, 1);
    if (first && active) {
      // this warp's slot row: stage, |h| max, fragments, digit sums
      const char* src = reinterpret_cast<const char*>(p.hact + (int64_t)slot * K);
      float* xs = M.xs + (size_t)slot * K;
      const int nch = K / 8;
      uint4 rr[8];
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (lane + 32 * i < nch) rr[i] = ld_u4(src + (size_t)(lane + 32 * i) * 16);
      unsigned amax = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int c = lane + 32 * i;
        if (c < nch) {
          float v[8];
          widen_u4<kBF16>(rr[i], v);
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            xs[c * 8 + q] = v[q];
            amax = max(amax, __float_as_uint(v[q]) & 0x7fffffffu);
          }
        }
      }
#pragma unroll
      for (int m = 16; m >= 1; m >>= 1) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, m));
      sh = fxa_shift(amax);
      __syncwarp();
      int raws[4] = {0, 0, 0, 0};
      fxa_build<2>(xs, K, sh, sh == kFxaNonFinite, iters_total, M.frag + slot * frag_stride, lane, 32, raws);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int m = 16; m >= 1; m >>= 1) raws[j] += __shfl_xor_sync(0xffffffffu, raws[j], m);
        tot[j] = raws[j] - 64 * iters_total * 256;
      }
      __syncwarp();
    }
    first = false;
    tmark(S, 2);
    if (active) {
      int acc[4] = {0, 0, 0, 0};
      contract_tile2<kStepNI>(wa, wb, iters_total, M.frag + slot * frag_stride, lane, acc);
      long long Sg, Sh;
      combine_digits(acc, tot, t, Sg, Sh);
      if (t == 0) {
        const bool nan_out = bad || sh == kFxaNonFinite;
        const float nanv = __int_as_float(0x7fc00000);
        const float vg = nan_out ? nanv : fxa_value(Sg, sh);
        const float vh = nan_out ? nanv : fxa_value(Sh, sh);
        const float ag = row_g < N ? ldf(al, row_g, p.alpha_f32) : 0.f;
        const float ah = row_h < N ? ldf(al, row_h, p.alpha_f32) : 0.f;
        S.y[slot][g] = bf16_round(__fmul_rn(vg, ag));
        S.y[slot][g + 8] = bf16_round(__fmul_rn(vh, ah));
      }
    }
    __syncthreads();
    tmark(S, 3);
    if (tid < 16) {
      const int row = item * 16 + tid;
      if (row < N) {
        float acc2 = 0.0f;
        for (int sl = 0; sl < p.topk; ++sl) acc2 = __fmaf_rn(S.wts[sl], S.y[sl][tid], acc2);
        acc2 = __fadd_rn(acc2, bf16_to_f32(p.resid[row]));
        p.x[row] = f32_to_bf16(acc2);
      }
    }
    __syncthreads();
    tmark(S, 4);
  }
}

// -------------------------------------------------------------- router ----
// v = x + o; CTA 0 stores resid = bf16(v) and normed = bf16(v * rstd * w);
// logits[e] = R128 dot(bf16(normed), gate[e]) (router_kernel<FUSE>).  One
// item per CTA: 2 experts; warp (e_local = w / 4, q = w % 4) owns R128
// partials 32q + lane.  The norm weights and this CTA's gate rows were
// staged in shared memory before the barrier.
__device__ __forceinline__ void router_phase(StepShared& S, const StepSmem& M, const StepParams& p) {
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int K = p.H;
  const int n_items = (p.E + kRouterExpertsPerItem - 1) / kRouterExpertsPerItem;
  if ((int)blockIdx.x >= n_items) return;
  float* vs = M.xr;  // x + o, fp32
  float* xs = M.xs;  // bf16(normed), fp32
  const int nch = K / 8;
  uint4 rx[4], ro[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = tid + i * kStepThreads;
    if (c < nch) {
      rx[i] = ld_u4(reinterpret_cast<const char*>(p.x) + (size_t)c * 16);
      ro[i] = ld_u4(reinterpret_cast<const char*>(p.o) + (size_t)c * 16);
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = tid + i * kStepThreads;
    if (c < nch) {
      float a[8], b[8];
      widen_u4<kBF16>(rx[i], a);
      widen_u4<kBF16>(ro[i], b);
#pragma unroll
      for (int e = 0; e < 8; ++e) vs[c * 8 + e] = __fadd_rn(a[e], b[e]);
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
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = tid + i * kStepThreads;
    if (c < nch) {
      uint32_t rq[4], nq[4];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const int k = c * 8 + e;
        const float v = vs[k];
        const float nv = __fmul_rn(__fmul_rn(v, rstd), ldf(M.post_norm, k, p.norm_f32));
        const uint16_t nb = f32_to_bf16(nv);
        xs[k] = bf16_to_f32(nb);
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
  }
  __syncthreads();
  tmark(S, 3);
  const int el = warp / 4, q = warp % 4;
  const int e = blockIdx.x * kRouterExpertsPerItem + el;
  if (e < p.E) {
    const int j = 32 * q + lane;
    float pj = 0.0f;
#pragma unroll 4
    for (int k = j; k < K; k += 128) pj = __fmaf_rn(xs[k], ldf(M.gate, (int64_t)el * K + k, p.gate_f32), pj);
    S.part[el][j] = pj;
  }
  __syncthreads();
  if (q == 0 && e < p.E) {
    const float logit = r128_smem_finish(S.part[el], lane);
    if (lane == 0) p.logits[e] = logit;
  }
  tmark(S, 4);
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
__device__ __forceinline__ void norm_rope_head(const uint16_t (&raw)[D / 32], const void* nw, int norm_f32,
                                               const void* cs, const void* sn, int cs_f32, int use_rope, int R,
                                               float eps, float* dst) {
  constexpr int U = D / 32;
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
  const uint16_t* vt16 = reinterpret_cast<const uint16_t*>(vtile);
  float* scores = reinterpret_cast<float*>(M.att + 2 * (size_t)P * D * 2);  // [8][P]
  float* pb = scores + 8 * P;                                                 // [8][P]
  float* qs = pb + 8 * P;                                                     // [8][D]
  float* ks = qs + 8 * D;                                                     // [D]
  const int n_items = p.Hkv * a.ns;
  const float ninf = __int_as_float(0xff800000);
  const int use_rope = (int)w.use_rope;
  const bool store_ok = a.pos >= 0 && a.pos < p.T && a.cb_ok;
  bool first = true;
  for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
    const int h = item / a.ns, s = item % a.ns;
    const int t0 = a.start + s * P;
    const int n = min(P, a.kv_len - t0);
    const int n_pre = max(0, (int)min((int64_t)n, a.pos - t0));
    if (!first && tid == 0) attn_issue<D>(p, a, w, item, M.att, &S.bar_kv);
    first = false;
    const bool has_new = a.pos >= t0 && a.pos < (int64_t)t0 + n && store_ok;
    // loads first: q head of warp g < G, the new K (warp 0) and V (warp 1) rows
    uint16_t rq[U], rk[U], rv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      rq[u] = warp < G ? p.qkv[(h * G + warp) * D + lane + 32 * u] : 0;
      rk[u] = (warp == 0 && has_new) ? p.qkv[(p.Hq + h) * D + lane + 32 * u] : 0;
      rv[u] = (warp == 1 && has_new) ? p.qkv[(p.Hq + p.Hkv + h) * D + lane + 32 * u] : 0;
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
    // scores: warp w takes position groups of 4 (gqa_cluster_kernel)
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
            for (int u = 0; u < U; ++u) pj[u & 3] = __fmaf_rn(qs[gg * D + lane + 32 * u], kk[u], pj[u & 3]);
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
        pp[u] = (tt < n) ? mexp(__fsub_rn(sv[u], m)) : 0.0f;
        if (tt < P) pb[gg * P + tt] = (tt < n) ? bf16_round(pp[u]) : 0.0f;
      }
      const float l = r128_lane_finish(pp[0], pp[1], pp[2], pp[3]);
      __syncwarp();
      float acc[U];
#pragma unroll
      for (int u = 0; u < U; ++u) acc[u] = 0.0f;
      int tt = 0;
      for (; tt + 4 <= n; tt += 4) {
        float pq[4], vv[4][U];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          pq[i] = pb[gg * P + tt + i];
#pragma unroll
          for (int u = 0; u < U; ++u) vv[i][u] = bf16_to_f32(vt16[(size_t)(tt + i) * D + lane + 32 * u]);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int u = 0; u < U; ++u) acc[u] = __fmaf_rn(pq[i], vv[i][u], acc[u]);
      }
      for (; tt < n; ++tt) {
        const float pt = pb[gg * P + tt];
#pragma unroll
        for (int u = 0; u < U; ++u) acc[u] = __fmaf_rn(pt, bf16_to_f32(vt16[(size_t)tt * D + lane + 32 * u]), acc[u]);
      }
      const int hq = h * G + gg;
      if (a.ns == 1) {
#pragma unroll
        for (int u = 0; u < U; ++u) p.attn[hq * D + lane + 32 * u] = f32_to_bf16(__fdiv_rn(acc[u], l));
      } else {
        float* wa = p.att_acc + ((int64_t)hq * p.NS + s) * D;
#pragma unroll
        for (int u = 0; u < U; ++u) wa[lane + 32 * u] = acc[u];
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
          float mj[8], lj[8], aj[8][U];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int j = j0 + i;
            if (j < a.ns) {
              mj[i] = __ldcg(ml + 2 * j);
              lj[i] = __ldcg(ml + 2 * j + 1);
#pragma unroll
              for (int u = 0; u < U; ++u) aj[i][u] = __ldcg(ac + (int64_t)j * D + lane + 32 * u);
            }
          }
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            if (j0 + i < a.ns) {
              const float wgt = mexp(__fsub_rn(mj[i], M2));
              den = __fmaf_rn(wgt, lj[i], den);
#pragma unroll
              for (int u = 0; u < U; ++u) num[u] = __fmaf_rn(wgt, aj[i][u], num[u]);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) p.attn[hq * D + lane + 32 * u] = f32_to_bf16(__fdiv_rn(num[u], den));
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
    // 1: RMSNorm -> QKV
    phase_marks(l, 0);
    wait_stage(p, &S.bar_in, ph_in);
    dense_gemv<4>(S, M, p.x, M.in_norm, p.norm_f32, p.eps, w.qkv_codes, w.qkv_alpha, p.alpha_f32, p.qkv,
               (p.Hq + 2 * p.Hkv) * D, p.H, p.wm_qkv);
    tmark(S, 7);
    if (!grid_barrier(p, epoch, &S.ok, next_tr())) break;
    // 2: attention (first item's final rows are in flight since the previous layer)
    phase_marks(l, 1);
    wait_stage(p, &S.bar_st, ph_st);
    attention_phase<D>(S, M, p, w, ag, ph_kv);
    tmark(S, 7);
    if (!grid_barrier(p, epoch, &S.ok, next_tr())) break;
    // 3: O projection
    phase_marks(l, 2);
    dense_gemv<4>(S, M, p.attn, nullptr, p.norm_f32, 0.0f, w.o_codes, w.o_alpha, p.alpha_f32, p.o, p.H, p.Hq * D,
               p.wm_o);
    tmark(S, 7);
    if (!grid_barrier(p, epoch, &S.ok, next_tr())) break;
    // 4: residual add + RMSNorm + router logits; the next layer's dense
    // weights into L2 once this CTA is done
    phase_marks(l, 3);
    router_phase(S, M, p);
    if (l + 1 < p.n_layers) prefetch_layer_dense(p, L[l + 1]);
    tmark(S, 7);
    if (!grid_barrier(p, epoch, &S.ok, next_tr())) break;
    // 5: top-k (every CTA), down rows of the selected experts into L2, SwiGLU
    phase_marks(l, 4);
    swiglu_phase(S, M, p, w);
    tmark(S, 7);
    if (!grid_barrier(p, epoch, &S.ok, next_tr())) break;
    // 6: down + combine + residual -> x; then the next layer's staging copies
    phase_marks(l, 5);
    down_phase(S, M, p, w);
    if (l + 1 < p.n_layers && tid == kLast) stage_layer<D>(S, p, M, L[l + 1], attn_geom(p, (int)L[l + 1].window));
    tmark(S, 7);
    if (l + 1 < p.n_layers && !grid_barrier(p, epoch, &S.ok, next_tr())) break;
  }
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
  int64_t qkv, attn, o, resid, normed, hact, logits, acc, ml, trace, total;
  int off_frag, off_xs, off_xr, off_att, off_layers, off_in, off_post, off_qn, off_kn, off_cos, off_sin, off_gate, smem;
};

StepLayout step_layout(int64_t H, int64_t Hq, int64_t Hkv, int64_t D, int64_t E, int64_t topk, int64_t I,
                       int64_t NS, int64_t P, int64_t R, int64_t n_layers) {
  StepLayout L{};
  int64_t off = kStepSyncBytes;
  L.qkv = off; off = align256(off + (Hq + 2 * Hkv) * D * 2);
  L.attn = off; off = align256(off + Hq * D * 2);
  L.o = off; off = align256(off + H * 2);
  L.resid = off; off = align256(off + H * 2);
  L.normed = off; off = align256(off + H * 2);
  L.hact = off; off = align256(off + topk * I * 2);
  L.logits = off; off = align256(off + E * 4);
  L.acc = off; off = align256(off + Hq * NS * D * 4);
  L.ml = off; off = align256(off + Hq * NS * 2 * 4);
  L.trace = off; off = align256(off + kStepTraceBytes);
  L.total = off;
  auto iters = [](int64_t K) { return (K / 16 + 15) / 16; };
  auto a128 = [](int64_t v) { return (v + 127) & ~int64_t(127); };
  const int64_t frag = std::max(std::max(iters(H), iters(Hq * D)) * 2048, topk * iters(I) * 2048);
  const int64_t xs = std::max(std::max(H, Hq * D), topk * I);
  const int64_t xr = std::max(H, Hq * D);
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

// Row tiles per item: the fewest that cover N within one wave of CTAs while
// each warp's K slice stays within max_ni register iterations.
int pick_wm(int64_t N, int64_t K, int grid, int min_wm, int rows_per_tile, int max_ni) {
  const int64_t it = (K / 16 + 15) / 16;
  int best = -1;
  for (int wm = min_wm; wm <= kStepWarps; wm *= 2) {
    const int wk = kStepWarps / wm;
    if ((it + wk - 1) / wk > max_ni) continue;
    if (best < 0) best = wm;
    const int64_t items = (N + (int64_t)rows_per_tile * wm - 1) / ((int64_t)rows_per_tile * wm);
    if (items <= grid) return wm;
    best = wm;
  }
  return best;
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
  p.wm_qkv = pick_wm((num_heads + 2 * num_kv_heads) * head_dim, hidden, grid, 1, 16, 4);
  p.wm_o = pick_wm(hidden, num_heads * head_dim, grid, 1, 16, 4);
  p.wm_sw = pick_wm(topk * inter, hidden, grid, 2, 8, kStepNI);
  if (p.wm_qkv < 0 || p.wm_o < 0 || p.wm_sw < 0) return kErrShape;
  char* ws = static_cast<char*>(workspace);
  p.qkv = reinterpret_cast<uint16_t*>(ws + L.qkv);
  p.attn = reinterpret_cast<uint16_t*>(ws + L.attn);
  p.o = reinterpret_cast<uint16_t*>(ws + L.o);
  p.resid = reinterpret_cast<uint16_t*>(ws + L.resid);
  p.normed = reinterpret_cast<uint16_t*>(ws + L.normed);
  p.hact = reinterpret_cast<uint16_t*>(ws + L.hact);
  p.logits = reinterpret_cast<float*>(ws + L.logits);
  p.att_acc = reinterpret_cast<float*>(ws + L.acc);
  p.att_ml = reinterpret_cast<float*>(ws + L.ml);
  p.sync = reinterpret_cast<unsigned*>(ws);
  // timestamps of every barrier (opt-in through sync word 2) when they fit
  p.trace = (n_layers * 6 * 2 * (int64_t)grid * 8 <= kStepTraceBytes) ? reinterpret_cast<int64_t*>(ws + L.trace)
                                                                      : nullptr;
  p.trace_bytes = kStepTraceBytes;
  p.att_tickets = reinterpret_cast<unsigned*>(ws + 256);
  p.err = err;
  p.off_frag = L.off_frag; p.off_xs = L.off_xs; p.off_xr = L.off_xr; p.off_att = L.off_att;
  p.off_layers = L.off_layers; p.off_in = L.off_in; p.off_post = L.off_post; p.off_qn = L.off_qn;
  p.off_kn = L.off_kn; p.off_cos = L.off_cos; p.off_sin = L.off_sin; p.off_gate = L.off_gate;
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
