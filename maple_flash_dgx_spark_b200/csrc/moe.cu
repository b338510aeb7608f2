// MoE router and expert combine.
//
// router_topk      reference kernels/router.py:141-217 (kernels :20-126)
// expert down+sum  reference kernels/ternary_expert.py:125-234 (down GEMV) followed
//                  by kernels/fused_norm.py:164-202 (moe_reduce_add), fused; and
//                  ternary_expert_down_sum (ternary_expert.py:471-556)
// moe_reduce_add   reference kernels/fused_norm.py:164-202
#include <cooperative_groups.h>

#include "bulk.cuh"
#include "fxa.cuh"
#include "launch.cuh"

namespace mb {

namespace cg = cooperative_groups;

// Thread-block cluster barrier halves (every thread of every CTA executes them).
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

constexpr int kTicketBytesMoe = 1 << 20;

// ----------------------------------------------------------------- router --
// Logits: one warp per (token, expert), R128 order over K (products x*g added
// with fmaf).  One CTA of a token then runs softmax, top-k by repeated argmax
// (ties -> lowest index), and the 1/(sum+1e-20) renorm: with CL (at most 8
// CTAs per token, one thread-block cluster) the CTAs write their logits into
// cluster rank 0's shared memory and rank 0 continues after a cluster
// barrier; otherwise the logits go through global scratch and the last CTA
// to take the token's ticket continues.
struct RouterParams {
  const void* x;       // [T, K]
  const void* gate;    // [E, K]
  int32_t* idx;        // [T, topk]
  float* wt;           // [T, topk]
  float* logits;       // [T, E] scratch
  unsigned* tickets;   // [T]
  // Fused residual add + RMSNorm in front of the router (FUSE): x is the
  // residual stream, y the attention output; every CTA forms v = x + y and
  // the normed row in the add_rms_norm kernel's order, CTA 0 of a token
  // writes residual_out = v and normed_out, and the logits use the normed row.
  const void* y;
  const void* norm_w;
  void* residual_out;
  void* normed_out;
  int64_t x_stride;
  int E, K, topk, norm_w_bf16;
  float eps;
};

constexpr int kRouterWarps = 8;

template <int XT, int GT, bool FUSE, bool CL>
__global__ void __launch_bounds__(256) router_kernel(RouterParams p) {
  extern __shared__ __align__(16) unsigned char rsm[];  // x as fp32 [K] | gate rows raw [8][K] | (FUSE) y, w [K]
  constexpr int kMaxE = 256;
  __shared__ float s_logit[kMaxE];  // CL: every expert's logit (rank 0's copy is filled)
  __shared__ int s_last;
  __shared__ float s_part[128];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int tok = blockIdx.y;
  const int e0 = blockIdx.x * kRouterWarps;
  if constexpr (CL) cluster_arrive_relaxed();  // this CTA has started
  // gate rows are weights: loaded before waiting for the activation
  const int ne = min(kRouterWarps, p.E - e0);
  const int ges = GT == kBF16 ? 2 : 4;
  float* xs = reinterpret_cast<float*>(rsm);
  unsigned char* gs = rsm + (size_t)p.K * sizeof(float);
  // Gate rows of this CTA's experts (contiguous), 16-byte loads issued together.
  {
    const char* gsrc = static_cast<const char*>(p.gate) + (int64_t)e0 * p.K * ges;
    const int nbytes = ne * p.K * ges;
    const bool vec = ((reinterpret_cast<uintptr_t>(gsrc) & 15) == 0) && (nbytes % 16 == 0);
    if (vec) {
      const int nch = nbytes / 16;
      uint4 r[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) if (tid + 256 * i < nch) r[i] = ld_stream_u4(gsrc + (size_t)(tid + 256 * i) * 16);
#pragma unroll
      for (int i = 0; i < 8; ++i) if (tid + 256 * i < nch) *reinterpret_cast<uint4*>(gs + (size_t)(tid + 256 * i) * 16) = r[i];
      for (int c = tid + 2048; c < nch; c += 256) *reinterpret_cast<uint4*>(gs + (size_t)c * 16) = ld_stream_u4(gsrc + (size_t)c * 16);
    } else {
      for (int b = tid; b < nbytes; b += 256) gs[b] = gsrc[b];
    }
  }
  float* ys = reinterpret_cast<float*>(gs + (size_t)kRouterWarps * p.K * ges);
  float* ws = ys + p.K;
  if constexpr (FUSE) {
    if (p.norm_w_bf16) stage_row<kBF16, 256, 4>(p.norm_w, p.K, ws, tid);
    else stage_row<kF32, 256, 4>(p.norm_w, p.K, ws, tid);
  }
  pdl_wait();
  pdl_trigger();
  const int es = XT == kBF16 ? 2 : 4;
  const char* xr = static_cast<const char*>(p.x) + tok * p.x_stride * es;
  if constexpr (FUSE) {
    // v = x + y straight from the two rows: thread j < 128 owns elements j,
    // j + 128, ... (its R128 sum-of-squares partial, in order) and keeps v in
    // xs; after one barrier every warp finishes the R128 sum itself.
    (void)ys;
    const char* yr = static_cast<const char*>(p.y) + tok * p.x_stride * es;
    if (tid < 128) {
      float ss = 0.0f;
      for (int k0 = tid; k0 < p.K; k0 += 128 * 16) {  // one memory round trip for K <= 2048
        float xv[16], yv[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int k = k0 + 128 * u;
          xv[u] = k < p.K ? load_f<XT>(xr, k) : 0.0f;
          yv[u] = k < p.K ? load_f<XT>(yr, k) : 0.0f;
        }
#pragma unroll
        for (int u = 0; u < 16; ++u) {
          const int k = k0 + 128 * u;
          if (k < p.K) {
            const float v = __fadd_rn(xv[u], yv[u]);
            ss = __fmaf_rn(v, v, ss);
            xs[k] = v;
          }
        }
      }
      s_part[tid] = ss;
    }
    __syncthreads();
    const float rstd = rstd_of(r128_smem_finish(s_part, lane), p.K, p.eps);
    char* res = static_cast<char*>(p.residual_out) + tok * p.x_stride * es;
    char* nrm = static_cast<char*>(p.normed_out) + tok * p.x_stride * es;
    for (int k = tid; k < p.K; k += 256) {
      const float v = xs[k];
      const float nv = __fmul_rn(__fmul_rn(v, rstd), ws[k]);
      float nq = nv;
      if constexpr (XT == kBF16) nq = bf16_to_f32(f32_to_bf16(nv));
      if (blockIdx.x == 0) {
        store_f<XT>(res, k, v);
        store_f<XT>(nrm, k, nv);
      }
      xs[k] = nq;  // the router reads the stored (rounded) normed row
    }
    __syncthreads();
  } else {
    stage_row<XT, 256, 2>(xr, p.K, xs, tid);
    __syncthreads();
  }
  if constexpr (CL) cluster_wait_acquire();  // every CTA of the cluster has started
  if (warp < ne) {
    const unsigned char* gr = gs + (size_t)warp * p.K * ges;
    // Lane l owns R128 partials j = l + 32u (elements j, j+128, ...).
    float pj[4] = {0.f, 0.f, 0.f, 0.f};
    for (int c = 0; c < p.K; c += 128) {
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int k = c + lane + 32 * u;
        if (k < p.K) pj[u] = __fmaf_rn(xs[k], load_f<GT>(gr, k), pj[u]);
      }
    }
    const float logit = r128_lane_finish(pj[0], pj[1], pj[2], pj[3]);
    if (lane == 0) {
      if constexpr (CL) *cg::this_cluster().map_shared_rank(&s_logit[e0 + warp], 0) = logit;
      else p.logits[(int64_t)tok * p.E + e0 + warp] = logit;
    }
  }
  if constexpr (CL) {
    cluster_arrive_release();
    cluster_wait_acquire();
    if (blockIdx.x != 0) return;
  } else {
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const unsigned old = atomicAdd(&p.tickets[tok], 1u);
      s_last = (old == gridDim.x - 1);
      if (s_last) atomicExch(&p.tickets[tok], 0u);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
  }
  // Softmax on warp 0 (lane l holds experts l + 32i), then the top-k: the
  // order in which repeated argmax (largest first, ties to the lowest index,
  // NaN never) would pick the experts is each expert's rank, computed by one
  // thread per expert.
  __shared__ float s_prob[kMaxE];
  __shared__ float s_sel_p[32];
  __shared__ int s_sel_i[32];
  const float ninf = __int_as_float(0xff800000);
  if (warp == 0) {
    float v[kMaxE / 32];
    float m = ninf;
#pragma unroll
    for (int i = 0; i < kMaxE / 32; ++i) {
      const int ee = lane + 32 * i;
      if constexpr (CL) v[i] = ee < p.E ? s_logit[ee] : ninf;
      else v[i] = ee < p.E ? __ldcg(&p.logits[(int64_t)tok * p.E + ee]) : ninf;
      m = fmaxf(m, v[i]);
    }
    m = warp_max(m);
    // R128 sum of exp: partial j = expert j, j+128 (sequential).
    float q0 = 0.f, q1 = 0.f, q2 = 0.f, q3 = 0.f;
#pragma unroll
    for (int i = 0; i < kMaxE / 32; ++i) {
      const int ee = lane + 32 * i;
      v[i] = ee < p.E ? mexp(__fsub_rn(v[i], m)) : 0.0f;
      const int j = (i & 3);
      if (j == 0) q0 = __fadd_rn(q0, v[i]);
      if (j == 1) q1 = __fadd_rn(q1, v[i]);
      if (j == 2) q2 = __fadd_rn(q2, v[i]);
      if (j == 3) q3 = __fadd_rn(q3, v[i]);
    }
    const float sum = r128_lane_finish(q0, q1, q2, q3);
#pragma unroll
    for (int i = 0; i < kMaxE / 32; ++i) {
      const int ee = lane + 32 * i;
      if (ee < p.E) s_prob[ee] = __fdiv_rn(v[i], sum);
    }
    s_sel_p[lane] = ninf;        // picks past the last finite expert: (-inf, INT_MAX)
    s_sel_i[lane] = 0x7fffffff;
  }
  __syncthreads();
  if (tid < p.E) {
    const float pi = s_prob[tid];
    if (pi == pi) {
      int rank = 0;
#pragma unroll 8
      for (int j = 0; j < p.E; ++j) {
        const float pj = s_prob[j];
        rank += (pj > pi || (pj == pi && j < tid)) ? 1 : 0;
      }
      if (rank < p.topk) {
        s_sel_p[rank] = pi;
        s_sel_i[rank] = tid;
      }
    }
  }
  __syncthreads();
  if (warp == 0) {
    float total = 0.0f;
    for (int r = 0; r < p.topk; ++r) total = __fadd_rn(total, s_sel_p[r]);
    const float inv = __fdiv_rn(1.0f, __fadd_rn(total, 1e-20f));
    if (lane < p.topk) {
      p.idx[(int64_t)tok * p.topk + lane] = s_sel_i[lane];
      p.wt[(int64_t)tok * p.topk + lane] = __fmul_rn(s_sel_p[lane], inv);
    }
  }
}

// ------------------------------------------------------- expert down + sum --
// One CTA per (16-row tile, token); warp s contracts top-k slot s's expert
// rows against that slot's activation h[t, s, :].  MODE 0 (model path, same
// rounding as ternary_expert_gemv + moe_reduce_add): y_s = bf16(alpha * S_s),
// out = bf16(fmaf-chain_s(w_s, y_s) + residual).  MODE 1
// (ternary_expert_down_sum): acc = fmaf(w_s * S_s, alpha, acc), no bf16 y_s.
struct DownParams {
  const void* h;          // [T, topk, K]
  const int32_t* ids;     // [T, topk]
  const float* wt;        // [T, topk]
  const uint32_t* codes;  // [E, N, K/16]
  const void* alpha;      // [E, N]
  const void* residual;   // [T, N] or nullptr
  void* out;              // [T, N]
  int64_t h_tok_stride, h_slot_stride, res_stride, out_stride;
  int E, N, K, nwords, topk, iters;
  int* err;               // device error word; non-null: expert rows staged by bulk copies
};

constexpr int kDownMaxIters = 8;
constexpr int kDownMaxTopk = 8;

// NI: K iterations held in registers (K <= 256 * NI).  The smaller
// instantiation (K <= 1024) needs few enough registers for a CTA to become
// resident beside two CTAs of the SwiGLU launch it follows, so it starts (and
// loads its expert rows) before that launch ends.
template <int XT, int AT, int MODE, int NI>
__global__ void __launch_bounds__(256, NI == 4 ? 3 : 1) down_sum_kernel(DownParams p) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ float s_y[kDownMaxTopk][16];
  __shared__ float s_a[kDownMaxTopk][16];  // MODE 1: the slots' row scales
  __shared__ float s_w[kDownMaxTopk];      // MODE 0: the slots' combine weights
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float res = 0.0f;  // residual of row tid (warp 0, lanes < 16)
  const int g = lane >> 2, t = lane & 3;
  const int tok = blockIdx.y;
  const int row_g = blockIdx.x * 16 + g, row_h = row_g + 8;
  // Per warp: the compact digit fragments of its slot row (fxa.cuh, direct
  // form), then (bulk) its expert's 16 code rows of this tile.  The rows are
  // one contiguous 16 x K/4-byte block that one bulk copy brings in whole:
  // per-thread 16-byte loads of them stall at issue while the SwiGLU launch
  // this one overlaps still holds the SM's outstanding requests.
  __shared__ uint64_t wbar[kDownMaxTopk];
  const bool bulk = p.err != nullptr;
  const unsigned rowb = (unsigned)p.nwords * 4u;
  const size_t per_warp = (size_t)p.iters * 128 * sizeof(uint2) + (bulk ? (size_t)16 * rowb : 0);
  uint2* frag = reinterpret_cast<uint2*>(smem + warp * per_warp);
  unsigned char* wtile = smem + warp * per_warp + (size_t)p.iters * 128 * sizeof(uint2);

  // Routing ids come from two launches back (complete once the previous
  // launch has passed its own wait), so the expert rows load before waiting.
  if (warp < p.topk) {
    int e = __ldcg(&p.ids[(int64_t)tok * p.topk + warp]);
    const bool bad = (e < 0 || e >= p.E);
    if (bad) e = 0;
    const uint32_t* codes = p.codes + (int64_t)e * p.N * p.nwords;
    const int row0 = blockIdx.x * 16, nrows = min(16, p.N - row0);
    if (bulk) {
      if (lane == 0) {
        mbar_init(&wbar[warp], 1);
        mbar_expect_tx(&wbar[warp], (unsigned)nrows * rowb);
        bulk_g2s(wtile, codes + (int64_t)row0 * p.nwords, (unsigned)nrows * rowb, &wbar[warp]);
      }
      __syncwarp();
    }
    uint4 wa[NI], wb[NI];
#pragma unroll
    for (int i = 0; i < NI; ++i) {
      wa[i] = make_uint4(0, 0, 0, 0);
      wb[i] = make_uint4(0, 0, 0, 0);
      const int word = i * 16 + 4 * t;
      if (!bulk && i < p.iters && word < p.nwords) {
        if (row_g < p.N) wa[i] = ld_stream_u4(codes + (int64_t)row_g * p.nwords + word);
        if (row_h < p.N) wb[i] = ld_stream_u4(codes + (int64_t)row_h * p.nwords + word);
      }
    }
    // The slot's row scales and combine weight come with the ids (static
    // weights / the router's output), so they load before the wait too.
    const void* al = static_cast<const char*>(p.alpha) + (int64_t)e * p.N * (AT == kBF16 ? 2 : 4);
    float ag = 0.0f, ah = 0.0f;
    if (t == 0) {
      if (row_g < p.N) ag = load_f<AT>(al, row_g);
      if (row_h < p.N) ah = load_f<AT>(al, row_h);
    }
    const float w = __ldcg(&p.wt[(int64_t)tok * p.topk + warp]);
    pdl_wait();
    // the residual row is read right after the wait, beside the activations
    if (warp == 0 && lane < 16 && p.residual != nullptr) {
      const int row = blockIdx.x * 16 + lane;
      if (row < p.N)
        res = load_f<XT>(static_cast<const char*>(p.residual) + tok * p.res_stride * (XT == kBF16 ? 2 : 4), row);
    }
    const void* hr = static_cast<const char*>(p.h) +
                     (tok * p.h_tok_stride + warp * p.h_slot_stride) * (XT == kBF16 ? 2 : 4);
    // Direct FXA prologue on one warp: lane l owns the 16-value blocks l,
    // l + 32, ... of the slot row in registers; the warp max gives the shift
    // and each lane writes its blocks' digit fragments (same digits, shift and
    // totals as fxa_warp_prologue2).
    constexpr int MAXB = NI / 2;  // K <= NI * 256 values = NI * 16 blocks over 32 lanes
    uint4 xb[MAXB][XBlk<XT>::kChunks];
    xblk_issue<XT, 32, MAXB>(hr, p.K, lane, xb);
    unsigned am = 0;
#pragma unroll
    for (int i = 0; i < MAXB; ++i) {
      if (lane + 32 * i < (p.K >> 4)) {
        float v[16];
        xblk_values<XT>(xb[i], v);
#pragma unroll
        for (int q = 0; q < 16; ++q) am = max(am, __float_as_uint(v[q]) & 0x7fffffffu);
      }
    }
    const int s = fxa_shift(__reduce_max_sync(0xffffffffu, am));
    int tot[4] = {0, 0, 0, 0};
#pragma unroll
    for (int i = 0; i < MAXB; ++i) {
      const int b = lane + 32 * i;
      if (b < (p.K >> 4)) {
        float v[16];
        xblk_values<XT>(xb[i], v);
        fxa_block_encode(v, b, s, s == kFxaNonFinite, frag, tot);
      }
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) tot[j] = __reduce_add_sync(0xffffffffu, tot[j]) - 64 * p.K;
    bool lost = false;  // bulk rows that never landed: reported, the slot's rows become NaN
    if (bulk) {
      const bool ready = mbar_wait_bounded(&wbar[warp], 0);
      if (!ready) {
        lost = true;
        if (lane == 0) atomicOr(p.err, kErrFlagTimeout);
        mbar_wait_bounded(&wbar[warp], 0);  // let the copy land before the CTA can exit
      } else {
#pragma unroll
        for (int i = 0; i < NI; ++i) {
          const int word = i * 16 + 4 * t;
          if (i < p.iters && word < p.nwords) {
            if (g < nrows) wa[i] = *reinterpret_cast<const uint4*>(wtile + (size_t)g * rowb + 4 * word);
            if (g + 8 < nrows) wb[i] = *reinterpret_cast<const uint4*>(wtile + (size_t)(g + 8) * rowb + 4 * word);
          }
        }
      }
    }
    __syncwarp();
    int acc[4] = {0, 0, 0, 0};
    contract_tile2c<NI>(wa, wb, p.iters, frag, lane, acc);
    long long Sg, Sh;
    combine_digits(acc, tot, t, Sg, Sh);
    if (t == 0) {
      const bool nan_out = bad || lost || s == kFxaNonFinite;
      const float nanv = __int_as_float(0x7fc00000);
      const float vg = nan_out ? nanv : fxa_value(Sg, s);
      const float vh = nan_out ? nanv : fxa_value(Sh, s);
      if constexpr (MODE == 0) {
        // the expert output is stored in the activation dtype before the combine
        float yg = __fmul_rn(vg, ag), yh = __fmul_rn(vh, ah);
        if constexpr (XT == kBF16) {
          yg = bf16_to_f32(f32_to_bf16(yg));
          yh = bf16_to_f32(f32_to_bf16(yh));
        }
        s_y[warp][g] = yg;
        s_y[warp][g + 8] = yh;
        if (lane == 0) s_w[warp] = w;
      } else {
        // alpha is applied in the combine below: acc = fmaf(w*S, alpha, acc)
        s_y[warp][g] = __fmul_rn(w, vg);
        s_y[warp][g + 8] = __fmul_rn(w, vh);
        s_a[warp][g] = ag;
        s_a[warp][g + 8] = ah;
      }
    }
  }
  pdl_wait();
  pdl_trigger();
  __syncthreads();
  if (tid < 16) {
    const int row = blockIdx.x * 16 + tid;
    if (row < p.N) {
      float acc = 0.0f;
      for (int sl = 0; sl < p.topk; ++sl) {
        if constexpr (MODE == 0) acc = __fmaf_rn(s_w[sl], s_y[sl][tid], acc);
        else acc = __fmaf_rn(s_y[sl][tid], s_a[sl][tid], acc);
      }
      if (p.residual != nullptr) acc = __fadd_rn(acc, res);
      store_f<XT>(static_cast<char*>(p.out) + tok * p.out_stride * (XT == kBF16 ? 2 : 4), row, acc);
    }
  }
}

// ------------------------------------------------------------ moe reduce --
template <int XT>
__global__ void moe_reduce_kernel(const void* x, const float* w, const void* residual, void* y,
                                  int64_t x_tok_stride, int64_t x_slot_stride, int64_t res_stride,
                                  int64_t y_stride, int N, int topk) {
  pdl_wait();
  pdl_trigger();
  const int tok = blockIdx.y;
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const int es = XT == kBF16 ? 2 : 4;
  float acc = 0.0f;
  for (int s = 0; s < topk; ++s)
    acc = __fmaf_rn(w[(int64_t)tok * topk + s],
                    load_f<XT>(static_cast<const char*>(x) + (tok * x_tok_stride + s * x_slot_stride) * es, n),
                    acc);
  if (residual != nullptr)
    acc = __fadd_rn(acc, load_f<XT>(static_cast<const char*>(residual) + tok * res_stride * es, n));
  store_f<XT>(static_cast<char*>(y) + tok * y_stride * es, n, acc);
}

}  // namespace mb

using namespace mb;

extern "C" int64_t maple_router_topk_workspace_bytes(int64_t tokens, int64_t n_experts) {
  return kTicketBytesMoe + tokens * n_experts * (int64_t)sizeof(float);
}

// Cluster variants get a (grid.x, 1, 1) cluster per token; the others launch
// plainly.  Both with PDL.
static void launch_router(void (*kern)(RouterParams), bool cl, dim3 grid, size_t smem, cudaStream_t st,
                          const RouterParams& p) {
  if (smem > 32 * 1024) cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (!cl) {
    launch_k(kern, grid, dim3(256), smem, st, p);
    return;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = grid.x;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl_enabled() ? 2 : 1;
  cudaLaunchKernelEx(&cfg, kern, p);
}

static int router_common(const void* x, int x_dtype, int64_t x_row_stride, int64_t tokens, int64_t k,
                         const void* gate, int gate_dtype, int64_t n_experts, int64_t topk, int32_t* idx, float* wt,
                         void* workspace, int64_t workspace_bytes, const void* y, const void* norm_w,
                         int norm_dtype, float eps, void* residual_out, void* normed_out, void* stream) {
  if (tokens < 0 || k <= 0 || n_experts <= 0 || topk <= 0) return kErrShape;
  if (tokens == 0) return kOk;
  if (topk > n_experts || topk > 32 || n_experts > 256) return kErrShape;
  if ((x_dtype != kF32 && x_dtype != kBF16) || (gate_dtype != kF32 && gate_dtype != kBF16)) return kErrDtype;
  if (!x || !gate || !idx || !wt) return kErrShape;
  if (tokens * (int64_t)sizeof(unsigned) > kTicketBytesMoe || tokens > 65535) return kErrShape;
  if (!workspace || workspace_bytes < maple_router_topk_workspace_bytes(tokens, n_experts)) return kErrWorkspace;
  RouterParams p{};
  p.x = x; p.gate = gate; p.idx = idx; p.wt = wt;
  p.tickets = static_cast<unsigned*>(workspace);
  p.logits = reinterpret_cast<float*>(static_cast<char*>(workspace) + kTicketBytesMoe);
  p.x_stride = x_row_stride; p.E = (int)n_experts; p.K = (int)k; p.topk = (int)topk;
  p.y = y; p.norm_w = norm_w; p.norm_w_bf16 = norm_dtype == kBF16; p.eps = eps;
  p.residual_out = residual_out; p.normed_out = normed_out;
  if (y != nullptr) {
    if (!norm_w || !residual_out || !normed_out) return kErrShape;
    if (norm_dtype != kF32 && norm_dtype != kBF16) return kErrDtype;
  }
  dim3 grid((unsigned)((n_experts + kRouterWarps - 1) / kRouterWarps), (unsigned)tokens);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool fuse = p.y != nullptr;
  const size_t smem = (size_t)k * sizeof(float) + (size_t)kRouterWarps * k * (gate_dtype == kBF16 ? 2 : 4) +
                      (fuse ? 2 * (size_t)k * sizeof(float) : 0);
  if (smem > 200 * 1024) return kErrShape;
  // At most 8 CTAs per token (64 experts): one portable cluster per token.
  const bool cl = grid.x <= 8;
#define MB_ROUTER(XT, GT)                                                                                       \
  do {                                                                                                          \
    if (fuse) {                                                                                                 \
      if (cl) launch_router(router_kernel<XT, GT, true, true>, true, grid, smem, st, p);                             \
      else launch_router(router_kernel<XT, GT, true, false>, false, grid, smem, st, p);                               \
    } else {                                                                                                    \
      if (cl) launch_router(router_kernel<XT, GT, false, true>, true, grid, smem, st, p);                            \
      else launch_router(router_kernel<XT, GT, false, false>, false, grid, smem, st, p);                              \
    }                                                                                                           \
  } while (0)
  if (x_dtype == kBF16) {
    if (gate_dtype == kBF16) MB_ROUTER(kBF16, kBF16); else MB_ROUTER(kBF16, kF32);
  } else {
    if (gate_dtype == kBF16) MB_ROUTER(kF32, kBF16); else MB_ROUTER(kF32, kF32);
  }
#undef MB_ROUTER
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_router_topk(const void* x, int x_dtype, int64_t x_row_stride, int64_t tokens,
                                 int64_t k, const void* gate, int gate_dtype, int64_t n_experts,
                                 int64_t topk, int32_t* idx, float* wt, void* workspace,
                                 int64_t workspace_bytes, void* stream) {
  return router_common(x, x_dtype, x_row_stride, tokens, k, gate, gate_dtype, n_experts, topk, idx, wt, workspace,
                       workspace_bytes, nullptr, nullptr, 0, 0.0f, nullptr, nullptr, stream);
}

extern "C" int maple_add_norm_router_topk(const void* x, const void* y, int x_dtype, int64_t row_stride,
                                          int64_t tokens, int64_t k, const void* norm_w, int norm_dtype, float eps,
                                          const void* gate, int gate_dtype, int64_t n_experts, int64_t topk,
                                          void* residual_out, void* normed_out, int32_t* idx, float* wt,
                                          void* workspace, int64_t workspace_bytes, void* stream) {
  if (!y) return kErrShape;
  return router_common(x, x_dtype, row_stride, tokens, k, gate, gate_dtype, n_experts, topk, idx, wt, workspace,
                       workspace_bytes, y, norm_w, norm_dtype, eps, residual_out, normed_out, stream);
}

namespace {
template <int XT, int AT, int MODE>
cudaError_t launch_down(const DownParams& p, int T, cudaStream_t st) {
  // compact fragments (+ the bulk-staged code rows)
  const size_t per_warp = (size_t)p.iters * 128 * sizeof(uint2) + (p.err ? (size_t)16 * p.nwords * 4 : 0);
  const size_t smem = per_warp * kDownMaxTopk;
  auto kern = p.iters <= 4 ? down_sum_kernel<XT, AT, MODE, 4> : down_sum_kernel<XT, AT, MODE, kDownMaxIters>;
  if (smem > 32 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  // whole carveout: room beside the expert SwiGLU CTAs this launch overlaps
  cudaError_t ce = cudaFuncSetAttribute(kern, cudaFuncAttributePreferredSharedMemoryCarveout,
                                        cudaSharedmemCarveoutMaxShared);
  if (ce != cudaSuccess) return ce;
  dim3 grid((p.N + 15) / 16, T);
  launch_k(kern, dim3(grid), dim3(256), smem, st, p);
  return cudaGetLastError();
}

template <int MODE>
int down_entry(const void* h, int h_dtype, int64_t h_tok_stride, int64_t h_slot_stride,
               const int32_t* ids, const float* wt, int64_t tokens, int64_t topk, int64_t k,
               const uint32_t* codes, int64_t n_experts, int64_t n, const void* alpha,
               int alpha_dtype, const void* residual, int64_t res_stride, void* out,
               int64_t out_stride, int* err, void* stream) {
  if (tokens < 0 || topk <= 0 || k <= 0 || n < 0 || n_experts <= 0) return kErrShape;
  if (tokens == 0 || n == 0) return kOk;
  if (topk > kDownMaxTopk || k % 64 != 0 || k > kDownMaxIters * 256 || tokens > 65535) return kErrShape;
  if ((h_dtype != kF32 && h_dtype != kBF16) || (alpha_dtype != kF32 && alpha_dtype != kBF16)) return kErrDtype;
  if (!h || !ids || !wt || !codes || !alpha || !out) return kErrShape;
  if ((reinterpret_cast<uintptr_t>(codes) & 15) != 0) return kErrAlign;
  DownParams p{};
  p.h = h; p.ids = ids; p.wt = wt; p.codes = codes; p.alpha = alpha; p.residual = residual; p.out = out;
  p.h_tok_stride = h_tok_stride; p.h_slot_stride = h_slot_stride; p.res_stride = res_stride;
  p.out_stride = out_stride; p.E = (int)n_experts; p.N = (int)n; p.K = (int)k; p.nwords = (int)(k / 16);
  p.topk = (int)topk; p.iters = (int)((k + 255) / 256); p.err = err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (h_dtype == kBF16)
    e = alpha_dtype == kBF16 ? launch_down<kBF16, kBF16, MODE>(p, (int)tokens, st)
                             : launch_down<kBF16, kF32, MODE>(p, (int)tokens, st);
  else
    e = alpha_dtype == kBF16 ? launch_down<kF32, kBF16, MODE>(p, (int)tokens, st)
                             : launch_down<kF32, kF32, MODE>(p, (int)tokens, st);
  return e == cudaSuccess ? kOk : kErrCuda;
}
}  // namespace

extern "C" int maple_ternary_expert_down_reduce(const void* h, int h_dtype, int64_t h_tok_stride,
                                                int64_t h_slot_stride, const int32_t* ids,
                                                const float* wt, int64_t tokens, int64_t topk,
                                                int64_t k, const uint32_t* codes, int64_t n_experts,
                                                int64_t n, const void* alpha, int alpha_dtype,
                                                const void* residual, int64_t res_stride, void* out,
                                                int64_t out_stride, int* err, void* stream) {
  return down_entry<0>(h, h_dtype, h_tok_stride, h_slot_stride, ids, wt, tokens, topk, k, codes,
                       n_experts, n, alpha, alpha_dtype, residual, res_stride, out, out_stride, err, stream);
}

extern "C" int maple_ternary_expert_down_sum(const void* h, int h_dtype, int64_t h_tok_stride,
                                             int64_t h_slot_stride, const int32_t* ids,
                                             const float* wt, int64_t tokens, int64_t topk,
                                             int64_t k, const uint32_t* codes, int64_t n_experts,
                                             int64_t n, const void* alpha, int alpha_dtype,
                                             const void* residual, int64_t res_stride, void* out,
                                             int64_t out_stride, int* err, void* stream) {
  return down_entry<1>(h, h_dtype, h_tok_stride, h_slot_stride, ids, wt, tokens, topk, k, codes,
                       n_experts, n, alpha, alpha_dtype, residual, res_stride, out, out_stride, err, stream);
}

extern "C" int maple_moe_reduce_add(const void* x, int x_dtype, int64_t x_tok_stride,
                                    int64_t x_slot_stride, const float* wt, int64_t tokens,
                                    int64_t topk, int64_t n, const void* residual,
                                    int64_t res_stride, void* y, int64_t y_stride, void* stream) {
  if (tokens < 0 || topk <= 0 || n < 0) return kErrShape;
  if (tokens == 0 || n == 0) return kOk;
  if (x_dtype != kF32 && x_dtype != kBF16) return kErrDtype;
  if (!x || !wt || !y || tokens > 65535) return kErrShape;
  dim3 grid((unsigned)((n + 127) / 128), (unsigned)tokens);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (x_dtype == kBF16)
    launch_k(moe_reduce_kernel<kBF16>, dim3(grid), dim3(128), 0, st, x, wt, residual, y, x_tok_stride, x_slot_stride,
                                                   res_stride, y_stride, (int)n, (int)topk);
  else
    launch_k(moe_reduce_kernel<kF32>, dim3(grid), dim3(128), 0, st, x, wt, residual, y, x_tok_stride, x_slot_stride,
                                                  res_stride, y_stride, (int)n, (int)topk);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}
