// Decode attention: per-head QK RMSNorm + RoPE + KV-cache store, and GQA
// flash-decode split along the sequence with an in-kernel log-sum-exp merge.
//
// Reference: kernels/decode_attn.py:362-439 (apply_qkv_decode, kernel
// :64-163) and :470-592 (decode_gqa_attn, kernels :166-359; split count
// gqa_splits :446-467).
//
// Canonical arithmetic (mirrored by the CPU oracle):
//   head RMS      sum of squares in R128 order, x_hat = (x * rstd) * w
//   RoPE          lo' = x_lo*cos_lo + (-x_hi)*sin_lo,  hi' = x_hi*cos_hi + x_lo*sin_hi
//   scores        s_gt = R128 dot(q_g, k_t) * scale
//   split         positions [start + s*P, ...) in chunks of P (the caller's
//                 split length); per split m = max_t s, p_t = exp(s_t - m),
//                 l = R128 sum of p_t over the split's positions,
//                 acc_d = sequential fmaf over t of bf16(p_t) * v_td
//   merge         w_s = exp(m_s - max m), out = (fmaf-chain w_s*acc_s) /
//                 (fmaf-chain w_s*l_s), sequential over splits
// K/V tiles of a split are staged in shared memory with cp.async.bulk (TMA
// bulk copy) completing on an mbarrier; the wait is bounded and a timeout is
// reported through the error word instead of hanging.
#include <cooperative_groups.h>

#include "bulk.cuh"
#include "common.cuh"
#include "launch.cuh"
#include "tmap.cuh"

namespace cg = cooperative_groups;

namespace mb {


// ------------------------------------------------------ QK norm + RoPE ----
struct QkvParams {
  const void* qkv;        // [B, (Hq + 2*Hkv) * D]
  const void* q_w;        // [D]
  const void* k_w;        // [D]
  const void* cos;        // [B, R]
  const void* sin;        // [B, R]
  void* q_out;            // [B, Hq, D]
  void* kc;               // [Bc, Hkv, T, D]
  void* vc;
  const int64_t* seqlen;  // [B]
  const int32_t* row_map; // [B] or nullptr
  int* err;
  int64_t qkv_sb, cs_sb, q_sb, q_sh, kc_sb, kc_sh, vc_sb, vc_sh;
  int Hq, Hkv, D, R, Bc, T;
  int64_t cs_table_len;   // > 0: cos/sin are tables indexed by clamp(pos); 0: one row per batch row
  int use_rope;
  float eps;
};

template <int XT, int WT, int CT>
__global__ void __launch_bounds__(32) qk_norm_rope_store_kernel(QkvParams p) {
  __shared__ float xh[256];
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x;
  const int head = blockIdx.x, b = blockIdx.y;
  const int D = p.D;
  const char* row = static_cast<const char*>(p.qkv) + b * p.qkv_sb * (XT == kBF16 ? 2 : 4);
  const int64_t pos = p.seqlen[b];
  int cb = b;
  if (p.row_map != nullptr) cb = p.row_map[b];
  const bool store_ok = pos >= 0 && pos < p.T && cb >= 0 && cb < p.Bc;
  if (head >= p.Hq && !store_ok) {
    if (lane == 0) atomicOr(p.err, kErrFlagBounds);
    return;
  }
  if (head >= p.Hq + p.Hkv) {  // V: raw copy into the cache
    const int base = (p.Hq + p.Hkv) * D + (head - p.Hq - p.Hkv) * D;
    char* dst = static_cast<char*>(p.vc) + (cb * p.vc_sb + (head - p.Hq - p.Hkv) * p.vc_sh + pos * D) * (XT == kBF16 ? 2 : 4);
    for (int d = lane; d < D; d += 32) store_f<XT>(dst, d, load_f<XT>(row, base + d));
    return;
  }
  const bool is_q = head < p.Hq;
  const int base = is_q ? head * D : p.Hq * D + (head - p.Hq) * D;
  const void* w = is_q ? p.q_w : p.k_w;
  float part[4] = {0.f, 0.f, 0.f, 0.f};
  float xv[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) xv[u] = (u * 32 < D) ? load_f<XT>(row, base + lane + 32 * u) : 0.0f;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    if (u * 32 < D) {
      xh[lane + 32 * u] = xv[u];
      part[u & 3] = __fmaf_rn(xv[u], xv[u], part[u & 3]);
    }
  }
  const float rstd = rstd_of(r128_lane_finish(part[0], part[1], part[2], part[3]), D, p.eps);
  for (int u = 0; u * 32 < D; ++u) {
    const int d = lane + 32 * u;
    xh[d] = __fmul_rn(__fmul_rn(xh[d], rstd), load_f<WT>(w, d));
  }
  __syncwarp();
  int64_t cs_row = b;
  if (p.cs_table_len > 0) cs_row = pos < 0 ? 0 : (pos >= p.cs_table_len ? p.cs_table_len - 1 : pos);
  const char* cs = static_cast<const char*>(p.cos) + cs_row * p.cs_sb * (CT == kBF16 ? 2 : 4);
  const char* sn = static_cast<const char*>(p.sin) + cs_row * p.cs_sb * (CT == kBF16 ? 2 : 4);
  const int half = p.R / 2;
  char* dst;
  if (is_q)
    dst = static_cast<char*>(p.q_out) + (b * p.q_sb + head * p.q_sh) * (XT == kBF16 ? 2 : 4);
  else
    dst = static_cast<char*>(p.kc) + (cb * p.kc_sb + (head - p.Hq) * p.kc_sh + pos * D) * (XT == kBF16 ? 2 : 4);
  for (int d = lane; d < D; d += 32) {
    float o = xh[d];
    if (p.use_rope && d < p.R) {
      if (d < half) {
        o = __fadd_rn(__fmul_rn(xh[d], load_f<CT>(cs, d)), __fmul_rn(-xh[d + half], load_f<CT>(sn, d)));
      } else {
        o = __fadd_rn(__fmul_rn(xh[d], load_f<CT>(cs, d)), __fmul_rn(xh[d - half], load_f<CT>(sn, d)));
      }
    }
    store_f<XT>(dst, d, o);
  }
}

// ---------------------------------------------------------- GQA decode ----
struct AttnParams {
  const void* q;          // [B, Hq, D]
  const void* kc;         // [Bc, Hkv, T, D]
  const void* vc;
  const int64_t* seqlen;  // [B]
  const int32_t* row_map; // [B] or nullptr
  void* out;              // [B, Hq, D]
  float* ws_acc;          // [B, Hq, NS, D]
  float* ws_ml;           // [B, Hq, NS, 2]
  unsigned* tickets;      // [B * Hkv]
  int* err;
  int64_t q_sb, q_sh, kc_sb, kc_sh, vc_sb, vc_sh, o_sb, o_sh;
  int Hq, Hkv, G, Bc, T, P, NS, window;
  int kv_final;           // 1: K/V at positions < seqlen[b] were final before the previous launch
  int defer_merge;        // 1: leave the split partials for gqa_merge_kernel (long contexts)
  float scale;
  // Fused QK RMSNorm + RoPE + K/V store (kernels with QK = true, decode rows
  // only): q heads and the new K/V row come from the QKV projection rows.
  const void* qkv;        // [B, (Hq + 2 Hkv) D]
  int64_t qkv_sb;
  const void* q_w;        // [D]
  const void* k_w;        // [D]
  const void* cos;        // [cs_len, R] tables read at clamp(seqlen[b])
  const void* sin;
  int64_t cs_sb, cs_len;
  int w_f32, cs_f32, R, use_rope;
  float eps;
};

__device__ __forceinline__ float ldf_rt(const void* p, int64_t i, int f32) {
  return f32 ? static_cast<const float*>(p)[i] : bf16_to_f32(static_cast<const uint16_t*>(p)[i]);
}

// acc[u] (dim lane + 32u) += sum over positions t < n of p[t] * V[t], one
// fmaf per position in position order; the shared-memory loads of four
// positions are issued together ahead of their fmafs.
template <int XT, int D>
__device__ __forceinline__ void pv_accumulate(const float* prow, const unsigned char* vtile, int n, int lane,
                                              float (&acc)[D / 32]) {
  constexpr int U = D / 32;
  constexpr int es = XT == kBF16 ? 2 : 4;
  int t = 0;
  for (; t + 4 <= n; t += 4) {
    float pt[4], vv[4][U];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      pt[i] = prow[t + i];
#pragma unroll
      for (int u = 0; u < U; ++u) vv[i][u] = load_f<XT>(vtile + (size_t)(t + i) * D * es, lane + 32 * u);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int u = 0; u < U; ++u) acc[u] = __fmaf_rn(pt[i], vv[i][u], acc[u]);
  }
  for (; t < n; ++t) {
    const float pt = prow[t];
#pragma unroll
    for (int u = 0; u < U; ++u) acc[u] = __fmaf_rn(pt, load_f<XT>(vtile + (size_t)t * D * es, lane + 32 * u), acc[u]);
  }
}

// QK mode: the q/k norm weights and the RoPE cos/sin row of position pos are
// static inputs of the launch, staged into shared memory c = [4][D] (q weight,
// k weight, cos, sin; zero cos/sin past the rotary dims) by the whole CTA.
template <int D>
__device__ __forceinline__ void qk_stage_consts(const AttnParams& p, int64_t pos, float* c) {
  const int64_t cs_row = pos < 0 ? 0 : (pos >= p.cs_len ? p.cs_len - 1 : pos);
  const char* cs = static_cast<const char*>(p.cos) + cs_row * p.cs_sb * (p.cs_f32 ? 4 : 2);
  const char* sn = static_cast<const char*>(p.sin) + cs_row * p.cs_sb * (p.cs_f32 ? 4 : 2);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    c[d] = ldf_rt(p.q_w, d, p.w_f32);
    c[D + d] = ldf_rt(p.k_w, d, p.w_f32);
    const bool r = p.use_rope && d < p.R;
    c[2 * D + d] = r ? ldf_rt(cs, d, p.cs_f32) : 0.0f;
    c[3 * D + d] = r ? ldf_rt(sn, d, p.cs_f32) : 0.0f;
  }
}

// One warp: RMSNorm (R128 over D) * w, then RoPE of one head whose values
// xv[u] (dim lane + 32u) are already loaded -- the arithmetic of
// qk_norm_rope_store_kernel; o[u] is the value of dim lane + 32u before its
// bf16 store.  w, cs, sn: the staged weight and cos/sin rows; xh: D floats of
// warp-private shared memory.
template <int D>
__device__ __forceinline__ void qk_norm_rope_vals(const AttnParams& p, const float (&xv)[D / 32], const float* w,
                                                  const float* cs, const float* sn, float* xh, float (&o)[D / 32]) {
  constexpr int U = D / 32;
  const int lane = threadIdx.x & 31;
  float part[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int u = 0; u < U; ++u) part[u & 3] = __fmaf_rn(xv[u], xv[u], part[u & 3]);
  const float rstd = rstd_of(r128_lane_finish(part[0], part[1], part[2], part[3]), D, p.eps);
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int d = lane + 32 * u;
    xh[d] = __fmul_rn(__fmul_rn(xv[u], rstd), w[d]);
  }
  __syncwarp();
  const int half = p.R / 2;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int d = lane + 32 * u;
    float v = xh[d];
    if (p.use_rope && d < p.R) {
      if (d < half)
        v = __fadd_rn(__fmul_rn(xh[d], cs[d]), __fmul_rn(-xh[d + half], sn[d]));
      else
        v = __fadd_rn(__fmul_rn(xh[d], cs[d]), __fmul_rn(xh[d - half], sn[d]));
    }
    o[u] = v;
  }
  __syncwarp();
}

// QK mode: the split's q heads into qsm ([8][D], bf16-rounded values; zero
// rows beyond G) and, in the split that holds position pos, the new K/V row
// into the cache and the tiles.  Warp w takes q heads w, w + nwarps, ...;
// warps 0 / 1 also take the new K / V row, whose loads are issued with the q
// loads.  c: the staged constants (qk_stage_consts, visible to all threads).
// Ends synchronised.
template <int XT, int D>
__device__ __forceinline__ void qk_fused_rows(const AttnParams& p, int b, int h, int cb, int64_t pos, int t0,
                                              int n, bool active, bool cb_ok, unsigned char* ktile,
                                              unsigned char* vtile, float* qsm, float* kscr, const float* c,
                                              int nwarps) {
  constexpr int U = D / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int es = XT == kBF16 ? 2 : 4;
  const char* row = static_cast<const char*>(p.qkv) + b * p.qkv_sb * es;
  const bool has_new = active && pos >= t0 && pos < (int64_t)t0 + n && pos < p.T && cb_ok;
  const bool do_k = has_new && warp == 0, do_v = has_new && warp == 1;
  float xn[U];
  if (do_k || do_v) {
    const int nb = do_k ? p.Hq * D + h * D : (p.Hq + p.Hkv) * D + h * D;
#pragma unroll
    for (int u = 0; u < U; ++u) xn[u] = load_f<XT>(row, nb + lane + 32 * u);
  }
  for (int g = warp; g < 8; g += nwarps) {
    if (g < p.G && active) {
      float xq[U], o[U];
#pragma unroll
      for (int u = 0; u < U; ++u) xq[u] = load_f<XT>(row, (h * p.G + g) * D + lane + 32 * u);
      qk_norm_rope_vals<D>(p, xq, c, c + 2 * D, c + 3 * D, qsm + g * D, o);
#pragma unroll
      for (int u = 0; u < U; ++u) qsm[g * D + lane + 32 * u] = XT == kBF16 ? bf16_to_f32(f32_to_bf16(o[u])) : o[u];
    } else {
#pragma unroll
      for (int u = 0; u < U; ++u) qsm[g * D + lane + 32 * u] = 0.0f;
    }
  }
  if (do_k) {
    float o[U];
    qk_norm_rope_vals<D>(p, xn, c + D, c + 2 * D, c + 3 * D, kscr, o);
    char* dst = static_cast<char*>(const_cast<void*>(p.kc)) + (cb * p.kc_sb + h * p.kc_sh + pos * D) * es;
    unsigned char* tt = ktile + (size_t)(pos - t0) * D * es;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      store_f<XT>(dst, lane + 32 * u, o[u]);
      store_f<XT>(tt, lane + 32 * u, o[u]);
    }
  } else if (do_v) {
    char* dst = static_cast<char*>(const_cast<void*>(p.vc)) + (cb * p.vc_sb + h * p.vc_sh + pos * D) * es;
    unsigned char* tt = vtile + (size_t)(pos - t0) * D * es;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      store_f<XT>(dst, lane + 32 * u, xn[u]);
      store_f<XT>(tt, lane + 32 * u, xn[u]);
    }
  }
  __syncthreads();
}

template <int XT, int D, bool QK>
__global__ void __launch_bounds__(128) gqa_decode_kernel(AttnParams p) {
  constexpr int U = D / 32;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t bar;
  __shared__ float s_m[8], s_l[8];
  __shared__ int s_last;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int P = p.P, G = p.G;
  const int es = XT == kBF16 ? 2 : 4;
  pdl_wait();
  pdl_trigger();

  const int64_t pos = p.seqlen[b];
  const int kv_len = (int)min(pos + 1, (int64_t)p.T);
  const int start = p.window > 0 ? max(0, kv_len - p.window) : 0;
  const int ns = kv_len > start ? (kv_len - start + P - 1) / P : 0;
  if (s >= ns) return;
  const int t0 = start + s * P;
  const int n = min(P, kv_len - t0);
  int cb = b;
  if (p.row_map != nullptr) cb = p.row_map[b];
  const bool cb_ok = cb >= 0 && cb < p.Bc;
  if (!cb_ok) {
    if (tid == 0) atomicOr(p.err, kErrFlagBounds);
    cb = 0;
  }

  unsigned char* ktile = smem;
  unsigned char* vtile = smem + (size_t)P * D * es;
  float* scores = reinterpret_cast<float*>(smem + 2 * (size_t)P * D * es);  // [8][P]
  float* pb = scores + 8 * P;                                                 // [8][P]
  float* qsm = pb + 8 * P;                                                    // QK: [8][D] q, then [D] K scratch

  // QK: only the rows before pos are in the cache; the newest is formed here
  const int n_copy = QK ? max(0, (int)min((int64_t)n, pos - t0)) : n;
  if (tid == 0) {
    mbar_init(&bar, 1);
    const unsigned bytes = (unsigned)(n_copy * D * es);
    mbar_expect_tx(&bar, 2 * bytes);
    const char* ksrc = static_cast<const char*>(p.kc) + (cb * p.kc_sb + h * p.kc_sh + (int64_t)t0 * D) * es;
    const char* vsrc = static_cast<const char*>(p.vc) + (cb * p.vc_sb + h * p.vc_sh + (int64_t)t0 * D) * es;
    if (bytes > 0) {
      bulk_g2s(ktile, ksrc, bytes, &bar);
      bulk_g2s(vtile, vsrc, bytes, &bar);
    }
  }
  // q of the group's heads while the copies are in flight.
  float qv[8][U];
  if constexpr (QK) {
    qk_stage_consts<D>(p, pos, qsm + 9 * D);
    __syncthreads();
    qk_fused_rows<XT, D>(p, b, h, cb, pos, t0, n, true, cb_ok, ktile, vtile, qsm, qsm + 8 * D, qsm + 9 * D, 4);
#pragma unroll
    for (int g = 0; g < 8; ++g)
#pragma unroll
      for (int u = 0; u < U; ++u) qv[g][u] = qsm[g * D + lane + 32 * u];
  } else {
#pragma unroll
    for (int g = 0; g < 8; ++g)
#pragma unroll
      for (int u = 0; u < U; ++u)
        qv[g][u] = g < G ? load_f<XT>(static_cast<const char*>(p.q) + (b * p.q_sb + (h * G + g) * p.q_sh) * es,
                                      lane + 32 * u)
                         : 0.0f;
  }
  __syncthreads();  // barrier initialised before anyone waits on it
  bool ready = false;
  for (int i = 0; i < kWaitSpins && !ready; ++i) ready = mbar_try_wait(&bar, 0);
  if (!ready) {
    if (tid == 0) atomicOr(p.err, kErrFlagTimeout);
    for (int i = 0; i < kWaitSpins && !ready; ++i) ready = mbar_try_wait(&bar, 0);
    return;
  }

  // Scores: warp w takes position groups of 4; 32 (position, head) partials
  // per lane reduced with a transposing butterfly (lane l ends with element l).
  for (int grp = warp; grp * 4 < n; grp += 4) {
    float v[32];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int t = grp * 4 + i;
      float kk[U];
#pragma unroll
      for (int u = 0; u < U; ++u) kk[u] = t < n ? load_f<XT>(ktile + (size_t)t * D * es, lane + 32 * u) : 0.0f;
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        float pj[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int u = 0; u < U; ++u) pj[u & 3] = __fmaf_rn(qv[g][u], kk[u], pj[u & 3]);
        v[i * 8 + g] = __fadd_rn(__fadd_rn(__fadd_rn(pj[0], pj[1]), pj[2]), pj[3]);
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
    const int t = grp * 4 + (lane >> 3), g = lane & 7;
    if (t < n && g < G) scores[g * P + t] = __fmul_rn(v[0], p.scale);
  }
  __syncthreads();

  // Softmax statistics of this split, one warp per head.
  const float ninf = __int_as_float(0xff800000);
  for (int g = warp; g < G; g += 4) {
    float sv[4];
    float m = ninf;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = lane + 32 * u;
      sv[u] = (t < n) ? scores[g * P + t] : ninf;
      m = fmaxf(m, sv[u]);
    }
    m = warp_max(m);
    float pp[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = lane + 32 * u;
      pp[u] = (t < n) ? mexp(__fsub_rn(sv[u], m)) : 0.0f;
      if (t < P) pb[g * P + t] = (t < n) ? bf16_to_f32(f32_to_bf16(pp[u])) : 0.0f;
    }
    const float l = r128_lane_finish(pp[0], pp[1], pp[2], pp[3]);
    if (lane == 0) { s_m[g] = m; s_l[g] = l; }
  }
  __syncthreads();

  // P.V with the bf16-rounded probabilities, sequential over positions.
  for (int g = warp; g < G; g += 4) {
    float acc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) acc[u] = 0.0f;
    pv_accumulate<XT, D>(pb + g * P, vtile, n, lane, acc);
    const int hq = h * G + g;
    if (ns == 1) {
      char* o = static_cast<char*>(p.out) + (b * p.o_sb + hq * p.o_sh) * es;
#pragma unroll
      for (int u = 0; u < U; ++u) store_f<XT>(o, lane + 32 * u, __fdiv_rn(acc[u], s_l[g]));
    } else {
      float* wa = p.ws_acc + (((int64_t)b * p.Hq + hq) * p.NS + s) * D;
#pragma unroll
      for (int u = 0; u < U; ++u) wa[lane + 32 * u] = acc[u];
      if (lane == 0) {
        float* wml = p.ws_ml + (((int64_t)b * p.Hq + hq) * p.NS + s) * 2;
        wml[0] = s_m[g];
        wml[1] = s_l[g];
      }
    }
  }
  if (ns == 1 || p.defer_merge) return;

  // Last split of (b, h) merges all splits in split order.
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    unsigned* tk = p.tickets + (int64_t)b * p.Hkv + h;
    const unsigned old = atomicAdd(tk, 1u);
    s_last = (old == static_cast<unsigned>(ns - 1));
    if (s_last) atomicExch(tk, 0u);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // One warp per query head: lanes own dims lane + 32u; splits in order, their
  // partials fetched four at a time.
  for (int g = warp; g < G; g += 4) {
    const int hq = h * G + g;
    const float* ml = p.ws_ml + ((int64_t)b * p.Hq + hq) * p.NS * 2;
    const float* ac = p.ws_acc + ((int64_t)b * p.Hq + hq) * p.NS * D;
    float M = ninf;
    for (int j = lane; j < ns; j += 32) M = fmaxf(M, __ldcg(ml + 2 * j));
    M = warp_max(M);
    float num[U];
#pragma unroll
    for (int u = 0; u < U; ++u) num[u] = 0.0f;
    float den = 0.0f;
    for (int j0 = 0; j0 < ns; j0 += 4) {
      float mj[4], lj[4], aj[4][U];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int j = j0 + i;
        if (j < ns) {
          mj[i] = __ldcg(ml + 2 * j);
          lj[i] = __ldcg(ml + 2 * j + 1);
#pragma unroll
          for (int u = 0; u < U; ++u) aj[i][u] = __ldcg(ac + (int64_t)j * D + lane + 32 * u);
        }
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if (j0 + i < ns) {
          const float w = mexp(__fsub_rn(mj[i], M));
          den = __fmaf_rn(w, lj[i], den);
#pragma unroll
          for (int u = 0; u < U; ++u) num[u] = __fmaf_rn(w, aj[i][u], num[u]);
        }
      }
    }
    char* o = static_cast<char*>(p.out) + (b * p.o_sb + hq * p.o_sh) * es;
#pragma unroll
    for (int u = 0; u < U; ++u) store_f<XT>(o, lane + 32 * u, __fdiv_rn(num[u], den));
  }
}


// Short contexts (at most 16 splits): the splits of one (row, kv head) form a
// thread-block cluster.  Each CTA leaves its split's (acc, m, l) in its own
// shared memory; after a cluster barrier the rank-0 CTA merges them in split
// order through distributed shared memory (same arithmetic as the workspace
// merge).  With kv_final, K/V rows of positions before seqlen[b] are copied
// before the PDL wait; only the newest position waits for the previous launch.
template <int XT, int D, bool QK>
__global__ void __launch_bounds__(256) gqa_cluster_kernel(AttnParams p) {
  constexpr int U = D / 32;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ uint64_t bar[2];
  cg::cluster_group cluster = cg::this_cluster();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int P = p.P, G = p.G;
  const int es = XT == kBF16 ? 2 : 4;
  unsigned char* ktile = smem;
  unsigned char* vtile = smem + (size_t)P * D * es;
  float* scores = reinterpret_cast<float*>(smem + 2 * (size_t)P * D * es);  // [8][P]
  float* pb = scores + 8 * P;                                                 // [8][P]
  float* part = pb + 8 * P;                                                   // [8][D] acc, then m[8], l[8]
  float* part_m = part + 8 * D;
  float* part_l = part_m + 8;
  float* kscr = part_l + 8;                                                   // QK: [D] K scratch
  float* qkc = kscr + D;                                                      // QK: [4][D] constants

  const int64_t pos = p.seqlen[b];
  const int kv_len = (int)min(pos + 1, (int64_t)p.T);
  const int start = p.window > 0 ? max(0, kv_len - p.window) : 0;
  const int ns = kv_len > start ? (kv_len - start + P - 1) / P : 0;
  const bool active = s < ns;
  const int t0 = start + s * P;
  const int n = active ? min(P, kv_len - t0) : 0;
  int cb = b;
  if (p.row_map != nullptr) cb = p.row_map[b];
  const bool cb_ok = cb >= 0 && cb < p.Bc;
  if (!cb_ok) cb = 0;
  const char* ksrc = static_cast<const char*>(p.kc) + (cb * p.kc_sb + h * p.kc_sh + (int64_t)t0 * D) * es;
  const char* vsrc = static_cast<const char*>(p.vc) + (cb * p.vc_sb + h * p.vc_sh + (int64_t)t0 * D) * es;
  // rows [0, n_pre) are final before the previous launch
  const int n_pre = (p.kv_final && active) ? max(0, min(n, (int)(pos - t0))) : 0;
  if (tid == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    if (n_pre > 0) {
      mbar_expect_tx(&bar[0], 2u * n_pre * D * es);
      bulk_g2s(ktile, ksrc, (unsigned)(n_pre * D * es), &bar[0]);
      bulk_g2s(vtile, vsrc, (unsigned)(n_pre * D * es), &bar[0]);
    }
  }
  if constexpr (QK) {
    qk_stage_consts<D>(p, pos, qkc);
    __syncthreads();
  }
  pdl_wait();
  pdl_trigger();
  if (tid == 0) {
    if (!cb_ok) atomicOr(p.err, kErrFlagBounds);
    if (!QK && n > n_pre) {
      const unsigned off = (unsigned)(n_pre * D * es), bytes = (unsigned)((n - n_pre) * D * es);
      mbar_expect_tx(&bar[1], 2u * bytes);
      bulk_g2s(ktile + off, ksrc + off, bytes, &bar[1]);
      bulk_g2s(vtile + off, vsrc + off, bytes, &bar[1]);
    }
  }
  float qv[8][U];
  if constexpr (QK) {
    // q heads and the newest K/V row from the QKV rows (the merge area holds q until P.V)
    qk_fused_rows<XT, D>(p, b, h, cb, pos, t0, n, active, cb_ok, ktile, vtile, part, kscr, qkc, 8);
#pragma unroll
    for (int g = 0; g < 8; ++g)
#pragma unroll
      for (int u = 0; u < U; ++u) qv[g][u] = part[g * D + lane + 32 * u];
  } else {
#pragma unroll
    for (int g = 0; g < 8; ++g)
#pragma unroll
      for (int u = 0; u < U; ++u)
        qv[g][u] = (g < G && active) ? load_f<XT>(static_cast<const char*>(p.q) + (b * p.q_sb + (h * G + g) * p.q_sh) * es,
                                                  lane + 32 * u)
                                     : 0.0f;
  }
  __syncthreads();  // barriers initialised before anyone waits; q read from shared memory
  bool ok = true;
  for (int k = 0; k < 2; ++k) {
    const bool need = (k == 0) ? n_pre > 0 : (!QK && n > n_pre);
    if (need) {
      bool ready = false;
      for (int i = 0; i < kWaitSpins && !ready; ++i) ready = mbar_try_wait(&bar[k], 0);
      if (!ready) {
        ok = false;
        if (tid == 0) atomicOr(p.err, kErrFlagTimeout);
        for (int i = 0; i < kWaitSpins && !ready; ++i) ready = mbar_try_wait(&bar[k], 0);
      }
    }
  }
  const bool work = active && ok;
  const float ninf = __int_as_float(0xff800000);
  if (work) {
    for (int grp = warp; grp * 4 < n; grp += 8) {
      float v[32];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int t = grp * 4 + i;
        float kk[U];
#pragma unroll
        for (int u = 0; u < U; ++u) kk[u] = t < n ? load_f<XT>(ktile + (size_t)t * D * es, lane + 32 * u) : 0.0f;
#pragma unroll
        for (int g = 0; g < 8; ++g) {
          float pj[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int u = 0; u < U; ++u) pj[u & 3] = __fmaf_rn(qv[g][u], kk[u], pj[u & 3]);
          v[i * 8 + g] = __fadd_rn(__fadd_rn(__fadd_rn(pj[0], pj[1]), pj[2]), pj[3]);
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
      const int t = grp * 4 + (lane >> 3), g = lane & 7;
      if (t < n && g < G) scores[g * P + t] = __fmul_rn(v[0], p.scale);
    }
  }
  __syncthreads();
  if (work && warp < G) {
    const int g = warp;
    float sv[4];
    float m = ninf;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = lane + 32 * u;
      sv[u] = (t < n) ? scores[g * P + t] : ninf;
      m = fmaxf(m, sv[u]);
    }
    m = warp_max(m);
    float pp[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const int t = lane + 32 * u;
      pp[u] = (t < n) ? mexp(__fsub_rn(sv[u], m)) : 0.0f;
      if (t < P) pb[g * P + t] = (t < n) ? bf16_to_f32(f32_to_bf16(pp[u])) : 0.0f;
    }
    const float l = r128_lane_finish(pp[0], pp[1], pp[2], pp[3]);
    __syncwarp();
    float acc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) acc[u] = 0.0f;
    pv_accumulate<XT, D>(pb + g * P, vtile, n, lane, acc);
#pragma unroll
    for (int u = 0; u < U; ++u) part[g * D + lane + 32 * u] = acc[u];
    if (lane == 0) {
      part_m[g] = m;
      part_l[g] = l;
    }
  }
  cluster.sync();
  // Merge: the cluster's CTAs share the G*D outputs; a thread reads the ns
  // splits' (m, l, acc) of its head and dimension from their CTAs' shared
  // memory with all loads issued together, then M = max_j m_j,
  // w_j = exp(m_j - M), den and num as fmaf chains in split order,
  // out = num / den.
  if (ns > 0) {
    constexpr int kMaxSplits = 16;
    const int cl = (int)gridDim.x;
    for (int o = s * (int)blockDim.x + tid; o < G * D; o += cl * (int)blockDim.x) {
      const int g = o / D, dd = o - g * D;
      float mj[kMaxSplits], lj[kMaxSplits], aj[kMaxSplits];
#pragma unroll
      for (int j = 0; j < kMaxSplits; ++j) {
        if (j < ns) {
          const float* rp = cluster.map_shared_rank(part, j);
          mj[j] = rp[8 * D + g];
          lj[j] = rp[8 * D + 8 + g];
          aj[j] = rp[g * D + dd];
        }
      }
      float M = ninf;
#pragma unroll
      for (int j = 0; j < kMaxSplits; ++j)
        if (j < ns) M = fmaxf(M, mj[j]);
      float num = 0.0f, den = 0.0f;
#pragma unroll
      for (int j = 0; j < kMaxSplits; ++j) {
        if (j < ns) {
          const float w = mexp(__fsub_rn(mj[j], M));
          den = __fmaf_rn(w, lj[j], den);
          num = __fmaf_rn(w, aj[j], num);
        }
      }
      char* out = static_cast<char*>(p.out) + (b * p.o_sb + (h * G + g) * p.o_sh) * es;
      store_f<XT>(out, dd, __fdiv_rn(num, den));
    }
  }
  cluster.sync();  // peers keep their shared memory until the merge has read it
}


// Merge of long contexts' split partials, one CTA per (row, query head) and
// one thread per dimension, so hundreds of splits are read by many SMs at
// once rather than by the last split's CTA.  Same arithmetic as the in-kernel
// merge: M = max_j m_j, w_j = exp(m_j - M), den and num as fmaf chains in
// split order, out = num / den.
template <int XT, int D>
__global__ void __launch_bounds__(D) gqa_merge_kernel(AttnParams p) {
  __shared__ float s_max[D / 32];
  const int d = threadIdx.x, lane = d & 31, warp = d >> 5;
  const int hq = blockIdx.x, b = blockIdx.y;
  const int es = XT == kBF16 ? 2 : 4;
  pdl_wait();
  pdl_trigger();
  const int64_t pos = p.seqlen[b];
  const int kv_len = (int)min(pos + 1, (int64_t)p.T);
  const int start = p.window > 0 ? max(0, kv_len - p.window) : 0;
  const int ns = kv_len > start ? (kv_len - start + p.P - 1) / p.P : 0;
  if (ns <= 1) return;  // a single split was stored directly
  const float* ml = p.ws_ml + ((int64_t)b * p.Hq + hq) * p.NS * 2;
  const float* ac = p.ws_acc + ((int64_t)b * p.Hq + hq) * p.NS * D;
  float M = __int_as_float(0xff800000);
  for (int j = d; j < ns; j += D) M = fmaxf(M, __ldcg(ml + 2 * j));
  M = warp_max(M);
  if (lane == 0) s_max[warp] = M;
  __syncthreads();
  M = s_max[0];
#pragma unroll
  for (int w = 1; w < D / 32; ++w) M = fmaxf(M, s_max[w]);
  float num = 0.0f, den = 0.0f;
  constexpr int kB = 8;
  for (int j0 = 0; j0 < ns; j0 += kB) {
    float mj[kB], lj[kB], aj[kB];
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      const int j = j0 + i;
      if (j < ns) {
        mj[i] = __ldcg(ml + 2 * j);
        lj[i] = __ldcg(ml + 2 * j + 1);
        aj[i] = __ldcg(ac + (int64_t)j * D + d);
      }
    }
#pragma unroll
    for (int i = 0; i < kB; ++i) {
      if (j0 + i < ns) {
        const float w = mexp(__fsub_rn(mj[i], M));
        den = __fmaf_rn(w, lj[i], den);
        num = __fmaf_rn(w, aj[i], num);
      }
    }
  }
  store_f<XT>(static_cast<char*>(p.out) + (b * p.o_sb + hq * p.o_sh) * es, d, __fdiv_rn(num, den));
}


// ---------------------------------------------------------------------------
// Tensor-core decode attention (bf16 caches, long contexts / large batches).
//
// The reference kernel's arithmetic (kernels/decode_attn.py:166-313): q.K^T as
// a bf16 dot with fp32 accumulation, an online softmax per query head, P
// rounded to bf16 for the P.V dot, fp32 accumulation -- on the bf16 tensor
// pipe (mma.sync m16n8k16) instead of CUDA-core fp32 fmas.  The GQA group's
// query heads are the MMA's M rows (8 used of 16), 8 positions or 8 output
// dims are its N, so the scores of one n-tile pair become the A operand of
// the P.V product in registers (no trip through shared memory).
//
// CTA = 4 warps = one (row, kv head, split of positions); the split streams
// through shared memory in chunks of 64 positions (16 per warp) with a
// 3-stage pipeline of tiled TMA loads (cp.async.bulk.tensor over a 4-D tensor
// map of the cache, boxes of 64 positions x 64 dims with the 128-byte swizzle,
// so the ldmatrix reads below are bank-conflict free).  Each warp
// keeps its own running max / sum / accumulator; the CTA merges its 4 warps
// and stores the split's (acc, m, l) for gqa_merge_kernel (or the output when
// the row has a single split).  Waits are bounded: a wait that gives up sets
// the error word, drains the copies in flight and returns.
constexpr int kTcChunk = 64;
constexpr int kTcStages = 3;

__device__ __forceinline__ void ldsm_x4(unsigned addr, unsigned& r0, unsigned& r1, unsigned& r2, unsigned& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(unsigned addr, unsigned& r0, unsigned& r1, unsigned& r2, unsigned& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
// c += A * B with A rows 8-15 zero (a1 = a3 = 0): only c[0], c[1] carry data.
__device__ __forceinline__ void mma_bf16_h8(float (&c)[4], unsigned a0, unsigned a2, unsigned b0, unsigned b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
      "{%0, %1, %2, %3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}
__device__ __forceinline__ unsigned pack_bf16x2(float lo, float hi) {
  return static_cast<unsigned>(f32_to_bf16(lo)) | (static_cast<unsigned>(f32_to_bf16(hi)) << 16);
}

// Byte offset of 16-byte unit U (dims 8U..8U+7) of row r in a K or V tile of
// 128-byte-swizzled 64 x 64 boxes (one box per 64 dims).
__device__ __forceinline__ unsigned tc_swz(int r, int U) {
  return (unsigned)((U >> 3) * 8192 + r * 128 + (((U & 7) ^ (r & 7)) << 4));
}

template <int D>
__global__ void __launch_bounds__(128) gqa_tc_kernel(AttnParams p, const __grid_constant__ CUtensorMap tmk,
                                                     const __grid_constant__ CUtensorMap tmv) {
  constexpr int HALVES = D / 64;                 // 64-dim boxes per row
  constexpr int TILE = HALVES * 8192;            // one K or V tile of 64 positions
  constexpr int STAGE = 2 * TILE;                // K tile, then V tile
  constexpr int NT = D / 8;                      // output n-tiles (8 dims each)
  extern __shared__ unsigned char smem_raw[];
  // the 128-byte swizzle repeats every 1024 bytes: tiles start 1024-aligned
  unsigned char* smem = reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar[kTcStages];
  __shared__ float s_m[4][8], s_l[4][8];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int s = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const float ninf = __int_as_float(0xff800000);
  pdl_wait();
  pdl_trigger();

  const int64_t pos = p.seqlen[b];
  const int kv_len = (int)min(pos + 1, (int64_t)p.T);
  const int start = p.window > 0 ? max(0, kv_len - p.window) : 0;
  const int ns = kv_len > start ? (kv_len - start + p.P - 1) / p.P : 0;
  if (s >= ns) return;
  const int t0 = start + s * p.P;
  const int hi = min(t0 + p.P, kv_len);
  const int nchunks = (hi - t0 + kTcChunk - 1) / kTcChunk;
  int cb = b;
  if (p.row_map != nullptr) cb = p.row_map[b];
  if (cb < 0 || cb >= p.Bc) {
    if (tid == 0) atomicOr(p.err, kErrFlagBounds);
    cb = 0;
  }

  if (tid == 0)
    for (int i = 0; i < kTcStages; ++i) mbar_init(&bar[i], 1);
  __syncthreads();

  // thread 0 issues chunk c: the full 64-position boxes of K and V (rows past
  // the cache's end arrive as zeros and count toward the transaction bytes)
  auto issue = [&](int c) {
    const int stage = c % kTcStages;
    const int c0 = t0 + c * kTcChunk;
    unsigned char* kt = smem + stage * STAGE;
    mbar_expect_tx(&bar[stage], (unsigned)STAGE);
#pragma unroll
    for (int hf = 0; hf < HALVES; ++hf) {
      tma_load_4d(kt + hf * 8192, &tmk, 64 * hf, c0, h, cb, &bar[stage]);
      tma_load_4d(kt + TILE + hf * 8192, &tmv, 64 * hf, c0, h, cb, &bar[stage]);
    }
  };
  if (tid == 0)
    for (int c = 0; c < min(kTcStages, nchunks); ++c) issue(c);

  // this thread's A fragments of q (rows g = query head of the group; rows
  // 8-15 of the MMA are zero): dims 16kk + 2t, +1 and 16kk + 8 + 2t, +1
  unsigned qa[D / 16][2];
  {
    const bool real = g < p.G;
    const unsigned* qrow = reinterpret_cast<const unsigned*>(
        static_cast<const char*>(p.q) + (b * p.q_sb + (h * p.G + (real ? g : 0)) * p.q_sh) * 2);
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      qa[kk][0] = real ? qrow[8 * kk + t] : 0u;
      qa[kk][1] = real ? qrow[8 * kk + 4 + t] : 0u;
    }
  }

  float m_run = ninf, l_run = 0.0f;
  float acc[NT][4];
#pragma unroll
  for (int j = 0; j < NT; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.0f;
  const int r0 = warp * 16;

  for (int c = 0; c < nchunks; ++c) {
    const int stage = c % kTcStages;
    const bool ok = mbar_wait_bounded(&bar[stage], (unsigned)((c / kTcStages) & 1));
    if (__syncthreads_or(!ok)) {
      // give up: report, let this CTA's copies land (bounded), return
      if (tid == 0) {
        atomicOr(p.err, kErrFlagTimeout);
        for (int c2 = c; c2 < min(c + kTcStages, nchunks); ++c2)
          mbar_wait_bounded(&bar[c2 % kTcStages], (unsigned)((c2 / kTcStages) & 1));
      }
      __syncthreads();
      return;
    }
    const int c0 = t0 + c * kTcChunk;
    const int n = min(kTcChunk, hi - c0);
    unsigned char* kt = smem + stage * STAGE;
    unsigned char* vt = kt + TILE;
    if (r0 < n) {
      if (n < r0 + 16) {
        // rows past the split's end hold other positions' bytes: zero V there
        // (P is 0 at masked positions, and 0 * anything non-finite is NaN)
        for (int r = n; r < r0 + 16; ++r)
          for (int i = lane; i < D / 8; i += 32)
            *reinterpret_cast<uint4*>(vt + tc_swz(r, i)) = make_uint4(0, 0, 0, 0);
        __syncwarp();
      }
      // S = q K^T for this warp's 16 positions (two n-tiles of 8)
      float sfr[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        sfr[j][0] = sfr[j][1] = sfr[j][2] = sfr[j][3] = 0.0f;
#pragma unroll
        for (int kp = 0; kp < D / 32; ++kp) {
          unsigned b0, b1, b2, b3;
          ldsm_x4(smem_u32(kt + tc_swz(r0 + 8 * j + (lane & 7), 4 * kp + (lane >> 3))), b0, b1, b2, b3);
          mma_bf16_h8(sfr[j], qa[2 * kp][0], qa[2 * kp][1], b0, b1);
          mma_bf16_h8(sfr[j], qa[2 * kp + 1][0], qa[2 * kp + 1][1], b2, b3);
        }
      }
      // online softmax of row g over positions r0 + {2t, 2t+1, 8+2t, 9+2t}
      float sv[4] = {sfr[0][0], sfr[0][1], sfr[1][0], sfr[1][1]};
      const int pr[4] = {r0 + 2 * t, r0 + 2 * t + 1, r0 + 8 + 2 * t, r0 + 9 + 2 * t};
      float mx = ninf;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sv[i] = pr[i] < n ? __fmul_rn(sv[i], p.scale) : ninf;
        mx = fmaxf(mx, sv[i]);
      }
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float m_new = fmaxf(m_run, mx);
      const float m_use = m_new == ninf ? 0.0f : m_new;
      const float alpha = __expf(__fsub_rn(m_run, m_use));
      float pv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pv[i] = __expf(__fsub_rn(sv[i], m_use));
      l_run = __fadd_rn(__fmul_rn(l_run, alpha), __fadd_rn(__fadd_rn(pv[0], pv[1]), __fadd_rn(pv[2], pv[3])));
      m_run = m_new;
#pragma unroll
      for (int j = 0; j < NT; ++j) {
        acc[j][0] = __fmul_rn(acc[j][0], alpha);
        acc[j][1] = __fmul_rn(acc[j][1], alpha);
      }
      const unsigned pa0 = pack_bf16x2(pv[0], pv[1]), pa2 = pack_bf16x2(pv[2], pv[3]);
      // O += P V: V fragments by transposed ldmatrix, two dim n-tiles per load
#pragma unroll
      for (int jp = 0; jp < D / 16; ++jp) {
        unsigned b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(vt + tc_swz(r0 + (lane & 7) + 8 * ((lane >> 3) & 1), 2 * jp + (lane >> 4))), b0, b1, b2,
                  b3);
        mma_bf16_h8(acc[2 * jp], pa0, pa2, b0, b1);
        mma_bf16_h8(acc[2 * jp + 1], pa0, pa2, b2, b3);
      }
    }
    __syncthreads();  // every warp is done with this stage
    if (tid == 0 && c + kTcStages < nchunks) {
      fence_proxy_async_smem();
      issue(c + kTcStages);
    }
  }

  // merge the four warps' states: row sums over the 4 threads of a row,
  // accumulators through the (now idle) stage memory
  l_run = __fadd_rn(l_run, __shfl_xor_sync(0xffffffffu, l_run, 1));
  l_run = __fadd_rn(l_run, __shfl_xor_sync(0xffffffffu, l_run, 2));
  float* wacc = reinterpret_cast<float*>(smem);  // [4 warps][8 heads][D]
  if (t == 0) {
    s_m[warp][g] = m_run;
    s_l[warp][g] = l_run;
  }
#pragma unroll
  for (int j = 0; j < NT; ++j) {
    wacc[(warp * 8 + g) * D + 8 * j + 2 * t] = acc[j][0];
    wacc[(warp * 8 + g) * D + 8 * j + 2 * t + 1] = acc[j][1];
  }
  __syncthreads();
  for (int i = tid; i < p.G * D; i += blockDim.x) {
    const int gg = i / D, d = i - gg * D;
    float M = s_m[0][gg];
#pragma unroll
    for (int w = 1; w < 4; ++w) M = fmaxf(M, s_m[w][gg]);
    float num = 0.0f, den = 0.0f;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
      const float wt = s_m[w][gg] == ninf ? 0.0f : __expf(__fsub_rn(s_m[w][gg], M));
      num = __fmaf_rn(wt, wacc[(w * 8 + gg) * D + d], num);
      den = __fmaf_rn(wt, s_l[w][gg], den);
    }
    const int hq = h * p.G + gg;
    if (ns == 1) {
      store_f<kBF16>(static_cast<char*>(p.out) + (b * p.o_sb + hq * p.o_sh) * 2, d, __fdiv_rn(num, den));
    } else {
      p.ws_acc[(((int64_t)b * p.Hq + hq) * p.NS + s) * D + d] = num;
      if (d == 0) {
        float* ml = p.ws_ml + (((int64_t)b * p.Hq + hq) * p.NS + s) * 2;
        ml[0] = M;
        ml[1] = den;
      }
    }
  }
}

// Split merge of the tensor-core path: one CTA per (row, query head), its 8
// warps take splits j = warp, warp + 8, ... with a running max / rescaled sum
// over D/32 dims per lane (16-byte loads), then the warps combine through
// shared memory.  Many splits are read at once instead of one after another
// (a batch-1 row of a 64K cache has 257 splits).
template <int D>
__global__ void __launch_bounds__(256) gqa_tc_merge_kernel(AttnParams p) {
  constexpr int V = D / 32;  // dims per lane
  __shared__ float s_m[8], s_l[8];
  __shared__ float s_acc[8][D];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int hq = blockIdx.x, b = blockIdx.y;
  const float ninf = __int_as_float(0xff800000);
  pdl_wait();
  pdl_trigger();
  const int64_t pos = p.seqlen[b];
  const int kv_len = (int)min(pos + 1, (int64_t)p.T);
  const int start = p.window > 0 ? max(0, kv_len - p.window) : 0;
  const int ns = kv_len > start ? (kv_len - start + p.P - 1) / p.P : 0;
  if (ns <= 1) return;  // a single split was stored directly
  const float* ml = p.ws_ml + ((int64_t)b * p.Hq + hq) * p.NS * 2;
  const float* ac = p.ws_acc + ((int64_t)b * p.Hq + hq) * p.NS * D;
  float m = ninf, l = 0.0f, acc[V];
#pragma unroll
  for (int v = 0; v < V; ++v) acc[v] = 0.0f;
  for (int j = warp; j < ns; j += 8) {
    const float mj = __ldcg(ml + 2 * j), lj = __ldcg(ml + 2 * j + 1);
    float aj[V];
    if constexpr (V == 4) {
      const float4 a4 = __ldcg(reinterpret_cast<const float4*>(ac + (int64_t)j * D) + lane);
      aj[0] = a4.x; aj[1] = a4.y; aj[2] = a4.z; aj[3] = a4.w;
    } else {
      const float2 a2 = __ldcg(reinterpret_cast<const float2*>(ac + (int64_t)j * D) + lane);
      aj[0] = a2.x; aj[1] = a2.y;
    }
    const float mn = fmaxf(m, mj);
    const float c_old = m == ninf ? 0.0f : __expf(__fsub_rn(m, mn));
    const float c_new = __expf(__fsub_rn(mj, mn));
    l = __fmaf_rn(lj, c_new, __fmul_rn(l, c_old));
#pragma unroll
    for (int v = 0; v < V; ++v) acc[v] = __fmaf_rn(aj[v], c_new, __fmul_rn(acc[v], c_old));
    m = mn;
  }
  if (lane == 0) {
    s_m[warp] = m;
    s_l[warp] = l;
  }
#pragma unroll
  for (int v = 0; v < V; ++v) s_acc[warp][V * lane + v] = acc[v];
  __syncthreads();
  if (tid < D) {
    float M = s_m[0];
#pragma unroll
    for (int w = 1; w < 8; ++w) M = fmaxf(M, s_m[w]);
    float num = 0.0f, den = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
      const float c = s_m[w] == ninf ? 0.0f : __expf(__fsub_rn(s_m[w], M));
      num = __fmaf_rn(c, s_acc[w][tid], num);
      den = __fmaf_rn(c, s_l[w], den);
    }
    store_f<kBF16>(static_cast<char*>(p.out) + (b * p.o_sb + hq * p.o_sh) * 2, tid, __fdiv_rn(num, den));
  }
}

}  // namespace mb

using namespace mb;

constexpr int kAttnTicketBytes = 1 << 20;

extern "C" int maple_apply_qkv_decode(const void* qkv, int x_dtype, int64_t batch, int64_t qkv_row_stride,
                                      const void* q_weight, const void* k_weight, int w_dtype,
                                      const void* cos, const void* sin, int cs_dtype, int64_t cs_row_stride,
                                      int64_t cs_table_len, void* q_out, int64_t q_sb, int64_t q_sh, void* k_cache, void* v_cache,
                                      int64_t cache_batch, int64_t cache_sb, int64_t cache_sh,
                                      int64_t max_len, const int64_t* seqlen, const int32_t* row_map,
                                      int64_t num_heads, int64_t num_kv_heads, int64_t head_dim,
                                      int64_t rotary_dim, int use_rope, float eps, int* err, void* stream) {
  if (batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || head_dim <= 0) return kErrShape;
  if (batch == 0) return kOk;
  if (head_dim % 32 != 0 || head_dim > 256 || rotary_dim < 0 || rotary_dim > head_dim || (rotary_dim & 1))
    return kErrShape;
  if (x_dtype != kF32 && x_dtype != kBF16) return kErrDtype;
  if ((w_dtype != kF32 && w_dtype != kBF16) || (cs_dtype != kF32 && cs_dtype != kBF16)) return kErrDtype;
  if (!qkv || !q_weight || !k_weight || !q_out || !k_cache || !v_cache || !seqlen || !err) return kErrShape;
  if (use_rope && (!cos || !sin)) return kErrShape;
  QkvParams p{};
  p.qkv = qkv; p.q_w = q_weight; p.k_w = k_weight; p.cos = cos; p.sin = sin; p.q_out = q_out;
  p.kc = k_cache; p.vc = v_cache; p.seqlen = seqlen; p.row_map = row_map; p.err = err;
  p.qkv_sb = qkv_row_stride; p.cs_sb = cs_row_stride; p.cs_table_len = cs_table_len; p.q_sb = q_sb; p.q_sh = q_sh;
  p.kc_sb = cache_sb; p.kc_sh = cache_sh; p.vc_sb = cache_sb; p.vc_sh = cache_sh;
  p.Hq = (int)num_heads; p.Hkv = (int)num_kv_heads; p.D = (int)head_dim; p.R = (int)rotary_dim;
  p.Bc = (int)cache_batch; p.T = (int)max_len; p.use_rope = use_rope; p.eps = eps;
  dim3 grid((unsigned)(num_heads + 2 * num_kv_heads), (unsigned)batch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
#define MB_QKV(XT, WT, CT) launch_k(qk_norm_rope_store_kernel<XT, WT, CT>, dim3(grid), dim3(32), 0, st, p)
  if (x_dtype == kBF16) {
    if (w_dtype == kBF16) { if (cs_dtype == kBF16) MB_QKV(kBF16, kBF16, kBF16); else MB_QKV(kBF16, kBF16, kF32); }
    else { if (cs_dtype == kBF16) MB_QKV(kBF16, kF32, kBF16); else MB_QKV(kBF16, kF32, kF32); }
  } else {
    if (w_dtype == kBF16) { if (cs_dtype == kBF16) MB_QKV(kF32, kBF16, kBF16); else MB_QKV(kF32, kBF16, kF32); }
    else { if (cs_dtype == kBF16) MB_QKV(kF32, kF32, kBF16); else MB_QKV(kF32, kF32, kF32); }
  }
#undef MB_QKV
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int64_t maple_decode_gqa_workspace_bytes(int64_t batch, int64_t num_heads, int64_t head_dim,
                                                    int64_t max_len, int64_t split_len) {
  if (split_len <= 0) return -1;
  const int64_t ns = (max_len + split_len - 1) / split_len;
  return kAttnTicketBytes + batch * num_heads * ns * (head_dim + 2) * (int64_t)sizeof(float);
}

static int gqa_common(const void* q, int x_dtype, int64_t batch, int64_t num_heads, int64_t q_sb, int64_t q_sh,
                      const void* k_cache, const void* v_cache, int64_t cache_batch, int64_t num_kv_heads,
                      int64_t cache_sb, int64_t cache_sh, int64_t max_len, int64_t head_dim,
                      const int64_t* seqlen, const int32_t* row_map, float scale, int64_t window,
                      int64_t split_len, int kv_final, void* out, int64_t o_sb, int64_t o_sh, void* workspace,
                      int64_t workspace_bytes, int* err, void* stream, const AttnParams* qk) {
  if (batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || max_len <= 0) return kErrShape;
  if (batch == 0) return kOk;
  if (num_heads % num_kv_heads != 0 || num_heads / num_kv_heads > 8) return kErrShape;
  if (head_dim != 64 && head_dim != 128 && head_dim != 256) return kErrShape;
  if (split_len != 32 && split_len != 64 && split_len != 128) return kErrShape;
  if (x_dtype != kF32 && x_dtype != kBF16) return kErrDtype;
  if ((!q && !qk) || !k_cache || !v_cache || !seqlen || !out || !err) return kErrShape;
  const int es = x_dtype == kBF16 ? 2 : 4;
  if ((reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15) ||
      ((cache_sb * es) & 15) || ((cache_sh * es) & 15))
    return kErrAlign;
  const int64_t ns = (max_len + split_len - 1) / split_len;
  if (batch * num_kv_heads * (int64_t)sizeof(unsigned) > kAttnTicketBytes || ns > 65535 || batch > 65535)
    return kErrShape;
  if (ns > 16 && (!workspace || workspace_bytes < maple_decode_gqa_workspace_bytes(batch, num_heads, head_dim,
                                                                                   max_len, split_len)))
    return kErrWorkspace;
  AttnParams p = qk ? *qk : AttnParams{};
  p.q = q; p.kc = k_cache; p.vc = v_cache; p.seqlen = seqlen; p.row_map = row_map; p.out = out; p.err = err;
  p.tickets = static_cast<unsigned*>(workspace);
  p.ws_acc = workspace ? reinterpret_cast<float*>(static_cast<char*>(workspace) + kAttnTicketBytes) : nullptr;
  p.ws_ml = p.ws_acc ? p.ws_acc + batch * num_heads * ns * head_dim : nullptr;
  p.q_sb = q_sb; p.q_sh = q_sh; p.kc_sb = cache_sb; p.kc_sh = cache_sh; p.vc_sb = cache_sb; p.vc_sh = cache_sh;
  p.o_sb = o_sb; p.o_sh = o_sh;
  p.Hq = (int)num_heads; p.Hkv = (int)num_kv_heads; p.G = (int)(num_heads / num_kv_heads);
  p.Bc = (int)cache_batch; p.T = (int)max_len; p.P = (int)split_len; p.NS = (int)ns;
  p.window = (int)window; p.scale = scale; p.kv_final = kv_final;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (ns <= 16) {
    // one cluster of CL >= ns CTAs per (row, kv head), merged in shared memory
    int cl = 1;
    while (cl < ns) cl *= 2;
    const size_t smem = 2 * (size_t)split_len * head_dim * es + 2 * 8 * (size_t)split_len * sizeof(float) +
                        (8 * (size_t)head_dim + 16) * sizeof(float) + (qk ? 5 * (size_t)head_dim * sizeof(float) : 0);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)cl, (unsigned)num_kv_heads, (unsigned)batch);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = cl;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 2 : 1;
    cudaError_t e = cudaSuccess;
#define MB_ATTC(XT, DD)                                                                                       \
  do {                                                                                                        \
    auto kern = qk ? gqa_cluster_kernel<XT, DD, true> : gqa_cluster_kernel<XT, DD, false>;                    \
    if (cl > 8) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);            \
    if (e == cudaSuccess && smem > 32 * 1024)                                                                 \
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                 \
    if (e == cudaSuccess) e = cudaLaunchKernelEx(&cfg, kern, p);                                              \
  } while (0)
    if (x_dtype == kBF16) {
      if (head_dim == 64) MB_ATTC(kBF16, 64); else if (head_dim == 128) MB_ATTC(kBF16, 128); else MB_ATTC(kBF16, 256);
    } else {
      if (head_dim == 64) MB_ATTC(kF32, 64); else if (head_dim == 128) MB_ATTC(kF32, 128); else MB_ATTC(kF32, 256);
    }
#undef MB_ATTC
    return e == cudaSuccess ? kOk : kErrCuda;
  }
  const size_t smem = 2 * (size_t)split_len * head_dim * es + 2 * 8 * (size_t)split_len * sizeof(float) +
                      (qk ? 13 * (size_t)head_dim * sizeof(float) : 0);
  dim3 grid((unsigned)ns, (unsigned)num_kv_heads, (unsigned)batch);
  cudaError_t e = cudaSuccess;
  // Long contexts: the splits' merge gets its own launch spread over
  // (row, query head) CTAs instead of one CTA per (row, kv head).
  p.defer_merge = ns >= 128 ? 1 : 0;
#define MB_ATT(XT, DD)                                                                        \
  do {                                                                                        \
    auto kern = qk ? gqa_decode_kernel<XT, DD, true> : gqa_decode_kernel<XT, DD, false>;       \
    if (smem > 32 * 1024) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    if (e == cudaSuccess) e = launch_k(kern, dim3(grid), dim3(128), smem, st, p);                               \
    if (e == cudaSuccess && p.defer_merge)                                                    \
      e = launch_k(gqa_merge_kernel<XT, DD>, dim3((unsigned)num_heads, (unsigned)batch), dim3(DD), 0, st, p);   \
  } while (0)
  if (x_dtype == kBF16) {
    if (head_dim == 64) MB_ATT(kBF16, 64); else if (head_dim == 128) MB_ATT(kBF16, 128); else MB_ATT(kBF16, 256);
  } else {
    if (head_dim == 64) MB_ATT(kF32, 64); else if (head_dim == 128) MB_ATT(kF32, 128); else MB_ATT(kF32, 256);
  }
#undef MB_ATT
  if (e != cudaSuccess) return kErrCuda;
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_decode_gqa_attn(const void* q, int x_dtype, int64_t batch, int64_t num_heads,
                                     int64_t q_sb, int64_t q_sh, const void* k_cache, const void* v_cache,
                                     int64_t cache_batch, int64_t num_kv_heads, int64_t cache_sb,
                                     int64_t cache_sh, int64_t max_len, int64_t head_dim,
                                     const int64_t* seqlen, const int32_t* row_map, float scale,
                                     int64_t window, int64_t split_len, int kv_final, void* out,
                                     int64_t o_sb, int64_t o_sh, void* workspace, int64_t workspace_bytes,
                                     int* err, void* stream) {
  return gqa_common(q, x_dtype, batch, num_heads, q_sb, q_sh, k_cache, v_cache, cache_batch, num_kv_heads, cache_sb,
                    cache_sh, max_len, head_dim, seqlen, row_map, scale, window, split_len, kv_final, out, o_sb, o_sh,
                    workspace, workspace_bytes, err, stream, nullptr);
}

extern "C" int maple_decode_gqa_attn_qk(const void* qkv, int x_dtype, int64_t batch, int64_t qkv_row_stride,
                                        const void* q_weight, const void* k_weight, int w_dtype, const void* cos,
                                        const void* sin, int cs_dtype, int64_t cs_row_stride, int64_t cs_table_len,
                                        int64_t rotary_dim, int use_rope, float eps, int64_t num_heads,
                                        const void* k_cache, const void* v_cache, int64_t cache_batch,
                                        int64_t num_kv_heads, int64_t cache_sb, int64_t cache_sh, int64_t max_len,
                                        int64_t head_dim, const int64_t* seqlen, const int32_t* row_map,
                                        float scale, int64_t window, int64_t split_len, void* out, int64_t o_sb,
                                        int64_t o_sh, void* workspace, int64_t workspace_bytes, int* err,
                                        void* stream) {
  if (!qkv || !q_weight || !k_weight) return kErrShape;
  if ((w_dtype != kF32 && w_dtype != kBF16) || (cs_dtype != kF32 && cs_dtype != kBF16)) return kErrDtype;
  if (rotary_dim < 0 || rotary_dim > head_dim || (rotary_dim & 1)) return kErrShape;
  if (use_rope && (!cos || !sin || cs_table_len <= 0)) return kErrShape;
  AttnParams qk{};
  qk.qkv = qkv; qk.qkv_sb = qkv_row_stride; qk.q_w = q_weight; qk.k_w = k_weight; qk.w_f32 = w_dtype == kF32;
  qk.cos = cos; qk.sin = sin; qk.cs_f32 = cs_dtype == kF32; qk.cs_sb = cs_row_stride; qk.cs_len = cs_table_len;
  qk.R = (int)rotary_dim; qk.use_rope = use_rope; qk.eps = eps;
  return gqa_common(nullptr, x_dtype, batch, num_heads, 0, 0, k_cache, v_cache, cache_batch, num_kv_heads, cache_sb,
                    cache_sh, max_len, head_dim, seqlen, row_map, scale, window, split_len, 1, out, o_sb, o_sh,
                    workspace, workspace_bytes, err, stream, &qk);
}

// Positions per CTA of the tensor-core attention.  A function of the cache
// length only, so a row's split boundaries (and so its rounding) do not depend
// on the batch: batched decode equals per-sequence decode, and expert-parallel
// ranks (the same cache length, fewer rows) equal one GPU, bit for bit.
// 512 positions where rows x kv heads fill the GPU (batched decode at 8-16K),
// 256 for short caches and for very long ones, whose few rows still need
// about four waves of CTAs.
static int64_t gqa_tc_split(int64_t max_len) { return (max_len >= 8192 && max_len < 32768) ? 512 : 256; }

extern "C" int64_t maple_decode_gqa_attn_tc_workspace_bytes(int64_t batch, int64_t num_heads, int64_t head_dim,
                                                            int64_t max_len) {
  if (batch <= 0 || max_len <= 0) return -1;
  return maple_decode_gqa_workspace_bytes(batch, num_heads, head_dim, max_len, gqa_tc_split(max_len));
}

extern "C" int maple_decode_gqa_attn_tc(const void* q, int x_dtype, int64_t batch, int64_t num_heads, int64_t q_sb,
                                        int64_t q_sh, const void* k_cache, const void* v_cache, int64_t cache_batch,
                                        int64_t num_kv_heads, int64_t cache_sb, int64_t cache_sh, int64_t max_len,
                                        int64_t head_dim, const int64_t* seqlen, const int32_t* row_map,
                                        float scale, int64_t window, void* out, int64_t o_sb, int64_t o_sh,
                                        void* workspace, int64_t workspace_bytes, int* err, void* stream) {
  if (batch < 0 || num_heads <= 0 || num_kv_heads <= 0 || max_len <= 0) return kErrShape;
  if (batch == 0) return kOk;
  if (x_dtype != kBF16) return kErrDtype;
  if (num_heads % num_kv_heads != 0 || num_heads / num_kv_heads > 8) return kErrShape;
  if (head_dim != 64 && head_dim != 128) return kErrShape;
  if (!q || !k_cache || !v_cache || !seqlen || !out || !err || batch > 65535) return kErrShape;
  if ((reinterpret_cast<uintptr_t>(k_cache) & 15) || (reinterpret_cast<uintptr_t>(v_cache) & 15) ||
      ((cache_sb * 2) & 15) || ((cache_sh * 2) & 15) || (reinterpret_cast<uintptr_t>(q) & 3) || (q_sb & 1) ||
      (q_sh & 1))
    return kErrAlign;
  const int64_t sp = gqa_tc_split(max_len);
  const int64_t ns = (max_len + sp - 1) / sp;
  if (ns > 65535) return kErrShape;
  if (ns > 1 && (!workspace || workspace_bytes < maple_decode_gqa_workspace_bytes(batch, num_heads, head_dim,
                                                                                  max_len, sp)))
    return kErrWorkspace;
  AttnParams p{};
  p.q = q; p.kc = k_cache; p.vc = v_cache; p.seqlen = seqlen; p.row_map = row_map; p.out = out; p.err = err;
  p.ws_acc = workspace ? reinterpret_cast<float*>(static_cast<char*>(workspace) + kAttnTicketBytes) : nullptr;
  p.ws_ml = p.ws_acc ? p.ws_acc + batch * num_heads * ns * head_dim : nullptr;
  p.q_sb = q_sb; p.q_sh = q_sh; p.kc_sb = cache_sb; p.kc_sh = cache_sh; p.vc_sb = cache_sb; p.vc_sh = cache_sh;
  p.o_sb = o_sb; p.o_sh = o_sh;
  p.Hq = (int)num_heads; p.Hkv = (int)num_kv_heads; p.G = (int)(num_heads / num_kv_heads);
  p.Bc = (int)cache_batch; p.T = (int)max_len; p.P = (int)sp; p.NS = (int)ns;
  p.window = (int)window; p.scale = scale;
  // 4-D maps of the caches: (dim, position, kv head, cache row), boxes of 64 x 64
  CUtensorMap tmk, tmv;
  if (!tmap_bf16_4d(k_cache, head_dim, max_len, num_kv_heads, cache_batch, head_dim, cache_sh, cache_sb, 64,
                    kTcChunk, &tmk) ||
      !tmap_bf16_4d(v_cache, head_dim, max_len, num_kv_heads, cache_batch, head_dim, cache_sh, cache_sb, 64,
                    kTcChunk, &tmv))
    return kErrCuda;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid((unsigned)ns, (unsigned)num_kv_heads, (unsigned)batch);
  cudaError_t e = cudaSuccess;
#define MB_TC(DD)                                                                                              \
  do {                                                                                                         \
    const size_t smem = (size_t)kTcStages * 2 * (DD / 64) * 8192 + 1024;                                       \
    e = cudaFuncSetAttribute(gqa_tc_kernel<DD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);       \
    if (e == cudaSuccess) e = launch_k(gqa_tc_kernel<DD>, grid, dim3(128), smem, st, p, tmk, tmv);             \
    if (e == cudaSuccess && ns > 1)                                                                            \
      e = launch_k(gqa_tc_merge_kernel<DD>, dim3((unsigned)num_heads, (unsigned)batch), dim3(256), 0, st, p);   \
  } while (0)
  if (head_dim == 64) MB_TC(64); else MB_TC(128);
#undef MB_TC
  if (e != cudaSuccess) return kErrCuda;
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}
