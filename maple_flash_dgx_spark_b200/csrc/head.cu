// Vocabulary side of the decode step: RTN-4 lm_head GEMV (dense and
// FlashHead-indexed), greedy argmax, the fused top-k / temperature / top-p
// sampler, and the embedding gather.
//
// Reference: kernels/rtn4.py:285-415 (rtn4_gemv, kernels :84-282),
// :514-611 (rtn4_indexed_gemv, kernel :418-511), :27-47 (rtn4_embedding);
// kernels/sampler.py:106-206 (fused_sample / fused_sample_batched, kernels
// :24-103); generate.py:147-148 (greedy argmax).
//
// RTN-4 contraction: w = s_g * c + b_g per group g, so
//   y = sum_g [ s_g * C_g + b_g * X_g ] * 2^-shift,
//   C_g = sum_{k in g} c_k X_k (exact, u8 codes x s8 FXA digits on the int8
//   tensor pipe), X_g = sum_{k in g} X_k (exact), accumulated in double in
//   group order as acc = (acc + s_g*C_g) + b_g*X_g, rounded once to fp32.
// Symmetric heads (biases == NULL) use b_g = -8 * s_g.
#include "bulk.cuh"
#include "fxa.cuh"
#include "launch.cuh"

namespace mb {

constexpr int kHeadTicketBytes = 1 << 20;
constexpr int kHeadPrefetch = 4;  // iterations in flight per warp

struct Rtn4Params {
  const void* x;           // [B, K]
  const uint32_t* codes;   // [rows, K/8] (or [n_clusters, C, K/8])
  const void* scales;      // [rows, K/G]
  const void* biases;      // [rows, K/G] or nullptr (symmetric)
  const int32_t* cluster_ids;  // indexed mode: [n_probes] or nullptr
  void* y;                 // [B, n_out]
  int64_t x_stride, y_stride;
  int n_out, K, nwords, G, iters, cluster_size, n_clusters;
};

template <int XT, int ST>
__global__ void __launch_bounds__(128) rtn4_gemv_kernel(Rtn4Params p) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ FxaBlock fb;
  __shared__ long long s_xg[64];  // per-group sums of X (K / G <= 64)
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int b = blockIdx.y;
  const int ngroups = p.K / p.G;
  const int iters = p.iters;
  uint2* frag = reinterpret_cast<uint2*>(smem);
  float* xsm = reinterpret_cast<float*>(smem + (size_t)iters * 128 * sizeof(uint2));

  // Persistent: this CTA streams 64-row blocks blockIdx.x, +gridDim.x, ...;
  // flattened (block, iteration) steps q keep kHeadPrefetch loads in flight
  // per lane across block boundaries.
  const int nblk = (p.n_out + 63) / 64;
  const int nb_my = blockIdx.x < nblk ? (nblk - 1 - blockIdx.x) / gridDim.x + 1 : 0;
  const int total = nb_my * iters;
  if (p.cluster_ids != nullptr) pdl_wait();  // probe ids come from the previous launch
  auto phys = [&](int r) -> int64_t {
    if (p.cluster_ids == nullptr) return r;
    const int probe = r / p.cluster_size, member = r - probe * p.cluster_size;
    int c = p.cluster_ids[probe];
    if (c < 0 || c >= p.n_clusters) c = 0;
    return (int64_t)c * p.cluster_size + member;
  };
  auto issue = [&](int q, uint4& ra, uint4& rb) {
    ra = make_uint4(0, 0, 0, 0);
    rb = make_uint4(0, 0, 0, 0);
    if (q >= total) return;
    const int blk = blockIdx.x + (q / iters) * gridDim.x, i = q - (q / iters) * iters;
    const int og = blk * 64 + 16 * warp + g, oh = og + 8;
    const int word = i * 16 + 4 * t;
    if (og < p.n_out) ra = ld_stream_u4(p.codes + phys(og) * p.nwords + word);
    if (oh < p.n_out) rb = ld_stream_u4(p.codes + phys(oh) * p.nwords + word);
  };
  uint4 wa[kHeadPrefetch], wb[kHeadPrefetch];
#pragma unroll
  for (int ii = 0; ii < kHeadPrefetch; ++ii) issue(ii, wa[ii], wb[ii]);

  pdl_wait();
  pdl_trigger();
  const void* xr = static_cast<const char*>(p.x) + b * p.x_stride * (XT == kBF16 ? 2 : 4);
  fxa_prologue<XT, kF32, false, 4, 128>(xr, nullptr, p.K, 0.0f, 0, iters, xsm, nullptr, frag, fb, s_xg, p.G);
  const int s = fb.s;
  const bool bad = (s == kFxaNonFinite);
  const float nanv = __int_as_float(0x7fc00000);
  const int es_s = ST == kBF16 ? 2 : 4;
  const int its_per_group = p.G >= 128 ? p.G / 128 : 1;
  const bool split_iter = p.G == 64;
  char* yr = static_cast<char*>(p.y) + b * p.y_stride * (XT == kBF16 ? 2 : 4);

  double acc_g = 0.0, acc_h = 0.0;
  int ca[4] = {0, 0, 0, 0}, cb[4] = {0, 0, 0, 0};
  int cur_blk = -1;
  bool ok_g = false, ok_h = false;
  const char *sc_g = nullptr, *sc_h = nullptr, *bi_g = nullptr, *bi_h = nullptr;
  int out_g = 0, out_h = 0;

  auto finish_group = [&](int (&c)[4], int gi) {
    const long long pg = (long long)c[0] + 128LL * c[1];
    const long long ph = (long long)c[2] + 128LL * c[3];
    const long long ug = __shfl_down_sync(0xffffffffu, pg, 1);
    const long long uh = __shfl_down_sync(0xffffffffu, ph, 1);
    if (t == 0) {
      const long long Cg = pg + 16384LL * ug, Ch = ph + 16384LL * uh;
      const double xg = (double)s_xg[gi];
      const float sg = ok_g ? load_f<ST>(sc_g, gi) : 0.f, shh = ok_h ? load_f<ST>(sc_h, gi) : 0.f;
      const float bg = bi_g ? (ok_g ? load_f<ST>(bi_g, gi) : 0.f) : __fmul_rn(-8.0f, sg);
      const float bh = bi_h ? (ok_h ? load_f<ST>(bi_h, gi) : 0.f) : __fmul_rn(-8.0f, shh);
      acc_g = __dadd_rn(__dadd_rn(acc_g, __dmul_rn((double)sg, (double)Cg)), __dmul_rn((double)bg, xg));
      acc_h = __dadd_rn(__dadd_rn(acc_h, __dmul_rn((double)shh, (double)Ch)), __dmul_rn((double)bh, xg));
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) c[j] = 0;
  };

  for (int q0 = 0; q0 < total; q0 += kHeadPrefetch) {
#pragma unroll
    for (int ii = 0; ii < kHeadPrefetch; ++ii) {
      const int q = q0 + ii;
      if (q < total) {
        const int blk = blockIdx.x + (q / iters) * gridDim.x, i = q - (q / iters) * iters;
        if (blk != cur_blk) {
          cur_blk = blk;
          out_g = blk * 64 + 16 * warp + g;
          out_h = out_g + 8;
          ok_g = out_g < p.n_out;
          ok_h = out_h < p.n_out;
          const int64_t pg = ok_g ? phys(out_g) : 0, ph = ok_h ? phys(out_h) : 0;
          sc_g = static_cast<const char*>(p.scales) + pg * ngroups * es_s;
          sc_h = static_cast<const char*>(p.scales) + ph * ngroups * es_s;
          bi_g = p.biases ? static_cast<const char*>(p.biases) + pg * ngroups * es_s : nullptr;
          bi_h = p.biases ? static_cast<const char*>(p.biases) + ph * ngroups * es_s : nullptr;
          acc_g = 0.0;
          acc_h = 0.0;
        }
        const uint32_t ga[4] = {wa[ii].x, wa[ii].y, wa[ii].z, wa[ii].w};
        const uint32_t gb[4] = {wb[ii].x, wb[ii].y, wb[ii].z, wb[ii].w};
        issue(q + kHeadPrefetch, wa[ii], wb[ii]);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          const uint32_t a0 = ga[m] & 0x0f0f0f0fu, a2 = (ga[m] >> 4) & 0x0f0f0f0fu;
          const uint32_t a1 = gb[m] & 0x0f0f0f0fu, a3 = (gb[m] >> 4) & 0x0f0f0f0fu;
          const uint2 bf = frag[(i * 4 + m) * 32 + lane];
          if (split_iter) {
            const uint2 lo = t < 2 ? bf : make_uint2(0u, 0u);
            const uint2 hi = t < 2 ? make_uint2(0u, 0u) : bf;
            mma_u8s8(ca, a0, a1, a2, a3, lo.x, lo.y);
            mma_u8s8(cb, a0, a1, a2, a3, hi.x, hi.y);
          } else {
            mma_u8s8(ca, a0, a1, a2, a3, bf.x, bf.y);
          }
        }
        if (split_iter) {
          finish_group(ca, 2 * i);
          finish_group(cb, 2 * i + 1);
        } else if ((i + 1) % its_per_group == 0) {
          finish_group(ca, i / its_per_group);
        }
        if (i == iters - 1 && t == 0) {
          if (ok_g) store_f<XT>(yr, out_g, bad ? nanv : __double2float_rn(acc_g * pow2d(-s)));
          if (ok_h) store_f<XT>(yr, out_h, bad ? nanv : __double2float_rn(acc_h * pow2d(-s)));
        }
      }
    }
  }
}

// ----------------------------------------------------------------- argmax --
// Greedy next token: first index of the maximum (NaN counts as the maximum,
// as torch.argmax does).  Blocks reduce 8192-element chunks; the last block
// of a row (ticket) merges.
__device__ __forceinline__ bool better(float a, int ia, float b, int ib) {
  const bool na = a != a, nb = b != b;
  if (na || nb) return na && (!nb || ia < ib);
  return a > b || (a == b && ia < ib);
}

template <int XT>
__global__ void __launch_bounds__(256) argmax_kernel(const void* logits, int64_t row_stride, int V,
                                                     float* ws_v, int* ws_i, unsigned* tickets,
                                                     int64_t* out) {
  __shared__ float sv[8];
  __shared__ int si[8];
  __shared__ int s_last;
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.y, nblk = gridDim.x;
  const char* row = static_cast<const char*>(logits) + b * row_stride * (XT == kBF16 ? 2 : 4);
  float bv = __int_as_float(0xff800000);
  int bi = 0x7fffffff;
  const int lo = blockIdx.x * 8192, hi = min(V, lo + 8192);
  constexpr int EPC = XT == kBF16 ? 8 : 4;   // elements per 16-byte vector
  constexpr int CPT = 8192 / EPC / 256;     // vectors per thread
  const int nvec = ((reinterpret_cast<uintptr_t>(row) & 15) == 0) ? (hi - lo) / EPC : 0;
  uint4 r[CPT];
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int c = tid + 256 * i;
    if (c < nvec) r[i] = ld_u4(row + (size_t)(lo + c * EPC) * (XT == kBF16 ? 2 : 4));
  }
#pragma unroll
  for (int i = 0; i < CPT; ++i) {
    const int c = tid + 256 * i;
    if (c < nvec) {
      float f[EPC];
      widen_u4<XT>(r[i], f);
#pragma unroll
      for (int e = 0; e < EPC; ++e)
        if (better(f[e], lo + c * EPC + e, bv, bi)) { bv = f[e]; bi = lo + c * EPC + e; }
    }
  }
  for (int k = lo + nvec * EPC + tid; k < hi; k += 256) {
    const float v = load_f<XT>(row, k);
    if (better(v, k, bv, bi)) { bv = v; bi = k; }
  }
  auto reduce = [&]() {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
      if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < 8; ++w)
        if (better(sv[w], si[w], bv, bi)) { bv = sv[w]; bi = si[w]; }
    }
  };
  reduce();
  if (nblk == 1) {
    if (tid == 0) out[b] = bi;
    return;
  }
  if (tid == 0) {
    ws_v[(int64_t)b * nblk + blockIdx.x] = bv;
    ws_i[(int64_t)b * nblk + blockIdx.x] = bi;
    __threadfence();
    const unsigned old = atomicAdd(&tickets[b], 1u);
    s_last = old == (unsigned)(nblk - 1);
    if (s_last) atomicExch(&tickets[b], 0u);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  bv = __int_as_float(0xff800000);
  bi = 0x7fffffff;
  for (int j = tid; j < nblk; j += 256) {
    const float v = __ldcg(&ws_v[(int64_t)b * nblk + j]);
    const int i = __ldcg(&ws_i[(int64_t)b * nblk + j]);
    if (better(v, i, bv, bi)) { bv = v; bi = i; }
  }
  __syncthreads();
  reduce();
  if (tid == 0) out[b] = bi;
}

// ---------------------------------------------------------------- sampler --
// Stage 1: top-K of each 4096-logit block by K rounds of argmax (ties ->
// lowest index).  Stage 2 (last block of the row): top-K of the candidates,
// p = exp((v - v_max) * inv_T), p /= R128 sum, nucleus keeps i while the
// sequential prefix before i is <= top_p, pick = #(prefix' <= u * total')
// clipped to K-1.
constexpr int kSampBlock = 4096;
constexpr int kSampMaxK = 64;

template <int XT>
__global__ void __launch_bounds__(256) sample_kernel(const void* logits, int64_t row_stride, int V, int K,
                                                     float inv_t, float top_p, const float* uniform,
                                                     float* cand_v, int* cand_i, unsigned* tickets,
                                                     int64_t* out) {
  __shared__ float sv[8];
  __shared__ int si[8];
  __shared__ int s_win;
  __shared__ int s_last;
  __shared__ float kv[kSampMaxK];
  __shared__ int ki[kSampMaxK];
  pdl_wait();
  pdl_trigger();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int b = blockIdx.y, nblk = gridDim.x;
  const char* row = static_cast<const char*>(logits) + b * row_stride * (XT == kBF16 ? 2 : 4);
  const float ninf = __int_as_float(0xff800000);
  constexpr int PER = kSampBlock / 256;
  float v[PER];
  const int base = blockIdx.x * kSampBlock;
#pragma unroll
  for (int j = 0; j < PER; ++j) {
    const int k = base + j * 256 + tid;
    v[j] = k < V ? load_f<XT>(row, k) : ninf;
  }
  auto block_best = [&](float& bv, int& bi) {
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
    }
    if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < 8; ++w)
        if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; }
      sv[0] = bv; si[0] = bi;
    }
    __syncthreads();
    bv = sv[0]; bi = si[0];
    __syncthreads();
  };
  float* cv = cand_v + (int64_t)b * nblk * K;
  int* ci = cand_i + (int64_t)b * nblk * K;
  for (int r = 0; r < K; ++r) {
    float bv = ninf;
    int bi = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int k = base + j * 256 + tid;
      if (v[j] > bv || (v[j] == bv && k < bi)) { bv = v[j]; bi = k; }
    }
    block_best(bv, bi);
    if (tid == 0) { cv[blockIdx.x * K + r] = bv; ci[blockIdx.x * K + r] = bi; }
#pragma unroll
    for (int j = 0; j < PER; ++j)
      if (base + j * 256 + tid == bi) v[j] = ninf;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned old = atomicAdd(&tickets[b], 1u);
    s_last = old == (unsigned)(nblk - 1);
    if (s_last) atomicExch(&tickets[b], 0u);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  // Stage 2: top-K of the nblk*K candidates, ordered (value desc, index asc).
  const int nc = nblk * K;
  for (int r = 0; r < K; ++r) {
    float bv = ninf;
    int bi = 0x7fffffff, bpos = -1;
    for (int j = tid; j < nc; j += 256) {
      const float x = __ldcg(&cv[j]);
      const int ix = __ldcg(&ci[j]);
      if (x > bv || (x == bv && ix < bi)) { bv = x; bi = ix; bpos = j; }
    }
    // carry the position along with the index for removal
#pragma unroll
    for (int m = 16; m >= 1; m >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
      const int op = __shfl_xor_sync(0xffffffffu, bpos, m);
      if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; bpos = op; }
    }
    if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
    __shared__ int sp[8];
    if (lane == 0) sp[warp] = bpos;
    __syncthreads();
    if (tid == 0) {
      for (int w = 1; w < 8; ++w)
        if (sv[w] > bv || (sv[w] == bv && si[w] < bi)) { bv = sv[w]; bi = si[w]; bpos = sp[w]; }
      kv[r] = bv; ki[r] = bi; s_win = bpos;
      if (bpos >= 0) cv[bpos] = ninf;
    }
    __syncthreads();
  }
  if (warp != 0) return;
  const float vmax = kv[0];
  float pr[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const int i = lane + 32 * u;
    pr[u] = i < K ? mexp(__fmul_rn(__fsub_rn(kv[i], vmax), inv_t)) : 0.0f;
  }
  const float sum = r128_lane_finish(pr[0], pr[1], 0.0f, 0.0f);
#pragma unroll
  for (int u = 0; u < 2; ++u) pr[u] = (lane + 32 * u < K) ? __fdiv_rn(pr[u], sum) : 0.0f;
  // Sequential prefixes on lane 0 (K <= 64).
  __shared__ float sp_[kSampMaxK];
  sp_[lane] = pr[0];
  sp_[lane + 32] = pr[1];
  __syncwarp();
  if (lane == 0) {
    float cum = 0.0f;
    for (int i = 0; i < K; ++i) {
      const float pi = sp_[i];
      cum = __fadd_rn(cum, pi);
      sp_[i] = (__fsub_rn(cum, pi) <= top_p) ? pi : 0.0f;
    }
  }
  __syncwarp();
  pr[0] = sp_[lane];
  pr[1] = sp_[lane + 32];
  const float total = r128_lane_finish(pr[0], pr[1], 0.0f, 0.0f);
  if (lane == 0) {
    const float u = __fmul_rn(uniform[b], total);
    float cum = 0.0f;
    int pick = 0;
    for (int i = 0; i < K; ++i) {
      cum = __fadd_rn(cum, sp_[i]);
      if (cum <= u) ++pick;
    }
    pick = min(pick, K - 1);
    out[b] = ki[pick];
  }
}

// ------------------------------------------------------------- embedding --
template <int OT, int TT>
__global__ void embed_bf16_kernel(const int64_t* ids, const void* table, int64_t V, int64_t H, void* out,
                                  int64_t out_stride, int* err) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.y;
  const int64_t id = ids[b];
  const bool ok = id >= 0 && id < V;
  if (!ok && threadIdx.x == 0 && blockIdx.x == 0) atomicOr(err, 2);
  for (int64_t k = blockIdx.x * blockDim.x + threadIdx.x; k < H; k += (int64_t)gridDim.x * blockDim.x) {
    const float v = ok ? load_f<TT>(static_cast<const char*>(table) + id * H * (TT == kBF16 ? 2 : 4), k) : 0.0f;
    store_f<OT>(static_cast<char*>(out) + b * out_stride * (OT == kBF16 ? 2 : 4), k, v);
  }
}

template <int OT, int ST>
__global__ void embed_rtn4_kernel(const int64_t* ids, const uint32_t* codes, const void* scales,
                                  const void* biases, int64_t V, int64_t H, int G, void* out,
                                  int64_t out_stride, int* err) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.y;
  const int64_t id = ids[b];
  const bool ok = id >= 0 && id < V;
  if (!ok && threadIdx.x == 0 && blockIdx.x == 0) atomicOr(err, 2);
  const int64_t ng = H / G;
  for (int64_t k = blockIdx.x * blockDim.x + threadIdx.x; k < H; k += (int64_t)gridDim.x * blockDim.x) {
    float v = 0.0f;
    if (ok) {
      const uint32_t w = codes[id * (H / 8) + k / 8];
      const float c = static_cast<float>((w >> (4 * (k & 7))) & 15u);
      const float s = load_f<ST>(scales, id * ng + k / G);
      const float bb = biases ? load_f<ST>(biases, id * ng + k / G) : __fmul_rn(-8.0f, s);
      v = __fadd_rn(__fmul_rn(c, s), bb);
    }
    store_f<OT>(static_cast<char*>(out) + b * out_stride * (OT == kBF16 ? 2 : 4), k, v);
  }
}

}  // namespace mb

namespace mb {
// ---------------------------------------------------- batched RTN-4 head --
// For B > 1 rows the head is streamed once per chunk of up to 2*NP rows
// instead of once per row: rtn4_encode_kernel FXA-encodes each row once (4-bit
// fragment layout, compact: entry (i*16 + l) for lane l < 16 of fragment
// i = it*4 + m) with its per-group sums X_g, and rtn4_gemm_kernel stages a
// chunk's digits in shared memory while a persistent grid of 8-warp CTAs
// streams 16-row tiles of the head, one MMA serving two rows (B columns 0-3
// row a, 4-7 row b).  The per-group double accumulation is the batch-1
// kernel's, so each row's logits are bit-identical to it.
constexpr int kXgStride = 64;  // group sums per row (K / G <= 64)

template <int XT>
__global__ void __launch_bounds__(256) rtn4_encode_kernel(const void* x, int64_t x_stride, int K, int G, uint2* frag,
                                                          int* meta, long long* xg) {
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ FxaBlock fb;
  __shared__ long long s_xg[kXgStride];
  const int iters = K / 128;
  uint2* fr = reinterpret_cast<uint2*>(smem);
  float* xsm = reinterpret_cast<float*>(smem + (size_t)iters * 128 * sizeof(uint2));
  const int64_t r = blockIdx.x;
  pdl_wait();
  pdl_trigger();
  const void* xr = static_cast<const char*>(x) + r * x_stride * (XT == kBF16 ? 2 : 4);
  fxa_prologue<XT, kF32, false, 4, 256>(xr, nullptr, K, 0.0f, 0, iters, xsm, nullptr, fr, fb, s_xg, G);
  uint4* o = reinterpret_cast<uint4*>(frag + r * iters * 64);
  const uint4* f4 = reinterpret_cast<const uint4*>(fr);
  for (int c = threadIdx.x; c < iters * 32; c += 256) o[c] = f4[(c >> 3) * 16 + (c & 7)];
  for (int g = threadIdx.x; g < kXgStride; g += 256) xg[r * kXgStride + g] = g < K / G ? s_xg[g] : 0;
  if (threadIdx.x < 8) meta[r * 8 + threadIdx.x] = threadIdx.x == 0 ? fb.s : 0;
}

struct Rtn4GemmParams {
  const uint32_t* codes;   // [n_out, K/8]
  const void* scales;      // [n_out, K/G]
  const void* biases;      // [n_out, K/G] or nullptr (symmetric)
  const uint2* frag;       // [B, iters*64]
  const int* meta;         // [B, 8]
  const long long* xg;     // [B, 64]
  void* y;                 // [B, n_out]
  int* err;
  int64_t y_stride;
  int n_out, K, nwords, G, iters, B;
};

template <int XT, int ST, int NP>
__global__ void __launch_bounds__(256, 1) rtn4_gemm_kernel(Rtn4GemmParams p) {
  constexpr int CH = 2 * NP;  // rows per chunk
  extern __shared__ __align__(16) unsigned char smem[];
  __shared__ uint64_t bar;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int g = lane >> 2, t = lane & 3;
  const int c0 = blockIdx.y * CH;
  const int nt = min(CH, p.B - c0);
  const int rowu2 = p.iters * 64;
  uint2* dig = reinterpret_cast<uint2*>(smem);
  long long* sxg = reinterpret_cast<long long*>(smem + (size_t)CH * rowu2 * sizeof(uint2));
  int* smeta = reinterpret_cast<int*>(sxg + CH * kXgStride);
  pdl_wait();
  pdl_trigger();
  if (tid == 0) mbar_init(&bar, 1);
  __syncthreads();
  if (tid == 0) {
    const unsigned b_dig = (unsigned)(nt * rowu2 * sizeof(uint2)), b_xg = (unsigned)(nt * kXgStride * 8),
                   b_meta = (unsigned)(nt * 32);
    mbar_expect_tx(&bar, b_dig + b_xg + b_meta);
    bulk_g2s(dig, p.frag + (int64_t)c0 * rowu2, b_dig, &bar);
    bulk_g2s(sxg, p.xg + (int64_t)c0 * kXgStride, b_xg, &bar);
    bulk_g2s(smeta, p.meta + (int64_t)c0 * 8, b_meta, &bar);
  }
  const bool ready = mbar_wait_bounded(&bar, 0);
  if (__syncthreads_or(!ready)) {
    if (tid == 0) atomicOr(p.err, kErrFlagTimeout);
    mbar_wait_bounded(&bar, 0);
    return;
  }
  const int ngroups = p.K / p.G;
  const bool split_iter = p.G == 64;
  const int ipg = p.G >= 128 ? p.G / 128 : 1;
  const int es_s = ST == kBF16 ? 2 : 4;
  const int ntiles = (p.n_out + 15) / 16;
  const int half = lane >> 4, l16 = lane & 15;
  const int my_tok = t >> 1;  // lanes t<2: row a of a pair, t>=2: row b
  const float nanv = __int_as_float(0x7fc00000);

  for (int tile = blockIdx.x * 8 + warp; tile < ntiles; tile += gridDim.x * 8) {
    const int rg = tile * 16 + g, rh = rg + 8;
    const bool ok_g = rg < p.n_out, ok_h = rh < p.n_out;
    const uint32_t* cgp = p.codes + (int64_t)(ok_g ? rg : 0) * p.nwords;
    const uint32_t* chp = p.codes + (int64_t)(ok_h ? rh : 0) * p.nwords;
    const char* sg_row = static_cast<const char*>(p.scales) + (int64_t)(ok_g ? rg : 0) * ngroups * es_s;
    const char* sh_row = static_cast<const char*>(p.scales) + (int64_t)(ok_h ? rh : 0) * ngroups * es_s;
    const char* bg_row = p.biases ? static_cast<const char*>(p.biases) + (int64_t)(ok_g ? rg : 0) * ngroups * es_s
                                  : nullptr;
    const char* bh_row = p.biases ? static_cast<const char*>(p.biases) + (int64_t)(ok_h ? rh : 0) * ngroups * es_s
                                  : nullptr;
    double accd[NP][2];
    int acc[NP][4], acc2[NP][4];
#pragma unroll
    for (int q = 0; q < NP; ++q) {
      accd[q][0] = accd[q][1] = 0.0;
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[q][j] = acc2[q][j] = 0;
    }
    auto load_w = [&](int it, uint4& ra, uint4& rb) {
      ra = make_uint4(0, 0, 0, 0);
      rb = make_uint4(0, 0, 0, 0);
      if (it < p.iters) {
        const int word = it * 16 + 4 * t;
        if (ok_g) ra = ld_stream_u4(cgp + word);
        if (ok_h) rb = ld_stream_u4(chp + word);
      }
    };
    auto finish = [&](int (&c)[NP][4], int gi) {
      float sg = 0.f, sh = 0.f, bg = 0.f, bh = 0.f;
      if ((t & 1) == 0) {
        sg = ok_g ? load_f<ST>(sg_row, gi) : 0.f;
        sh = ok_h ? load_f<ST>(sh_row, gi) : 0.f;
        bg = bg_row ? (ok_g ? load_f<ST>(bg_row, gi) : 0.f) : __fmul_rn(-8.0f, sg);
        bh = bh_row ? (ok_h ? load_f<ST>(bh_row, gi) : 0.f) : __fmul_rn(-8.0f, sh);
      }
#pragma unroll
      for (int q = 0; q < NP; ++q) {
        const long long pg = (long long)c[q][0] + 128LL * c[q][1];
        const long long ph = (long long)c[q][2] + 128LL * c[q][3];
        const long long ug = __shfl_down_sync(0xffffffffu, pg, 1);
        const long long uh = __shfl_down_sync(0xffffffffu, ph, 1);
        if ((t & 1) == 0) {
          const long long Cg = pg + 16384LL * ug, Ch = ph + 16384LL * uh;
          const double xgv = (double)sxg[(2 * q + my_tok) * kXgStride + gi];
          accd[q][0] = __dadd_rn(__dadd_rn(accd[q][0], __dmul_rn((double)sg, (double)Cg)), __dmul_rn((double)bg, xgv));
          accd[q][1] = __dadd_rn(__dadd_rn(accd[q][1], __dmul_rn((double)sh, (double)Ch)), __dmul_rn((double)bh, xgv));
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) c[q][j] = 0;
      }
    };
    uint4 wa[4], wb[4];
#pragma unroll
    for (int ii = 0; ii < 4; ++ii) load_w(ii, wa[ii], wb[ii]);
    for (int it0 = 0; it0 < p.iters; it0 += 4) {
#pragma unroll
      for (int ii = 0; ii < 4; ++ii) {
        const int it = it0 + ii;
        if (it < p.iters) {
          const uint32_t ga[4] = {wa[ii].x, wa[ii].y, wa[ii].z, wa[ii].w};
          const uint32_t gb[4] = {wb[ii].x, wb[ii].y, wb[ii].z, wb[ii].w};
          load_w(it + 4, wa[ii], wb[ii]);
#pragma unroll
          for (int m = 0; m < 4; ++m) {
            const uint32_t a0 = ga[m] & 0x0f0f0f0fu, a2 = (ga[m] >> 4) & 0x0f0f0f0fu;
            const uint32_t a1 = gb[m] & 0x0f0f0f0fu, a3 = (gb[m] >> 4) & 0x0f0f0f0fu;
            const int ent = (it * 4 + m) * 16 + l16;
#pragma unroll
            for (int q = 0; q < NP; ++q) {
              const uint2 bv = dig[(size_t)(2 * q + half) * rowu2 + ent];
              if (split_iter) {
                const uint2 lo = t < 2 ? bv : make_uint2(0u, 0u);
                const uint2 hi = t < 2 ? make_uint2(0u, 0u) : bv;
                mma_u8s8(acc[q], a0, a1, a2, a3, lo.x, lo.y);
                mma_u8s8(acc2[q], a0, a1, a2, a3, hi.x, hi.y);
              } else {
                mma_u8s8(acc[q], a0, a1, a2, a3, bv.x, bv.y);
              }
            }
          }
          if (split_iter) {
            finish(acc, 2 * it);
            finish(acc2, 2 * it + 1);
          } else if ((it + 1) % ipg == 0) {
            finish(acc, it / ipg);
          }
        }
      }
    }
    if ((t & 1) == 0) {
#pragma unroll
      for (int q = 0; q < NP; ++q) {
        const int tok = 2 * q + my_tok;
        if (tok < nt) {
          const int s = smeta[tok * 8];
          const bool bad = s == kFxaNonFinite;
          char* yr = static_cast<char*>(p.y) + (int64_t)(c0 + tok) * p.y_stride * (XT == kBF16 ? 2 : 4);
          if (ok_g) store_f<XT>(yr, rg, bad ? nanv : __double2float_rn(accd[q][0] * pow2d(-s)));
          if (ok_h) store_f<XT>(yr, rh, bad ? nanv : __double2float_rn(accd[q][1] * pow2d(-s)));
        }
      }
    }
  }
}

// ------------------------------------------------- per-row sampler draws --
// One uniform in [0, 1) per row from a counter-based generator: the
// splitmix64 finaliser of (row seed, step), the step a device counter that
// the kernel advances, so a captured decode graph draws fresh values on every
// replay.  Stands in for the per-request torch.Generator draws of
// server.py:591-596 (the sampler's parity is defined on the uniform).
__device__ __forceinline__ uint64_t row_mix(uint64_t z) {
  z += 0x9E3779B97F4A7C15ULL;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

__global__ void __launch_bounds__(1024) row_uniform_kernel(const uint64_t* seeds, int64_t* counter, int B, float* out) {
  pdl_wait();
  pdl_trigger();
  const uint64_t step = static_cast<uint64_t>(counter[0]);
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const uint64_t h = row_mix(row_mix(seeds[b]) ^ (step * 0xD1B54A32D192ED03ULL));
    out[b] = static_cast<float>(h >> 40) * (1.0f / 16777216.0f);
  }
  __syncthreads();
  if (threadIdx.x == 0) counter[0] = static_cast<int64_t>(step + 1);
}

int rtn4_launch(Rtn4Params& p, int x_dtype, int s_dtype, int64_t batch, void* stream) {
  const size_t smem = (size_t)p.iters * 128 * sizeof(uint2) + (size_t)p.K * sizeof(float);
  const int nblk = (p.n_out + 63) / 64;
  dim3 grid((unsigned)(nblk < 148 * 4 ? nblk : 148 * 4), (unsigned)batch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
#define MB_R4(XT, ST)                                                                        \
  do {                                                                                       \
    auto kern = rtn4_gemv_kernel<XT, ST>;                                                    \
    if (smem > 32 * 1024) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    if (e == cudaSuccess) launch_k(kern, dim3(grid), dim3(128), smem, st, p);                                  \
  } while (0)
  if (x_dtype == kBF16) { if (s_dtype == kBF16) MB_R4(kBF16, kBF16); else MB_R4(kBF16, kF32); }
  else { if (s_dtype == kBF16) MB_R4(kF32, kBF16); else MB_R4(kF32, kF32); }
#undef MB_R4
  if (e != cudaSuccess) return kErrCuda;
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int rtn4_checks(int x_dtype, int s_dtype, int64_t k, int64_t group) {
  if ((x_dtype != kF32 && x_dtype != kBF16) || (s_dtype != kF32 && s_dtype != kBF16)) return kErrDtype;
  if (k <= 0 || k % 128 != 0 || k > 8192) return kErrShape;
  if (group != 64 && (group % 128 != 0 || group > k)) return kErrShape;
  if (k % group != 0 || k / group > 64) return kErrShape;
  return kOk;
}
}  // namespace mb

using namespace mb;

extern "C" int maple_rtn4_gemv(const void* x, int x_dtype, int64_t batch, int64_t k, int64_t x_row_stride,
                               const uint32_t* codes, int64_t n, const void* scales, const void* biases,
                               int s_dtype, int64_t group_size, void* y, int64_t y_row_stride, void* stream) {
  if (batch < 0 || n < 0) return kErrShape;
  if (batch == 0 || n == 0) return kOk;
  if (int rc = rtn4_checks(x_dtype, s_dtype, k, group_size)) return rc;
  if (!x || !codes || !scales || !y) return kErrShape;
  if ((reinterpret_cast<uintptr_t>(codes) & 15) != 0) return kErrAlign;
  if (batch > 65535 || n > (1LL << 31) - 64) return kErrShape;
  Rtn4Params p{};
  p.x = x; p.codes = codes; p.scales = scales; p.biases = biases; p.y = y;
  p.x_stride = x_row_stride; p.y_stride = y_row_stride;
  p.n_out = (int)n; p.K = (int)k; p.nwords = (int)(k / 8); p.G = (int)group_size; p.iters = (int)(k / 128);
  return rtn4_launch(p, x_dtype, s_dtype, batch, stream);
}

extern "C" int maple_rtn4_indexed_gemv(const void* x, int x_dtype, int64_t batch, int64_t k,
                                       int64_t x_row_stride, const uint32_t* codes, int64_t n_clusters,
                                       int64_t cluster_size, const void* scales, const void* biases,
                                       int s_dtype, int64_t group_size, const int32_t* cluster_ids,
                                       int64_t n_probes, void* y, int64_t y_row_stride, void* stream) {
  if (batch < 0 || n_clusters <= 0 || cluster_size <= 0 || n_probes < 0) return kErrShape;
  if (batch == 0 || n_probes == 0) return kOk;
  if (int rc = rtn4_checks(x_dtype, s_dtype, k, group_size)) return rc;
  if (!x || !codes || !scales || !y || !cluster_ids) return kErrShape;
  if ((reinterpret_cast<uintptr_t>(codes) & 15) != 0) return kErrAlign;
  Rtn4Params p{};
  p.x = x; p.codes = codes; p.scales = scales; p.biases = biases; p.y = y; p.cluster_ids = cluster_ids;
  p.x_stride = x_row_stride; p.y_stride = y_row_stride;
  p.n_out = (int)(n_probes * cluster_size); p.K = (int)k; p.nwords = (int)(k / 8); p.G = (int)group_size;
  p.iters = (int)(k / 128); p.cluster_size = (int)cluster_size; p.n_clusters = (int)n_clusters;
  return rtn4_launch(p, x_dtype, s_dtype, batch, stream);
}

extern "C" int64_t maple_rtn4_frag_bytes(int64_t rows, int64_t k) {
  if (rows < 0 || k <= 0) return -1;
  return rows * (k / 128) * 64 * 8 + rows * (32 + kXgStride * 8);
}

// Batched head: scratch (maple_rtn4_frag_bytes) holds the encoded rows, their
// metadata and group sums.
extern "C" int maple_rtn4_gemm(const void* x, int x_dtype, int64_t batch, int64_t k, int64_t x_row_stride,
                               const uint32_t* codes, int64_t n, const void* scales, const void* biases, int s_dtype,
                               int64_t group_size, void* y, int64_t y_row_stride, void* scratch,
                               int64_t scratch_bytes, int* err, void* stream) {
  if (batch < 0 || n < 0) return kErrShape;
  if (batch == 0 || n == 0) return kOk;
  if (int rc = rtn4_checks(x_dtype, s_dtype, k, group_size)) return rc;
  if (k > 4096) return kErrShape;
  if (!x || !codes || !scales || !y || !err || !scratch) return kErrShape;
  if ((reinterpret_cast<uintptr_t>(codes) | reinterpret_cast<uintptr_t>(scratch)) & 15) return kErrAlign;
  if (((reinterpret_cast<uintptr_t>(x) & 15) != 0) || ((x_row_stride * (x_dtype == kBF16 ? 2 : 4)) & 15))
    return kErrAlign;
  if (scratch_bytes < maple_rtn4_frag_bytes(batch, k)) return kErrWorkspace;
  if (batch > 65535 * 16 || n > (1LL << 31) - 64) return kErrShape;
  const int K = (int)k, iters = K / 128;
  uint2* frag = static_cast<uint2*>(scratch);
  int* meta = reinterpret_cast<int*>(static_cast<char*>(scratch) + batch * iters * 64 * 8);
  long long* xg = reinterpret_cast<long long*>(meta + batch * 8);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
  const size_t esmem = (size_t)iters * 128 * sizeof(uint2) + (size_t)K * sizeof(float);
  if (x_dtype == kBF16) {
    if (esmem > 32 * 1024) e = cudaFuncSetAttribute(rtn4_encode_kernel<kBF16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)esmem);
    if (e == cudaSuccess) e = launch_k(rtn4_encode_kernel<kBF16>, dim3((unsigned)batch), dim3(256), esmem, st, x, x_row_stride, K, (int)group_size, frag, meta, xg);
  } else {
    if (esmem > 32 * 1024) e = cudaFuncSetAttribute(rtn4_encode_kernel<kF32>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)esmem);
    if (e == cudaSuccess) e = launch_k(rtn4_encode_kernel<kF32>, dim3((unsigned)batch), dim3(256), esmem, st, x, x_row_stride, K, (int)group_size, frag, meta, xg);
  }
  if (e != cudaSuccess) return kErrCuda;
  Rtn4GemmParams p{};
  p.codes = codes; p.scales = scales; p.biases = biases; p.frag = frag; p.meta = meta; p.xg = xg; p.y = y; p.err = err;
  p.y_stride = y_row_stride; p.n_out = (int)n; p.K = K; p.nwords = K / 8; p.G = (int)group_size; p.iters = iters;
  p.B = (int)batch;
  const int np = K <= 2048 ? 8 : 4;
  const int chunks = (int)((batch + 2 * np - 1) / (2 * np));
  const int ntiles = (int)((n + 15) / 16);
  int gx = 148 / chunks;
  if (gx < 1) gx = 1;
  if (gx > (ntiles + 7) / 8) gx = (ntiles + 7) / 8;
  const size_t smem = (size_t)2 * np * iters * 64 * sizeof(uint2) + (size_t)2 * np * (kXgStride * 8 + 32);
  dim3 grid((unsigned)gx, (unsigned)chunks);
#define MB_RG(XT, ST, NP)                                                                                    \
  do {                                                                                                       \
    auto kern = rtn4_gemm_kernel<XT, ST, NP>;                                                                \
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);                  \
    if (e == cudaSuccess) e = launch_k(kern, grid, dim3(256), smem, st, p);                                  \
  } while (0)
  if (np == 8) {
    if (x_dtype == kBF16) { if (s_dtype == kBF16) MB_RG(kBF16, kBF16, 8); else MB_RG(kBF16, kF32, 8); }
    else { if (s_dtype == kBF16) MB_RG(kF32, kBF16, 8); else MB_RG(kF32, kF32, 8); }
  } else {
    if (x_dtype == kBF16) { if (s_dtype == kBF16) MB_RG(kBF16, kBF16, 4); else MB_RG(kBF16, kF32, 4); }
    else { if (s_dtype == kBF16) MB_RG(kF32, kBF16, 4); else MB_RG(kF32, kF32, 4); }
  }
#undef MB_RG
  return e == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_row_uniform(const uint64_t* seeds, int64_t batch, int64_t* counter, float* out,
                                 void* stream) {
  if (batch < 0 || batch > 65535) return kErrShape;
  if (batch == 0) return kOk;
  if (!seeds || !counter || !out) return kErrShape;
  cudaError_t e = launch_k(row_uniform_kernel, dim3(1), dim3(1024), 0, static_cast<cudaStream_t>(stream), seeds,
                           counter, (int)batch, out);
  return e == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int64_t maple_argmax_workspace_bytes(int64_t batch, int64_t vocab) {
  const int64_t nblk = (vocab + 8191) / 8192;
  return kHeadTicketBytes + batch * nblk * 8;
}

extern "C" int maple_argmax(const void* logits, int x_dtype, int64_t batch, int64_t vocab, int64_t row_stride,
                            int64_t* out, void* workspace, int64_t workspace_bytes, void* stream) {
  if (batch < 0 || vocab <= 0) return kErrShape;
  if (batch == 0) return kOk;
  if (x_dtype != kF32 && x_dtype != kBF16) return kErrDtype;
  if (!logits || !out || batch > 65535 || vocab > (1LL << 31) - 8192) return kErrShape;
  const int64_t nblk = (vocab + 8191) / 8192;
  if (nblk > 1 && (!workspace || workspace_bytes < maple_argmax_workspace_bytes(batch, vocab))) return kErrWorkspace;
  if (batch * 4 > kHeadTicketBytes) return kErrShape;
  unsigned* tickets = static_cast<unsigned*>(workspace);
  float* wv = workspace ? reinterpret_cast<float*>(static_cast<char*>(workspace) + kHeadTicketBytes) : nullptr;
  int* wi = wv ? reinterpret_cast<int*>(wv + batch * nblk) : nullptr;
  dim3 grid((unsigned)nblk, (unsigned)batch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (x_dtype == kBF16) launch_k(argmax_kernel<kBF16>, dim3(grid), dim3(256), 0, st, logits, row_stride, (int)vocab, wv, wi, tickets, out);
  else launch_k(argmax_kernel<kF32>, dim3(grid), dim3(256), 0, st, logits, row_stride, (int)vocab, wv, wi, tickets, out);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int64_t maple_fused_sample_workspace_bytes(int64_t batch, int64_t vocab, int64_t top_k) {
  const int64_t nblk = (vocab + kSampBlock - 1) / kSampBlock;
  return kHeadTicketBytes + batch * nblk * top_k * 8;
}

extern "C" int maple_fused_sample(const void* logits, int x_dtype, int64_t batch, int64_t vocab,
                                  int64_t row_stride, const float* uniform, float temperature, float top_p,
                                  int64_t top_k, int64_t* out, void* workspace, int64_t workspace_bytes,
                                  void* stream) {
  if (batch < 0 || vocab <= 0) return kErrShape;
  if (batch == 0) return kOk;
  if (top_k <= 0 || top_k > kSampMaxK || !(temperature > 0.0f)) return kErrShape;
  if (x_dtype != kF32 && x_dtype != kBF16) return kErrDtype;
  if (!logits || !uniform || !out || batch > 65535) return kErrShape;
  if (!workspace || workspace_bytes < maple_fused_sample_workspace_bytes(batch, vocab, top_k)) return kErrWorkspace;
  if (batch * 4 > kHeadTicketBytes) return kErrShape;
  const int64_t nblk = (vocab + kSampBlock - 1) / kSampBlock;
  unsigned* tickets = static_cast<unsigned*>(workspace);
  float* cv = reinterpret_cast<float*>(static_cast<char*>(workspace) + kHeadTicketBytes);
  int* ci = reinterpret_cast<int*>(cv + batch * nblk * top_k);
  const float inv_t = (float)(1.0 / (double)temperature);
  dim3 grid((unsigned)nblk, (unsigned)batch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (x_dtype == kBF16)
    launch_k(sample_kernel<kBF16>, dim3(grid), dim3(256), 0, st, logits, row_stride, (int)vocab, (int)top_k, inv_t, top_p, uniform,
                                               cv, ci, tickets, out);
  else
    launch_k(sample_kernel<kF32>, dim3(grid), dim3(256), 0, st, logits, row_stride, (int)vocab, (int)top_k, inv_t, top_p, uniform,
                                              cv, ci, tickets, out);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_embedding(const int64_t* ids, int64_t batch, const void* table, int t_dtype, int64_t vocab,
                               int64_t hidden, void* out, int out_dtype, int64_t out_row_stride, int* err,
                               void* stream) {
  if (batch < 0 || vocab <= 0 || hidden <= 0) return kErrShape;
  if (batch == 0) return kOk;
  if ((t_dtype != kF32 && t_dtype != kBF16) || (out_dtype != kF32 && out_dtype != kBF16)) return kErrDtype;
  if (!ids || !table || !out || !err || batch > 65535) return kErrShape;
  dim3 grid((unsigned)((hidden + 255) / 256), (unsigned)batch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (out_dtype == kBF16) {
    if (t_dtype == kBF16) launch_k(embed_bf16_kernel<kBF16, kBF16>, dim3(grid), dim3(256), 0, st, ids, table, vocab, hidden, out, out_row_stride, err);
    else launch_k(embed_bf16_kernel<kBF16, kF32>, dim3(grid), dim3(256), 0, st, ids, table, vocab, hidden, out, out_row_stride, err);
  } else {
    if (t_dtype == kBF16) launch_k(embed_bf16_kernel<kF32, kBF16>, dim3(grid), dim3(256), 0, st, ids, table, vocab, hidden, out, out_row_stride, err);
    else launch_k(embed_bf16_kernel<kF32, kF32>, dim3(grid), dim3(256), 0, st, ids, table, vocab, hidden, out, out_row_stride, err);
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_rtn4_embedding(const int64_t* ids, int64_t batch, const uint32_t* codes, const void* scales,
                                    const void* biases, int s_dtype, int64_t vocab, int64_t hidden,
                                    int64_t group_size, void* out, int out_dtype, int64_t out_row_stride, int* err,
                                    void* stream) {
  if (batch < 0 || vocab <= 0 || hidden <= 0 || group_size <= 0) return kErrShape;
  if (batch == 0) return kOk;
  if (hidden % 8 != 0 || hidden % group_size != 0) return kErrShape;
  if ((s_dtype != kF32 && s_dtype != kBF16) || (out_dtype != kF32 && out_dtype != kBF16)) return kErrDtype;
  if (!ids || !codes || !scales || !out || !err || batch > 65535) return kErrShape;
  dim3 grid((unsigned)((hidden + 255) / 256), (unsigned)batch);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (out_dtype == kBF16) {
    if (s_dtype == kBF16) launch_k(embed_rtn4_kernel<kBF16, kBF16>, dim3(grid), dim3(256), 0, st, ids, codes, scales, biases, vocab, hidden, (int)group_size, out, out_row_stride, err);
    else launch_k(embed_rtn4_kernel<kBF16, kF32>, dim3(grid), dim3(256), 0, st, ids, codes, scales, biases, vocab, hidden, (int)group_size, out, out_row_stride, err);
  } else {
    if (s_dtype == kBF16) launch_k(embed_rtn4_kernel<kF32, kBF16>, dim3(grid), dim3(256), 0, st, ids, codes, scales, biases, vocab, hidden, (int)group_size, out, out_row_stride, err);
    else launch_k(embed_rtn4_kernel<kF32, kF32>, dim3(grid), dim3(256), 0, st, ids, codes, scales, biases, vocab, hidden, (int)group_size, out, out_row_stride, err);
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}
