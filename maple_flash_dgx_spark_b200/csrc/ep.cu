// Expert-parallel combine: the weighted top-k sum over expert outputs that
// came back from the ranks owning the experts.
//
// Reference: kernels/fused_norm.py:164-202 (moe_reduce_add) on the output of
// kernels/ternary_expert.py:125-234, and model.py:465-474 (the MoE block).
// Under expert parallelism (experts [r*E/W, (r+1)*E/W) on rank r) every rank
// computes the slots routed to its experts for all tokens; an all-to-all
// returns to each token's rank the W candidate rows per slot,
// recv[r][t*top_k + j], of which the owner's is the real one.  The sum is the
// single-GPU moe_reduce_add arithmetic (fmaf over j in slot order, then the
// residual), so expert-parallel decode is bit-identical to one GPU.
#include "bulk.cuh"
#include "common.cuh"
#include "launch.cuh"

namespace mb {

template <int XT>
__global__ void ep_combine_kernel(const void* recv, int64_t rank_stride, const int* ids, const float* w,
                                  const void* residual, void* y, int N, int topk, int E, int per_rank, int W) {
  pdl_wait();
  pdl_trigger();
  const int tok = blockIdx.y;
  const int n = blockIdx.x * blockDim.x + threadIdx.x;
  if (n >= N) return;
  const int es = XT == kBF16 ? 2 : 4;
  float acc = 0.0f;
  for (int j = 0; j < topk; ++j) {
    int e = ids[(int64_t)tok * topk + j];
    if (e < 0 || e >= E) e = 0;  // listed under expert 0, whose rank wrote a NaN row
    const int r = min(e / per_rank, W - 1);
    const char* row = static_cast<const char*>(recv) + (r * rank_stride + ((int64_t)tok * topk + j) * N) * es;
    acc = __fmaf_rn(w[(int64_t)tok * topk + j], load_f<XT>(row, n), acc);
  }
  if (residual != nullptr) acc = __fadd_rn(acc, load_f<XT>(static_cast<const char*>(residual) + (int64_t)tok * N * es, n));
  store_f<XT>(static_cast<char*>(y) + (int64_t)tok * N * es, n, acc);
}

}  // namespace mb

using namespace mb;

extern "C" int maple_ep_combine(const void* recv, int x_dtype, int64_t world, int64_t tokens, int64_t topk, int64_t n,
                                const int32_t* expert_ids, const float* topk_weight, int64_t n_experts,
                                const void* residual, void* y, void* stream) {
  if (world <= 0 || tokens < 0 || topk <= 0 || n <= 0 || n_experts <= 0 || n_experts % world != 0) return kErrShape;
  if (tokens == 0) return kOk;
  if (!recv || !expert_ids || !topk_weight || !y || tokens > 65535) return kErrShape;
  if (x_dtype != kBF16 && x_dtype != kF32) return kErrDtype;
  const int64_t rank_stride = tokens * topk * n;
  dim3 grid((unsigned)((n + 127) / 128), (unsigned)tokens);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = x_dtype == kBF16
                      ? launch_k(ep_combine_kernel<kBF16>, grid, dim3(128), 0, st, recv, rank_stride, expert_ids,
                                 topk_weight, residual, y, (int)n, (int)topk, (int)n_experts,
                                 (int)(n_experts / world), (int)world)
                      : launch_k(ep_combine_kernel<kF32>, grid, dim3(128), 0, st, recv, rank_stride, expert_ids,
                                 topk_weight, residual, y, (int)n, (int)topk, (int)n_experts,
                                 (int)(n_experts / world), (int)world);
  return e == cudaSuccess ? kOk : kErrCuda;
}

// ------------------------------------------------------------------------
// Expert-parallel exchange over NVLink peer memory (no NCCL), in tagged
// words: every 8 data bytes travel as one 16-byte store {d0, seq, d1, seq}
// into the receiver's buffer, and the receiver polls the words themselves
// until both tags equal the call's sequence number.  A 16-byte store reaches
// the peer as two 8-byte halves, each whole, so a half whose tag is current
// carries current data: no fence and no separate flag is needed (a
// system-scope fence costs microseconds per call, more than the data).  The
// cost is twice the bytes on the link, which at these sizes (kilobytes per
// row) is far below the latency saved.
//
// Every rank holds one symmetric buffer (same size and layout on all ranks,
// mapped into the others through CUDA IPC, zero-filled).  Sequence numbers
// come from a per-rank device counter that the last CTA of each call
// advances, so the calls can live in a CUDA graph; every rank makes the same
// calls in the same order, so the numbers agree.  A buffer area is written
// for call n+1 only after its reader finished call n: the writer must first
// pass an exchange that needs data the reader sends after reading.  Every
// poll is bounded (one budget per thread); a thread that runs out sets bit 1
// of the error word and stops waiting.  Both kernels are launched with
// programmatic dependent launch and read everything after the wait.
namespace mb {

constexpr int kP2PChunks = 16;         // CTAs per source rank in the dispatch
constexpr int kP2PUnroll = 4;          // words in flight per thread
constexpr int kP2PSpins = 1 << 20;     // polls per thread before giving up (about a second)
constexpr int kP2PMaxWorld = 8;
constexpr int kP2PMaxTopk = 8;
constexpr unsigned kP2PBadSlot = 0x80000000u;  // moe_plan's mark of an out-of-range expert id

struct P2PParams {
  unsigned char* base[kP2PMaxWorld];  // every rank's symmetric buffer (this rank's at [rank])
  int64_t off_ll;                     // this call's tagged-word area
  int rank, world;
  unsigned* seq;     // this rank's call counter
  unsigned* ticket;  // this rank's last-CTA ticket
  int* err;
};

__device__ __forceinline__ void st_tagged(uint4* p, uint2 d, unsigned tag) {
  asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};\n" ::"l"(p), "r"(d.x), "r"(tag), "r"(d.y),
               "r"(tag)
               : "memory");
}
__device__ __forceinline__ uint4 ld_tagged(const uint4* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}
__device__ __forceinline__ bool tagged_ready(const uint4& v, unsigned tag) { return v.y == tag && v.w == tag; }

// Re-poll one word until its tags are current or the thread's budget runs out.
__device__ __forceinline__ void poll_tagged(const uint4* p, uint4& v, unsigned tag, int& spins) {
  while (!tagged_ready(v, tag) && spins < kP2PSpins) {
    ++spins;
    v = ld_tagged(p);
  }
}

// The last CTA to finish advances this rank's call counter.
__device__ __forceinline__ void p2p_finish(const P2PParams& q, unsigned seq, bool ok) {
  if (!ok) atomicOr(q.err, kErrFlagTimeout);
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned t = atomicAdd(q.ticket, 1u);
    if (t == gridDim.x - 1) {
      *q.ticket = 0u;
      *q.seq = seq;
    }
  }
}

// Dispatch.  Row r of rank s is nx 8-byte words of x followed by ni words of
// its top-k ids (two per word, zero-padded); it travels as word row s*T + r
// of every rank's area.  grid = world * kP2PChunks: CTA (d, c) sends chunk c
// of this rank's rows to rank d, then receives chunk c of rank d's rows from
// this rank's own area into the dense outputs rows_out [world*T][nx words]
// and ids_out [world*T][topk].
__global__ void __launch_bounds__(256) p2p_dispatch_kernel(P2PParams q, const uint2* x, int64_t x_stride8, int nx,
                                                           int T, const int* ids, int topk, uint2* rows_out,
                                                           int* ids_out) {
  pdl_wait();
  pdl_trigger();
  const int d = blockIdx.x / kP2PChunks, c = blockIdx.x % kP2PChunks;
  const unsigned seq = *q.seq + 1u;
  const int ni = (topk + 1) / 2, wpr = nx + ni;
  const int per = (T + kP2PChunks - 1) / kP2PChunks;
  const int r0 = min(T, c * per), r1 = min(T, r0 + per);
  const int n = (r1 - r0) * wpr;
  uint4* dst = reinterpret_cast<uint4*>(q.base[d] + q.off_ll) + ((int64_t)q.rank * T + r0) * wpr;
  for (int i0 = threadIdx.x; i0 < n; i0 += kP2PUnroll * blockDim.x) {
    uint2 v[kP2PUnroll];
#pragma unroll
    for (int u = 0; u < kP2PUnroll; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i < n) {
        const int r = i / wpr, w = i - r * wpr;
        if (w < nx) {
          v[u] = x[(int64_t)(r0 + r) * x_stride8 + w];
        } else {
          const int j = 2 * (w - nx);
          const int* id = ids + (int64_t)(r0 + r) * topk + j;
          v[u] = make_uint2(static_cast<unsigned>(id[0]), j + 1 < topk ? static_cast<unsigned>(id[1]) : 0u);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < kP2PUnroll; ++u)
      if (i0 + u * blockDim.x < n) st_tagged(dst + i0 + u * blockDim.x, v[u], seq);
  }
  const uint4* src = reinterpret_cast<const uint4*>(q.base[q.rank] + q.off_ll) + ((int64_t)d * T + r0) * wpr;
  int spins = 0;
  for (int i0 = threadIdx.x; i0 < n; i0 += kP2PUnroll * blockDim.x) {
    uint4 v[kP2PUnroll];
#pragma unroll
    for (int u = 0; u < kP2PUnroll; ++u)
      if (i0 + u * blockDim.x < n) v[u] = ld_tagged(src + i0 + u * blockDim.x);
#pragma unroll
    for (int u = 0; u < kP2PUnroll; ++u) {
      const int i = i0 + u * blockDim.x;
      if (i >= n) continue;
      poll_tagged(src + i, v[u], seq, spins);
      const int r = i / wpr, w = i - r * wpr;
      const int64_t row = (int64_t)d * T + r0 + r;
      if (w < nx) {
        rows_out[row * nx + w] = make_uint2(v[u].x, v[u].z);
      } else {
        const int j = 2 * (w - nx);
        ids_out[row * topk + j] = static_cast<int>(v[u].x);
        if (j + 1 < topk) ids_out[row * topk + j + 1] = static_cast<int>(v[u].z);
      }
    }
  }
  p2p_finish(q, seq, spins < kP2PSpins);
}

// Combine.  Phase 1: the rows this rank's experts computed, y[s] for the
// slots s its plan lists (slot s = (owner*T + t)*topk + j of the gathered
// tokens, nx words each), go as word row t*topk + j of the owner's area;
// every slot has exactly one computing rank.  Phase 2: out[t] = sum_j
// w[t,j] * row(t*topk + j) (+ residual) for this rank's T tokens, 16 bytes
// per thread, in moe_reduce_add's order (fmaf over j, then the residual add).
template <int XT>
__global__ void __launch_bounds__(256) p2p_combine_kernel(P2PParams q, const uint2* y, const int* offsets,
                                                          const unsigned* slots, int n_local, int T, int topk,
                                                          int nx, const float* w, const uint4* residual,
                                                          uint4* out) {
  pdl_wait();
  pdl_trigger();
  const unsigned seq = *q.seq + 1u;
  const int n_mine = offsets[n_local];
  const int slots_all = q.world * T * topk;
  const int stride = gridDim.x * blockDim.x;
  // phase 1, one warp per listed slot row, kRowUnroll words in flight per lane
  constexpr int kRowUnroll = 8;
  const int lane = threadIdx.x & 31;
  const int nwarps = gridDim.x * (blockDim.x >> 5);
  bool bounds_ok = true;
  for (int r = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); r < n_mine; r += nwarps) {
    const int sl = static_cast<int>(slots[r] & ~kP2PBadSlot);
    if (sl >= slots_all) {
      bounds_ok = false;
      continue;
    }
    const int owner = sl / (T * topk);
    uint4* dst = reinterpret_cast<uint4*>(q.base[owner] + q.off_ll) + (int64_t)(sl - owner * T * topk) * nx;
    const uint2* src = y + (int64_t)sl * nx;
    for (int w0 = lane; w0 < nx; w0 += 32 * kRowUnroll) {
      uint2 v[kRowUnroll];
#pragma unroll
      for (int u = 0; u < kRowUnroll; ++u)
        if (w0 + 32 * u < nx) v[u] = src[w0 + 32 * u];
#pragma unroll
      for (int u = 0; u < kRowUnroll; ++u)
        if (w0 + 32 * u < nx) st_tagged(dst + w0 + 32 * u, v[u], seq);
    }
  }
  if (!bounds_ok) atomicOr(q.err, kErrFlagBounds);

  constexpr int EPV = XT == kBF16 ? 8 : 4;  // elements per 16 data bytes
  const int v16 = nx / 2;
  const uint4* ll = reinterpret_cast<const uint4*>(q.base[q.rank] + q.off_ll);
  int spins = 0;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < T * v16; i += stride) {
    const int t = i / v16, v = i - t * v16;
    uint4 a[kP2PMaxTopk], b[kP2PMaxTopk];
#pragma unroll
    for (int j = 0; j < kP2PMaxTopk; ++j) {
      if (j < topk) {
        const uint4* p = ll + (int64_t)(t * topk + j) * nx + 2 * v;
        a[j] = ld_tagged(p);
        b[j] = ld_tagged(p + 1);
      }
    }
    float acc[EPV];
#pragma unroll
    for (int e = 0; e < EPV; ++e) acc[e] = 0.0f;
#pragma unroll
    for (int j = 0; j < kP2PMaxTopk; ++j) {
      if (j < topk) {
        const uint4* p = ll + (int64_t)(t * topk + j) * nx + 2 * v;
        poll_tagged(p, a[j], seq, spins);
        poll_tagged(p + 1, b[j], seq, spins);
        const unsigned d4[4] = {a[j].x, a[j].z, b[j].x, b[j].z};
        const float wj = w[t * topk + j];
#pragma unroll
        for (int e = 0; e < EPV; ++e) {
          const float ye = XT == kBF16 ? bf16_to_f32(static_cast<uint16_t>(d4[e >> 1] >> (16 * (e & 1))))
                                       : __uint_as_float(d4[e]);
          acc[e] = __fmaf_rn(wj, ye, acc[e]);
        }
      }
    }
    if (residual != nullptr) {
      const uint4 r = residual[(int64_t)t * v16 + v];
      const unsigned r4[4] = {r.x, r.y, r.z, r.w};
#pragma unroll
      for (int e = 0; e < EPV; ++e)
        acc[e] = __fadd_rn(acc[e], XT == kBF16 ? bf16_to_f32(static_cast<uint16_t>(r4[e >> 1] >> (16 * (e & 1))))
                                               : __uint_as_float(r4[e]));
    }
    unsigned o4[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if constexpr (XT == kBF16)
        o4[e] = static_cast<unsigned>(f32_to_bf16(acc[2 * e])) | (static_cast<unsigned>(f32_to_bf16(acc[2 * e + 1])) << 16);
      else
        o4[e] = __float_as_uint(acc[e]);
    }
    out[(int64_t)t * v16 + v] = make_uint4(o4[0], o4[1], o4[2], o4[3]);
  }
  p2p_finish(q, seq, spins < kP2PSpins);
}

inline int p2p_fill(P2PParams& q, void* const* bases, int world, int rank, int64_t off_ll, unsigned* seq,
                    unsigned* ticket, int* err) {
  if (world < 1 || world > kP2PMaxWorld || rank < 0 || rank >= world || !bases || !seq || !ticket || !err)
    return kErrShape;
  for (int r = 0; r < world; ++r) {
    if (!bases[r] || (reinterpret_cast<uintptr_t>(bases[r]) & 15)) return kErrAlign;
    q.base[r] = static_cast<unsigned char*>(bases[r]);
  }
  if (off_ll & 15) return kErrAlign;
  q.off_ll = off_ll;
  q.rank = rank;
  q.world = world;
  q.seq = seq;
  q.ticket = ticket;
  q.err = err;
  return kOk;
}

// Combine grid: enough threads for one 16-byte output vector each in phase 2,
// 32..128 CTAs.
inline int p2p_combine_ctas(int64_t tokens, int64_t v16) {
  const int64_t want = (tokens * v16 + 255) / 256;
  return (int)(want < 32 ? 32 : want > 128 ? 128 : want);
}

}  // namespace mb

using namespace mb;

extern "C" int64_t maple_p2p_dispatch_bytes(int64_t world, int64_t tokens_per_rank, int64_t n, int x_dtype,
                                            int64_t topk) {
  if (world < 1 || tokens_per_rank <= 0 || n <= 0 || topk <= 0) return -1;
  const int64_t es = x_dtype == kBF16 ? 2 : 4;
  return world * tokens_per_rank * ((n * es + 7) / 8 + (topk + 1) / 2) * 16;
}

extern "C" int64_t maple_p2p_combine_bytes(int64_t tokens_per_rank, int64_t topk, int64_t n, int x_dtype) {
  if (tokens_per_rank <= 0 || n <= 0 || topk <= 0) return -1;
  const int64_t es = x_dtype == kBF16 ? 2 : 4;
  return tokens_per_rank * topk * ((n * es + 7) / 8) * 16;
}

extern "C" int maple_p2p_dispatch(void* const* peer_bases, int world, int rank, int64_t off_ll, const void* x,
                                  int x_dtype, int64_t x_row_stride, int64_t tokens_per_rank, int64_t n,
                                  const int32_t* expert_ids, int64_t topk, void* rows_out, int32_t* ids_out,
                                  unsigned* seq, unsigned* ticket, int* err, void* stream) {
  P2PParams q{};
  if (int rc = p2p_fill(q, peer_bases, world, rank, off_ll, seq, ticket, err)) return rc;
  if (tokens_per_rank <= 0 || n <= 0 || topk <= 0 || x_row_stride < n) return kErrShape;
  if (x_dtype != kBF16 && x_dtype != kF32) return kErrDtype;
  const int es = x_dtype == kBF16 ? 2 : 4;
  if ((n * es) % 16 != 0 || (x_row_stride * es) % 8 != 0) return kErrAlign;
  if (!x || !expert_ids || !rows_out || !ids_out) return kErrShape;
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(rows_out)) & 15) return kErrAlign;
  if (world * tokens_per_rank * (n * es / 8 + topk) > (1LL << 30)) return kErrShape;
  return launch_k(p2p_dispatch_kernel, dim3(world * kP2PChunks), dim3(256), 0, static_cast<cudaStream_t>(stream), q,
                  static_cast<const uint2*>(x), x_row_stride * es / 8, (int)(n * es / 8), (int)tokens_per_rank,
                  expert_ids, (int)topk, static_cast<uint2*>(rows_out), ids_out) == cudaSuccess
             ? kOk
             : kErrCuda;
}

extern "C" int maple_p2p_combine(void* const* peer_bases, int world, int rank, int64_t off_ll, const void* y,
                                 int x_dtype, const int32_t* plan_offsets, const uint32_t* plan_slots,
                                 int64_t n_local_experts, int64_t tokens_per_rank, int64_t topk, int64_t n,
                                 const float* topk_weight, const void* residual, void* out, unsigned* seq,
                                 unsigned* ticket, int* err, void* stream) {
  P2PParams q{};
  if (int rc = p2p_fill(q, peer_bases, world, rank, off_ll, seq, ticket, err)) return rc;
  if (tokens_per_rank <= 0 || topk <= 0 || topk > kP2PMaxTopk || n <= 0 || n_local_experts <= 0) return kErrShape;
  if (x_dtype != kBF16 && x_dtype != kF32) return kErrDtype;
  const int es = x_dtype == kBF16 ? 2 : 4;
  if ((n * es) % 16 != 0) return kErrAlign;
  if (!y || !plan_offsets || !plan_slots || !topk_weight || !out) return kErrShape;
  if ((reinterpret_cast<uintptr_t>(y) | reinterpret_cast<uintptr_t>(out) | reinterpret_cast<uintptr_t>(residual)) &
      15)
    return kErrAlign;
  if (world * tokens_per_rank * topk * (n * es / 8) > (1LL << 30)) return kErrShape;
  const int64_t nx = n * es / 8;
  const dim3 grid((unsigned)p2p_combine_ctas(tokens_per_rank, nx / 2));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e =
      x_dtype == kBF16
          ? launch_k(p2p_combine_kernel<kBF16>, grid, dim3(256), 0, st, q, static_cast<const uint2*>(y), plan_offsets,
                     plan_slots, (int)n_local_experts, (int)tokens_per_rank, (int)topk, (int)nx, topk_weight,
                     static_cast<const uint4*>(residual), static_cast<uint4*>(out))
          : launch_k(p2p_combine_kernel<kF32>, grid, dim3(256), 0, st, q, static_cast<const uint2*>(y), plan_offsets,
                     plan_slots, (int)n_local_experts, (int)tokens_per_rank, (int)topk, (int)nx, topk_weight,
                     static_cast<const uint4*>(residual), static_cast<uint4*>(out));
  return e == cudaSuccess ? kOk : kErrCuda;
}
