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
// Expert-parallel exchange over NVLink peer memory (no NCCL).  Every rank
// holds one symmetric buffer (same size and layout on all ranks, mapped into
// the others through CUDA IPC): a dispatch receive area, a combine receive
// area, and flags.  Data moves by plain 16-byte stores into the peers'
// buffers; a store-release of a flag (or a release add on a counter) at
// system scope follows the data, and the receiver polls it with load-acquire
// in a bounded loop (a wait that gives up sets bit 1 of the error word and
// the kernel returns).  Sequence numbers come from a per-rank device counter
// that the last CTA of each call advances, so the calls can live in a CUDA
// graph.  These kernels are launched without programmatic dependent launch:
// all of their CTAs are resident together (grids of at most 64 CTAs) while
// some of them wait.
namespace mb {

constexpr int kP2PChunks = 4;          // CTAs per destination in the all-gather
constexpr int kP2PCombineCtas = 64;
constexpr int kP2PSpins = 1 << 20;     // bounded polls (about a second)
constexpr int kP2PMaxWorld = 8;

struct P2PParams {
  unsigned char* base[kP2PMaxWorld];  // every rank's symmetric buffer (this rank's at [rank])
  int64_t off_recv, off_flags;
  int rank, world;
  unsigned* seq;     // this rank's call counter
  unsigned* ticket;  // this rank's last-CTA ticket
  int* err;
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_add_release_sys(unsigned* p, unsigned v) {
  asm volatile("red.release.sys.global.add.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}

// Wait until *p >= target (wrap-aware); false on timeout.
__device__ __forceinline__ bool wait_geq(const unsigned* p, unsigned target) {
  for (int i = 0; i < kP2PSpins; ++i)
    if ((int)(ld_acquire_sys(p) - target) >= 0) return true;
  return false;
}

// The last CTA to finish advances this rank's call counter.
__device__ __forceinline__ void p2p_finish(const P2PParams& q, unsigned seq) {
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

// All-gather: this rank's `bytes` from src go to offset rank*bytes of every
// rank's receive area.  grid = world * kP2PChunks; CTA 0 waits for all.
__global__ void __launch_bounds__(256) p2p_allgather_kernel(P2PParams q, const uint4* src, int64_t n16) {
  const int d = blockIdx.x / kP2PChunks, c = blockIdx.x % kP2PChunks;
  const unsigned seq = *q.seq + 1u;
  uint4* dst = reinterpret_cast<uint4*>(q.base[d] + q.off_recv) + (int64_t)q.rank * n16;
  const int64_t per = (n16 + kP2PChunks - 1) / kP2PChunks;
  const int64_t lo = c * per, hi = min(n16, lo + per);
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) dst[i] = src[i];
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0)
    st_release_sys(reinterpret_cast<unsigned*>(q.base[d] + q.off_flags) + q.rank * kP2PChunks + c, seq);
  if (blockIdx.x == 0) {
    const unsigned* mine = reinterpret_cast<const unsigned*>(q.base[q.rank] + q.off_flags);
    bool ok = true;
    for (int f = threadIdx.x; f < q.world * kP2PChunks; f += blockDim.x) ok = wait_geq(mine + f, seq) && ok;
    if (!ok) atomicOr(q.err, 1);
  }
  p2p_finish(q, seq);
}

// Combine: phase 1 sends every slot row this rank computed (its experts) to
// the rank owning the slot's token, at recv[rank][slot - owner*T*k]; phase 2
// waits for all ranks and forms out[t] = sum_j w[t,j] * recv[owner(e_tj)][t*k+j]
// (+ residual) in moe_reduce_add's order.
template <int XT>
__global__ void __launch_bounds__(256) p2p_combine_kernel(P2PParams q, const void* y, const int* ids_all, int T,
                                                          int topk, int N, int E, const int* ids_mine,
                                                          const float* w_mine, const void* residual, void* out) {
  const int es = XT == kBF16 ? 2 : 4;
  const unsigned seq = *q.seq + 1u;
  const int per = E / q.world;
  const int e_first = q.rank * per;
  const int slots = q.world * T * topk;
  const int n16 = N * es / 16;
  for (int s = blockIdx.x; s < slots; s += gridDim.x) {
    int e = ids_all[s];
    if (e < 0 || e >= E) e = 0;
    if (e < e_first || e >= e_first + per) continue;
    const int owner = s / (T * topk);
    const uint4* src = reinterpret_cast<const uint4*>(static_cast<const char*>(y) + (int64_t)s * N * es);
    uint4* dst = reinterpret_cast<uint4*>(q.base[owner] + q.off_recv +
                                          ((int64_t)q.rank * T * topk + (s - owner * T * topk)) * N * es);
    for (int i = threadIdx.x; i < n16; i += blockDim.x) dst[i] = src[i];
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0)
    for (int d = 0; d < q.world; ++d)
      red_add_release_sys(reinterpret_cast<unsigned*>(q.base[d] + q.off_flags) + kP2PMaxWorld * kP2PChunks + q.rank,
                          1u);
  const unsigned* cnt = reinterpret_cast<const unsigned*>(q.base[q.rank] + q.off_flags) + kP2PMaxWorld * kP2PChunks;
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if (threadIdx.x < q.world && !wait_geq(cnt + threadIdx.x, seq * gridDim.x)) {
    atomicOr(q.err, 1);
    s_ok = 0;
  }
  __syncthreads();
  if (s_ok) {
    const char* recv = reinterpret_cast<const char*>(q.base[q.rank] + q.off_recv);
    const int64_t rank_stride = (int64_t)T * topk * N;
    for (int t = blockIdx.x; t < T; t += gridDim.x) {
      for (int n = threadIdx.x; n < N; n += blockDim.x) {
        float acc = 0.0f;
        for (int j = 0; j < topk; ++j) {
          int e = ids_mine[t * topk + j];
          if (e < 0 || e >= E) e = 0;
          const int r = min(e / per, q.world - 1);
          acc = __fmaf_rn(w_mine[t * topk + j], load_f<XT>(recv + (r * rank_stride + ((int64_t)t * topk + j) * N) * es, n),
                          acc);
        }
        if (residual != nullptr) acc = __fadd_rn(acc, load_f<XT>(static_cast<const char*>(residual) + (int64_t)t * N * es, n));
        store_f<XT>(static_cast<char*>(out) + (int64_t)t * N * es, n, acc);
      }
    }
  }
  p2p_finish(q, seq);
}

inline int p2p_fill(P2PParams& q, void* const* bases, int world, int rank, int64_t off_recv, int64_t off_flags,
                    unsigned* seq, unsigned* ticket, int* err) {
  if (world < 1 || world > kP2PMaxWorld || rank < 0 || rank >= world || !bases || !seq || !ticket || !err)
    return kErrShape;
  for (int r = 0; r < world; ++r) {
    if (!bases[r] || (reinterpret_cast<uintptr_t>(bases[r]) & 15)) return kErrAlign;
    q.base[r] = static_cast<unsigned char*>(bases[r]);
  }
  if ((off_recv | off_flags) & 15) return kErrAlign;
  q.off_recv = off_recv;
  q.off_flags = off_flags;
  q.rank = rank;
  q.world = world;
  q.seq = seq;
  q.ticket = ticket;
  q.err = err;
  return kOk;
}

}  // namespace mb

using namespace mb;

extern "C" int64_t maple_p2p_flag_bytes(void) {
  return (int64_t)(kP2PMaxWorld * kP2PChunks + kP2PMaxWorld) * 4;
}

extern "C" int maple_p2p_allgather(void* const* peer_bases, int world, int rank, int64_t off_recv, int64_t off_flags,
                                   const void* src, int64_t bytes_per_rank, unsigned* seq, unsigned* ticket, int* err,
                                   void* stream) {
  P2PParams q{};
  if (int rc = p2p_fill(q, peer_bases, world, rank, off_recv, off_flags, seq, ticket, err)) return rc;
  if (bytes_per_rank < 0 || bytes_per_rank % 16 != 0) return kErrShape;
  if (!src || (reinterpret_cast<uintptr_t>(src) & 15)) return kErrAlign;
  p2p_allgather_kernel<<<world * kP2PChunks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      q, static_cast<const uint4*>(src), bytes_per_rank / 16);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_p2p_combine(void* const* peer_bases, int world, int rank, int64_t off_recv, int64_t off_flags,
                                 const void* y, int x_dtype, const int32_t* ids_all, int64_t tokens_per_rank,
                                 int64_t topk, int64_t n, int64_t n_experts, const int32_t* ids_mine,
                                 const float* w_mine, const void* residual, void* out, unsigned* seq,
                                 unsigned* ticket, int* err, void* stream) {
  P2PParams q{};
  if (int rc = p2p_fill(q, peer_bases, world, rank, off_recv, off_flags, seq, ticket, err)) return rc;
  if (tokens_per_rank <= 0 || topk <= 0 || n <= 0 || n_experts <= 0 || n_experts % world != 0) return kErrShape;
  if (x_dtype != kBF16 && x_dtype != kF32) return kErrDtype;
  if ((n * (x_dtype == kBF16 ? 2 : 4)) % 16 != 0) return kErrAlign;
  if (!y || !ids_all || !ids_mine || !w_mine || !out || (reinterpret_cast<uintptr_t>(y) & 15)) return kErrShape;
  if (world * tokens_per_rank * topk > (1LL << 30)) return kErrShape;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (x_dtype == kBF16)
    p2p_combine_kernel<kBF16><<<kP2PCombineCtas, 256, 0, st>>>(q, y, ids_all, (int)tokens_per_rank, (int)topk, (int)n,
                                                               (int)n_experts, ids_mine, w_mine, residual, out);
  else
    p2p_combine_kernel<kF32><<<kP2PCombineCtas, 256, 0, st>>>(q, y, ids_all, (int)tokens_per_rank, (int)topk, (int)n,
                                                              (int)n_experts, ids_mine, w_mine, residual, out);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}
