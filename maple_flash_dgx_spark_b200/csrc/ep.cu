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
