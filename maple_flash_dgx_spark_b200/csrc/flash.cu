// FlashHead support: top-k cluster selection and the logit scatter.
//
// Reference: flash_head.py:330-369 (FlashHead.__call__): centroid scores ->
// torch.topk(n_probes) -> rtn4_indexed_gemv over the probed clusters ->
// index_put into a -inf row of the vocabulary.
//
// topk_select_kernel: one CTA radix-selects the k largest of n scores.  Keys
// are the scores mapped to order-preserving uint32 (NaN above +inf, as
// torch.topk ranks NaN highest); ties at the k-th key go to the lowest
// indices.  The selected indices are written in ascending index order (the
// set is what FlashHead uses; the order only permutes the probe rows).
#include "common.cuh"
#include "launch.cuh"

namespace mb {

__device__ __forceinline__ uint32_t order_key(float f) {
  if (f != f) return 0xffffffffu;
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

template <int XT>
__global__ void __launch_bounds__(1024) topk_select_kernel(const void* x, int n, int k, int* out) {
  __shared__ unsigned hist[256];
  __shared__ uint32_t s_prefix, s_mask;
  __shared__ int s_need;
  __shared__ int warp_gt[32], warp_eq[32];
  __shared__ int s_base_gt, s_base_eq;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();
  pdl_trigger();
  if (tid == 0) {
    s_prefix = 0;
    s_mask = 0;
    s_need = k;
  }
  __syncthreads();
  // Radix select (MSB first): after the 4 passes, s_prefix is the k-th key and
  // s_need is how many keys equal to it are taken.
  for (int pass = 0; pass < 4; ++pass) {
    const int shift = 24 - 8 * pass;
    for (int i = tid; i < 256; i += 1024) hist[i] = 0;
    __syncthreads();
    const uint32_t prefix = s_prefix, mask = s_mask;
    for (int i = tid; i < n; i += 1024) {
      const uint32_t key = order_key(load_f<XT>(x, i));
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      int need = s_need;
      int d = 255;
      for (; d > 0; --d) {
        if ((int)hist[d] >= need) break;
        need -= (int)hist[d];
      }
      s_prefix = prefix | ((uint32_t)d << shift);
      s_mask = mask | (255u << shift);
      s_need = need;
    }
    __syncthreads();
  }
  const uint32_t kth = s_prefix;
  const int take_eq = s_need;
  // Compaction in index order: keys above kth, then the first take_eq equal ones.
  if (tid == 0) {
    s_base_gt = 0;
    s_base_eq = 0;
  }
  __syncthreads();
  for (int c0 = 0; c0 < n; c0 += 1024) {
    const int i = c0 + tid;
    uint32_t key = 0;
    if (i < n) key = order_key(load_f<XT>(x, i));
    const bool gt = i < n && key > kth, eq = i < n && key == kth;
    const unsigned bg = __ballot_sync(0xffffffffu, gt), be = __ballot_sync(0xffffffffu, eq);
    if (lane == 0) {
      warp_gt[warp] = __popc(bg);
      warp_eq[warp] = __popc(be);
    }
    __syncthreads();
    int off_gt = s_base_gt, off_eq = s_base_eq;
    for (int w = 0; w < warp; ++w) {
      off_gt += warp_gt[w];
      off_eq += warp_eq[w];
    }
    const unsigned below = (1u << lane) - 1u;
    const int r_gt = off_gt + __popc(bg & below), r_eq = off_eq + __popc(be & below);
    const bool take = gt || (eq && r_eq < take_eq);
    // position in the output = selected keys with a lower index
    const int r_sel = r_gt + min(r_eq, take_eq);
    if (take) out[r_sel] = i;
    __syncthreads();
    if (tid == 0) {
      int tg = 0, te = 0;
      for (int w = 0; w < 32; ++w) {
        tg += warp_gt[w];
        te += warp_eq[w];
      }
      s_base_gt += tg;
      s_base_eq += te;
    }
    __syncthreads();
  }
}

template <int XT>
__global__ void fill_kernel(void* out, int64_t n, float v) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    store_f<XT>(out, i, v);
}

// out[token_map[cluster_ids[p]][i]] = probe[p*cs + i]; out[force_ids[j]] = force[j].
template <int XT>
__global__ void flash_scatter_kernel(const void* probe, const int* cluster_ids, int n_probes, int cs,
                                     const int* token_map, int n_clusters, const void* force, const int64_t* force_ids,
                                     int n_force, void* out, int64_t V, int* err) {
  pdl_wait();
  pdl_trigger();
  const int64_t total = (int64_t)n_probes * cs + n_force;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t tok;
    float v;
    if (i < (int64_t)n_probes * cs) {
      const int p = (int)(i / cs), r = (int)(i - (int64_t)p * cs);
      const int c = cluster_ids[p];
      if (c < 0 || c >= n_clusters) {
        atomicOr(err, 2);
        continue;
      }
      tok = token_map[(int64_t)c * cs + r];
      v = load_f<XT>(probe, i);
    } else {
      const int j = (int)(i - (int64_t)n_probes * cs);
      tok = force_ids[j];
      v = load_f<XT>(force, j);
    }
    if (tok < 0 || tok >= V) {
      atomicOr(err, 2);
      continue;
    }
    store_f<XT>(out, tok, v);
  }
}

}  // namespace mb

using namespace mb;

extern "C" int maple_topk_select(const void* x, int x_dtype, int64_t n, int64_t k, int32_t* out, void* stream) {
  if (n < 0 || k < 0 || k > n || n > (1LL << 30)) return kErrShape;
  if (k == 0) return kOk;
  if (!x || !out) return kErrShape;
  if (x_dtype != kBF16 && x_dtype != kF32) return kErrDtype;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = x_dtype == kBF16
                      ? launch_k(topk_select_kernel<kBF16>, dim3(1), dim3(1024), 0, st, x, (int)n, (int)k, out)
                      : launch_k(topk_select_kernel<kF32>, dim3(1), dim3(1024), 0, st, x, (int)n, (int)k, out);
  return e == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_flash_scatter(const void* probe, int x_dtype, const int32_t* cluster_ids, int64_t n_probes,
                                   int64_t cluster_size, const int32_t* token_map, int64_t n_clusters,
                                   const void* force, const int64_t* force_ids, int64_t n_force, void* out,
                                   int64_t vocab, int* err, void* stream) {
  if (n_probes < 0 || cluster_size <= 0 || n_clusters <= 0 || n_force < 0 || vocab <= 0) return kErrShape;
  if (!out || !err || (n_probes > 0 && (!probe || !cluster_ids || !token_map)) ||
      (n_force > 0 && (!force || !force_ids)))
    return kErrShape;
  if (x_dtype != kBF16 && x_dtype != kF32) return kErrDtype;
  if (n_probes * cluster_size + n_force > (1LL << 31)) return kErrShape;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const float ninf = -__builtin_huge_valf();
  const int fill_blocks = (int)((vocab + 255) / 256 < 1184 ? (vocab + 255) / 256 : 1184);
  const int64_t total = n_probes * cluster_size + n_force;
  const int sc_blocks = (int)((total + 255) / 256 < 1184 ? (total + 255) / 256 : 1184);
  cudaError_t e;
  if (x_dtype == kBF16) {
    e = launch_k(fill_kernel<kBF16>, dim3(fill_blocks), dim3(256), 0, st, out, vocab, ninf);
    if (e == cudaSuccess && total > 0)
      e = launch_k(flash_scatter_kernel<kBF16>, dim3(sc_blocks), dim3(256), 0, st, probe, cluster_ids, (int)n_probes,
                   (int)cluster_size, token_map, (int)n_clusters, force, force_ids, (int)n_force, out, vocab, err);
  } else {
    e = launch_k(fill_kernel<kF32>, dim3(fill_blocks), dim3(256), 0, st, out, vocab, ninf);
    if (e == cudaSuccess && total > 0)
      e = launch_k(flash_scatter_kernel<kF32>, dim3(sc_blocks), dim3(256), 0, st, probe, cluster_ids, (int)n_probes,
                   (int)cluster_size, token_map, (int)n_clusters, force, force_ids, (int)n_force, out, vocab, err);
  }
  return e == cudaSuccess ? kOk : kErrCuda;
}
