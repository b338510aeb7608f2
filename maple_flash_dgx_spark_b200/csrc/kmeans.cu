// Balanced spherical k-means of the lm_head rows for FlashHead (offline, at
// checkpoint conversion).
//
// Reference: maple_run/flash_head.py:30-110 (_balanced_spherical_kmeans):
// per iteration, assign every row to its most similar centroid; for each
// over-full cluster keep its cluster_size most similar members and evict the
// rest; reassign the evicted rows one by one to their most similar cluster
// that is not yet full; recompute the centroids as normalised member means.
//
// B200 design.  The assignment is an N x K x D contraction (151936 x 4748 x
// 2048 for the configs' head): km_dots_kernel is a tiled fp32 GEMM whose
// epilogue keeps, per row, the best centroid of its 128-centroid tile, so the
// N x K similarity matrix is never written; km_argmax_kernel picks the best
// tile.  The evicted rows' full similarity rows are written (a few thousand
// rows), and the sequential reassignment runs in one warp with the cluster
// counts and "full" flags in shared memory: a row takes its precomputed best
// open cluster unless that cluster filled meanwhile, in which case the warp
// rescans the row.  The centroid update gathers each cluster's members (in
// ascending row order) per CTA.
//
// Canonical arithmetic (restated by oracle.c orc_km_*): every similarity is
// one fp32 fmaf chain over k = 0..D-1 from 0.0f, so eviction and
// reassignment see exactly the assignment's values; a centroid is the plain
// fp32 sum of its members in ascending row order, divided by the count, then
// by (sqrt(R128 sum of squares) + 1e-8); ties go to the lowest cluster index.
#include "common.cuh"
#include "launch.cuh"

namespace mb {

constexpr int kKmBM = 128, kKmBN = 128, kKmBK = 16;  // GEMM tile: rows x centroids x k
constexpr int kKmMaxClusters = 8192;

// (value, index) order for an argmax with ties to the lowest index.
__device__ __forceinline__ bool km_better(float v, int i, float bv, int bi) {
  return v > bv || (v == bv && i < bi);
}

// Similarities of rows a[rows[r]] (or a[r]) with centroids b[c]: MODE 0 writes
// per (centroid tile, row) the best (value, index) of the tile; MODE 1 writes
// every similarity out[r * nb + c].  256 threads, each an 8 x 8 block of
// outputs; k runs in order for every output.
template <int MODE>
__global__ void __launch_bounds__(256) km_dots_kernel(const float* __restrict__ a, const int* __restrict__ rows,
                                                      int na, const float* __restrict__ b, int nb, int d,
                                                      float* out_val, int* out_idx) {
  __shared__ __align__(16) float As[2][kKmBK][kKmBM];
  __shared__ __align__(16) float Bs[2][kKmBK][kKmBN];
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  const int r0 = blockIdx.x * kKmBM, c0 = blockIdx.y * kKmBN;
  // loader: thread loads 8 consecutive k of one row of A and of B
  const int lr = tid >> 1, lk = (tid & 1) * 8;
  const int ar = r0 + lr, bc = c0 + lr;
  const float* ap = nullptr;
  if (ar < na) ap = a + (int64_t)(rows ? rows[ar] : ar) * d;
  const float* bp = bc < nb ? b + (int64_t)bc * d : nullptr;
  float4 ra0, ra1, rb0, rb1;
  auto gload = [&](int k0) {
    const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
    ra0 = ap ? *reinterpret_cast<const float4*>(ap + k0 + lk) : z;
    ra1 = ap ? *reinterpret_cast<const float4*>(ap + k0 + lk + 4) : z;
    rb0 = bp ? *reinterpret_cast<const float4*>(bp + k0 + lk) : z;
    rb1 = bp ? *reinterpret_cast<const float4*>(bp + k0 + lk + 4) : z;
  };
  auto sstore = [&](int buf) {
    const float av[8] = {ra0.x, ra0.y, ra0.z, ra0.w, ra1.x, ra1.y, ra1.z, ra1.w};
    const float bv[8] = {rb0.x, rb0.y, rb0.z, rb0.w, rb1.x, rb1.y, rb1.z, rb1.w};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      As[buf][lk + j][lr] = av[j];
      Bs[buf][lk + j][lr] = bv[j];
    }
  };
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
  gload(0);
  sstore(0);
  __syncthreads();
  const int nk = d / kKmBK;
  for (int t = 0; t < nk; ++t) {
    const int cur = t & 1;
    if (t + 1 < nk) gload((t + 1) * kKmBK);
#pragma unroll
    for (int kk = 0; kk < kKmBK; ++kk) {
      const float4 x0 = *reinterpret_cast<const float4*>(&As[cur][kk][ty * 8]);
      const float4 x1 = *reinterpret_cast<const float4*>(&As[cur][kk][ty * 8 + 4]);
      const float4 y0 = *reinterpret_cast<const float4*>(&Bs[cur][kk][tx * 8]);
      const float4 y1 = *reinterpret_cast<const float4*>(&Bs[cur][kk][tx * 8 + 4]);
      const float xa[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
      const float yb[8] = {y0.x, y0.y, y0.z, y0.w, y1.x, y1.y, y1.z, y1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = __fmaf_rn(xa[i], yb[j], acc[i][j]);
    }
    if (t + 1 < nk) {
      sstore(cur ^ 1);
      __syncthreads();
    }
  }
  if constexpr (MODE == 1) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = r0 + ty * 8 + i;
      if (r >= na) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = c0 + tx * 8 + j;
        if (c < nb) out_val[(int64_t)r * nb + c] = acc[i][j];
      }
    }
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = c0 + tx * 8 + j;
        if (c < nb && km_better(acc[i][j], c, bv, bi)) {
          bv = acc[i][j];
          bi = c;
        }
      }
      // the 16 threads of a half warp share these rows
#pragma unroll
      for (int m = 8; m >= 1; m >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
        if (km_better(ov, oi, bv, bi)) {
          bv = ov;
          bi = oi;
        }
      }
      const int r = r0 + ty * 8 + i;
      if (tx == 0 && r < na) {
        out_val[(int64_t)blockIdx.y * na + r] = bv;
        out_idx[(int64_t)blockIdx.y * na + r] = bi;
      }
    }
  }
}

// labels[r], best[r]: the best of the per-tile candidates, tiles in order.
__global__ void km_argmax_kernel(const float* cand_val, const int* cand_idx, int ntiles, int n, int* labels,
                                 float* best) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= n) return;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int t = 0; t < ntiles; ++t) {
    const float v = cand_val[(int64_t)t * n + r];
    const int i = cand_idx[(int64_t)t * n + r];
    if (km_better(v, i, bv, bi)) {
      bv = v;
      bi = i;
    }
  }
  labels[r] = bi;
  best[r] = bv;
}

// Best open cluster of each evicted row (one warp per row), at the start of
// the reassignment: -1 when every cluster is full.
__global__ void km_best_open_kernel(const float* sims, int n_e, int k, const int* recount, int cs, int* best) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (warp >= n_e) return;
  const float* row = sims + (int64_t)warp * k;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  for (int c = lane; c < k; c += 32)
    if (recount[c] < cs && km_better(row[c], c, bv, bi)) {
      bv = row[c];
      bi = c;
    }
#pragma unroll
  for (int m = 16; m >= 1; m >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, m);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, m);
    if (km_better(ov, oi, bv, bi)) {
      bv = ov;
      bi = oi;
    }
  }
  if (lane == 0) best[warp] = bi == 0x7fffffff ? -1 : bi;
}

// The sequential reassignment (flash_head.py:82-96), one warp: evicted row e
// (in order) takes the most similar cluster not yet full; counts and "full"
// flags live in shared memory.
__global__ void __launch_bounds__(32) km_reassign_kernel(const float* sims, const int* evict, const int* best0,
                                                         int n_e, int k, const int* recount_in, int cs,
                                                         int* labels) {
  extern __shared__ int cnt[];  // [k]
  const int lane = threadIdx.x;
  for (int c = lane; c < k; c += 32) cnt[c] = recount_in[c];
  __syncwarp();
  for (int e0 = 0; e0 < n_e; e0 += 32) {
    const int my_b = e0 + lane < n_e ? best0[e0 + lane] : -1;
    const int my_pt = e0 + lane < n_e ? evict[e0 + lane] : 0;
    const int m = min(32, n_e - e0);
    for (int j = 0; j < m; ++j) {
      int b = __shfl_sync(0xffffffffu, my_b, j);
      const int pt = __shfl_sync(0xffffffffu, my_pt, j);
      if (b < 0 || cnt[b] >= cs) {  // filled since: rescan this row over the open clusters
        const float* row = sims + (int64_t)(e0 + j) * k;
        float bv = -INFINITY;
        int bi = 0x7fffffff;
        for (int c = lane; c < k; c += 32)
          if (cnt[c] < cs && km_better(row[c], c, bv, bi)) {
            bv = row[c];
            bi = c;
          }
#pragma unroll
        for (int s = 16; s >= 1; s >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, s);
          const int oi = __shfl_xor_sync(0xffffffffu, bi, s);
          if (km_better(ov, oi, bv, bi)) {
            bv = ov;
            bi = oi;
          }
        }
        b = bi;
        if (b == 0x7fffffff) {  // every cluster full: the first with room (never, when N = K * cs)
          int f = 0x7fffffff;
          for (int c = lane; c < k; c += 32)
            if (cnt[c] < cs) f = min(f, c);
#pragma unroll
          for (int s = 16; s >= 1; s >>= 1) f = min(f, __shfl_xor_sync(0xffffffffu, f, s));
          b = f == 0x7fffffff ? 0 : f;
        }
      }
      if (lane == 0) {
        labels[pt] = b;
        cnt[b] += 1;
      }
      __syncwarp();
    }
  }
}

// Centroid j = normalised mean of its members (members[offsets[j] ..
// offsets[j+1]), ascending rows): 128 threads per cluster, plain fp32 adds in
// member order, then the R128 sum of squares.
__global__ void __launch_bounds__(128) km_update_kernel(const float* w, int d, const int* members,
                                                        const int* offsets, float* cent) {
  extern __shared__ float row[];  // [d]
  __shared__ float part[128];
  const int j = blockIdx.x, tid = threadIdx.x;
  const int m0 = offsets[j], m1 = offsets[j + 1];
  const float cf = static_cast<float>(m1 - m0 > 0 ? m1 - m0 : 1);
  for (int k = tid; k < d; k += 128) {
    float s = 0.0f;
    for (int m = m0; m < m1; ++m) s = __fadd_rn(s, w[(int64_t)members[m] * d + k]);
    row[k] = __fdiv_rn(s, cf);
  }
  __syncthreads();
  float p = 0.0f;
  for (int k = tid; k < d; k += 128) p = __fmaf_rn(row[k], row[k], p);
  part[tid] = p;
  __syncthreads();
  __shared__ float s_nrm;
  if (tid < 32) {
    const float ss = r128_smem_finish(part, tid);
    if (tid == 0) s_nrm = __fadd_rn(__fsqrt_rn(ss), 1e-8f);
  }
  __syncthreads();
  for (int k = tid; k < d; k += 128) cent[(int64_t)j * d + k] = __fdiv_rn(row[k], s_nrm);
}

// Per block of 1024 rows: the double sum, in row order, of each row's
// similarity to its centroid (one fmaf chain per row).
__global__ void __launch_bounds__(256) km_objective_kernel(const float* w, int n, int d, const int* labels,
                                                           const float* cent, double* partial) {
  __shared__ float dots[1024];
  const int b0 = blockIdx.x * 1024;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // each warp: 128 rows, lane-strided over rows, k in order per row
  for (int i = warp * 128 + lane; i < warp * 128 + 128; i += 32) {
    const int r = b0 + i;
    float acc = 0.0f;
    if (r < n) {
      const float* wr = w + (int64_t)r * d;
      const float* cr = cent + (int64_t)labels[r] * d;
      for (int k = 0; k < d; ++k) acc = __fmaf_rn(wr[k], cr[k], acc);
    }
    dots[i] = acc;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double s = 0.0;
    const int m = min(1024, n - b0);
    for (int i = 0; i < m; ++i) s += static_cast<double>(dots[i]);
    partial[blockIdx.x] = s;
  }
}

// Rows scaled by 1 / (sqrt(R128 sum of squares) + 1e-8), one block of 128 per row.
__global__ void __launch_bounds__(128) km_normalize_kernel(float* v, int d) {
  __shared__ float part[128];
  __shared__ float s_nrm;
  float* r = v + (int64_t)blockIdx.x * d;
  float p = 0.0f;
  for (int k = threadIdx.x; k < d; k += 128) p = __fmaf_rn(r[k], r[k], p);
  part[threadIdx.x] = p;
  __syncthreads();
  if (threadIdx.x < 32) {
    const float ss = r128_smem_finish(part, threadIdx.x);
    if (threadIdx.x == 0) s_nrm = __fadd_rn(__fsqrt_rn(ss), 1e-8f);
  }
  __syncthreads();
  for (int k = threadIdx.x; k < d; k += 128) r[k] = __fdiv_rn(r[k], s_nrm);
}

}  // namespace mb

using namespace mb;

static bool km_shape_ok(int64_t n, int64_t d) { return n > 0 && n < (1LL << 31) && d > 0 && d % kKmBK == 0; }

extern "C" int64_t maple_km_assign_workspace_bytes(int64_t n, int64_t k) {
  if (n <= 0 || k <= 0) return -1;
  return ((k + kKmBN - 1) / kKmBN) * n * 8;
}

extern "C" int maple_km_assign(const float* w, int64_t n, int64_t d, const float* cent, int64_t k, int32_t* labels,
                               float* best, void* workspace, int64_t workspace_bytes, void* stream) {
  if (!km_shape_ok(n, d) || k <= 0 || k > kKmMaxClusters) return kErrShape;
  if (!w || !cent || !labels || !best || !workspace) return kErrShape;
  if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(cent)) & 15) return kErrAlign;
  if (workspace_bytes < maple_km_assign_workspace_bytes(n, k)) return kErrWorkspace;
  const int ntiles = (int)((k + kKmBN - 1) / kKmBN);
  float* cv = static_cast<float*>(workspace);
  int* ci = reinterpret_cast<int*>(cv + (int64_t)ntiles * n);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  km_dots_kernel<0><<<dim3((unsigned)((n + kKmBM - 1) / kKmBM), ntiles), 256, 0, st>>>(w, nullptr, (int)n, cent,
                                                                                       (int)k, (int)d, cv, ci);
  km_argmax_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(cv, ci, ntiles, (int)n, labels, best);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_km_dots(const float* w, const int32_t* rows, int64_t n_rows, int64_t d, const float* cent,
                             int64_t k, float* out, void* stream) {
  if (!km_shape_ok(n_rows, d) || k <= 0 || k > kKmMaxClusters) return kErrShape;
  if (!w || !rows || !cent || !out) return kErrShape;
  if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(cent)) & 15) return kErrAlign;
  km_dots_kernel<1><<<dim3((unsigned)((n_rows + kKmBM - 1) / kKmBM), (unsigned)((k + kKmBN - 1) / kKmBN)), 256, 0,
                      static_cast<cudaStream_t>(stream)>>>(w, rows, (int)n_rows, cent, (int)k, (int)d, out, nullptr);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_km_reassign(const float* sims, const int32_t* evict, int64_t n_evict, int64_t k,
                                 const int32_t* recount, int64_t cluster_size, int32_t* labels, int32_t* scratch,
                                 void* stream) {
  if (n_evict < 0 || k <= 0 || k > kKmMaxClusters || cluster_size <= 0) return kErrShape;
  if (n_evict == 0) return kOk;
  if (!sims || !evict || !recount || !labels || !scratch || n_evict >= (1LL << 31)) return kErrShape;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  km_best_open_kernel<<<(unsigned)((n_evict * 32 + 255) / 256), 256, 0, st>>>(sims, (int)n_evict, (int)k, recount,
                                                                             (int)cluster_size, scratch);
  const size_t smem = (size_t)k * sizeof(int);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(km_reassign_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return kErrCuda;
  km_reassign_kernel<<<1, 32, smem, st>>>(sims, evict, scratch, (int)n_evict, (int)k, recount, (int)cluster_size,
                                          labels);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_km_update(const float* w, int64_t d, const int32_t* members, const int32_t* offsets, int64_t k,
                               float* cent, void* stream) {
  if (d <= 0 || k <= 0 || !w || !members || !offsets || !cent) return kErrShape;
  const size_t smem = (size_t)d * sizeof(float);
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(km_update_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return kErrCuda;
  km_update_kernel<<<(unsigned)k, 128, smem, static_cast<cudaStream_t>(stream)>>>(w, (int)d, members, offsets, cent);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int64_t maple_km_objective_blocks(int64_t n) { return n <= 0 ? -1 : (n + 1023) / 1024; }

extern "C" int maple_km_objective(const float* w, int64_t n, int64_t d, const int32_t* labels, const float* cent,
                                  double* partial, void* stream) {
  if (!km_shape_ok(n, d) || !w || !labels || !cent || !partial) return kErrShape;
  km_objective_kernel<<<(unsigned)((n + 1023) / 1024), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      w, (int)n, (int)d, labels, cent, partial);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_km_normalize(float* v, int64_t rows, int64_t d, void* stream) {
  if (rows <= 0 || d <= 0 || !v) return kErrShape;
  km_normalize_kernel<<<(unsigned)rows, 128, 0, static_cast<cudaStream_t>(stream)>>>(v, (int)d);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}
