// RMSNorm and residual-add + RMSNorm.
// Reference: kernels/fused_norm.py:105-125 (rms_norm, kernel :11-29) and
// :128-161 (add_rms_norm, kernel :32-57).  One CTA (128 threads) per row;
// the sum of squares is R128 order (thread j owns elements j, j+128, ...).
#include "common.cuh"
#include "launch.cuh"

namespace mb {

template <int XT, int WT, bool ADD>
__global__ void __launch_bounds__(128) rms_norm_kernel(const void* x, const void* y, const void* w,
                                                       void* residual, void* out, int64_t x_stride,
                                                       int64_t y_stride, int64_t r_stride,
                                                       int64_t o_stride, int N, float eps) {
  extern __shared__ float srow[];  // x | y | w, N floats each
  __shared__ float part[128];
  __shared__ float s_rstd;
  const int tid = threadIdx.x;
  const int row = blockIdx.x;
  const int es = XT == kBF16 ? 2 : 4;
  float* xs = srow;
  float* ys = srow + N;
  float* wsm = srow + 2 * N;
  stage_row<WT, 128, 4>(w, N, wsm, tid);  // weights: before waiting
  pdl_wait();
  pdl_trigger();
  stage_row<XT, 128, 4>(static_cast<const char*>(x) + row * x_stride * es, N, xs, tid);
  if constexpr (ADD) stage_row<XT, 128, 4>(static_cast<const char*>(y) + row * y_stride * es, N, ys, tid);
  __syncthreads();
  float ss = 0.0f;
  for (int k = tid; k < N; k += 128) {
    float v = xs[k];
    if constexpr (ADD) {
      v = __fadd_rn(v, ys[k]);
      store_f<XT>(static_cast<char*>(residual) + row * r_stride * es, k, v);
      xs[k] = v;
    }
    ss = __fmaf_rn(v, v, ss);
  }
  part[tid] = ss;
  __syncthreads();
  if (tid < 32) {
    const float tot = r128_smem_finish(part, tid);
    if (tid == 0) s_rstd = rstd_of(tot, N, eps);
  }
  __syncthreads();
  const float rstd = s_rstd;
  char* orow = static_cast<char*>(out) + row * o_stride * es;
  for (int k = tid; k < N; k += 128) store_f<XT>(orow, k, __fmul_rn(__fmul_rn(xs[k], rstd), wsm[k]));
}

template <bool ADD>
int launch_norm(const void* x, const void* y, int x_dtype, int64_t rows, int64_t n, int64_t xs,
                int64_t ys, const void* w, int w_dtype, float eps, void* residual, int64_t rs,
                void* out, int64_t os, void* stream) {
  if (rows < 0 || n <= 0) return kErrShape;
  if (rows == 0) return kOk;
  if ((x_dtype != kF32 && x_dtype != kBF16) || (w_dtype != kF32 && w_dtype != kBF16)) return kErrDtype;
  if (!x || !w || !out || (ADD && (!y || !residual))) return kErrShape;
  if (n > 16384 || rows > (1LL << 31) - 1) return kErrShape;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const size_t smem = 3 * (size_t)n * sizeof(float);
  if (smem > 32 * 1024) {
    cudaFuncSetAttribute(rms_norm_kernel<kBF16, kBF16, ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(rms_norm_kernel<kBF16, kF32, ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(rms_norm_kernel<kF32, kBF16, ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(rms_norm_kernel<kF32, kF32, ADD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  }
  const dim3 grid((unsigned)rows);
  if (x_dtype == kBF16) {
    if (w_dtype == kBF16)
      launch_k(rms_norm_kernel<kBF16, kBF16, ADD>, dim3(grid), dim3(128), smem, st, x, y, w, residual, out, xs, ys, rs, os, (int)n, eps);
    else
      launch_k(rms_norm_kernel<kBF16, kF32, ADD>, dim3(grid), dim3(128), smem, st, x, y, w, residual, out, xs, ys, rs, os, (int)n, eps);
  } else {
    if (w_dtype == kBF16)
      launch_k(rms_norm_kernel<kF32, kBF16, ADD>, dim3(grid), dim3(128), smem, st, x, y, w, residual, out, xs, ys, rs, os, (int)n, eps);
    else
      launch_k(rms_norm_kernel<kF32, kF32, ADD>, dim3(grid), dim3(128), smem, st, x, y, w, residual, out, xs, ys, rs, os, (int)n, eps);
  }
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace mb

using namespace mb;

extern "C" int maple_rms_norm(const void* x, int x_dtype, int64_t rows, int64_t n,
                              int64_t x_row_stride, const void* w, int w_dtype, float eps,
                              void* out, int64_t out_row_stride, void* stream) {
  return launch_norm<false>(x, nullptr, x_dtype, rows, n, x_row_stride, 0, w, w_dtype, eps, nullptr,
                            0, out, out_row_stride, stream);
}

extern "C" int maple_add_rms_norm(const void* x, const void* y, int x_dtype, int64_t rows, int64_t n,
                                  int64_t x_row_stride, int64_t y_row_stride, const void* w,
                                  int w_dtype, float eps, void* residual, int64_t residual_row_stride,
                                  void* out, int64_t out_row_stride, void* stream) {
  return launch_norm<true>(x, y, x_dtype, rows, n, x_row_stride, y_row_stride, w, w_dtype, eps,
                           residual, residual_row_stride, out, out_row_stride, stream);
}
