// Packing and quantisation of checkpoints on the GPU (conversion path).
//
// Reference: pack.py:23-149 (pack_2bit / unpack_2bit / pack_4bit /
// unpack_4bit / quantize_rtn / dequantize_rtn / ternarize), NumPy on the CPU.
// These kernels reproduce its results bit for bit:
//   * packing sums the shifted codes in 64 bits and keeps the low 32 (what
//     the reference's uint64 np.sum + astype(uint32) does, also for codes
//     that overflow their field);
//   * ternarize reproduces NumPy's float32 pairwise summation order for
//     np.mean / np.sum along a contiguous last axis: a span of n > 128
//     values splits at n2 = n/2 rounded down to a multiple of 8 and returns
//     sum(first n2) + sum(rest); a span of 8..128 values is summed into 8
//     interleaved accumulators, combined as ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)),
//     then the n % 8 tail added in order; a span below 8 is summed in order
//     from 0.  mean = sum / float32(n);
//   * quantize_rtn is float32 min/max, scale = (max-min)/15, q =
//     clip(rint((w-min)/scale), 0, 15) with scale 0 -> code 0; dequantize is
//     code*scale (rounded) + bias (rounded).
// The row-wise kernels stage one row in shared memory per warp; the
// pairwise leaves (<= 128 values each) are summed by separate lanes and
// combined by lane 0 along the same split tree.
#include "common.cuh"
#include "launch.cuh"

namespace mb {

constexpr int kMaxLeaves = 256;  // rows up to 16384 values (leaves hold >= 64)

// Leaves of the pairwise split tree of [off, off+n), in order.
__device__ void pw_leaves(int off, int n, int* loff, int* llen, int& cnt) {
  if (n <= 128) {
    if (cnt < kMaxLeaves) {
      loff[cnt] = off;
      llen[cnt] = n;
    }
    ++cnt;
    return;
  }
  int n2 = n / 2;
  n2 -= n2 % 8;
  pw_leaves(off, n2, loff, llen, cnt);
  pw_leaves(off + n2, n - n2, loff, llen, cnt);
}

// One leaf (n <= 128) of values produced by f(i).
template <typename F>
__device__ float pw_leaf(int n, F f) {
  if (n < 8) {
    float r = 0.0f;
    for (int i = 0; i < n; ++i) r = __fadd_rn(r, f(i));
    return r;
  }
  float r[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) r[j] = f(j);
  int i = 8;
  for (; i < n - (n % 8); i += 8)
#pragma unroll
    for (int j = 0; j < 8; ++j) r[j] = __fadd_rn(r[j], f(i + j));
  float res = __fadd_rn(__fadd_rn(__fadd_rn(r[0], r[1]), __fadd_rn(r[2], r[3])),
                        __fadd_rn(__fadd_rn(r[4], r[5]), __fadd_rn(r[6], r[7])));
  for (; i < n; ++i) res = __fadd_rn(res, f(i));
  return res;
}

// Combine leaf sums along the split tree of a span of n values.
__device__ float pw_combine(int n, const float* sums, int& idx) {
  if (n <= 128) return sums[idx++];
  int n2 = n / 2;
  n2 -= n2 % 8;
  const float a = pw_combine(n2, sums, idx);
  const float b = pw_combine(n - n2, sums, idx);
  return __fadd_rn(a, b);
}

// ------------------------------------------------------------ packing ----
template <int BITS>
__global__ void pack_kernel(const uint8_t* codes, int64_t n_words, uint32_t* out) {
  constexpr int PER = 32 / BITS;
  pdl_wait();
  pdl_trigger();
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < n_words; w += (int64_t)gridDim.x * blockDim.x) {
    const uint8_t* c = codes + w * PER;
    unsigned long long s = 0;
#pragma unroll
    for (int i = 0; i < PER; ++i) s += (unsigned long long)c[i] << (BITS * i);
    out[w] = static_cast<uint32_t>(s);
  }
}

template <int BITS>
__global__ void unpack_kernel(const uint32_t* words, int64_t n_words, uint8_t* out) {
  constexpr int PER = 32 / BITS;
  constexpr uint32_t M = (1u << BITS) - 1u;
  pdl_wait();
  pdl_trigger();
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < n_words; w += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t v = words[w];
#pragma unroll
    for (int i = 0; i < PER; ++i) out[w * PER + i] = static_cast<uint8_t>((v >> (BITS * i)) & M);
  }
}

// ---------------------------------------------------------- ternarize ----
// One warp per row: |w| staged in shared memory, threshold = ts * mean|w|,
// alpha = sum(|w| * mask) / max(count, 1), codes sign(w)*mask + 1.
template <int WT, int AT>
__global__ void __launch_bounds__(32) ternarize_kernel(const void* w, int K, float ts, uint32_t* packed, void* alpha) {
  extern __shared__ float aw[];
  __shared__ int loff[kMaxLeaves], llen[kMaxLeaves];
  __shared__ float lsum[kMaxLeaves];
  __shared__ float s_thr;
  const int lane = threadIdx.x;
  const int64_t r = blockIdx.x;
  pdl_wait();
  pdl_trigger();
  const char* row = static_cast<const char*>(w) + r * (int64_t)K * (WT == kBF16 ? 2 : 4);
  for (int k = lane; k < K; k += 32) aw[k] = fabsf(load_f<WT>(row, k));
  int nl = 0;
  if (lane == 0) pw_leaves(0, K, loff, llen, nl);
  __syncwarp();
  nl = __shfl_sync(0xffffffffu, nl, 0);
  for (int l = lane; l < nl; l += 32) {
    const float* a = aw + loff[l];
    lsum[l] = pw_leaf(llen[l], [&](int i) { return a[i]; });
  }
  __syncwarp();
  if (lane == 0) {
    int idx = 0;
    const float mean = __fdiv_rn(pw_combine(K, lsum, idx), (float)K);
    s_thr = __fmul_rn(ts, mean);
  }
  __syncwarp();
  const float thr = s_thr;
  int cnt = 0;
  for (int k = lane; k < K; k += 32) cnt += aw[k] > thr ? 1 : 0;
  for (int m = 16; m >= 1; m >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, m);
  for (int l = lane; l < nl; l += 32) {
    const float* a = aw + loff[l];
    lsum[l] = pw_leaf(llen[l], [&](int i) { return a[i] > thr ? a[i] : 0.0f; });
  }
  __syncwarp();
  if (lane == 0) {
    int idx = 0;
    const float num = pw_combine(K, lsum, idx);
    const float den = (float)(cnt > 0 ? cnt : 1);
    store_f<AT>(alpha, r, __fdiv_rn(num, den));
  }
  uint32_t* out = packed + r * (int64_t)(K / 16);
  for (int q = lane; q < K / 16; q += 32) {
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int k = q * 16 + i;
      const float v = load_f<WT>(row, k);
      const bool keep = aw[k] > thr;
      const uint32_t code = keep ? (v > 0.0f ? 2u : (v < 0.0f ? 0u : 1u)) : 1u;
      word |= code << (2 * i);
    }
    out[q] = word;
  }
}

// ------------------------------------------------------------------ RTN ----
// One thread per group of G values.
template <int WT>
__global__ void quantize_rtn_kernel(const void* w, int64_t n_groups, int G, uint32_t* packed, float* scales,
                                    float* biases) {
  pdl_wait();
  pdl_trigger();
  for (int64_t gi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; gi < n_groups;
       gi += (int64_t)gridDim.x * blockDim.x) {
    const char* src = static_cast<const char*>(w) + gi * G * (WT == kBF16 ? 2 : 4);
    float lo = load_f<WT>(src, 0), hi = lo;
    for (int i = 1; i < G; ++i) {
      const float v = load_f<WT>(src, i);
      lo = fminf(lo, v);
      hi = fmaxf(hi, v);
    }
    const float scale = __fdiv_rn(__fsub_rn(hi, lo), 15.0f);
    const bool zero = scale == 0.0f;
    const float safe = zero ? 1.0f : scale;
    uint32_t* out = packed + gi * (G / 8);
    for (int q = 0; q < G / 8; ++q) {
      uint32_t word = 0;
      for (int i = 0; i < 8; ++i) {
        float c = rintf(__fdiv_rn(__fsub_rn(load_f<WT>(src, q * 8 + i), lo), safe));
        c = fminf(fmaxf(c, 0.0f), 15.0f);
        const uint32_t code = zero ? 0u : static_cast<uint32_t>(c);
        word |= code << (4 * i);
      }
      out[q] = word;
    }
    scales[gi] = scale;
    biases[gi] = lo;
  }
}

__global__ void dequantize_rtn_kernel(const uint32_t* packed, const float* scales, const float* biases, int64_t n,
                                      int G, float* out) {
  pdl_wait();
  pdl_trigger();
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const uint32_t code = (packed[i >> 3] >> (4 * (i & 7))) & 15u;
    const int64_t g = i / G;
    out[i] = __fadd_rn(__fmul_rn((float)code, scales[g]), biases[g]);
  }
}

inline unsigned grid_for(int64_t n) {
  const int64_t b = (n + 255) / 256;
  return (unsigned)(b < 148 * 16 ? (b > 0 ? b : 1) : 148 * 16);
}

}  // namespace mb

using namespace mb;

extern "C" int maple_pack_codes(const uint8_t* codes, int64_t n_codes, int bits, uint32_t* out, void* stream) {
  if (n_codes < 0 || (bits != 2 && bits != 4) || n_codes % (32 / bits)) return kErrShape;
  if (n_codes == 0) return kOk;
  if (!codes || !out) return kErrShape;
  const int64_t nw = n_codes / (32 / bits);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = bits == 2 ? launch_k(pack_kernel<2>, dim3(grid_for(nw)), dim3(256), 0, st, codes, nw, out)
                            : launch_k(pack_kernel<4>, dim3(grid_for(nw)), dim3(256), 0, st, codes, nw, out);
  return e == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_unpack_codes(const uint32_t* words, int64_t n_words, int bits, uint8_t* out, void* stream) {
  if (n_words < 0 || (bits != 2 && bits != 4)) return kErrShape;
  if (n_words == 0) return kOk;
  if (!words || !out) return kErrShape;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = bits == 2 ? launch_k(unpack_kernel<2>, dim3(grid_for(n_words)), dim3(256), 0, st, words, n_words, out)
                            : launch_k(unpack_kernel<4>, dim3(grid_for(n_words)), dim3(256), 0, st, words, n_words, out);
  return e == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_ternarize(const void* w, int w_dtype, int64_t rows, int64_t k, float threshold_scale,
                               uint32_t* packed, void* alpha, int alpha_dtype, void* stream) {
  if (rows < 0 || k <= 0 || k % 128 != 0 || k > 16384) return kErrShape;
  if (rows == 0) return kOk;
  if (!w || !packed || !alpha || rows > (1LL << 31) - 1) return kErrShape;
  if ((w_dtype != kBF16 && w_dtype != kF32) || (alpha_dtype != kBF16 && alpha_dtype != kF32)) return kErrDtype;
  const size_t smem = (size_t)k * sizeof(float);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaSuccess;
#define MB_TERN(WT, AT)                                                                                   \
  do {                                                                                                    \
    auto kern = ternarize_kernel<WT, AT>;                                                                 \
    if (smem > 32 * 1024) e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem); \
    if (e == cudaSuccess)                                                                                 \
      e = launch_k(kern, dim3((unsigned)rows), dim3(32), smem, st, w, (int)k, threshold_scale, packed, alpha); \
  } while (0)
  if (w_dtype == kBF16) {
    if (alpha_dtype == kBF16) MB_TERN(kBF16, kBF16); else MB_TERN(kBF16, kF32);
  } else {
    if (alpha_dtype == kBF16) MB_TERN(kF32, kBF16); else MB_TERN(kF32, kF32);
  }
#undef MB_TERN
  return e == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_quantize_rtn(const void* w, int w_dtype, int64_t rows, int64_t k, int64_t group_size,
                                  uint32_t* packed, float* scales, float* biases, void* stream) {
  if (rows < 0 || k <= 0 || group_size <= 0 || group_size % 8 != 0 || k % group_size != 0) return kErrShape;
  if (rows == 0) return kOk;
  if (!w || !packed || !scales || !biases) return kErrShape;
  if (w_dtype != kBF16 && w_dtype != kF32) return kErrDtype;
  const int64_t ng = rows * (k / group_size);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = w_dtype == kBF16
                      ? launch_k(quantize_rtn_kernel<kBF16>, dim3(grid_for(ng)), dim3(256), 0, st, w, ng,
                                 (int)group_size, packed, scales, biases)
                      : launch_k(quantize_rtn_kernel<kF32>, dim3(grid_for(ng)), dim3(256), 0, st, w, ng,
                                 (int)group_size, packed, scales, biases);
  return e == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_dequantize_rtn(const uint32_t* packed, const float* scales, const float* biases, int64_t rows,
                                    int64_t k, int64_t group_size, float* out, void* stream) {
  if (rows < 0 || k <= 0 || group_size <= 0 || k % group_size != 0 || k % 8 != 0) return kErrShape;
  if (rows == 0) return kOk;
  if (!packed || !scales || !biases || !out) return kErrShape;
  const int64_t n = rows * k;
  cudaError_t e = launch_k(dequantize_rtn_kernel, dim3(grid_for(n)), dim3(256), 0, static_cast<cudaStream_t>(stream),
                           packed, scales, biases, n, (int)group_size, out);
  return e == cudaSuccess ? kOk : kErrCuda;
}
