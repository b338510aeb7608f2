// Deterministic synthetic weights for benchmarks and tests (the synthetic
// architecture of the benchmark configs; no checkpoint exists for it).
//
// Every value is a pure function of (seed, stream, index) through integer
// hashing (splitmix64 finaliser), then at most one fp32 multiply-add and one
// rounding, so an independent CPU implementation reproduces the tensors bit
// for bit.  Distributions:
//   ternary code   16 bits u of a hash: t = 0 if u < 26214 (p = 0.4),
//                  -1 if u < 45875, else +1; stored as code t + 1
//   normal(0, s)   Irwin-Hall sum of four 16-bit uniforms, centred and scaled:
//                  (sum - 131070) * c, c = fp32(s / sqrt(4 * (65536^2 - 1) / 12))
//   abs / offset   |normal| + offset, then bf16 or fp32
//   RTN-4 sym      w ~ normal(0, s) per element; per group scale = absmax / 7,
//                  q = clamp(rint(w / scale), -8, 7), code q + 8, stored scale bf16
#include "common.cuh"

namespace mb {

__host__ __device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ULL;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ULL;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBULL;
  return z ^ (z >> 31);
}

__host__ __device__ __forceinline__ uint64_t stream_key(uint64_t seed, uint64_t stream) {
  return mix64(mix64(seed) ^ (stream * 0x9E3779B97F4A7C15ULL));
}

__device__ __forceinline__ uint64_t hash_at(uint64_t key, uint64_t i) {
  return mix64(key ^ (i * 0xD1B54A32D192ED03ULL));
}

__device__ __forceinline__ float normal_at(uint64_t key, uint64_t i, float c) {
  const uint64_t h = hash_at(key, i);
  const int s = (int)(h & 0xffff) + (int)((h >> 16) & 0xffff) + (int)((h >> 32) & 0xffff) + (int)(h >> 48);
  return __fmul_rn(static_cast<float>(s - 131070), c);
}

__global__ void synth_ternary_kernel(uint64_t key, int64_t n_words, uint32_t* out) {
  for (int64_t w = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; w < n_words;
       w += (int64_t)gridDim.x * blockDim.x) {
    uint32_t word = 0;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint64_t h = hash_at(key, 4 * w + q);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint32_t u = (h >> (16 * j)) & 0xffffu;
        const uint32_t code = u < 26214u ? 1u : (u < 45875u ? 0u : 2u);
        word |= code << (2 * (4 * q + j));
      }
    }
    out[w] = word;
  }
}

template <int OT>
__global__ void synth_normal_kernel(uint64_t key, int64_t n, float c, float offset, int use_abs, void* out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = normal_at(key, i, c);
    if (use_abs) v = fabsf(v);
    v = __fadd_rn(v, offset);
    store_f<OT>(out, i, v);
  }
}

// One thread per (row, group).
__global__ void synth_rtn4_sym_kernel(uint64_t key, int64_t rows, int k, int group, float c, uint32_t* codes,
                                      uint16_t* scales) {
  const int ng = k / group;
  for (int64_t rg = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; rg < rows * ng;
       rg += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = rg / ng;
    const int g = (int)(rg - r * ng);
    const int64_t base = r * k + (int64_t)g * group;
    float amax = 0.0f;
    for (int i = 0; i < group; ++i) amax = fmaxf(amax, fabsf(normal_at(key, base + i, c)));
    const float sc = __fdiv_rn(amax, 7.0f);
    for (int w = 0; w < group / 8; ++w) {
      uint32_t word = 0;
      for (int j = 0; j < 8; ++j) {
        float q = 0.0f;
        if (sc > 0.0f) q = fminf(fmaxf(rintf(__fdiv_rn(normal_at(key, base + 8 * w + j, c), sc)), -8.0f), 7.0f);
        word |= static_cast<uint32_t>(static_cast<int>(q) + 8) << (4 * j);
      }
      codes[(base >> 3) + w] = word;
    }
    scales[rg] = f32_to_bf16(sc);
  }
}

__global__ void synth_tokens_kernel(uint64_t key, int64_t n, int64_t vocab, int64_t* out) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    out[i] = (int64_t)(hash_at(key, i) % (uint64_t)vocab);
}

}  // namespace mb

using namespace mb;

namespace {
float normal_scale_const(double scale) { return (float)(scale / sqrt(4.0 * (65536.0 * 65536.0 - 1.0) / 12.0)); }
unsigned grid_for(int64_t n) {
  const int64_t b = (n + 255) / 256;
  return (unsigned)(b < 148 * 32 ? (b > 0 ? b : 1) : 148 * 32);
}
}  // namespace

extern "C" int maple_synth_ternary(uint64_t seed, uint64_t stream_id, int64_t n_words, uint32_t* out, void* stream) {
  if (n_words < 0 || (!out && n_words)) return kErrShape;
  if (n_words == 0) return kOk;
  synth_ternary_kernel<<<grid_for(n_words), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      stream_key(seed, stream_id), n_words, out);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_synth_normal(uint64_t seed, uint64_t stream_id, int64_t n, double scale, float offset,
                                  int use_abs, int out_dtype, void* out, void* stream) {
  if (n < 0 || (!out && n)) return kErrShape;
  if (n == 0) return kOk;
  if (out_dtype != kF32 && out_dtype != kBF16) return kErrDtype;
  const uint64_t key = stream_key(seed, stream_id);
  const float c = normal_scale_const(scale);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (out_dtype == kBF16) synth_normal_kernel<kBF16><<<grid_for(n), 256, 0, st>>>(key, n, c, offset, use_abs, out);
  else synth_normal_kernel<kF32><<<grid_for(n), 256, 0, st>>>(key, n, c, offset, use_abs, out);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_synth_rtn4_sym(uint64_t seed, uint64_t stream_id, int64_t rows, int64_t k, int64_t group,
                                    double scale, uint32_t* codes, uint16_t* scales_bf16, void* stream) {
  if (rows < 0 || k <= 0 || group <= 0 || k % group || group % 8) return kErrShape;
  if (rows == 0) return kOk;
  if (!codes || !scales_bf16) return kErrShape;
  synth_rtn4_sym_kernel<<<grid_for(rows * (k / group)), 256, 0, static_cast<cudaStream_t>(stream)>>>(
      stream_key(seed, stream_id), rows, (int)k, (int)group, normal_scale_const(scale), codes, scales_bf16);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

extern "C" int maple_synth_tokens(uint64_t seed, uint64_t stream_id, int64_t n, int64_t vocab, int64_t* out,
                                  void* stream) {
  if (n < 0 || vocab <= 0 || (!out && n)) return kErrShape;
  if (n == 0) return kOk;
  synth_tokens_kernel<<<grid_for(n), 256, 0, static_cast<cudaStream_t>(stream)>>>(stream_key(seed, stream_id), n,
                                                                                  vocab, out);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}
