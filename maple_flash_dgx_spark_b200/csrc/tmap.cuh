// Tensor maps (TMA descriptors) for tiled cp.async.bulk.tensor loads.
//
// Host side: cuTensorMapEncodeTiled, reached through the runtime's driver
// entry point (no link against libcuda), with a small cache keyed by the
// tensor's address and geometry so repeated launches over the same buffers
// (every decode step, every layer) encode each map once.  Device side: the
// 4-D tiled load into shared memory completing on an mbarrier.  Loads only,
// from this GPU's own memory, each CTA fetching its own tiles.
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstring>
#include <mutex>
#include <unordered_map>

namespace mb {

// 4-D bf16 tensor [d3][d2][d1][d0] with d0 contiguous; strides in elements
// (s1 for d1, s2 for d2, s3 for d3, each a multiple of 8); box {b0, b1, 1, 1}
// with b0 * 2 bytes = 128 (so the 128-byte swizzle covers one box row).
struct TmapKey {
  uintptr_t addr;
  int64_t d0, d1, d2, d3, s1, s2, s3;
  int b0, b1;
  bool operator==(const TmapKey& o) const { return std::memcmp(this, &o, sizeof(TmapKey)) == 0; }
};

struct TmapKeyHash {
  size_t operator()(const TmapKey& k) const {
    const uint64_t* w = reinterpret_cast<const uint64_t*>(&k);
    uint64_t h = 1469598103934665603ull;
    for (size_t i = 0; i < sizeof(TmapKey) / 8; ++i) h = (h ^ w[i]) * 1099511628211ull;
    return static_cast<size_t>(h);
  }
};

// Encodes (or returns the cached) map; false if the driver refuses it.
inline bool tmap_bf16_4d(const void* base, int64_t d0, int64_t d1, int64_t d2, int64_t d3, int64_t s1, int64_t s2,
                         int64_t s3, int b0, int b1, CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> cache;
  static PFN_cuTensorMapEncodeTiled encode = nullptr;
  TmapKey key{};
  key.addr = reinterpret_cast<uintptr_t>(base);
  key.d0 = d0; key.d1 = d1; key.d2 = d2; key.d3 = d3; key.s1 = s1; key.s2 = s2; key.s3 = s3;
  key.b0 = b0; key.b1 = b1;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return true;
  }
  if (encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr)
      return false;
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(fn);
  }
  const cuuint64_t dims[4] = {(cuuint64_t)d0, (cuuint64_t)d1, (cuuint64_t)d2, (cuuint64_t)d3};
  const cuuint64_t strides[3] = {(cuuint64_t)s1 * 2, (cuuint64_t)s2 * 2, (cuuint64_t)s3 * 2};
  const cuuint32_t box[4] = {(cuuint32_t)b0, (cuuint32_t)b1, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUtensorMap m;
  const CUresult r = encode(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, m);
  *out = m;
  return true;
}

// 2-D tensor [d1][d0] of `esize`-byte elements (row stride d0 elements, a
// multiple of 16 bytes) with boxes of b0 x b1 elements, cached like the 4-D
// maps; `swz128`: the 128-byte swizzle (b0 * esize must then be 128).
inline bool tmap_2d(const void* base, CUtensorMapDataType dtype, int esize, int64_t d0, int64_t d1, int b0, int b1,
                    bool swz128, CUtensorMap* out) {
  static std::mutex mu;
  static std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> cache;
  static PFN_cuTensorMapEncodeTiled encode = nullptr;
  TmapKey key{};
  key.addr = reinterpret_cast<uintptr_t>(base);
  key.d0 = d0; key.d1 = d1; key.b0 = b0; key.b1 = b1;
  key.s1 = esize; key.s2 = (int64_t)dtype; key.s3 = swz128;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return true;
  }
  if (encode == nullptr) {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess || fn == nullptr)
      return false;
    encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled>(fn);
  }
  const cuuint64_t dims[2] = {(cuuint64_t)d0, (cuuint64_t)d1};
  const cuuint64_t strides[1] = {(cuuint64_t)(d0 * esize)};
  const cuuint32_t box[2] = {(cuuint32_t)b0, (cuuint32_t)b1};
  const cuuint32_t estr[2] = {1, 1};
  CUtensorMap m;
  const CUresult r = encode(&m, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE,
                            swz128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return false;
  if (cache.size() > 4096) cache.clear();
  cache.emplace(key, m);
  *out = m;
  return true;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];\n" ::"r"(static_cast<unsigned>(__cvta_generic_to_shared(dst))),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y),
      "r"(static_cast<unsigned>(__cvta_generic_to_shared(bar)))
      : "memory");
}

// Tiled 4-D load of one box into shared memory (x = innermost coordinate,
// whose byte offset must be a multiple of 16), completing on `bar`.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int x, int y, int z, int w,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, "
      "%5}], [%6];\n" ::"r"(static_cast<unsigned>(__cvta_generic_to_shared(dst))),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w),
      "r"(static_cast<unsigned>(__cvta_generic_to_shared(bar)))
      : "memory");
}

}  // namespace mb
