// Host-side cache of 2-D bf16 TMA descriptors (CUtensorMap), shared by the
// attention and GEMM launchers.
//
// A descriptor is a pure function of (base address, dims, row stride, box,
// swizzle), so it is encoded once and reused.  The cache is keyed on that full
// tuple and compares every field on a hit: two buffers that differ in any field
// never share a descriptor.  It holds at most kMaxEntries descriptors and is
// cleared when full (a re-encode costs a few microseconds of host time).
#pragma once

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <mutex>
#include <unordered_map>

namespace pse {

struct TmapKey {
  uint64_t ptr, inner, outer, stride;  // base, dims (elements), row stride (bytes)
  uint32_t box_inner, box_outer, swizzle;
  bool operator==(const TmapKey& o) const {
    return ptr == o.ptr && inner == o.inner && outer == o.outer && stride == o.stride &&
           box_inner == o.box_inner && box_outer == o.box_outer && swizzle == o.swizzle;
  }
};

struct TmapKeyHash {
  size_t operator()(const TmapKey& k) const {
    uint64_t h = 1469598103934665603ull;
    const uint64_t f[7] = {k.ptr, k.inner, k.outer, k.stride, k.box_inner, k.box_outer, k.swizzle};
    for (uint64_t v : f) h = (h ^ v) * 1099511628211ull;
    return (size_t)h;
  }
};

class TmapCache {
 public:
  static constexpr size_t kMaxEntries = 4096;

  // Returns 0 and the descriptor for a [outer x inner] bf16 matrix whose rows
  // are `stride` bytes apart, box [box_outer x box_inner], 128-byte swizzle,
  // L2 promotion 256 B, out-of-range elements read as zero; PSE_EINVAL-style
  // nonzero codes on failure (the caller's error space).
  int get(const void* ptr, uint64_t inner, uint64_t outer, uint64_t stride, uint32_t box_inner, uint32_t box_outer,
          int err_code, CUtensorMap* out) {
    const TmapKey key{reinterpret_cast<uint64_t>(ptr), inner, outer, stride, box_inner, box_outer, 128u};
    std::lock_guard<std::mutex> lk(mu_);
    auto it = maps_.find(key);
    if (it != maps_.end()) {
      *out = it->second;
      return 0;
    }
    if (!encode_) {
      cudaDriverEntryPointQueryResult q;
      void* fn = nullptr;
      cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
      if (e != cudaSuccess) return (int)e;
      if (q != cudaDriverEntryPointSuccess || !fn) return err_code;
      encode_ = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    CUtensorMap m;
    const cuuint64_t dims[2] = {(cuuint64_t)inner, (cuuint64_t)outer};
    const cuuint64_t strides[1] = {(cuuint64_t)stride};
    const cuuint32_t box[2] = {box_inner, box_outer};
    const cuuint32_t estr[2] = {1, 1};
    CUresult r = encode_(&m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return err_code;
    if (maps_.size() >= kMaxEntries) maps_.clear();
    maps_.emplace(key, m);
    *out = m;
    return 0;
  }

  size_t size() {
    std::lock_guard<std::mutex> lk(mu_);
    return maps_.size();
  }

 private:
  std::mutex mu_;
  PFN_cuTensorMapEncodeTiled_v12000 encode_ = nullptr;
  std::unordered_map<TmapKey, CUtensorMap, TmapKeyHash> maps_;
};

}  // namespace pse
