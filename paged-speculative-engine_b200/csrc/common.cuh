// Shared device helpers for libpse (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "pse.h"

#define PSE_LAUNCH_CHECK()                        \
  do {                                            \
    cudaError_t e__ = cudaGetLastError();         \
    if (e__ != cudaSuccess) return (int)e__;      \
  } while (0)

namespace pse {

constexpr int kNumSMs = 148;

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }

template <typename T>
__device__ __forceinline__ T from_f32(float v);
template <>
__device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <>
__device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }

__device__ __forceinline__ float load_as_f32(const void* p, int64_t i, int dtype) {
  return dtype == PSE_BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i])
                           : reinterpret_cast<const float*>(p)[i];
}

__device__ __forceinline__ void store_from_f32(void* p, int64_t i, float v, int dtype) {
  if (dtype == PSE_BF16)
    reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else
    reinterpret_cast<float*>(p)[i] = v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ int warp_sum_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Inclusive scan over a warp.
__device__ __forceinline__ int warp_inclusive_scan(int v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

__device__ __forceinline__ double warp_inclusive_scan_d(double v) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    double n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  return v;
}

// Block-wide exclusive scan of ints (blockDim.x a multiple of 32, <= 1024).
// `tmp` must hold 33 ints of shared memory.  Returns the exclusive prefix and
// writes the block total into *total.
__device__ __forceinline__ int block_exclusive_scan(int v, int* tmp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  int inc = warp_inclusive_scan(v);
  if (lane == 31) tmp[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    int w = lane < nwarps ? tmp[lane] : 0;
    int wi = warp_inclusive_scan(w);
    if (lane < nwarps) tmp[lane] = wi - w;
    if (lane == nwarps - 1) tmp[32] = wi;
  }
  __syncthreads();
  int res = tmp[warp] + inc - v;
  *total = tmp[32];
  __syncthreads();
  return res;
}

__host__ __device__ __forceinline__ int ceil_div(int a, int b) { return (a + b - 1) / b; }

// ---------------------------------------------------------------- programmatic dependent launch
// A kernel launched with launch_pdl may start while the kernel before it on
// the stream is still running: everything before pdl_wait() overlaps that
// kernel's tail, so a kernel must call pdl_wait() before it reads or writes
// any memory an earlier kernel touches (all of them call it first thing).
// pdl_trigger() lets the next kernel launch once every CTA of this one has
// issued it (or exited).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }

// Whether the small per-token kernels launch with programmatic dependent
// launch (pse_launch_overlap); on by default.
bool pdl_enabled();

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args... args) {
  if (!pdl_enabled()) {
    kern<<<grid, block, smem, s>>>(args...);
    return cudaGetLastError();
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

__device__ __forceinline__ int blocks_for(int n_tokens, int block_size) {
  return n_tokens == 0 ? 0 : (n_tokens - 1) / block_size + 1;
}

// ---------------------------------------------------------------- which keys a query sees
// Query w of a row whose call starts at cache position `base`.  tree_b == 0:
// causal, keys <= base + w.  tree_b = b > 0 (a token-tree call): the call's
// tokens are tree nodes in depth-major order from depth tree_d0 -- node
// n = tree_d0 * b + w sits at position L + n (L = base - tree_d0 * b, the
// row's length at the tree's root), is branch n % b at depth n / b, and sees
// the keys below L plus its own branch's nodes at depths up to its own.
struct KeyVis {
  int lim;  // every key <= lim is visible (-1: none)
  int L, br, dep;
};

__device__ __forceinline__ KeyVis key_vis(int base, int w, int tree_b, int tree_d0) {
  if (tree_b <= 0) return KeyVis{base + w, 0, 0, -1};
  const int n = tree_d0 * tree_b + w, L = base - tree_d0 * tree_b;
  return KeyVis{L - 1, L, n % tree_b, n / tree_b};
}

__device__ __forceinline__ bool key_visible(const KeyVis& v, int tok, int tree_b) {
  if (tok <= v.lim) return true;
  if (tree_b <= 0 || tok < v.L) return false;
  const int m = tok - v.L;
  return m % tree_b == v.br && m / tree_b <= v.dep;
}

constexpr KeyVis kNoKeys{-1, 0, 0, -1};

}  // namespace pse
