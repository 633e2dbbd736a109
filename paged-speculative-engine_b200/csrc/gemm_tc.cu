// Projection GEMMs on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// C[M, N] = A[M, K] . W[N, K]^T (+ bias) (-> GELU), bf16 operands, fp32
// accumulation in tensor memory, bf16 or fp32 output: the nn.Linear layers of
// engine/model.py:73-74, 127-129, 156 (qkv, out, MLP, lm_head).
//
// One CTA computes one 128 x BN tile.  Warp 0 (one thread) streams 128 x 64
// slabs of A and BN x 64 slabs of W through a TMA + mbarrier ring (128-byte
// swizzle, the layout tcgen05 reads natively); warp 1 allocates BN columns of
// tensor memory and issues tcgen05.mma (M=128, N=BN, K=16, one thread) from
// shared-memory descriptors, committing each stage back to the producer with
// tcgen05.commit; warps 4..7 drain the accumulator with tcgen05.ld (each warp
// owns its 32-lane quarter of TMEM), apply bias / GELU and store.  All waits
// are bounded; an expired wait latches PSE_STATUS_TIMEOUT and the CTA still
// releases its tensor memory.

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tmap_cache.h"

namespace pse {
namespace gemm {

constexpr int BM = 128, BK = 64;
constexpr int kThreads = 256;
constexpr uint32_t kSpinLimit = 1u << 24;

__host__ __device__ constexpr int stages_for(int bn) { return bn == 256 ? 3 : 4; }

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(su32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i >= 64) __nanosleep(64);
  }
  return false;
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(su32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(su32(bar))
      : "memory");
}

// Shared-memory matrix descriptor of a K-major tile in the 128-byte swizzle
// layout: rows 128 bytes apart, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);        // start address
  d |= (uint64_t)1 << 16;                       // leading byte offset (16 B units; unused for SW128 K-major)
  d |= (uint64_t)(1024 >> 4) << 32;             // stride byte offset between 8-row groups
  d |= (uint64_t)1 << 46;                       // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                       // layout: 128-byte swizzle
  return d;
}

// Instruction descriptor: bf16 x bf16 -> fp32, both K-major, M = 128, N = bn.
__host__ __device__ constexpr uint32_t instr_desc(int bn) {
  return (1u << 4)                 // D format fp32
         | (1u << 7)               // A format bf16
         | (1u << 10)              // B format bf16
         | ((uint32_t)(bn >> 3) << 17)
         | ((uint32_t)(BM >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int j = 0; j < 16; ++j) v[j] = __uint_as_float(r[j]);
}

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.f + erff(x * 0.70710678118654752440f)); }

struct Args {
  void* c;
  int64_t ldc;
  const __nv_bfloat16* bias;
  int M, N, K;
  int act;      // 0 none, 1 GELU
  int out_f32;  // 1: fp32 C, 0: bf16 C
  int32_t* status;
};

template <int BN>
__global__ void __launch_bounds__(kThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a,
                                                              const __grid_constant__ CUtensorMap tma_b, Args a) {
  constexpr int S = stages_for(BN);
  constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;                    // [S][A_BYTES]
  uint8_t* sb = smem + S * A_BYTES;      // [S][B_BYTES]
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + S * B_BYTES);
  uint64_t* empty = full + S;
  uint64_t* acc_bar = empty + S;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_bar + 1);
  int* failed = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
  const int KB = a.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_bar, 1);
    *failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                 "r"(BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % S;
        if (!mbar_wait(&empty[s], ((kb / S) & 1) ^ 1)) {
          *failed = 1;
          break;
        }
        mbar_expect_tx(&full[s], A_BYTES + B_BYTES);
        tma_load_2d(sa + s * A_BYTES, &tma_a, kb * BK, m0, &full[s]);
        tma_load_2d(sb + s * B_BYTES, &tma_b, kb * BK, n0, &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(BN);
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % S;
        if (!mbar_wait(&full[s], (kb / S) & 1)) {
          *failed = 1;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t a_base = su32(sa + s * A_BYTES), b_base = su32(sb + s * B_BYTES);
#pragma unroll
        for (int k = 0; k < BK / 16; ++k)
          mma_bf16(tmem, smem_desc(a_base + k * 32), smem_desc(b_base + k * 32), idesc, (kb | k) != 0);
        mma_commit(&empty[s]);  // the stage's smem is free once these MMAs have read it
      }
      mma_commit(acc_bar);      // accumulator complete (or, on failure, everything issued has retired)
    }
  } else if (warp >= 4) {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const bool ok = mbar_wait(acc_bar, 0);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    if (!ok) {
      *failed = 1;
    } else {
      const int row = m0 + 32 * q + lane;
      for (int c0 = 0; c0 < BN; c0 += 16) {
        float v[16];
        tmem_ld16(tmem + ((uint32_t)(32 * q) << 16) + c0, v);
        const int col = n0 + c0;
        if (row >= a.M || col >= a.N) continue;
        if (a.bias) {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] += col + j < a.N ? __bfloat162float(a.bias[col + j]) : 0.f;
        }
        if (a.act == 1) {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = gelu_erf(v[j]);
        }
        const bool full_chunk = col + 16 <= a.N;
        if (a.out_f32) {
          float* cr = reinterpret_cast<float*>(a.c) + (int64_t)row * a.ldc + col;
          if (full_chunk) {
#pragma unroll
            for (int j = 0; j < 16; j += 4) *reinterpret_cast<float4*>(cr + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
          } else {
            for (int j = 0; j < 16 && col + j < a.N; ++j) cr[j] = v[j];
          }
        } else {
          __nv_bfloat16* cr = reinterpret_cast<__nv_bfloat16*>(a.c) + (int64_t)row * a.ldc + col;
          if (full_chunk) {
            uint4 w[2];
            __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(w);
#pragma unroll
            for (int j = 0; j < 8; ++j) h[j] = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
            *reinterpret_cast<uint4*>(cr) = w[0];
            *reinterpret_cast<uint4*>(cr + 8) = w[1];
          } else {
            for (int j = 0; j < 16 && col + j < a.N; ++j) cr[j] = __float2bfloat16_rn(v[j]);
          }
        }
      }
    }
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  }
  __syncthreads();
  if (*reinterpret_cast<volatile int*>(failed)) {
    if (threadIdx.x == 0) {
      if (a.status) atomicOr(a.status, PSE_STATUS_TIMEOUT);
      // the MMA thread always commits acc_bar last: once it fires, every MMA
      // it issued has retired and tensor memory can be released
      mbar_wait(acc_bar, 0);
    }
    __syncthreads();
  }
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN));
  }
}

// ---------------------------------------------------------------- host side
TmapCache g_maps;

// [rows x cols] bf16 row-major with leading dimension ld (elements); box
// [box_rows x 64 columns], 128-byte swizzle, out-of-range reads as zero.
int tensor_map(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows, CUtensorMap* out) {
  return g_maps.get(ptr, (uint64_t)cols, (uint64_t)rows, (uint64_t)ld * 2, (uint32_t)BK, (uint32_t)box_rows, PSE_EINVAL,
                    out);
}

template <int BN>
constexpr size_t smem_bytes() {
  return 1024 + (size_t)stages_for(BN) * (BM * BK * 2 + BN * BK * 2) + (2 * stages_for(BN) + 1) * 8 + 16;
}

template <int BN>
int launch(const CUtensorMap& ma, const CUtensorMap& mb, const Args& a, cudaStream_t s) {
  auto kern = gemm_tc_kernel<BN>;
  constexpr size_t smem = smem_bytes<BN>();
  static_assert(smem <= 227 * 1024, "shared memory budget");
  static const cudaError_t opt = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (opt != cudaSuccess) return (int)opt;
  dim3 grid((unsigned)ceil_div(a.N, BN), (unsigned)ceil_div(a.M, BM));
  kern<<<grid, kThreads, smem, s>>>(ma, mb, a);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

}  // namespace gemm
}  // namespace pse

using namespace pse;

extern "C" int pse_gemm_bf16(const void* a, int64_t lda, const void* w, int64_t ldw, const void* bias, void* c,
                             int64_t ldc, int32_t m, int32_t n, int32_t k, int32_t act, int32_t out_f32,
                             int32_t* status, void* stream) {
  if (m < 0 || n < 0 || k < 0 || act < 0 || act > 1) return PSE_EINVAL;
  if (m == 0 || n == 0) return PSE_OK;
  if (!a || !w || !c) return PSE_EINVAL;
  // TMA: 16-byte aligned bases and row pitches; K in whole 64-element slabs
  if (k % gemm::BK != 0 || lda % 8 != 0 || ldw % 8 != 0 || ldc % (out_f32 ? 4 : 8) != 0) return PSE_EINVAL;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(c)) & 15)
    return PSE_EINVAL;
  const int bn = n >= 2048 ? 256 : 128;
  CUtensorMap ma, mb;
  int rc = gemm::tensor_map(a, m, k, lda, gemm::BM, &ma);
  if (rc) return rc;
  rc = gemm::tensor_map(w, n, k, ldw, bn, &mb);
  if (rc) return rc;
  gemm::Args args{c, ldc, reinterpret_cast<const __nv_bfloat16*>(bias), m, n, k, act, out_f32, status};
  cudaStream_t s = (cudaStream_t)stream;
  return bn == 256 ? gemm::launch<256>(ma, mb, args, s) : gemm::launch<128>(ma, mb, args, s);
}
