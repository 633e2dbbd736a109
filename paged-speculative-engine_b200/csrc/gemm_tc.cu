// Projection GEMMs on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// C[M, N] = A[M, K] . W[N, K]^T (+ bias) (-> GELU), bf16 operands, fp32
// accumulation in tensor memory, bf16 or fp32 output: the nn.Linear layers of
// engine/model.py:73-74, 127-129, 156 (qkv, out, MLP, lm_head).
//
// Persistent, warp-specialised kernel: min(tiles, SMs) CTAs walk the 128 x BN
// output tiles (M fastest, so the CTAs working at one time share weight
// columns through L2).  Per CTA:
//   warp 0 (one thread)  streams 128 x 64 slabs of A and BN x 64 slabs of W
//                        through a TMA + mbarrier ring (128-byte swizzle, the
//                        layout tcgen05 reads natively);
//   warp 1 (one thread)  issues tcgen05.mma (M=128, N=BN, K=16) from shared
//                        memory descriptors into one of two TMEM accumulators
//                        (2 x BN columns), returning each stage to the
//                        producer with tcgen05.commit;
//   warps 2..5           drain the other accumulator with tcgen05.ld (each warp
//                        its 32-lane TMEM quarter), add the bias, apply GELU,
//                        and store -- overlapping the next tile's MMAs.
// BN (64 / 128 / 256) is chosen per shape for SM coverage.
//
// Programmatic dependent launch: the CTAs may start while the previous kernel
// finishes (barrier set-up, TMEM allocation and descriptor prefetch overlap
// its tail) and wait for it before the first operand load; once a CTA has
// issued its last load it lets the next kernel launch.
//
// All waits are bounded; an expired wait latches PSE_STATUS_TIMEOUT, every
// role stops, the producer waits (bounded) for its copies in flight and the
// CTA releases its tensor memory after its last MMA has retired.

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tmap_cache.h"

namespace pse {
namespace gemm {

constexpr int BM = 128, BK = 64;
constexpr int kEpiWarps = 8;  // two per TMEM lane quarter, each draining half of the tile's columns
constexpr int kThreads = 64 + 32 * kEpiWarps;
constexpr uint32_t kSpinLimit = 1u << 24;

// ring depth per tile width: ~192 KB of stages
__host__ __device__ constexpr int stages_for(int bn) { return bn == 256 ? 4 : bn == 128 ? 6 : 8; }

__device__ __forceinline__ uint32_t su32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(bar)) : "memory");
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
    if (i >= 64) __nanosleep(32);
  }
  return false;
}
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(su32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(su32(bar))
      : "memory");
}
__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
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

__device__ __forceinline__ float gelu_erf(float x) { return 0.5f * x * (1.f + erff(x * 0.70710678118654752440f)); }

struct Args {
  void* c;
  int64_t ldc;
  const __nv_bfloat16* bias;
  int M, N, K;
  int tiles_m, tiles;
  int act;      // 0 none, 1 GELU
  int out_f32;  // 1: fp32 C, 0: bf16 C
  int32_t* status;
};

// Issue a 32-column accumulator load of this thread's TMEM lane; the values
// may be used only after tmem_ld_wait on the same registers.
__device__ __forceinline__ void tmem_ld32_issue(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// Wait for this thread's accumulator loads; the registers are in-out operands
// so no use of them is scheduled before the wait.
__device__ __forceinline__ void tmem_ld_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// Epilogue of one 32-column chunk of one accumulator row (bias, GELU, store).
__device__ __forceinline__ void store_chunk(const Args& a, int row, int col, float* v) {
  if (row >= a.M || col >= a.N) return;
  const bool full_chunk = col + 32 <= a.N;
  if (a.bias) {
    if (full_chunk) {
      const uint4* bp = reinterpret_cast<const uint4*>(a.bias + col);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const uint4 w = __ldg(bp + j);
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 f = __bfloat1622float2(h[e]);
          v[8 * j + 2 * e] += f.x;
          v[8 * j + 2 * e + 1] += f.y;
        }
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += col + j < a.N ? __bfloat162float(a.bias[col + j]) : 0.f;
    }
  }
  if (a.act == 1) {
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = gelu_erf(v[j]);
  }
  if (a.out_f32) {
    float* cr = reinterpret_cast<float*>(a.c) + (int64_t)row * a.ldc + col;
    if (full_chunk) {
#pragma unroll
      for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(cr + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col + j < a.N) cr[j] = v[j];
    }
  } else {
    __nv_bfloat16* cr = reinterpret_cast<__nv_bfloat16*>(a.c) + (int64_t)row * a.ldc + col;
    if (full_chunk) {
#pragma unroll
      for (int j = 0; j < 32; j += 8) {
        uint4 w;
        __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&w);
#pragma unroll
        for (int e = 0; e < 4; ++e) h[e] = __floats2bfloat162_rn(v[j + 2 * e], v[j + 2 * e + 1]);
        *reinterpret_cast<uint4*>(cr + j) = w;
      }
    } else {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col + j < a.N) cr[j] = __float2bfloat16_rn(v[j]);
    }
  }
}

// Drain `ncols` (a multiple of 32) accumulator columns of this thread's TMEM
// lane starting at `taddr`, output row `row`, output columns from `col0`: the
// load of the next 32 columns is in flight while the current ones are stored.
__device__ __forceinline__ void drain_cols(const Args& a, uint32_t taddr, int row, int col0, int ncols) {
  uint32_t r0[32], r1[32];
  float v[32];
  tmem_ld32_issue(taddr, r0);
  tmem_ld_wait(r0);
#pragma unroll 1
  for (int c = 0; c < ncols; c += 64) {
    const bool more1 = c + 32 < ncols, more2 = c + 64 < ncols;
    if (more1) tmem_ld32_issue(taddr + c + 32, r1);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r0[j]);
    store_chunk(a, row, col0 + c, v);
    if (!more1) break;
    tmem_ld_wait(r1);
    if (more2) tmem_ld32_issue(taddr + c + 64, r0);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r1[j]);
    store_chunk(a, row, col0 + c + 32, v);
    if (more2) tmem_ld_wait(r0);
  }
}

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
  uint64_t* acc_full = empty + S;        // [2] accumulator ready for the epilogue
  uint64_t* acc_empty = acc_full + 2;    // [2] accumulator drained
  uint64_t* done_bar = acc_empty + 2;    // every MMA of this CTA retired
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  int* failed = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int KB = a.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kEpiWarps);
    }
    mbar_init(done_bar, 1);
    *failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_map(&tma_a);
    prefetch_map(&tma_b);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                 "r"(2 * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  // A (and the bias) may come from the kernel just before this one
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;  // k-slabs issued, over all of this CTA's tiles
      bool ok = true;
      for (int t = blockIdx.x; ok && t < a.tiles; t += gridDim.x) {
        const int m0 = (t % a.tiles_m) * BM, n0 = (t / a.tiles_m) * BN;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(&empty[s], ((it / S) & 1) ^ 1)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], A_BYTES + B_BYTES);
          tma_load_2d(sa + s * A_BYTES, &tma_a, kb * BK, m0, &full[s]);
          tma_load_2d(sb + s * B_BYTES, &tma_b, kb * BK, n0, &full[s]);
        }
      }
      // every operand this CTA needs is on its way: the next kernel may launch
      asm volatile("griddepcontrol.launch_dependents;");
      if (!ok) {
        *failed = 1;
        // copies still in flight land in shared memory: wait for them (bounded)
        for (uint32_t t2 = it > (uint32_t)S ? it - S : 0; t2 < it; ++t2) mbar_wait(&full[t2 % S], (t2 / S) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      constexpr uint32_t idesc = instr_desc(BN);
      uint32_t it = 0, local = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < a.tiles; t += gridDim.x, ++local) {
        const uint32_t buf = local & 1;
        if (!mbar_wait(&acc_empty[buf], ((local >> 1) & 1) ^ 1)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + buf * BN;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(&full[s], (it / S) & 1)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_base = su32(sa + s * A_BYTES), b_base = su32(sb + s * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_bf16(d, smem_desc(a_base + k * 32), smem_desc(b_base + k * 32), idesc, (kb | k) != 0);
          mma_commit(&empty[s]);  // the stage's smem is free once these MMAs have read it
        }
        if (ok) mma_commit(&acc_full[buf]);  // accumulator complete
      }
      if (!ok) *failed = 1;
      mma_commit(done_bar);  // fires once every MMA issued above has retired
    }
  } else {
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    uint32_t local = 0;
    for (int t = blockIdx.x; t < a.tiles; t += gridDim.x, ++local) {
      const uint32_t buf = local & 1;
      const bool ok = mbar_wait(&acc_full[buf], (local >> 1) & 1);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      if (!ok) {
        *failed = 1;
        break;
      }
      const int m0 = (t % a.tiles_m) * BM, n0 = (t / a.tiles_m) * BN;
      const int row = m0 + 32 * q + lane;
      const int half = (warp - 2) / 4;  // which half of the tile's columns this warp drains
      const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + buf * BN + half * (BN / 2);
      drain_cols(a, tbase, row, n0 + half * (BN / 2), BN / 2);
      // this accumulator may take the tile after next
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[buf]);
    }
  }
  __syncthreads();
  if (warp == 1) {
    // the MMA thread committed done_bar after its last MMA: once it fires, the
    // tensor memory those MMAs write can be released
    const bool retired = mbar_wait(done_bar, 0);
    if (lane == 0 && (!retired || *reinterpret_cast<volatile int*>(failed)) && a.status)
      atomicOr(a.status, PSE_STATUS_TIMEOUT);
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
  }
}

// ---------------------------------------------------------------- two-SM tiles
//
// A cluster of two CTAs (one per SM) computes 256 x BN output tiles with
// tcgen05.mma.cta_group::2 (M = 256): CTA r loads rows [128 r, 128 r + 128) of
// the tile's A slab and rows [r BN/2, (r+1) BN/2) of its W slab into its own
// shared memory, and the MMA issued by rank 0 reads A from each CTA's own
// buffer and W from both, writing each CTA's 128 accumulator rows into that
// CTA's tensor memory.  Per SM and k-slab this moves 16 KB + BN x 64 B for a
// 128 x BN x 64 product, two thirds of the single-CTA tile's operand traffic
// at BN = 256 -- what bounds the single-CTA kernel on the wide projections is
// that traffic out of L2.
//
// Barriers (each CTA keeps the same layout): full[s] of rank 0 counts both
// CTAs' bytes of stage s (each CTA's copies signal it, rank 0 expects the
// total); empty[s], acc_full[b] and done of both CTAs are signalled by rank 0's
// commits (one per CTA); acc_empty[b] of rank 0 collects the epilogue warps
// of both CTAs.  Loads are plain (each CTA fetches its own operands).

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// shared::cluster address of `p` (this CTA's shared memory) in CTA `rank`.
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(su32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(su32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void mma_pair(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// Arrive on `bar` (a shared::cluster address, this CTA's or the peer's) once
// every tcgen05.mma this thread issued so far has completed.
__device__ __forceinline__ void mma_commit_pair(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
}

// Instruction descriptor of the pair MMA: M = 256, N = bn.
__host__ __device__ constexpr uint32_t instr_desc_pair(int bn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(256 >> 4) << 24);
}

__host__ __device__ constexpr int pair_stages(int bn) { return bn == 256 ? 6 : 8; }

template <int BN>
__global__ void __launch_bounds__(kThreads, 1) gemm_pair_kernel(const __grid_constant__ CUtensorMap tma_a,
                                                                const __grid_constant__ CUtensorMap tma_b, Args a) {
  constexpr int S = pair_stages(BN);
  constexpr int A_BYTES = BM * BK * 2, B_BYTES = (BN / 2) * BK * 2;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + S * A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + S * B_BYTES);
  uint64_t* empty = full + S;
  uint64_t* acc_full = empty + S;
  uint64_t* acc_empty = acc_full + 2;
  uint64_t* done_bar = acc_empty + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done_bar + 1);
  int* failed = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_rank();
  const int pair = blockIdx.x >> 1, n_pairs = gridDim.x >> 1;
  const int KB = a.K / BK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 2 * kEpiWarps);
    }
    mbar_init(done_bar, 1);
    *failed = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    prefetch_map(&tma_a);
    prefetch_map(&tma_b);
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                 "r"(2 * BN));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  // both CTAs' barriers exist before either signals the other's
  cluster_sync_all();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  asm volatile("griddepcontrol.wait;" ::: "memory");

  if (warp == 0) {
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = pair; ok && t < a.tiles; t += n_pairs) {
        const int m0 = (t % a.tiles_m) * (2 * BM) + (int)rank * BM;
        const int n0 = (t / a.tiles_m) * BN + (int)rank * (BN / 2);
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(&empty[s], ((it / S) & 1) ^ 1)) {
            ok = false;
            break;
          }
          const uint32_t bar0 = peer_addr(&full[s], 0);  // rank 0's barrier counts both CTAs' bytes
          if (rank == 0) mbar_expect_tx(&full[s], 2 * (A_BYTES + B_BYTES));
          tma_load_2d_pair(sa + s * A_BYTES, &tma_a, kb * BK, m0, bar0);
          tma_load_2d_pair(sb + s * B_BYTES, &tma_b, kb * BK, n0, bar0);
        }
      }
      asm volatile("griddepcontrol.launch_dependents;");
      if (!ok) {
        *failed = 1;
        __nanosleep(20000);  // copies in flight land within microseconds
        if (rank == 0)
          for (uint32_t t2 = it > (uint32_t)S ? it - S : 0; t2 < it; ++t2) mbar_wait(&full[t2 % S], (t2 / S) & 1);
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      constexpr uint32_t idesc = instr_desc_pair(BN);
      uint32_t it = 0, local = 0;
      bool ok = true;
      for (int t = pair; ok && t < a.tiles; t += n_pairs, ++local) {
        const uint32_t buf = local & 1;
        if (!mbar_wait(&acc_empty[buf], ((local >> 1) & 1) ^ 1)) {
          ok = false;
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t d = tmem + buf * BN;
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % S;
          if (!mbar_wait(&full[s], (it / S) & 1)) {
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint32_t a_base = su32(sa + s * A_BYTES), b_base = su32(sb + s * B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k)
            mma_pair(d, smem_desc(a_base + k * 32), smem_desc(b_base + k * 32), idesc, (kb | k) != 0);
          mma_commit_pair(peer_addr(&empty[s], 0));  // both CTAs' stage s is free once these MMAs have read it
          mma_commit_pair(peer_addr(&empty[s], 1));
        }
        if (ok) {
          mma_commit_pair(peer_addr(&acc_full[buf], 0));
          mma_commit_pair(peer_addr(&acc_full[buf], 1));
        }
      }
      if (!ok) *failed = 1;
      mma_commit_pair(peer_addr(done_bar, 0));
      mma_commit_pair(peer_addr(done_bar, 1));
    }
  } else {
    const int q = warp & 3;
    uint32_t local = 0;
    for (int t = pair; t < a.tiles; t += n_pairs, ++local) {
      const uint32_t buf = local & 1;
      const bool ok = mbar_wait(&acc_full[buf], (local >> 1) & 1);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      if (!ok) {
        *failed = 1;
        break;
      }
      const int m0 = (t % a.tiles_m) * (2 * BM) + (int)rank * BM;
      const int n0 = (t / a.tiles_m) * BN;
      const int row = m0 + 32 * q + lane;
      const int half = (warp - 2) / 4;
      const uint32_t tbase = tmem + ((uint32_t)(32 * q) << 16) + buf * BN + half * (BN / 2);
      drain_cols(a, tbase, row, n0 + half * (BN / 2), BN / 2);
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(peer_addr(&acc_empty[buf], 0));
    }
  }
  __syncthreads();
  if (warp == 1) {
    // rank 0's last commit fires once every MMA writing this CTA's tensor memory has retired
    const bool retired = mbar_wait(done_bar, 0);
    if (lane == 0 && (!retired || *reinterpret_cast<volatile int*>(failed)) && a.status)
      atomicOr(a.status, PSE_STATUS_TIMEOUT);
    __syncwarp();
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  }
  // neither CTA leaves while the other may still signal its barriers
  cluster_sync_all();
  if (warp == 1) asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * BN));
}

// ---------------------------------------------------------------- host side
TmapCache g_maps;
bool g_pair_tiles = true;

// [rows x cols] bf16 row-major with leading dimension ld (elements); box
// [box_rows x 64 columns], 128-byte swizzle, out-of-range reads as zero.
int tensor_map(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows, CUtensorMap* out) {
  return g_maps.get(ptr, (uint64_t)cols, (uint64_t)rows, (uint64_t)ld * 2, (uint32_t)BK, (uint32_t)box_rows, PSE_EINVAL,
                    out);
}

template <int BN>
constexpr size_t smem_bytes() {
  return 1024 + (size_t)stages_for(BN) * (BM * BK * 2 + BN * BK * 2) + (2 * stages_for(BN) + 5) * 8 + 16;
}

int sm_count() {
  static int sms = [] {
    int dev = 0, n = kNumSMs;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : kNumSMs;
  }();
  return sms;
}

// Tile width: the widest of 256 / 128 / 64 whose tiles cover the SMs (the
// MMA rate per tile column grows with N); narrower tiles only when the wider
// ones leave most SMs idle.
int pick_bn(int m, int n) {
  const int tm = ceil_div(m, BM), sms = sm_count();
  const int t256 = tm * ceil_div(n, 256), t128 = tm * ceil_div(n, 128);
  if (t256 >= (sms * 2) / 3 || n > 4096) return 256;
  if (t128 >= (sms * 2) / 3) return 128;
  return 64;
}

template <int BN>
constexpr size_t pair_smem_bytes() {
  return 1024 + (size_t)pair_stages(BN) * (BM * BK * 2 + (BN / 2) * BK * 2) + (2 * pair_stages(BN) + 5) * 8 + 16;
}

// Two-SM tiles (256 x 256) where they keep most SMs busy; single-CTA tiles otherwise.
bool use_pair(int m, int n) {
  const int pairs = ceil_div(m, 2 * BM) * ceil_div(n, 256);
  return pairs * 2 >= (sm_count() * 2) / 3;
}

template <int BN>
int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, Args a, cudaStream_t s) {
  auto kern = gemm_pair_kernel<BN>;
  constexpr size_t smem = pair_smem_bytes<BN>();
  static_assert(smem <= 227 * 1024, "shared memory budget");
  static const cudaError_t opt = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (opt != cudaSuccess) return (int)opt;
  a.tiles_m = ceil_div(a.M, 2 * BM);
  a.tiles = a.tiles_m * ceil_div(a.N, BN);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  // as many pairs as fit at once (one CTA per SM), at most one per tile
  static int max_pairs = 0;
  if (max_pairs == 0) {
    cfg.gridDim = dim3((unsigned)(2 * (sm_count() / 2)), 1, 1);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = sm_count() / 2;
    }
    max_pairs = n;
  }
  const int pairs = a.tiles < max_pairs ? a.tiles : max_pairs;
  cfg.gridDim = dim3((unsigned)(2 * pairs), 1, 1);
  const cudaError_t le = cudaLaunchKernelEx(&cfg, kern, ma, mb, a);
  if (le != cudaSuccess) return (int)le;
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

template <int BN>
int launch(const CUtensorMap& ma, const CUtensorMap& mb, Args a, cudaStream_t s) {
  auto kern = gemm_tc_kernel<BN>;
  constexpr size_t smem = smem_bytes<BN>();
  static_assert(smem <= 227 * 1024, "shared memory budget");
  static const cudaError_t opt = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (opt != cudaSuccess) return (int)opt;
  a.tiles_m = ceil_div(a.M, BM);
  a.tiles = a.tiles_m * ceil_div(a.N, BN);
  const int grid = a.tiles < sm_count() ? a.tiles : sm_count();
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl_enabled() ? 1 : 0;
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t le = cudaLaunchKernelEx(&cfg, kern, ma, mb, a);
  if (le != cudaSuccess) return (int)le;
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
  if (k == 0 || k % gemm::BK != 0 || lda % 8 != 0 || ldw % 8 != 0 || ldc % (out_f32 ? 4 : 8) != 0) return PSE_EINVAL;
  if ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(c) |
       reinterpret_cast<uintptr_t>(bias)) & 15)
    return PSE_EINVAL;
  gemm::Args args{c, ldc, reinterpret_cast<const __nv_bfloat16*>(bias), m, n, k, 0, 0, act, out_f32, status};
  cudaStream_t s = (cudaStream_t)stream;
  CUtensorMap ma, mb;
  int rc = gemm::tensor_map(a, m, k, lda, gemm::BM, &ma);
  if (rc) return rc;
  if (gemm::g_pair_tiles && gemm::use_pair(m, n)) {
    rc = gemm::tensor_map(w, n, k, ldw, 128, &mb);  // each CTA of a pair loads half of the 256 W rows
    if (rc) return rc;
    return gemm::launch_pair<256>(ma, mb, args, s);
  }
  const int bn = gemm::pick_bn(m, n);
  rc = gemm::tensor_map(w, n, k, ldw, bn, &mb);
  if (rc) return rc;
  if (bn == 256) return gemm::launch<256>(ma, mb, args, s);
  if (bn == 128) return gemm::launch<128>(ma, mb, args, s);
  return gemm::launch<64>(ma, mb, args, s);
}

extern "C" int pse_gemm_pair_tiles(int32_t on) {
  gemm::g_pair_tiles = on != 0;
  return PSE_OK;
}
