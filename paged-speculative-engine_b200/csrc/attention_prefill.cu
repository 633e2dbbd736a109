// Paged attention for wide calls (prompt prefill) on the 5th-generation tensor
// cores, sm_100a.
//
// Same contract as pse_paged_attention (engine/model.py:99-116 over the paged
// layout of engine/paged_cache.py:83-88) for calls with many query rows per
// (row, KV head): the K/V of a prompt is re-read by every query tile from L2,
// so these calls are bound by the tensor cores, the softmax's exponentials and
// shared-memory traffic, not by HBM.
//
// A query tile is 128 rows: the GQA group's heads over 128 / group consecutive
// tokens, head-major (tile row r = group head r / (128 / group), token
// r % (128 / group)).  Persistent CTAs take work items round-robin, heaviest
// first.  Warp roles:
//   warp 8       TMA producer: each item's Q tile(s) into one of two buffers
//                ahead of use, and the K and V pages of each 128-key tile into
//                a shared-memory ring (128-byte swizzle; each head_dim half of
//                a tile's 128 keys is one 16 KB K-major block), completing on
//                mbarriers;
//   warp 9       allocates the 512 TMEM columns and issues tcgen05.mma from
//                one thread: S = Q K^T (M 128, N 128, K 16; Q and K in shared
//                memory) into a TMEM score buffer, O += P V (M 128, N
//                head_dim, K 16; P in TMEM, V in shared memory as an MN-major
//                operand) into the TMEM output; tcgen05.commit hands each
//                result on;
//   warps 0..7   the softmax, one thread per (tile row, warpgroup): tcgen05.ld
//                of the scores, causal mask, exp2 online softmax (max and sum
//                over 8 independent chains, ex2.approx), P as bf16 pairs into
//                TMEM with tcgen05.st, rescale of the row's TMEM output when
//                its reference maximum grows by more than 2^8, and at the
//                item's end O / l to global memory.
// P never touches shared memory: with K, V and Q the only operands read from
// it, shared-memory bandwidth (which bounds these small-N MMAs) goes to them.
// Two arrangements of the softmax warpgroups:
//   prefill_attn_kernel (head_dim 64 or 128): one query tile per item; the two
//                warpgroups split its 128 key columns and exchange each row's
//                maximum every tile;
//   prefill_pair_kernel (head_dim 64): two query tiles per item (tiles 2m and
//                2m + 1 of one row and KV head), one per warpgroup, sharing
//                every K/V tile.
// Scores of tile j+1 are computed while the softmax of tile j runs, P V of
// tile j while the softmax of tile j+1 runs, and the next item's Q and first
// scores while this item's output is written.
//
// Query tokens at or past the row's length (padding of a length-grouped
// prefill, which never allocates them) get zero output.  Every wait is bounded
// and watches an abort flag: on expiry the kernel latches PSE_STATUS_TIMEOUT,
// every role stops, the MMA thread's last commit still retires before tensor
// memory is released, and in-flight copies are waited for before exit.

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"

namespace pse {
namespace pf {

constexpr int BQ = 128;   // query rows per item = TMEM lanes
constexpr int BKV = 128;  // keys per tile
// warps 0..7: softmax (warp w handles TMEM lanes 32 * (w % 4) .. +31 and key
// columns 64 * (w / 4) .. +63 of each tile); warp 8: TMA; warp 9: MMA
constexpr int kSoftmaxThreads = 256;
constexpr int kProducerWarp = 8, kMmaWarp = 9;
constexpr int kThreads = 10 * 32;
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;    // score buffers at columns 0 and 128
constexpr uint32_t kColO = 256;  // output accumulator
constexpr uint32_t kColP = 384;  // P (bf16 pairs, 64 columns): the A operand of O += P V
constexpr int kHalfBytes = BKV * 128;  // one 64-column half of a 128-row tile (16 KB)

#ifndef PSE_PF_STAGES64
#define PSE_PF_STAGES64 3
#endif
template <int HD>
__host__ __device__ constexpr int n_stages() { return HD == 64 ? PSE_PF_STAGES64 : 2; }
// Q tiles in flight: two (the next item's Q lands while this one runs).
template <int HD>
__host__ __device__ constexpr int n_qbufs() { return 2; }

struct Args {
  const int32_t* block_table;
  const int32_t* nblocks;
  const int32_t* seq_len;
  int max_blocks, block_size, num_blocks, num_slots, kv_heads;
  __nv_bfloat16* out;
  int64_t out_tok_stride;
  const int32_t* slots;
  const int32_t* base_len;
  const int32_t* row_order;
  int rows, width, q_heads, group, tpt, n_qtiles, n_items;
  float scale_log2;
  int32_t* status;
  int oob_row;
};

// One work item: query tokens [w0, w_end) of row i for every head of KV head
// hk's group; tile row r is head hk * group + r / tpt at token w0 + r % tpt.
struct Item {
  int i, hk, slot, base, len, w0, w_end, kmax, n_tiles;
};

__device__ __forceinline__ Item decode(const Args& a, int e) {
  Item it;
  const int per_qt = a.rows * a.kv_heads;
  const int qt = a.n_qtiles - 1 - e / per_qt;  // heaviest query tile first
  const int rem = e % per_qt;
  const int ri = rem / a.kv_heads;
  it.hk = rem % a.kv_heads;
  it.i = a.row_order ? a.row_order[ri] : ri;
  it.slot = a.slots[it.i];
  it.base = a.base_len[it.i];
  it.w0 = qt * a.tpt;
  it.w_end = min(it.w0 + a.tpt, a.width);
  const bool ok = it.w_end > it.w0 && it.slot >= 0 && it.slot < a.num_slots && it.base >= 0;
  it.len = ok ? a.seq_len[it.slot] : 0;
  it.kmax = min(it.base + it.w_end, it.len);
  it.n_tiles = (ok && it.base + it.w0 < it.len && it.kmax > 0) ? (it.kmax + BKV - 1) / BKV : 0;
  return it;
}

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
// Bounded wait that also gives up once another role has aborted.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  for (uint32_t n = 0; n < kSpinLimit; ++n) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((n & 15) == 15 && *abort_flag) return false;
    if (n >= 64) __nanosleep(32);
  }
  *abort_flag = 1;
  return false;
}
// Bounded wait used only on the exit path (no abort check).
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  for (uint32_t n = 0; n < kSpinLimit; ++n) {
    if (mbar_try_wait(bar, parity)) return;
    if (n >= 64) __nanosleep(64);
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(su32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(su32(bar))
      : "memory");
}

// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 format).
// K-major operand: rows 128 B apart, 8-row groups 1024 B apart; the K offset
// of a 16-element step inside the 128-byte row is added to the start address.
__device__ __forceinline__ uint64_t desc_kmajor(uint32_t addr) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;               // leading byte offset: unused for swizzled K-major
  d |= (uint64_t)(1024 >> 4) << 32;     // stride byte offset: 8-row groups
  d |= (uint64_t)1 << 46;               // descriptor version
  d |= (uint64_t)2 << 61;               // 128-byte swizzle
  return d;
}
// MN-major operand (V for O += P V: N = head_dim contiguous, K = keys): a
// swizzle atom is 64 N-elements x 8 K-rows (1024 B); atoms along N are
// `lbo` bytes apart, 8-row groups along K 1024 B apart.
__device__ __forceinline__ uint64_t desc_mnmajor(uint32_t addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}
// Instruction descriptor: bf16 x bf16 -> fp32, M = 128, N = n; b_mn: B is MN-major.
__host__ __device__ constexpr uint32_t instr_desc(int n, int b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)b_mn << 16) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(BQ >> 4) << 24);
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
// A operand in tensor memory: row r of A is lane r, 16-bit elements packed two
// to a 32-bit column (K = 16 per instruction = 8 columns).
__device__ __forceinline__ void mma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(su32(bar))
               : "memory");
}

#define PF_R32(r)                                                                                                   \
  "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),       \
      "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),        \
      "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),       \
      "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
#define PF_W32(r)                                                                                                   \
  "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),      \
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),   \
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),   \
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])

// 32 consecutive columns of this thread's TMEM lane (no wait).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : PF_R32(r)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      PF_W32(r)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}


__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int HD>
constexpr size_t smem_bytes() {
  // align slack + Q buffers + ring (K and V per stage) + barriers + the two
  // softmax warpgroups' row exchange (2 x 2 x 128 maxima, 2 x 128 sums)
  return 1024 + (size_t)n_qbufs<HD>() * BQ * HD * 2 + (size_t)n_stages<HD>() * 2 * BKV * HD * 2 + 256 +
         (size_t)6 * BQ * 4;
}

template <int HD>
__global__ void __launch_bounds__(kThreads, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                        const __grid_constant__ CUtensorMap tmq, Args a) {
  constexpr int S = n_stages<HD>();
  constexpr int kTileBytes = BKV * HD * 2;  // one of K or V
  constexpr int kQBytes = BQ * HD * 2;
  constexpr int kHalves = HD / 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int QB = n_qbufs<HD>();
  uint8_t* q_s = smem;                        // [QB][128 x HD] K-major
  uint8_t* ring = q_s + QB * kQBytes;         // [S][K tile | V tile]
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + S * 2 * kTileBytes);
  uint64_t* empty = full + S;
  uint64_t* s_full = empty + S;     // [2] scores of a tile ready (one per score buffer)
  uint64_t* q_full = s_full + 2;    // [QB] an item's Q landed (one per Q buffer)
  uint64_t* q_empty = q_full + 2;   // [QB] an item's score MMAs retired: its Q buffer is free
  uint64_t* p_full = q_empty + 2;   // P written, output rescaled (128 arrivals)
  uint64_t* pv_done = p_full + 1;   // O += P V of a tile retired
  uint64_t* final_bar = pv_done + 1;
  uint64_t* pair_bar = final_bar + 1;  // [4] softmax warp pairs' exchanges (64 arrivals)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pair_bar + 4);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* issued = abort_flag + 1;   // K/V tiles whose copies the producer issued
  int* issued_q = issued + 1;     // Q tiles whose copies the producer issued
  float* xmax = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + 256);  // [2 tiles][2 halves][128]
  float* xsum = xmax + 4 * BQ;                                                      // [2 halves][128]
  volatile int* vabort = abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&s_full[b], 1);
      mbar_init(&q_full[b], 1);
      mbar_init(&q_empty[b], 1);
    }
    mbar_init(p_full, kSoftmaxThreads);
    mbar_init(pv_done, 1);
    mbar_init(final_bar, 1);
    for (int x = 0; x < 4; ++x) mbar_init(&pair_bar[x], 64);
    *abort_flag = 0;
    *issued = 0;
    *issued_q = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == kProducerWarp) {
    // ------------------------------------------------------------ producer
    const int bs = a.block_size, ppt = BKV / bs;  // pages per tile (<= 8)
    int g = 0, nq = 0;
    bool run = true;
    for (int e = blockIdx.x; run && e < a.n_items; e += gridDim.x) {
      const Item it = decode(a, e);
      if (it.n_tiles == 0) continue;
      // the item's Q: one [tpt tokens x 64 columns] box per group head and half
      if (lane == 0) {
        const int qb = nq % QB;
        if (!mbar_wait(&q_empty[qb], ((nq / QB) & 1) ^ 1, vabort)) {
          run = false;
        } else {
          mbar_expect_tx(&q_full[qb], kQBytes);
          *issued_q = nq + 1;
          const int y = it.i * a.width + it.w0;
          for (int gq = 0; gq < a.group; ++gq)
#pragma unroll
            for (int c = 0; c < kHalves; ++c)
              tma_load_2d(q_s + qb * kQBytes + c * kHalfBytes + gq * a.tpt * 128, &tmq,
                          (it.hk * a.group + gq) * HD + c * 64, y, &q_full[qb]);
        }
      }
      run = __shfl_sync(0xffffffffu, run ? 1 : 0, 0) != 0;
      if (!run) break;
      ++nq;
      auto page = [&](int j) -> int {  // block of page `lane` of tile j (lanes < ppt)
        if (lane >= ppt || j >= it.n_tiles) return -1;
        const int pi = j * ppt + lane;
        if (pi >= a.nblocks[it.slot] || pi >= a.max_blocks || pi * bs >= it.kmax) return -1;
        const int b = a.block_table[(int64_t)it.slot * a.max_blocks + pi];
        return (b >= 0 && b < a.num_blocks) ? b : -1;
      };
      int cur = page(0);
      for (int j = 0; j < it.n_tiles; ++j) {
        const int nxt = page(j + 1);
        const int s = g % S;
        int stop = 0;
        if (lane == 0) {
          if (!mbar_wait(&empty[s], ((g / S) & 1) ^ 1, vabort)) {
            stop = 1;
          } else {
            mbar_expect_tx(&full[s], 2 * kTileBytes);
            *issued = g + 1;
          }
        }
        stop = __shfl_sync(0xffffffffu, stop, 0);
        if (stop) {
          run = false;
          break;
        }
        uint8_t* kst = ring + s * 2 * kTileBytes;
        uint8_t* vst = kst + kTileBytes;
        for (int p = 0; p < ppt; ++p) {
          const int blk = __shfl_sync(0xffffffffu, cur, p);
          if (lane == 0) {
            const int y = blk >= 0 ? (blk * a.kv_heads + it.hk) * bs : a.oob_row;
#pragma unroll
            for (int c = 0; c < kHalves; ++c) {
              const int off = c * kHalfBytes + p * bs * 128;
              tma_load_2d(kst + off, &tmk, c * 64, y, &full[s]);
              tma_load_2d(vst + off, &tmv, c * 64, y, &full[s]);
            }
          }
        }
        cur = nxt;
        ++g;
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc_s = instr_desc(BKV, 0);
      constexpr uint32_t idesc_o = instr_desc(HD, 1);
      // V's head_dim halves are 16 KB apart; with one half the field is unused
      // and gets the 8-row-group stride, so no reading of it leaves the tile
      constexpr uint32_t kVAtomStride = HD == 128 ? (uint32_t)kHalfBytes : 1024u;
      int g = 0, items = 0;
      bool run = true;
      for (int e = blockIdx.x; run && e < a.n_items; e += gridDim.x) {
        const Item it = decode(a, e);
        if (it.n_tiles == 0) continue;
        const int qb = items % QB;
        if (!mbar_wait(&q_full[qb], (items / QB) & 1, vabort)) break;
        tc_fence_after();
        const uint32_t q_base = su32(q_s + qb * kQBytes);
        int s_prev = 0;
        for (int j = 0; j <= it.n_tiles; ++j) {
          if (j < it.n_tiles) {
            const int s = g % S;
            if (!mbar_wait(&full[s], (g / S) & 1, vabort)) {
              run = false;
              break;
            }
            tc_fence_after();
            const uint32_t kb = su32(ring + s * 2 * kTileBytes);
            const uint32_t d = tmem + kColS + (uint32_t)(g & 1) * BKV;
#pragma unroll
            for (int kk = 0; kk < HD / 16; ++kk) {
              const uint32_t off = (uint32_t)((kk >> 2) * kHalfBytes + (kk & 3) * 32);
              mma_bf16(d, desc_kmajor(q_base + off), desc_kmajor(kb + off), idesc_s, kk > 0);
            }
            mma_commit(&s_full[g & 1]);
            if (j + 1 == it.n_tiles) mma_commit(&q_empty[qb]);  // the item's last read of Q
          }
          if (j >= 1) {
            // O += P V for the previous tile once its softmax is done
            const int gp = g - 1;
            if (!mbar_wait(p_full, gp & 1, vabort)) {
              run = false;
              break;
            }
            tc_fence_after();
            const uint32_t vb = su32(ring + s_prev * 2 * kTileBytes + kTileBytes);
#pragma unroll
            for (int kk = 0; kk < BKV / 16; ++kk)
              mma_bf16_ts(tmem + kColO, tmem + kColP + kk * 8, desc_mnmajor(vb + kk * 16 * 128, kVAtomStride),
                          idesc_o, (j > 1 || kk > 0) ? 1u : 0u);
            mma_commit(pv_done);
            mma_commit(&empty[s_prev]);
          }
          if (j < it.n_tiles) {
            s_prev = g % S;
            ++g;
          }
        }
        ++items;
      }
      mma_commit(final_bar);  // retires after every MMA this thread issued
    }
  } else {
    // ------------------------------------------------------------ softmax
    // Warps w and w + 4 share tile rows 32 * (w % 4) .. +31: each takes 64 of
    // a tile's 128 key columns, half of P and half of the output columns; the
    // pair exchanges the row maximum every tile (and the row sum at the end)
    // through shared memory behind the pair's mbarrier (a bounded wait: a warp
    // that gives up never leaves its partner blocked).
    const int half = warp >> 2, q4 = warp & 3;
    const int r = 32 * q4 + lane;  // tile row = TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q4) << 16);
    const int gq = r / a.tpt, wr = r % a.tpt;
    const float sl2 = a.scale_log2;
    constexpr int kCols = BKV / 2;   // key columns of this warp
    constexpr int kOCols = HD / 2;   // output columns of this warp
    int nx = 0;  // exchanges so far (the pair's barrier phase)
    auto pair_wait = [&]() -> bool {  // after this thread's arrive: wait for the partner's
      const bool ok = mbar_wait(&pair_bar[q4], nx & 1, vabort);
      ++nx;
      return __all_sync(0xffffffffu, ok);
    };
    int g = 0;
    bool run = true;
    for (int e = blockIdx.x; run && e < a.n_items; e += gridDim.x) {
      const Item it = decode(a, e);
      const int w = it.w0 + wr;
      const bool row_ok = gq < a.group && w < it.w_end;
      const int pos = it.base + w;
      const bool valid = row_ok && pos < it.len;
      const int h = it.hk * a.group + gq;
      __nv_bfloat16* orow = a.out + ((int64_t)it.i * a.width + w) * a.out_tok_stride + (int64_t)h * HD + half * kOCols;
      if (it.n_tiles == 0) {
        if (row_ok) {
#pragma unroll
          for (int c = 0; c < kOCols / 8; ++c) *reinterpret_cast<uint4*>(orow + c * 8) = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      const int lim = row_ok ? min(pos + 1, it.kmax) : it.kmax;  // keys [0, lim) visible to this row
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < it.n_tiles; ++j) {
        // waits are made warp-uniform: the tcgen05.ld / st below are warp-wide
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[g & 1], (g >> 1) & 1, vabort))) {
          run = false;
          break;
        }
        tc_fence_after();
        float sc[kCols];
        const int key0 = j * BKV + half * kCols;
        auto load_scores = [&]() {  // this warp's 64 raw scores of the tile, masked
          uint32_t* u = reinterpret_cast<uint32_t*>(sc);
          const uint32_t col = kColS + (uint32_t)(g & 1) * BKV + half * kCols;
#pragma unroll
          for (int c = 0; c < kCols / 32; ++c) tmem_ld32(lane_base + col + c * 32, u + c * 32);
          tmem_wait_ld();
          if (key0 + kCols > lim) {
#pragma unroll
            for (int c = 0; c < kCols; ++c) sc[c] = key0 + c < lim ? sc[c] : -INFINITY;
          }
        };
        float s8[8];
        auto exps = [&](float msub) {  // sc <- 2^(score * scale - msub), partial sums in s8
#pragma unroll
          for (int x = 0; x < 8; ++x) s8[x] = 0.f;
#pragma unroll
          for (int c = 0; c < kCols; ++c) {
            sc[c] = ex2(fmaf(sc[c], sl2, -msub));
            s8[c & 7] += sc[c];
          }
        };
        load_scores();
        // maximum of the raw scores (8 independent chains), published to the pair
        float m8[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) m8[x] = sc[x];
#pragma unroll
        for (int c = 8; c < kCols; ++c) m8[c & 7] = fmaxf(m8[c & 7], sc[c]);
        const float pm = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                               fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7])));
        float* xm = xmax + (g & 1) * 2 * BQ;
        xm[half * BQ + r] = pm;
        mbar_arrive(&pair_bar[q4]);
        // From the second tile on, the exponentials are taken against the
        // row's current reference maximum while the partner's maximum is in
        // flight; they are redone (from the scores, still in TMEM) only when
        // the pair's maximum moved past that reference.
        if (j > 0) exps(m_used == -INFINITY ? 0.f : m_used);
        if (!pair_wait()) {
          run = false;
          break;
        }
        const float mx = fmaxf(pm, xm[(half ^ 1) * BQ + r]) * sl2;
        // the row's reference maximum moves only when it would grow by more
        // than 8 (exponents stay <= 2^8); the output is rescaled then.  Both
        // warps of the pair see the same maximum, so they decide alike.
        float corr = 1.f;
        bool rescale = false;
        const bool moved = mx > m_used + 8.f;
        if (moved) {
          if (m_used != -INFINITY) {
            corr = ex2(m_used - mx);
            rescale = j > 0;
          }
          m_used = mx;
        }
        if (j == 0 || __any_sync(0xffffffffu, moved)) {
          if (j > 0) load_scores();
          exps(m_used == -INFINITY ? 0.f : m_used);
        }
        l = l * corr + (((s8[0] + s8[1]) + (s8[2] + s8[3])) + ((s8[4] + s8[5]) + (s8[6] + s8[7])));
        // the previous tile's P V has retired: P's buffer and the output are free
        if (g > 0 && !__all_sync(0xffffffffu, mbar_wait(pv_done, (g - 1) & 1, vabort))) {
          run = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int c = 0; c < kOCols / 32; ++c) {
            uint32_t o[32];
            const uint32_t ta = lane_base + kColO + half * kOCols + c * 32;
            tmem_ld32(ta, o);
            tmem_wait_ld();
#pragma unroll
            for (int x = 0; x < 32; ++x) o[x] = __float_as_uint(__uint_as_float(o[x]) * corr);
            tmem_st32(ta, o);
          }
          tmem_wait_st();
        }
        {
          // this warp's 64 keys of P as bf16 pairs into TMEM (the PV MMA's A operand)
          uint32_t pk[kCols / 2];
#pragma unroll
          for (int c = 0; c < kCols / 2; ++c) pk[c] = pack_bf16(sc[2 * c], sc[2 * c + 1]);
          tmem_st32(lane_base + kColP + half * (kCols / 2), pk);
          tmem_wait_st();
        }
        tc_fence_before();
        mbar_arrive(p_full);
        ++g;
      }
      if (!run) break;
      // the item's output: O / l once the last P V has retired; the row's sum
      // is the pair's two partial sums (same reference maximum)
      xsum[half * BQ + r] = l;
      mbar_arrive(&pair_bar[q4]);
      if (!pair_wait()) break;
      const float L = l + xsum[(half ^ 1) * BQ + r];
      if (!__all_sync(0xffffffffu, mbar_wait(pv_done, (g - 1) & 1, vabort))) break;
      tc_fence_after();
      const float inv = valid && L > 0.f ? 1.f / L : 0.f;
#pragma unroll
      for (int c = 0; c < kOCols / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(lane_base + kColO + half * kOCols + c * 32, o);
        tmem_wait_ld();
        if (row_ok) {
#pragma unroll
          for (int x = 0; x < 32; x += 8) {
            uint4 v;
            v.x = pack_bf16(__uint_as_float(o[x + 0]) * inv, __uint_as_float(o[x + 1]) * inv);
            v.y = pack_bf16(__uint_as_float(o[x + 2]) * inv, __uint_as_float(o[x + 3]) * inv);
            v.z = pack_bf16(__uint_as_float(o[x + 4]) * inv, __uint_as_float(o[x + 5]) * inv);
            v.w = pack_bf16(__uint_as_float(o[x + 6]) * inv, __uint_as_float(o[x + 7]) * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + x) = v;
          }
        }
      }
      tc_fence_before();
    }
  }

  __syncthreads();
  if (*vabort) {
    if (tid == 0) atomicOr(a.status, PSE_STATUS_TIMEOUT);
    if (warp == kProducerWarp && lane == 0) {
      // copies still in flight land before the CTA's shared memory goes away
      const int n = *issued;
      for (int t = n > S ? n - S : 0; t < n; ++t) mbar_drain(&full[t % S], (t / S) & 1);
      const int nq = *issued_q;
      for (int t = nq > QB ? nq - QB : 0; t < nq; ++t) mbar_drain(&q_full[t % QB], (t / QB) & 1);
    }
  }
  if (warp == kMmaWarp) {
    // every MMA has retired before tensor memory is released
    if (lane == 0) mbar_drain(final_bar, 0);
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

template <int HD>
int launch(const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mq, const Args& a, cudaStream_t s) {
  auto kern = prefill_attn_kernel<HD>;
  constexpr size_t smem = smem_bytes<HD>();
  static_assert(smem <= 227 * 1024, "shared memory budget");
  static const cudaError_t opt = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (opt != cudaSuccess) return (int)opt;
  int sms = kNumSMs, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = a.n_items < sms ? a.n_items : sms;
  if (grid <= 0) return PSE_OK;
  kern<<<grid, kThreads, smem, s>>>(mk, mv, mq, a);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

// ---------------------------------------------------------------- two query tiles per CTA
// head_dim 64: each softmax warpgroup owns one query tile of a pair (tiles 2m
// and 2m + 1 of one row and KV head), so the pair shares every K/V tile, no
// row statistics cross warpgroups, and one warpgroup's waits overlap the
// other's exponentials on the SMSP's MUFU.

struct PairItem {
  int i, hk, slot, base, len;
  int w0[2], w_end[2], kmax[2], n[2];
  int kmax_all, n_max;
};

__device__ __forceinline__ PairItem decode_pair(const Args& a, int e) {
  PairItem it;
  const int per = a.rows * a.kv_heads;
  const int n_pairs = (a.n_qtiles + 1) / 2;
  const int m = n_pairs - 1 - e / per;  // heaviest pair first
  const int rem = e % per;
  const int ri = rem / a.kv_heads;
  it.hk = rem % a.kv_heads;
  it.i = a.row_order ? a.row_order[ri] : ri;
  it.slot = a.slots[it.i];
  it.base = a.base_len[it.i];
  const bool ok = it.slot >= 0 && it.slot < a.num_slots && it.base >= 0;
  it.len = ok ? a.seq_len[it.slot] : 0;
  it.kmax_all = 0;
  it.n_max = 0;
#pragma unroll
  for (int k = 0; k < 2; ++k) {
    it.w0[k] = (2 * m + k) * a.tpt;
    it.w_end[k] = min(it.w0[k] + a.tpt, a.width);
    it.kmax[k] = min(it.base + it.w_end[k], it.len);
    it.n[k] = (ok && it.w_end[k] > it.w0[k] && it.base + it.w0[k] < it.len && it.kmax[k] > 0)
                  ? (it.kmax[k] + BKV - 1) / BKV
                  : 0;
    if (it.n[k] > 0) it.kmax_all = max(it.kmax_all, it.kmax[k]);
    it.n_max = max(it.n_max, it.n[k]);
  }
  return it;
}

// Warps 0..15 are four softmax warpgroups: warpgroup 2k + h handles query tile
// k's key columns 64h .. 64h + 63 (each thread 64 scores: no spills at the
// register cap of 18 warps, four softmax warps per SMSP); warp 16 TMA, warp 17
// MMA.
constexpr int kPairThreads = 18 * 32;
constexpr int kPairProducer = 16, kPairMma = 17;
constexpr int kPairSoftmax = 256;  // softmax threads per query tile

constexpr size_t pair_smem_bytes() {
  // align slack + Q (two buffers x two tiles) + ring + barriers + the column
  // halves' row exchange (2 tiles x 2 query tiles x 2 halves x 128 maxima,
  // 2 query tiles x 2 halves x 128 sums)
  return 1024 + (size_t)2 * 2 * BQ * 64 * 2 + (size_t)3 * 2 * BKV * 64 * 2 + 256 + (size_t)12 * BQ * 4;
}

__global__ void __launch_bounds__(kPairThreads, 1)
    prefill_pair_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                        const __grid_constant__ CUtensorMap tmq, Args a) {
  constexpr int HD = 64, S = 3;
  constexpr int kTileBytes = BKV * HD * 2;  // one of K or V (16 KB)
  constexpr int kQBytes = BQ * HD * 2;      // one query tile (16 KB)
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* q_s = smem;                      // [2 buffers][2 tiles][128 x 64] K-major
  uint8_t* ring = q_s + 4 * kQBytes;        // [S][K tile | V tile]
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + S * 2 * kTileBytes);
  uint64_t* empty = full + S;
  uint64_t* s_full = empty + S;     // [2] per query tile: its scores of a tile are in TMEM
  uint64_t* s_free = s_full + 2;    // [2] per query tile: they have been loaded (256 arrivals)
  uint64_t* p_full = s_free + 2;    // [2] per query tile: P written, output rescaled (256 arrivals)
  uint64_t* pv_done = p_full + 2;   // [2] per query tile: its O += P V retired
  uint64_t* q_full = pv_done + 2;   // [2] per Q buffer: the item's two Q tiles landed
  uint64_t* q_empty = q_full + 2;   // [2] per Q buffer: the item's score MMAs retired
  uint64_t* final_bar = q_empty + 2;
  uint64_t* pair_bar = final_bar + 1;  // [2 query tiles][4 lane quarters]: column halves' exchange (64)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(pair_bar + 8);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* issued = abort_flag + 1;
  int* issued_q = issued + 1;
  float* xmax = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(full) + 256);  // [2][2][2][128]
  float* xsum = xmax + 8 * BQ;                                                      // [2][2][128]
  volatile int* vabort = abort_flag;

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int k = 0; k < 2; ++k) {
      mbar_init(&s_full[k], 1);
      mbar_init(&s_free[k], kPairSoftmax);
      mbar_init(&p_full[k], kPairSoftmax);
      mbar_init(&pv_done[k], 1);
      mbar_init(&q_full[k], 1);
      mbar_init(&q_empty[k], 1);
    }
    mbar_init(final_bar, 1);
    for (int x = 0; x < 8; ++x) mbar_init(&pair_bar[x], 64);
    *abort_flag = 0;
    *issued = 0;
    *issued_q = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kPairMma) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int n_items = a.rows * a.kv_heads * ((a.n_qtiles + 1) / 2);

  if (warp == kPairProducer) {
    // ------------------------------------------------------------ producer
    const int bs = a.block_size, ppt = BKV / bs;
    int g = 0, nq = 0;
    bool run = true;
    for (int e = blockIdx.x; run && e < n_items; e += gridDim.x) {
      const PairItem it = decode_pair(a, e);
      if (it.n_max == 0) continue;
      if (lane == 0) {
        const int qb = nq & 1;
        if (!mbar_wait(&q_empty[qb], ((nq >> 1) & 1) ^ 1, vabort)) {
          run = false;
        } else {
          mbar_expect_tx(&q_full[qb], 2 * kQBytes);
          *issued_q = nq + 1;
          for (int k = 0; k < 2; ++k) {
            const int y = it.i * a.width + it.w0[k];
            for (int gq = 0; gq < a.group; ++gq)
              tma_load_2d(q_s + (qb * 2 + k) * kQBytes + gq * a.tpt * 128, &tmq, (it.hk * a.group + gq) * HD, y,
                          &q_full[qb]);
          }
        }
      }
      run = __shfl_sync(0xffffffffu, run ? 1 : 0, 0) != 0;
      if (!run) break;
      ++nq;
      auto page = [&](int j) -> int {
        if (lane >= ppt || j >= it.n_max) return -1;
        const int pi = j * ppt + lane;
        if (pi >= a.nblocks[it.slot] || pi >= a.max_blocks || pi * bs >= it.kmax_all) return -1;
        const int b = a.block_table[(int64_t)it.slot * a.max_blocks + pi];
        return (b >= 0 && b < a.num_blocks) ? b : -1;
      };
      int cur = page(0);
      for (int j = 0; j < it.n_max; ++j) {
        const int nxt = page(j + 1);
        const int s = g % S;
        int stop = 0;
        if (lane == 0) {
          if (!mbar_wait(&empty[s], ((g / S) & 1) ^ 1, vabort)) {
            stop = 1;
          } else {
            mbar_expect_tx(&full[s], 2 * kTileBytes);
            *issued = g + 1;
          }
        }
        stop = __shfl_sync(0xffffffffu, stop, 0);
        if (stop) {
          run = false;
          break;
        }
        uint8_t* kst = ring + s * 2 * kTileBytes;
        uint8_t* vst = kst + kTileBytes;
        for (int p = 0; p < ppt; ++p) {
          const int blk = __shfl_sync(0xffffffffu, cur, p);
          if (lane == 0) {
            const int y = blk >= 0 ? (blk * a.kv_heads + it.hk) * bs : a.oob_row;
            tma_load_2d(kst + p * bs * 128, &tmk, 0, y, &full[s]);
            tma_load_2d(vst + p * bs * 128, &tmv, 0, y, &full[s]);
          }
        }
        cur = nxt;
        ++g;
      }
    }
  } else if (warp == kPairMma) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      constexpr uint32_t idesc_s = instr_desc(BKV, 0);
      constexpr uint32_t idesc_o = instr_desc(HD, 1);
      int g = 0, items = 0;
      int gs[2] = {0, 0}, gp[2] = {0, 0};  // score / P V tiles issued per warpgroup
      bool run = true;
      for (int e = blockIdx.x; run && e < n_items; e += gridDim.x) {
        const PairItem it = decode_pair(a, e);
        if (it.n_max == 0) continue;
        const int qb = items & 1;
        if (!mbar_wait(&q_full[qb], (items >> 1) & 1, vabort)) break;
        tc_fence_after();
        int s_prev = 0;
        for (int j = 0; run && j <= it.n_max; ++j) {
          if (j < it.n_max) {
            const int s = g % S;
            if (!mbar_wait(&full[s], (g / S) & 1, vabort)) {
              run = false;
              break;
            }
            tc_fence_after();
            const uint32_t kb = su32(ring + s * 2 * kTileBytes);
            for (int k = 0; k < 2; ++k) {
              if (j >= it.n[k]) continue;
              // the warpgroup has loaded its previous scores out of this buffer
              if (gs[k] > 0 && !mbar_wait(&s_free[k], (gs[k] - 1) & 1, vabort)) {
                run = false;
                break;
              }
              tc_fence_after();
              const uint32_t qa = su32(q_s + (qb * 2 + k) * kQBytes);
#pragma unroll
              for (int kk = 0; kk < HD / 16; ++kk)
                mma_bf16(tmem + kColS + k * BKV, desc_kmajor(qa + kk * 32), desc_kmajor(kb + kk * 32), idesc_s,
                         kk > 0);
              mma_commit(&s_full[k]);
              ++gs[k];
            }
            if (!run) break;
            if (j + 1 == it.n_max) mma_commit(&q_empty[qb]);  // the item's last read of its Q tiles
          }
          if (j >= 1) {
            const uint32_t vb = su32(ring + s_prev * 2 * kTileBytes + kTileBytes);
            for (int k = 0; k < 2; ++k) {
              if (j - 1 >= it.n[k]) continue;
              if (!mbar_wait(&p_full[k], gp[k] & 1, vabort)) {
                run = false;
                break;
              }
              tc_fence_after();
              // one head_dim half: the atom stride field is unused (8-row-group stride)
#pragma unroll
              for (int kk = 0; kk < BKV / 16; ++kk)
                mma_bf16_ts(tmem + kColO + k * HD, tmem + kColP + k * (BKV / 2) + kk * 8,
                            desc_mnmajor(vb + kk * 16 * 128, 1024u), idesc_o, (j > 1 || kk > 0) ? 1u : 0u);
              mma_commit(&pv_done[k]);
              ++gp[k];
            }
            if (!run) break;
            mma_commit(&empty[s_prev]);
          }
          if (j < it.n_max) {
            s_prev = g % S;
            ++g;
          }
        }
        ++items;
      }
      mma_commit(final_bar);
    }
  } else {
    // ------------------------------------------------------------ softmax
    const int k = warp >> 3;            // query tile of the pair
    const int half = (warp >> 2) & 1;   // key columns 64 * half .. + 63, output columns 32 * half .. + 31
    const int q4 = warp & 3;
    const int r = 32 * q4 + lane;       // tile row = TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t)(32 * q4) << 16);
    const uint32_t s_col = kColS + k * BKV + half * (BKV / 2), o_col = kColO + k * HD + half * (HD / 2);
    const uint32_t p_col = kColP + k * (BKV / 2) + half * (BKV / 4);
    const int gq = r / a.tpt, wr = r % a.tpt;
    const float sl2 = a.scale_log2;
    constexpr int kCols = BKV / 2, kOCols = HD / 2;
    uint64_t* const xbar = &pair_bar[k * 4 + q4];
    int nx = 0;  // exchanges with the other column half so far (its barrier phase)
    auto exchange = [&]() -> bool {  // after this thread's arrive: wait for the partner's
      const bool ok = mbar_wait(xbar, nx & 1, vabort);
      ++nx;
      return __all_sync(0xffffffffu, ok);
    };
    int gk = 0;  // tiles of this query tile processed
    bool run = true;
    for (int e = blockIdx.x; run && e < n_items; e += gridDim.x) {
      const PairItem it = decode_pair(a, e);
      const int w = it.w0[k] + wr;
      const bool row_ok = gq < a.group && w < it.w_end[k];
      const int pos = it.base + w;
      const bool valid = row_ok && pos < it.len;
      const int h = it.hk * a.group + gq;
      __nv_bfloat16* orow = a.out + ((int64_t)it.i * a.width + w) * a.out_tok_stride + (int64_t)h * HD + half * kOCols;
      const int n = it.n[k];
      if (n == 0) {
        if (row_ok) {
#pragma unroll
          for (int c = 0; c < kOCols / 8; ++c) *reinterpret_cast<uint4*>(orow + c * 8) = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      const int lim = row_ok ? min(pos + 1, it.kmax[k]) : it.kmax[k];
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < n; ++j) {
        if (!__all_sync(0xffffffffu, mbar_wait(&s_full[k], gk & 1, vabort))) {
          run = false;
          break;
        }
        tc_fence_after();
        float sc[kCols];
        {
          uint32_t* u = reinterpret_cast<uint32_t*>(sc);
#pragma unroll
          for (int c = 0; c < kCols / 32; ++c) tmem_ld32(lane_base + s_col + c * 32, u + c * 32);
          tmem_wait_ld();
        }
        // the scores are in registers: the MMA may write the next ones
        tc_fence_before();
        mbar_arrive(&s_free[k]);
        const int key0 = j * BKV + half * kCols;
        if (key0 + kCols > lim) {
#pragma unroll
          for (int c = 0; c < kCols; ++c) sc[c] = key0 + c < lim ? sc[c] : -INFINITY;
        }
        float m4[4];
#pragma unroll
        for (int x = 0; x < 4; ++x) m4[x] = sc[x];
#pragma unroll
        for (int c = 4; c < kCols; ++c) m4[c & 3] = fmaxf(m4[c & 3], sc[c]);
        const float pm = fmaxf(fmaxf(m4[0], m4[1]), fmaxf(m4[2], m4[3]));
        float* xm = xmax + ((gk & 1) * 4 + k * 2) * BQ;
        xm[half * BQ + r] = pm;
        mbar_arrive(xbar);
        if (!exchange()) {
          run = false;
          break;
        }
        const float mx = fmaxf(pm, xm[(half ^ 1) * BQ + r]) * sl2;
        // the row's reference maximum moves only when it would grow by more
        // than 8 (exponents stay <= 2^8); the output is rescaled then.  Both
        // column halves see the same maximum, so they decide alike.
        float corr = 1.f;
        bool rescale = false;
        if (mx > m_used + 8.f) {
          if (m_used != -INFINITY) {
            corr = ex2(m_used - mx);
            rescale = j > 0;
          }
          m_used = mx;
        }
        const float msub = m_used == -INFINITY ? 0.f : m_used;
        float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < kCols; ++c) {
          sc[c] = ex2(fmaf(sc[c], sl2, -msub));
          s4[c & 3] += sc[c];
        }
        l = l * corr + ((s4[0] + s4[1]) + (s4[2] + s4[3]));
        // this query tile's previous P V has retired: its P and output are free
        if (gk > 0 && !__all_sync(0xffffffffu, mbar_wait(&pv_done[k], (gk - 1) & 1, vabort))) {
          run = false;
          break;
        }
        tc_fence_after();
        {
          // this half's 64 keys of P as bf16 pairs into TMEM (the PV MMA's A operand)
          uint32_t pk[kCols / 2];
#pragma unroll
          for (int c = 0; c < kCols / 2; ++c) pk[c] = pack_bf16(sc[2 * c], sc[2 * c + 1]);
          tmem_st32(lane_base + p_col, pk);
        }
        if (__any_sync(0xffffffffu, rescale)) {
          uint32_t o[32];
          tmem_ld32(lane_base + o_col, o);
          tmem_wait_ld();
#pragma unroll
          for (int x = 0; x < 32; ++x) o[x] = __float_as_uint(__uint_as_float(o[x]) * corr);
          tmem_st32(lane_base + o_col, o);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[k]);
        ++gk;
      }
      if (!run) break;
      // the item's output: O / l once the last P V has retired; the row's sum
      // is the two halves' partial sums (same reference maximum)
      xsum[(k * 2 + half) * BQ + r] = l;
      mbar_arrive(xbar);
      if (!exchange()) break;
      const float L = l + xsum[(k * 2 + (half ^ 1)) * BQ + r];
      if (!__all_sync(0xffffffffu, mbar_wait(&pv_done[k], (gk - 1) & 1, vabort))) break;
      tc_fence_after();
      const float inv = valid && L > 0.f ? 1.f / L : 0.f;
      uint32_t o[32];
      tmem_ld32(lane_base + o_col, o);
      tmem_wait_ld();
      if (row_ok) {
#pragma unroll
        for (int x = 0; x < 32; x += 8) {
          uint4 v;
          v.x = pack_bf16(__uint_as_float(o[x + 0]) * inv, __uint_as_float(o[x + 1]) * inv);
          v.y = pack_bf16(__uint_as_float(o[x + 2]) * inv, __uint_as_float(o[x + 3]) * inv);
          v.z = pack_bf16(__uint_as_float(o[x + 4]) * inv, __uint_as_float(o[x + 5]) * inv);
          v.w = pack_bf16(__uint_as_float(o[x + 6]) * inv, __uint_as_float(o[x + 7]) * inv);
          *reinterpret_cast<uint4*>(orow + x) = v;
        }
      }
      tc_fence_before();
    }
  }

  __syncthreads();
  if (*vabort) {
    if (tid == 0) atomicOr(a.status, PSE_STATUS_TIMEOUT);
    if (warp == kPairProducer && lane == 0) {
      const int n = *issued;
      for (int t = n > S ? n - S : 0; t < n; ++t) mbar_drain(&full[t % S], (t / S) & 1);
      const int nq = *issued_q;
      for (int t = nq > 2 ? nq - 2 : 0; t < nq; ++t) mbar_drain(&q_full[t & 1], (t >> 1) & 1);
    }
  }
  if (warp == kPairMma) {
    if (lane == 0) mbar_drain(final_bar, 0);
    __syncwarp();
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

int launch_pair(const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mq, const Args& a, cudaStream_t s) {
  constexpr size_t smem = pair_smem_bytes();
  static_assert(smem <= 227 * 1024, "shared memory budget");
  static const cudaError_t opt =
      cudaFuncSetAttribute(prefill_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (opt != cudaSuccess) return (int)opt;
  int sms = kNumSMs, dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long items = (long long)a.rows * a.kv_heads * ((a.n_qtiles + 1) / 2);
  const int grid = items < sms ? (int)items : sms;
  if (grid <= 0) return PSE_OK;
  prefill_pair_kernel<<<grid, kPairThreads, smem, s>>>(mk, mv, mq, a);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

}  // namespace pf

namespace tc {
int tensor_map(const void* pool, int num_blocks, int kv_heads, int bs, int hd, CUtensorMap* out);
}
namespace gemm {
int tensor_map(const void* ptr, int64_t rows, int64_t cols, int64_t ld, int box_rows, CUtensorMap* out);
}

// Calls this kernel serves: bf16 pools, head_dim 64 / 128, pages that tile a
// 128-key tile, 16-byte aligned query / output rows, GQA groups of 1..16 heads
// dividing 128 (a group head's Q box of 128 / group tokens stays 1 KB aligned),
// and at least 64 query rows per (row, KV head).
// head_dim 64 runs the two-query-tile kernel unless switched off (parity tests
// compare the two)
bool g_prefill_pair = true;

bool prefill_eligible(const pse_block_state& st, const pse_kv_layer& kv, const void* q, int64_t q_tok_stride,
                      const void* out, int64_t out_tok_stride, int q_heads, int width) {
  if (kv.dtype != PSE_BF16 || (kv.head_dim != 64 && kv.head_dim != 128)) return false;
  if (st.block_size < 16 || st.block_size > pf::BKV || pf::BKV % st.block_size != 0) return false;
  if (!st.seq_len) return false;
  const int group = q_heads / kv.kv_heads;
  if (group < 1 || group > 16 || pf::BQ % group != 0) return false;
  if (group * (long long)width < 64) return false;
  if ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(out)) & 15) return false;
  if ((q_tok_stride * 2) % 16 != 0 || (out_tok_stride * 2) % 16 != 0) return false;
  if ((reinterpret_cast<uintptr_t>(kv.k_pool) | reinterpret_cast<uintptr_t>(kv.v_pool)) & 15) return false;
  const long long rows = (long long)st.num_blocks * kv.kv_heads * st.block_size;
  if (rows + st.block_size >= (1ll << 31)) return false;
  return true;
}

int prefill_attention(const pse_block_state& st, const pse_kv_layer& kv, const void* q, int64_t q_tok_stride,
                      void* out, int64_t out_tok_stride, const int32_t* slots, const int32_t* base_len, int rows,
                      int width, int q_heads, float scale, const int32_t* row_order, cudaStream_t s) {
  pf::Args a;
  a.block_table = st.block_table;
  a.nblocks = st.nblocks;
  a.seq_len = st.seq_len;
  a.max_blocks = st.max_blocks;
  a.block_size = st.block_size;
  a.num_blocks = st.num_blocks;
  a.num_slots = st.num_slots;
  a.kv_heads = kv.kv_heads;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.out_tok_stride = out_tok_stride;
  a.slots = slots;
  a.base_len = base_len;
  a.row_order = row_order;
  a.rows = rows;
  a.width = width;
  a.q_heads = q_heads;
  a.group = q_heads / kv.kv_heads;
  a.tpt = pf::BQ / a.group;
  a.n_qtiles = ceil_div(width, a.tpt);
  const long long n_items = (long long)rows * kv.kv_heads * a.n_qtiles;
  if (n_items >= (1ll << 31)) return PSE_EINVAL;
  a.n_items = (int)n_items;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.status = st.status;
  a.oob_row = st.num_blocks * kv.kv_heads * st.block_size;
  CUtensorMap mk, mv;
  int rc = tc::tensor_map(kv.k_pool, st.num_blocks, kv.kv_heads, st.block_size, kv.head_dim, &mk);
  if (rc) return rc;
  rc = tc::tensor_map(kv.v_pool, st.num_blocks, kv.kv_heads, st.block_size, kv.head_dim, &mv);
  if (rc) return rc;
  // Q viewed as [rows * width tokens, q_heads * head_dim] with the caller's token stride
  CUtensorMap mq;
  rc = gemm::tensor_map(q, (int64_t)rows * width, (int64_t)q_heads * kv.head_dim, q_tok_stride, a.tpt, &mq);
  if (rc) return rc;
  if (kv.head_dim == 64) return g_prefill_pair ? pf::launch_pair(mk, mv, mq, a, s) : pf::launch<64>(mk, mv, mq, a, s);
  return pf::launch<128>(mk, mv, mq, a, s);
}

}  // namespace pse
