// Paged attention for wide calls (prompt prefill) on the 5th-generation tensor
// cores, sm_100a.
//
// Same contract as pse_paged_attention (engine/model.py:99-116 over the paged
// layout of engine/paged_cache.py:83-88) for calls with many query rows per
// (row, KV head): the K/V of a prompt is re-read by every query tile from L2,
// so these calls are bound by math and by the softmax, not by HBM.
//
// Work item = (row, KV head, 128-query-row tile); the 128 query rows are the
// GQA group's heads over 128 / group consecutive tokens, head-major.
// Persistent CTAs take items round-robin, heaviest (last query tile) first.
// Per CTA:
//   warp 4       TMA producer: loads each item's Q tile into one of two
//                buffers ahead of use, walks the row's block table and copies
//                the K and V pages of each 128-key tile into a shared-memory
//                ring (128-byte swizzle; each head_dim half of the 128 keys is
//                one 16 KB K-major block), completing on mbarriers;
//   warp 5       allocates 512 TMEM columns and issues tcgen05.mma from one
//                thread: S = Q K^T (M 128, N 128, K 16) into one of two TMEM
//                score buffers, then O += P V (M 128, N head_dim, K 16) into
//                the TMEM output accumulator with V as an MN-major operand;
//                tcgen05.commit hands each result to the next stage;
//   warps 0..3   one thread per query row (its TMEM lane): tcgen05.ld of the
//                row's 128 scores, causal mask, exp2 online softmax (max and
//                sum over 8 independent chains, ex2.approx), P as bf16
//                into shared memory for the second MMA, rescale of the row's
//                TMEM output when its running maximum grows by more than 2^8,
//                and at the item's end O / l to global memory.
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
constexpr int kProducerWarp = 4, kMmaWarp = 5;  // warps 0..3: softmax
constexpr int kThreads = 6 * 32;
constexpr uint32_t kSpinLimit = 1u << 22;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kColS = 0;    // score buffers at columns 0 and 128
constexpr uint32_t kColO = 256;  // output accumulator
constexpr int kHalfBytes = BKV * 128;  // one 64-column half of a 128-row tile (16 KB)

template <int HD>
__host__ __device__ constexpr int n_stages() { return HD == 64 ? 3 : 2; }

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
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Byte offset of 16-byte chunk c (8 bf16 columns) of row r in a K-major
// 128-row operand made of 64-column halves (16 KB each), 128-byte swizzle.
__device__ __forceinline__ uint32_t chunk_off(int r, int c) {
  return (uint32_t)((c >> 3) * kHalfBytes + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int HD>
constexpr size_t smem_bytes() {
  // align slack + Q (two buffers) + P + ring (K and V per stage) + barriers
  return 1024 + (size_t)2 * BQ * HD * 2 + (size_t)BQ * BKV * 2 + (size_t)n_stages<HD>() * 2 * BKV * HD * 2 + 256;
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
  uint8_t* q_s = smem;                        // [2][128 x HD] K-major
  uint8_t* p_s = q_s + 2 * kQBytes;           // [128 x 128] K-major
  uint8_t* ring = p_s + BQ * BKV * 2;         // [S][K tile | V tile]
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + S * 2 * kTileBytes);
  uint64_t* empty = full + S;
  uint64_t* s_full = empty + S;     // [2] scores of a tile ready (one per score buffer)
  uint64_t* q_full = s_full + 2;    // [2] an item's Q landed (one per Q buffer)
  uint64_t* q_empty = q_full + 2;   // [2] an item's score MMAs retired: its Q buffer is free
  uint64_t* p_full = q_empty + 2;   // P written, output rescaled (128 arrivals)
  uint64_t* pv_done = p_full + 1;   // O += P V of a tile retired
  uint64_t* final_bar = pv_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(final_bar + 1);
  int* abort_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* issued = abort_flag + 1;   // K/V tiles whose copies the producer issued
  int* issued_q = issued + 1;     // Q tiles whose copies the producer issued
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
    mbar_init(p_full, BQ);
    mbar_init(pv_done, 1);
    mbar_init(final_bar, 1);
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
        const int qb = nq & 1;
        if (!mbar_wait(&q_empty[qb], ((nq >> 1) & 1) ^ 1, vabort)) {
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
      const uint32_t p_base = su32(p_s);
      int g = 0, items = 0;
      bool run = true;
      for (int e = blockIdx.x; run && e < a.n_items; e += gridDim.x) {
        const Item it = decode(a, e);
        if (it.n_tiles == 0) continue;
        const int qb = items & 1;
        if (!mbar_wait(&q_full[qb], (items >> 1) & 1, vabort)) break;
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
            for (int kk = 0; kk < BKV / 16; ++kk) {
              const uint32_t poff = (uint32_t)((kk >> 2) * kHalfBytes + (kk & 3) * 32);
              mma_bf16(tmem + kColO, desc_kmajor(p_base + poff), desc_mnmajor(vb + kk * 16 * 128, kVAtomStride),
                       idesc_o, (j > 1 || kk > 0) ? 1u : 0u);
            }
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
    const int r = tid;  // tile row = TMEM lane
    const uint32_t lane_base = tmem + ((uint32_t)(32 * warp) << 16);
    const int gq = r / a.tpt, wr = r % a.tpt;
    const float sl2 = a.scale_log2;
    int g = 0;
    bool run = true;
    for (int e = blockIdx.x; run && e < a.n_items; e += gridDim.x) {
      const Item it = decode(a, e);
      const int w = it.w0 + wr;
      const bool row_ok = gq < a.group && w < it.w_end;
      const int pos = it.base + w;
      const bool valid = row_ok && pos < it.len;
      const int h = it.hk * a.group + gq;
      __nv_bfloat16* orow = a.out + ((int64_t)it.i * a.width + w) * a.out_tok_stride + (int64_t)h * HD;
      if (it.n_tiles == 0) {
        if (row_ok) {
#pragma unroll
          for (int c = 0; c < HD / 8; ++c) *reinterpret_cast<uint4*>(orow + c * 8) = make_uint4(0, 0, 0, 0);
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
        float sc[BKV];
        {
          uint32_t* u = reinterpret_cast<uint32_t*>(sc);
          const uint32_t col = kColS + (uint32_t)(g & 1) * BKV;
#pragma unroll
          for (int c = 0; c < BKV / 32; ++c) tmem_ld32(lane_base + col + c * 32, u + c * 32);
          tmem_wait_ld();
        }
        const int key0 = j * BKV;
        if (key0 + BKV > lim) {
#pragma unroll
          for (int c = 0; c < BKV; ++c) sc[c] = key0 + c < lim ? sc[c] : -INFINITY;
        }
        // maximum of the raw scores (8 independent chains)
        float m8[8];
#pragma unroll
        for (int x = 0; x < 8; ++x) m8[x] = sc[x];
#pragma unroll
        for (int c = 8; c < BKV; ++c) m8[c & 7] = fmaxf(m8[c & 7], sc[c]);
        const float mx = fmaxf(fmaxf(fmaxf(m8[0], m8[1]), fmaxf(m8[2], m8[3])),
                               fmaxf(fmaxf(m8[4], m8[5]), fmaxf(m8[6], m8[7]))) * sl2;
        // the row's reference maximum moves only when it would grow by more
        // than 8 (exponents stay <= 2^8); the output is rescaled then
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
        float s8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int c = 0; c < BKV; ++c) {
          sc[c] = ex2(fmaf(sc[c], sl2, -msub));
          s8[c & 7] += sc[c];
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
          for (int c = 0; c < HD / 32; ++c) {
            uint32_t o[32];
            tmem_ld32(lane_base + kColO + c * 32, o);
            tmem_wait_ld();
#pragma unroll
            for (int x = 0; x < 32; ++x) o[x] = __float_as_uint(__uint_as_float(o[x]) * corr);
            tmem_st32(lane_base + kColO + c * 32, o);
          }
          tmem_wait_st();
        }
#pragma unroll
        for (int c = 0; c < BKV / 8; ++c) {
          uint4 v;
          v.x = pack_bf16(sc[8 * c + 0], sc[8 * c + 1]);
          v.y = pack_bf16(sc[8 * c + 2], sc[8 * c + 3]);
          v.z = pack_bf16(sc[8 * c + 4], sc[8 * c + 5]);
          v.w = pack_bf16(sc[8 * c + 6], sc[8 * c + 7]);
          *reinterpret_cast<uint4*>(p_s + chunk_off(r, c)) = v;
        }
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(p_full);
        ++g;
      }
      if (!run) break;
      // the item's output: O / l once the last P V has retired
      if (!__all_sync(0xffffffffu, mbar_wait(pv_done, (g - 1) & 1, vabort))) break;
      tc_fence_after();
      const float inv = valid && l > 0.f ? 1.f / l : 0.f;
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(lane_base + kColO + c * 32, o);
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
      for (int t = nq > 2 ? nq - 2 : 0; t < nq; ++t) mbar_drain(&q_full[t & 1], (t >> 1) & 1);
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
  return kv.head_dim == 64 ? pf::launch<64>(mk, mv, mq, a, s) : pf::launch<128>(mk, mv, mq, a, s);
}

}  // namespace pse
