// Paged attention for bf16 pools on sm_100a: TMA page loads + tensor-core math.
//
// Same contract as the generic kernel in attention.cu (engine/model.py:99-116
// over the paged layout of engine/paged_cache.py:83-88), specialised for the
// shapes that carry the bandwidth: bf16 K/V, head_dim 64 or 128, block_size
// 16 / 32 / 64, up to 32 query rows (GQA group x width) per tile.
//
// CTA = 1 producer warp + 4 consumer warps, one (row, KV head, query tile,
// KV split).  The producer walks the row's block table and, for every page of
// a 64-token tile, issues 2-D TMA loads (cp.async.bulk.tensor, 128-byte
// swizzle) of the page's K and V boxes [block_size x 64 columns] into a
// 3-stage shared-memory ring, completing on an mbarrier with the transaction
// byte count.  Pages past the row's end are requested at an out-of-range row,
// so the TMA unit fills them with zeros and the byte count never changes.
// Consumers run S = Q K^T and O += P V with mma.sync m16n8k16 (bf16 in, fp32
// accumulate), fragments fetched with ldmatrix from the swizzled tiles (the
// swizzle makes every ldmatrix conflict-free), an exp2-domain online softmax
// per row, and release the stage through an "empty" mbarrier.  Warps split
// the tile's tokens (and, with 32 query rows, the two 16-row m-tiles); their
// partial (max, sum, O) are merged at the item's last tile, through that
// tile's own stage buffers, before the stage is released.
//
// Every mbarrier wait is bounded; on expiry the kernel latches
// PSE_STATUS_TIMEOUT in the cache status word and stops issuing work.

#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "tmap_cache.h"

namespace pse {
namespace tc {

#ifndef PSE_TC_CONSUMERS
#define PSE_TC_CONSUMERS 4
#endif
#ifndef PSE_TC_STAGES64
#define PSE_TC_STAGES64 3
#endif
#ifndef PSE_TC_STAGES128
#define PSE_TC_STAGES128 3
#endif
#ifndef PSE_TC_MINB64
#define PSE_TC_MINB64 4
#endif
#ifndef PSE_TC_MINB128
#define PSE_TC_MINB128 2
#endif

constexpr int kConsumers = PSE_TC_CONSUMERS;
static_assert(kConsumers % 2 == 0, "the item merge puts half the consumer warps' partials in each stage buffer");
constexpr int kThreads = (kConsumers + 1) * 32;
constexpr int kTile = 16 * kConsumers;  // tokens per pipeline stage (16 per consumer warp)
constexpr uint32_t kSpinLimit = 1u << 22;

// Ring depth: 3 x 16 KB stages for head_dim 64 (4 CTAs per SM), 3 x 32 KB for
// head_dim 128 (2 CTAs per SM): up to 192 KB of K/V in flight per SM.  HBM
// needs ~200+ KB in flight per SM to approach its peak (a 128 KB ring reached
// ~60% of it), so the ring takes nearly all of shared memory; the item merge
// reuses the last tile's stage instead of a buffer of its own.  The persistent
// CTAs never let the ring drain between work items.
__host__ __device__ constexpr int stages_for(int hd) { return hd == 64 ? PSE_TC_STAGES64 : PSE_TC_STAGES128; }

struct Args {
  const int32_t* block_table;
  const int32_t* nblocks;
  int max_blocks, block_size, num_blocks, num_slots;
  int kv_heads, head_dim;
  const __nv_bfloat16* q;
  int64_t q_tok_stride;
  __nv_bfloat16* out;
  int64_t out_tok_stride;
  const int32_t* slots;
  const int32_t* base_len;
  int rows, width, q_heads;
  float scale_log2;
  int split_tokens, n_splits, n_qtiles;
  float* ws;
  int32_t* status;
  int oob_row;  // first row index past the pool's 2-D view (zero-fill requests)
  int n_items;  // rows * kv_heads * n_qtiles * n_splits
  int* counter; // work counter (zeroed before the launch)
  const int32_t* row_order;  // rows in the order items are handed out (nullable: 0..rows-1)
  int self_reset;            // the last CTA zeroes counter[0..1] (counter[1] counts CTAs done)
  int tree_b, tree_d0;       // token-tree call (key_vis in common.cuh); tree_b == 0: causal
};

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

// Bounded wait for the phase of parity `parity` to complete.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i >= 32) __nanosleep(32);
  }
  return false;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(su32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(su32(bar))
      : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma16816(float* c, uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Byte offset of element (row r, column d) inside a [rows x HD] bf16 tile
// stored as HD/64 column halves of [rows x 128 B] with the 128-byte swizzle
// (16-byte chunk c of row r stored at chunk c ^ (r % 8)).
template <int HD>
__device__ __forceinline__ uint32_t sw_off(int rows, int r, int d) {
  return (uint32_t)(((d >> 6) * rows + r) * 128 + ((((d & 63) >> 3) ^ (r & 7)) << 4) + (d & 7) * 2);
}

// Page-major tile: tokens t = page * bs + row; each page holds HD/64 boxes.
template <int HD>
__device__ __forceinline__ uint32_t kv_off(int bs, int t, int d) {
  const int page = t / bs, r = t % bs;
  return (uint32_t)(((page * (HD / 64) + (d >> 6)) * bs + r) * 128 + ((((d & 63) >> 3) ^ (r & 7)) << 4) +
                    (d & 7) * 2);
}

// One work item = (row, KV head, query tile, KV split).
struct Item {
  int i, hk, split, slot, base, r0, nr, k_lo, k_hi, n_tiles;
};

template <int QROWS>
__device__ __forceinline__ Item decode_item(const Args& a, int e) {
  Item it;
  const int group = a.q_heads / a.kv_heads;
  const int qtile = e % a.n_qtiles;
  e /= a.n_qtiles;
  it.hk = e % a.kv_heads;
  e /= a.kv_heads;
  it.i = a.row_order ? a.row_order[e % a.rows] : e % a.rows;
  it.split = e / a.rows;
  it.slot = a.slots[it.i];
  it.base = a.base_len[it.i];
  it.r0 = qtile * QROWS;
  it.nr = min(QROWS, group * a.width - it.r0);
  const int w_last = (it.r0 + it.nr - 1) / group;
  it.k_lo = it.split * a.split_tokens;
  it.k_hi = min(it.k_lo + a.split_tokens, it.base + w_last + 1);
  const bool ok = it.nr > 0 && it.slot >= 0 && it.slot < a.num_slots && it.base >= 0;
  it.n_tiles = (ok && it.k_hi > it.k_lo) ? (it.k_hi - it.k_lo + kTile - 1) / kTile : 0;
  return it;
}

constexpr int kFirst = 1, kLast = 2, kEmpty = 4, kEnd = 8;

// TREE: a token-tree call (the key_vis rule); the causal instantiation
// compiles without any of it.
template <int HD, int MT, bool TREE>
__global__ void __launch_bounds__(kThreads, HD == 64 ? PSE_TC_MINB64 : PSE_TC_MINB128) attn_tc_kernel(const __grid_constant__ CUtensorMap tmk,
                                                          const __grid_constant__ CUtensorMap tmv, Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kStages = stages_for(HD);
  constexpr int kTileBytes = kTile * HD * 2;  // one of K or V for a stage
  constexpr int kQRows = 16 * MT;
  uint8_t* stage_k = smem;                          // [kStages][kTileBytes]
  uint8_t* stage_v = smem + kStages * kTileBytes;   // [kStages][kTileBytes]
  uint8_t* q_s = smem + 2 * kStages * kTileBytes;   // [kQRows x HD] swizzled
  float* mw = reinterpret_cast<float*>(q_s + kQRows * HD * 2);  // [kConsumers][16]
  float* lw = mw + kConsumers * 16;                               // [kConsumers][16]
  uint64_t* full = reinterpret_cast<uint64_t*>(lw + kConsumers * 16);
  uint64_t* empty = full + kStages;
  int* desc_item = reinterpret_cast<int*>(empty + kStages);
  int* desc_tile = desc_item + kStages;
  int* desc_flags = desc_tile + kStages;
  int* abort_flag = desc_flags + kStages;
  int* issued = abort_flag + 1;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int bs = a.block_size;
  const int group = a.q_heads / a.kv_heads;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kConsumers);
    }
    *abort_flag = 0;
    *issued = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  if (warp == kConsumers) {
    // ------------------------------------------------------------ producer
    // The whole warp walks the work items; lane 0 owns the barriers and issues
    // the TMA copies.  Block-table entries are read 32 pages per coalesced warp
    // load, one chunk ahead, and the next work item is claimed, decoded and its
    // first table chunk fetched while the current item's last chunk is being
    // issued, so no copy ever waits on a dependent global read.
    const unsigned FULL = 0xffffffffu;
    const int ppt = kTile / bs;  // pages per tile
    auto claim = [&]() -> int {
      int e = 0;
      if (lane == 0) e = atomicAdd(a.counter, 1);
      return __shfl_sync(FULL, e, 0);
    };
    auto page_block = [&](const Item& it, int j) -> int {  // j: page index within the item
      if (j >= it.n_tiles * ppt) return -1;
      const int pi = it.k_lo / bs + j;
      if (pi >= a.nblocks[it.slot] || pi * bs >= it.k_hi) return -1;
      const int blk = a.block_table[(int64_t)it.slot * a.max_blocks + pi];
      return (blk >= 0 && blk < a.num_blocks) ? blk : -1;
    };
    // lane 0: acquire stage s for tile t (bounded); returns false on timeout
    auto acquire = [&](int tt_global) -> bool {
      if (mbar_wait(&empty[tt_global % kStages], ((tt_global / kStages) & 1) ^ 1)) return true;
      atomicOr(a.status, PSE_STATUS_TIMEOUT);
      atomicExch(abort_flag, 1);
      return false;
    };
    int t = 0;
    int e = claim();
    Item it{};
    int cur = -1;
    if (e < a.n_items) {
      it = decode_item<kQRows>(a, e);
      cur = page_block(it, lane);
    }
    // Everything above reads data the kernels before the K/V append wrote; the
    // pages themselves may come from that append, which this launch is allowed
    // to overlap (programmatic dependent launch): wait for it to finish here.
    asm volatile("griddepcontrol.wait;" ::: "memory");
    bool run = true;
    while (run && e < a.n_items) {
      const int e_next = claim();
      Item it_next{};
      int cur_next = -1;
      bool next_ready = false;
      if (it.n_tiles == 0) {
        int stop = 0;
        if (lane == 0) {
          if (acquire(t)) {
            const int s = t % kStages;
            desc_item[s] = e;
            desc_tile[s] = 0;
            desc_flags[s] = kFirst | kLast | kEmpty;
            mbar_arrive(&full[s]);
          } else {
            stop = 1;
          }
        }
        if (__shfl_sync(FULL, stop, 0)) break;
        ++t;
      }
      const int n_pages = it.n_tiles * ppt;
      for (int c0 = 0; c0 < n_pages; c0 += 32) {
        int nxt;
        if (c0 + 32 < n_pages) {
          nxt = page_block(it, c0 + 32 + lane);
        } else {
          if (e_next < a.n_items) {
            it_next = decode_item<kQRows>(a, e_next);
            cur_next = page_block(it_next, lane);
          }
          next_ready = true;
          nxt = -1;
        }
        const int tiles_here = min(32 / ppt, it.n_tiles - c0 / ppt);
        for (int tl = 0; tl < tiles_here; ++tl) {
          const int tt = c0 / ppt + tl;
          int blks[kTile / 16];
#pragma unroll
          for (int p = 0; p < kTile / 16; ++p) blks[p] = __shfl_sync(FULL, cur, (tl * ppt + p) & 31);
          int stop = 0;
          if (lane == 0) {
            if (!acquire(t)) {
              stop = 1;
            } else {
              const int s = t % kStages;
              desc_item[s] = e;
              desc_tile[s] = tt;
              desc_flags[s] = (tt == 0 ? kFirst : 0) | (tt == it.n_tiles - 1 ? kLast : 0);
              *issued = t + 1;
              mbar_expect_tx(&full[s], 2 * kTileBytes);
#pragma unroll
              for (int p = 0; p < kTile / 16; ++p) {
                if (p < ppt) {
                  const int y = blks[p] >= 0 ? (blks[p] * a.kv_heads + it.hk) * bs : a.oob_row;
#pragma unroll
                  for (int c = 0; c < HD / 64; ++c) {
                    const int off = ((p * (HD / 64) + c) * bs) * 128;
                    tma_load_2d(stage_k + s * kTileBytes + off, &tmk, c * 64, y, &full[s]);
                    tma_load_2d(stage_v + s * kTileBytes + off, &tmv, c * 64, y, &full[s]);
                  }
                }
              }
            }
          }
          if (__shfl_sync(FULL, stop, 0)) {
            run = false;
            break;
          }
          ++t;
        }
        if (!run) break;
        cur = nxt;
      }
      if (!run) break;
      if (!next_ready && e_next < a.n_items) {
        it_next = decode_item<kQRows>(a, e_next);
        cur_next = page_block(it_next, lane);
      }
      e = e_next;
      it = it_next;
      cur = cur_next;
    }
    if (run && lane == 0) {
      if (acquire(t)) {
        desc_flags[t % kStages] = kEnd;
        mbar_arrive(&full[t % kStages]);
      }
    }
  } else {
    // ------------------------------------------------------------ consumers
    // Q (and the output rows) may belong to the kernel just before this launch
    asm volatile("griddepcontrol.wait;" ::: "memory");
    const int mt = warp % MT;                       // this warp's 16-row m-tile
    const int tok_base = (warp / MT) * (16 * MT);   // this warp's token slice of a tile
    const int gid = lane >> 2, tid4 = lane & 3;
    const int lm = lane >> 3, lj = lane & 7;
    // ldmatrix source offsets are fixed for the whole kernel (block size and
    // the warp's token slice never change): compute them once.
    uint32_t q_off[HD / 16], k_off[MT][HD / 16], v_off[MT][HD / 16];
#pragma unroll
    for (int kk = 0; kk < HD / 16; ++kk) {
      q_off[kk] = su32(q_s) + sw_off<HD>(kQRows, mt * 16 + (lm & 1) * 8 + lj, kk * 16 + (lm >> 1) * 8);
#pragma unroll
      for (int sub = 0; sub < MT; ++sub) {
        const int t0 = tok_base + sub * 16;
        k_off[sub][kk] = kv_off<HD>(bs, t0 + (lm >> 1) * 8 + lj, kk * 16 + (lm & 1) * 8);
        v_off[sub][kk] = kv_off<HD>(bs, t0 + (lm & 1) * 8 + lj, kk * 16 + (lm >> 1) * 8);
      }
    }
    float o[HD / 8][4];
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
    KeyVis vis0 = kNoKeys, vis1 = kNoKeys;
    int qpos_min = -1;
    Item it{};
    for (int t = 0;; ++t) {
      const int s = t % kStages;
      if (!mbar_wait(&full[s], (t / kStages) & 1)) {
        atomicOr(a.status, PSE_STATUS_TIMEOUT);
        atomicExch(abort_flag, 1);
        break;
      }
      const int flags = desc_flags[s];
      if (flags & kEnd) break;
      if (flags & kFirst) {
        it = decode_item<kQRows>(a, desc_item[s]);
        // every consumer warp is done with the previous item (its Q and merge area)
        asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32));
        if (!(flags & kEmpty)) {
          for (int e = tid; e < kQRows * (HD / 2); e += kConsumers * 32) {
            const int r = e / (HD / 2), d = (e % (HD / 2)) * 2;
            uint32_t v = 0;
            if (r < it.nr) {
              const int rr = it.r0 + r, w = rr / group, g = rr % group;
              v = *reinterpret_cast<const uint32_t*>(a.q + ((int64_t)it.i * a.width + w) * a.q_tok_stride +
                                                     (int64_t)(it.hk * group + g) * HD + d);
            }
            *reinterpret_cast<uint32_t*>(q_s + sw_off<HD>(kQRows, r, d)) = v;
          }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32));
#pragma unroll
        for (int n = 0; n < HD / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
        m0 = m1 = -INFINITY;
        l0 = l1 = 0.f;
        const int ra = mt * 16 + gid, rb = ra + 8;
        const int tb = TREE ? a.tree_b : 0;
        vis0 = ra < it.nr ? key_vis(it.base, (it.r0 + ra) / group, tb, a.tree_d0) : kNoKeys;
        vis1 = rb < it.nr ? key_vis(it.base, (it.r0 + rb) / group, tb, a.tree_d0) : kNoKeys;
        // smallest visibility limit over this m-tile's valid rows: tokens at or
        // below it are visible to every row of the tile
        const int nr_mt = min(16, it.nr - mt * 16);
        qpos_min = nr_mt > 0 ? key_vis(it.base, (it.r0 + mt * 16) / group, tb, a.tree_d0).lim : -1;
      }
      if (!(flags & kEmpty)) {
        const int tt = desc_tile[s];
        const uint32_t kb = su32(stage_k + s * kTileBytes), vb = su32(stage_v + s * kTileBytes);
#pragma unroll
        for (int sub = 0; sub < MT; ++sub) {
          const int tok_abs = it.k_lo + tt * kTile + tok_base + sub * 16;
          float sc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            uint32_t a0, a1, a2, a3, b0, b1, b2, b3;
            ldsm_x4(q_off[kk], a0, a1, a2, a3);
            ldsm_x4(kb + k_off[sub][kk], b0, b1, b2, b3);
            mma16816(sc[0], a0, a1, a2, a3, b0, b1);
            mma16816(sc[1], a0, a1, a2, a3, b2, b3);
          }
          // Masking only where the slice reaches past the row end or the causal
          // limit of some row; interior slices just scale.
          const bool interior = tok_abs + 15 < it.k_hi && tok_abs + 15 <= qpos_min;
          float mx0 = -INFINITY, mx1 = -INFINITY;
          if (interior) {
#pragma unroll
            for (int n = 0; n < 2; ++n) {
#pragma unroll
              for (int c = 0; c < 4; ++c) sc[n][c] *= a.scale_log2;
              mx0 = fmaxf(mx0, fmaxf(sc[n][0], sc[n][1]));
              mx1 = fmaxf(mx1, fmaxf(sc[n][2], sc[n][3]));
            }
          } else {
#pragma unroll
            for (int n = 0; n < 2; ++n) {
#pragma unroll
              for (int c = 0; c < 2; ++c) {
                const int tok = tok_abs + n * 8 + 2 * tid4 + c;
                const bool live = tok < it.k_hi;
                const int tb = TREE ? a.tree_b : 0;
                sc[n][c] = (live && key_visible(vis0, tok, tb)) ? sc[n][c] * a.scale_log2 : -INFINITY;
                sc[n][2 + c] = (live && key_visible(vis1, tok, tb)) ? sc[n][2 + c] * a.scale_log2 : -INFINITY;
                mx0 = fmaxf(mx0, sc[n][c]);
                mx1 = fmaxf(mx1, sc[n][2 + c]);
              }
            }
          }
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
          mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
          mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
          const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
          const float ms0 = mn0 == -INFINITY ? 0.f : mn0, ms1 = mn1 == -INFINITY ? 0.f : mn1;
          // rescale the running output only when some row's maximum moved
          if (__any_sync(0xffffffffu, mn0 != m0 || mn1 != m1)) {
            const float c0 = exp2f(m0 - ms0), c1 = exp2f(m1 - ms1);
            l0 *= c0;
            l1 *= c1;
#pragma unroll
            for (int n = 0; n < HD / 8; ++n) {
              o[n][0] *= c0;
              o[n][1] *= c0;
              o[n][2] *= c1;
              o[n][3] *= c1;
            }
          }
          m0 = mn0;
          m1 = mn1;
          float p[2][4];
#pragma unroll
          for (int n = 0; n < 2; ++n) {
            p[n][0] = exp2f(sc[n][0] - ms0);
            p[n][1] = exp2f(sc[n][1] - ms0);
            p[n][2] = exp2f(sc[n][2] - ms1);
            p[n][3] = exp2f(sc[n][3] - ms1);
          }
          l0 += p[0][0] + p[0][1] + p[1][0] + p[1][1];
          l1 += p[0][2] + p[0][3] + p[1][2] + p[1][3];
          const uint32_t pa0 = pack_bf16(p[0][0], p[0][1]), pa1 = pack_bf16(p[0][2], p[0][3]);
          const uint32_t pa2 = pack_bf16(p[1][0], p[1][1]), pa3 = pack_bf16(p[1][2], p[1][3]);
#pragma unroll
          for (int n2 = 0; n2 < HD / 16; ++n2) {
            uint32_t b0, b1, b2, b3;
            ldsm_x4_t(vb + v_off[sub][n2], b0, b1, b2, b3);
            mma16816(o[2 * n2], pa0, pa1, pa2, pa3, b0, b1);
            mma16816(o[2 * n2 + 1], pa0, pa1, pa2, pa3, b2, b3);
          }
        }
      }
      __syncwarp();
      if (!(flags & kLast)) {
        if (lane == 0) mbar_arrive(&empty[s]);
      } else {
        // Merge the warps' partial (max, sum, O) of this item and write it out.
        // The partial O go through this tile's own stage buffers (K and V, two
        // warps each), which stay with the consumers until the merge is done.
        float L0 = l0 + __shfl_xor_sync(0xffffffffu, l0, 1);
        L0 += __shfl_xor_sync(0xffffffffu, L0, 2);
        float L1 = l1 + __shfl_xor_sync(0xffffffffu, l1, 1);
        L1 += __shfl_xor_sync(0xffffffffu, L1, 2);
        constexpr int kHalf = kConsumers / 2;  // warps per stage buffer
        float* const ow_k = reinterpret_cast<float*>(stage_k + s * kTileBytes);
        float* const ow_v = reinterpret_cast<float*>(stage_v + s * kTileBytes);
        auto ow_at = [&](int w2, int r) -> float* {
          return (w2 < kHalf ? ow_k : ow_v) + ((w2 % kHalf) * 16 + r) * HD;
        };
        // every consumer warp is done with this stage's K / V and with the previous item's merge
        asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32));
        if (tid4 == 0) {
          mw[warp * 16 + gid] = m0;
          mw[warp * 16 + gid + 8] = m1;
          lw[warp * 16 + gid] = L0;
          lw[warp * 16 + gid + 8] = L1;
        }
        float* const own0 = ow_at(warp, gid);
        float* const own1 = ow_at(warp, gid + 8);
#pragma unroll
        for (int n = 0; n < HD / 8; ++n) {
          const int d = n * 8 + 2 * tid4;
          *reinterpret_cast<float2*>(own0 + d) = make_float2(o[n][0], o[n][1]);
          *reinterpret_cast<float2*>(own1 + d) = make_float2(o[n][2], o[n][3]);
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kConsumers * 32));
        for (int e = tid; e < it.nr * HD; e += kConsumers * 32) {
          const int r = e / HD, d = e % HD;
          const int mtr = r / 16, rl = r % 16;
          float M = -INFINITY;
          for (int w2 = mtr; w2 < kConsumers; w2 += MT) M = fmaxf(M, mw[w2 * 16 + rl]);
          float L = 0.f, acc = 0.f;
          for (int w2 = mtr; w2 < kConsumers; w2 += MT) {
            const float f = M == -INFINITY ? 0.f : exp2f(mw[w2 * 16 + rl] - M);
            L += lw[w2 * 16 + rl] * f;
            acc += ow_at(w2, rl)[d] * f;
          }
          const int rr = it.r0 + r, w = rr / group, g = rr % group, h = it.hk * group + g;
          const int64_t tokrow = (int64_t)it.i * a.width + w;
          if (a.n_splits == 1) {
            a.out[tokrow * a.out_tok_stride + (int64_t)h * HD + d] = __float2bfloat16_rn(L > 0.f ? acc / L : 0.f);
          } else {
            float* ws = a.ws + (((int64_t)it.split * a.rows * a.width + tokrow) * a.q_heads + h) * (HD + 2);
            ws[d] = acc;
            if (d == 0) {
              ws[HD] = M == -INFINITY ? -INFINITY : M * 0.69314718055994531f;  // natural-log units
              ws[HD + 1] = L;
            }
          }
        }
        // the merge wrote the stage with generic-proxy stores: order them before
        // the producer's next TMA write into it, then release the stage
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
      }
    }
  }
  __syncthreads();
  // With self_reset the work counter is left zero for the next call: the
  // last CTA to finish (every CTA has stopped claiming by then) zeroes it.
  if (a.self_reset && tid == 0) {
    __threadfence();
    if (atomicAdd(a.counter + 1, 1) == (int)gridDim.x - 1) {
      a.counter[0] = 0;
      a.counter[1] = 0;
    }
  }
  // Error path only: before the CTA's shared memory is released, wait (bounded)
  // for the copies of the last tiles the producer issued.
  if (tid == kConsumers * 32 && *reinterpret_cast<volatile int*>(abort_flag)) {
    const int n = *issued;
    for (int t = n > kStages ? n - kStages : 0; t < n; ++t) mbar_wait(&full[t % kStages], (t / kStages) & 1);
  }
}

// ---------------------------------------------------------------- host side
TmapCache g_maps;

// 2-D view of one layer's pool: rows = num_blocks * kv_heads * block_size,
// columns = head_dim; box = [block_size rows x 64 columns], 128-byte swizzle.
int tensor_map(const void* pool, int num_blocks, int kv_heads, int bs, int hd, CUtensorMap* out) {
  return g_maps.get(pool, (uint64_t)hd, (uint64_t)num_blocks * kv_heads * bs, (uint64_t)hd * 2, 64u, (uint32_t)bs,
                    PSE_EINVAL, out);
}

template <int HD>
constexpr size_t smem_bytes(int mt) {
  return 1024 + 2 * stages_for(HD) * (size_t)kTile * HD * 2 + (size_t)16 * mt * HD * 2 +
         (size_t)(2 * kConsumers * 16) * 4 + 2 * stages_for(HD) * 8 + 3 * stages_for(HD) * 4 + 16;
}

// Persistent launch: as many CTAs as fit on the GPU at once (never more than
// work items); each pulls items from the work counter until it runs dry.
template <int HD, int MT, bool TREE>
int launch(const CUtensorMap& mk, const CUtensorMap& mv, const Args& a, cudaStream_t s) {
  auto kern = attn_tc_kernel<HD, MT, TREE>;
  constexpr size_t smem = smem_bytes<HD>(MT);
  static_assert(smem <= 227 * 1024, "shared memory budget");
  static const cudaError_t opt = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (opt != cudaSuccess) return (int)opt;
  static int per_sm = 0;
  if (per_sm == 0) {
    int n = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreads, smem);
    if (e != cudaSuccess) return (int)e;
    per_sm = n > 0 ? n : 1;
  }
  int sms = kNumSMs;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int grid = a.n_items < per_sm * sms ? a.n_items : per_sm * sms;
  if (!a.self_reset) {
    cudaError_t e = cudaMemsetAsync(a.counter, 0, sizeof(int), s);
    if (e != cudaSuccess) return (int)e;
  }
  // Programmatic dependent launch: the CTAs may start (and run their
  // prologue) while the preceding kernel -- the K/V append, which signals
  // early -- finishes; the producer waits for it before its first page copy.
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.gridDim = dim3((unsigned)grid, 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t le = cudaLaunchKernelEx(&cfg, kern, mk, mv, a);
  if (le != cudaSuccess) return (int)le;
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

}  // namespace tc

bool tc_eligible(const pse_block_state& st, const pse_kv_layer& kv, int q_heads, int width) {
  if (kv.dtype != PSE_BF16) return false;
  if (kv.head_dim != 64 && kv.head_dim != 128) return false;
  if (st.block_size != 16 && st.block_size != 32 && st.block_size != 64) return false;
  if ((reinterpret_cast<uintptr_t>(kv.k_pool) | reinterpret_cast<uintptr_t>(kv.v_pool)) & 15) return false;
  const long long rows = (long long)st.num_blocks * kv.kv_heads * st.block_size;
  if (rows + st.block_size >= (1ll << 31)) return false;
  (void)q_heads;
  (void)width;
  return true;
}

int tc_attention(const pse_block_state& st, const pse_kv_layer& kv, const void* q, int64_t q_tok_stride, void* out,
                 int64_t out_tok_stride, const int32_t* slots, const int32_t* base_len, int rows, int width,
                 int q_heads, float scale, int split_tokens, int n_splits, void* ws, int* counter,
                 const int32_t* row_order, bool self_reset, int tree_b, int tree_d0, cudaStream_t s) {
  const int n_qrows = (q_heads / kv.kv_heads) * width;
  const int MT = n_qrows <= 16 ? 1 : 2;
  tc::Args a;
  a.block_table = st.block_table;
  a.nblocks = st.nblocks;
  a.max_blocks = st.max_blocks;
  a.block_size = st.block_size;
  a.num_blocks = st.num_blocks;
  a.num_slots = st.num_slots;
  a.kv_heads = kv.kv_heads;
  a.head_dim = kv.head_dim;
  a.q = reinterpret_cast<const __nv_bfloat16*>(q);
  a.q_tok_stride = q_tok_stride;
  a.out = reinterpret_cast<__nv_bfloat16*>(out);
  a.out_tok_stride = out_tok_stride;
  a.slots = slots;
  a.base_len = base_len;
  a.rows = rows;
  a.width = width;
  a.q_heads = q_heads;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.split_tokens = split_tokens;
  a.n_splits = n_splits;
  a.n_qtiles = ceil_div(n_qrows, 16 * MT);
  a.ws = reinterpret_cast<float*>(ws);
  a.status = st.status;
  a.oob_row = st.num_blocks * kv.kv_heads * st.block_size;
  a.n_items = rows * kv.kv_heads * a.n_qtiles * n_splits;
  a.counter = counter;
  a.self_reset = self_reset ? 1 : 0;
  a.row_order = row_order;
  a.tree_b = tree_b;
  a.tree_d0 = tree_d0;
  if (!counter) return PSE_EINVAL;
  CUtensorMap mk, mv;
  int rc = tc::tensor_map(kv.k_pool, st.num_blocks, kv.kv_heads, st.block_size, kv.head_dim, &mk);
  if (rc) return rc;
  rc = tc::tensor_map(kv.v_pool, st.num_blocks, kv.kv_heads, st.block_size, kv.head_dim, &mv);
  if (rc) return rc;
  if (tree_b > 0) {
    if (kv.head_dim == 64)
      return MT == 1 ? tc::launch<64, 1, true>(mk, mv, a, s) : tc::launch<64, 2, true>(mk, mv, a, s);
    return MT == 1 ? tc::launch<128, 1, true>(mk, mv, a, s) : tc::launch<128, 2, true>(mk, mv, a, s);
  }
  if (kv.head_dim == 64) return MT == 1 ? tc::launch<64, 1, false>(mk, mv, a, s) : tc::launch<64, 2, false>(mk, mv, a, s);
  return MT == 1 ? tc::launch<128, 1, false>(mk, mv, a, s) : tc::launch<128, 2, false>(mk, mv, a, s);
}

}  // namespace pse
