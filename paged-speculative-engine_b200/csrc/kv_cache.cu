// Device block pool: free list, per-row block tables, KV append and gather.
//
// The free list is the reference's LIFO stack (engine/paged_cache.py:32-56)
// kept as an array plus a top index in device memory.  A batched call over
// many rows reproduces the reference's sequential per-row order exactly: row
// i's pops / pushes start at the exclusive prefix sum of the earlier rows'
// counts (single CTA, chunks of blockDim rows, block-wide scans).

#include <cstdio>

#include "common.cuh"

namespace pse {
namespace {

constexpr int kScanThreads = 1024;

__global__ void block_init_kernel(pse_block_state st) {
  const int64_t tid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = tid; i < st.num_blocks; i += stride) {
    st.free_stack[i] = (int32_t)i;
    st.block_free[i] = 1;
  }
  const int64_t table_n = (int64_t)st.num_slots * st.max_blocks;
  for (int64_t i = tid; i < table_n; i += stride) st.block_table[i] = -1;
  for (int64_t i = tid; i < st.num_slots; i += stride) {
    st.seq_len[i] = 0;
    st.nblocks[i] = 0;
  }
  if (tid == 0) {
    *st.free_top = st.num_blocks;
    *st.status = 0;
  }
}

__global__ void block_alloc_one_kernel(pse_block_state st, int32_t* out_id) {
  if (*st.status != 0) {
    *out_id = -1;
    return;
  }
  int top = *st.free_top;
  if (top <= 0) {
    *out_id = -1;
    atomicOr(st.status, PSE_STATUS_OOM);
    return;
  }
  int blk = st.free_stack[top - 1];
  st.block_free[blk] = 0;
  *st.free_top = top - 1;
  *out_id = blk;
}

__global__ void block_free_one_kernel(pse_block_state st, const int32_t* block_id) {
  if (*st.status != 0) return;
  int blk = *block_id;
  if (blk < 0 || blk >= st.num_blocks) {
    atomicOr(st.status, PSE_STATUS_BAD_BLOCK);
    return;
  }
  if (st.block_free[blk]) {
    atomicOr(st.status, PSE_STATUS_DOUBLE_FREE);
    return;
  }
  int top = *st.free_top;
  st.free_stack[top] = blk;
  st.block_free[blk] = 1;
  *st.free_top = top + 1;
}

// engine/paged_cache.py:116-130 for every row of one forward, rows in order.
__global__ void __launch_bounds__(kScanThreads) reserve_kernel(pse_block_state st, const int32_t* slots, int rows,
                                                              int width, const int32_t* widths, int32_t* base_len) {
  __shared__ int scan_tmp[33];
  const int tid = threadIdx.x;
  const bool latched = *st.status != 0;
  // Pass 1: lengths before the call, and capacity checks that must leave the
  // state untouched (slot range, table width).
  int bad = 0;
  for (int i = tid; i < rows; i += blockDim.x) {
    int slot = slots[i];
    if (slot < 0 || slot >= st.num_slots) {
      bad |= PSE_STATUS_BAD_BLOCK;
      base_len[i] = 0;
      continue;
    }
    int len = st.seq_len[slot];
    base_len[i] = len;
    const int w = widths ? widths[i] : width;
    if (w < 0)
      bad |= PSE_STATUS_BAD_BLOCK;
    else if (blocks_for(len + w, st.block_size) > st.max_blocks)
      bad |= PSE_STATUS_TABLE_OVERFLOW;
  }
  bad = __syncthreads_or(bad) ? 1 : 0;
  if (bad || latched) {
    if (bad && tid == 0) {
      // Record which kind (recomputed by one thread; rare path).
      int bits = 0;
      for (int i = 0; i < rows; ++i) {
        int slot = slots[i];
        if (slot < 0 || slot >= st.num_slots) {
          bits |= PSE_STATUS_BAD_BLOCK;
          continue;
        }
        const int w = widths ? widths[i] : width;
        if (w < 0)
          bits |= PSE_STATUS_BAD_BLOCK;
        else if (blocks_for(st.seq_len[slot] + w, st.block_size) > st.max_blocks)
          bits |= PSE_STATUS_TABLE_OVERFLOW;
      }
      atomicOr(st.status, bits);
    }
    return;
  }
  const int top = *st.free_top;
  int running = 0;
  int oom = 0;
  for (int c0 = 0; c0 < rows; c0 += blockDim.x) {
    const int i = c0 + tid;
    int slot = 0, len = 0, nb = 0, need = 0, w = 0;
    if (i < rows) {
      slot = slots[i];
      len = base_len[i];
      nb = st.nblocks[slot];
      w = widths ? widths[i] : width;
      need = max(blocks_for(len + w, st.block_size) - nb, 0);
    }
    int total = 0;
    const int off = block_exclusive_scan(need, scan_tmp, &total) + running;
    if (i < rows) {
      const int got = min(max(top - off, 0), need);
      int32_t* row = st.block_table + (int64_t)slot * st.max_blocks;
      for (int m = 0; m < got; ++m) {
        const int blk = st.free_stack[top - 1 - (off + m)];
        row[nb + m] = blk;
        st.block_free[blk] = 0;
      }
      st.nblocks[slot] = nb + got;
      if (off + need <= top)
        st.seq_len[slot] = len + w;
      else
        oom = 1;
    }
    running += total;
  }
  oom = __syncthreads_or(oom);
  if (tid == 0) {
    *st.free_top = top - min(running, top);
    if (oom) atomicOr(st.status, PSE_STATUS_OOM);
  }
}

// engine/paged_cache.py:140-154 (forward == false) and :156-160 (release:
// forward == true, every block, lengths to zero), rows in call order.
__global__ void __launch_bounds__(kScanThreads) free_rows_kernel(pse_block_state st, const int32_t* slots, int rows,
                                                                const int32_t* new_len, const int32_t* base_len,
                                                                const int32_t* accepted, int release) {
  __shared__ int scan_tmp[33];
  __shared__ int first_bad;
  const int tid = threadIdx.x;
  if (*st.status != 0) return;
  if (tid == 0) first_bad = rows;
  __syncthreads();
  // The reference raises at the first offending row; rows after it are untouched.
  for (int i = tid; i < rows; i += blockDim.x) {
    int slot = slots[i];
    bool badrow = slot < 0 || slot >= st.num_slots;
    if (!badrow && !release) {
      int n = new_len ? new_len[i] : base_len[i] + accepted[i];
      badrow = n < 0 || n > st.seq_len[slot];
    }
    if (badrow) atomicMin(&first_bad, i);
  }
  __syncthreads();
  const int limit = first_bad;
  const int top = *st.free_top;
  int running = 0;
  int flags = 0;
  for (int c0 = 0; c0 < limit; c0 += blockDim.x) {
    const int i = c0 + tid;
    int slot = 0, nb = 0, f = 0, n = 0;
    if (i < limit) {
      slot = slots[i];
      nb = st.nblocks[slot];
      n = release ? 0 : (new_len ? new_len[i] : base_len[i] + accepted[i]);
      f = max(nb - blocks_for(n, st.block_size), 0);
    }
    int total = 0;
    const int off = block_exclusive_scan(f, scan_tmp, &total) + running;
    if (i < limit) {
      int32_t* row = st.block_table + (int64_t)slot * st.max_blocks;
      for (int m = 0; m < f; ++m) {
        const int idx = release ? m : nb - 1 - m;
        const int blk = row[idx];
        row[idx] = -1;
        const int pos = top + off + m;
        if (blk < 0 || blk >= st.num_blocks || pos >= st.num_blocks) {
          flags |= PSE_STATUS_BAD_BLOCK;
          continue;
        }
        if (st.block_free[blk]) flags |= PSE_STATUS_DOUBLE_FREE;
        st.block_free[blk] = 1;
        st.free_stack[pos] = blk;
      }
      st.nblocks[slot] = nb - f;
      st.seq_len[slot] = n;
    }
    running += total;
  }
  if (flags) atomicOr(st.status, flags);
  __syncthreads();
  if (tid == 0) {
    *st.free_top = min(top + running, st.num_blocks);
    if (limit < rows) atomicOr(st.status, release ? PSE_STATUS_BAD_BLOCK : PSE_STATUS_TRUNCATE_LONG);
  }
}

// Scatter of new K/V tokens into their blocks (engine/paged_cache.py:131-136).
// CTAs walk the new tokens (row, w); a token's block is looked up once and its
// threads copy one VEC-element piece of one head each (32-bit index math).
template <typename T, int VEC>
__global__ void append_kernel(pse_block_state st, T* __restrict__ k_pool, T* __restrict__ v_pool, int kv_heads,
                              int head_dim, const T* __restrict__ k_src, const T* __restrict__ v_src,
                              int64_t tok_stride, int64_t head_stride, const int32_t* __restrict__ slots,
                              const int32_t* __restrict__ base_len, int rows, int width) {
  // new K/V may come from the kernel just before (this launch may overlap it)
  pdl_wait();
  // the attention kernel that follows may launch now (it waits for this
  // kernel's writes before it copies any page)
  pdl_trigger();
  const int vecs = head_dim / VEC;
  const int per_tok = kv_heads * vecs;
  const int n_tok = rows * width;
  for (int tkn = blockIdx.x; tkn < n_tok; tkn += gridDim.x) {
    const int i = tkn / width, w = tkn - (tkn / width) * width;
    const int slot = slots[i];
    if (slot < 0 || slot >= st.num_slots) continue;
    const int pos = base_len[i] + w;
    if (pos < 0) continue;
    const int bi = pos / st.block_size;
    if (bi >= st.nblocks[slot]) continue;  // block never reserved (pool exhausted)
    const int blk = st.block_table[(int64_t)slot * st.max_blocks + bi];
    if (blk < 0 || blk >= st.num_blocks) continue;
    const int64_t dst_tok = ((int64_t)blk * kv_heads * st.block_size + pos % st.block_size) * head_dim;
    const int64_t src_tok = (int64_t)tkn * tok_stride;
    for (int e = threadIdx.x; e < per_tok; e += blockDim.x) {
      const int h = e / vecs, v = e - (e / vecs) * vecs;
      const int64_t dst = dst_tok + (int64_t)h * st.block_size * head_dim + v * VEC;
      const int64_t src = src_tok + (int64_t)h * head_stride + v * VEC;
      if constexpr (VEC * sizeof(T) == 16) {
        *reinterpret_cast<uint4*>(k_pool + dst) = *reinterpret_cast<const uint4*>(k_src + src);
        *reinterpret_cast<uint4*>(v_pool + dst) = *reinterpret_cast<const uint4*>(v_src + src);
      } else {
#pragma unroll
        for (int q = 0; q < VEC; ++q) {
          k_pool[dst + q] = k_src[src + q];
          v_pool[dst + q] = v_src[src + q];
        }
      }
    }
  }
}

template <typename T>
__global__ void gather_kernel(pse_block_state st, const T* __restrict__ k_pool, const T* __restrict__ v_pool,
                              int kv_heads, int head_dim, const int32_t* __restrict__ slots, int rows, int max_len,
                              T* __restrict__ k_out, T* __restrict__ v_out) {
  const int64_t total = (int64_t)rows * kv_heads * max_len * head_dim;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int d = (int)(e % head_dim);
    int64_t r = e / head_dim;
    const int t = (int)(r % max_len);
    r /= max_len;
    const int h = (int)(r % kv_heads);
    const int i = (int)(r / kv_heads);
    const int slot = slots[i];
    T kv = from_f32<T>(0.f), vv = from_f32<T>(0.f);
    if (slot >= 0 && slot < st.num_slots && t < st.seq_len[slot]) {
      const int bi = t / st.block_size;
      if (bi < st.nblocks[slot]) {
        const int blk = st.block_table[(int64_t)slot * st.max_blocks + bi];
        if (blk >= 0 && blk < st.num_blocks) {
          const int64_t src = (((int64_t)blk * kv_heads + h) * st.block_size + t % st.block_size) * head_dim + d;
          kv = k_pool[src];
          vv = v_pool[src];
        }
      }
    }
    k_out[e] = kv;
    v_out[e] = vv;
  }
}

inline int grid_for(int64_t work, int threads) {
  int64_t g = (work + threads - 1) / threads;
  if (g > (int64_t)kNumSMs * 32) g = (int64_t)kNumSMs * 32;
  return g < 1 ? 1 : (int)g;
}

bool g_pdl = true;

bool state_ok(const pse_block_state& st) {
  return st.block_table && st.seq_len && st.nblocks && st.free_stack && st.free_top && st.block_free && st.status &&
         st.num_blocks >= 0 && st.block_size > 0 && st.max_blocks > 0 && st.num_slots > 0;
}

template <typename T>
int launch_append(const pse_block_state& st, const pse_kv_layer& kv, const void* k_src, const void* v_src,
                  int64_t tok_stride, int64_t head_stride, const int32_t* slots, const int32_t* base_len, int rows,
                  int width, cudaStream_t s) {
  constexpr int V16 = 16 / sizeof(T);
  const bool vec_ok = kv.head_dim % V16 == 0 && tok_stride % V16 == 0 && head_stride % V16 == 0 &&
                      reinterpret_cast<uintptr_t>(k_src) % 16 == 0 && reinterpret_cast<uintptr_t>(v_src) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(kv.k_pool) % 16 == 0 && reinterpret_cast<uintptr_t>(kv.v_pool) % 16 == 0;
  if ((int64_t)rows * width >= (1ll << 31)) return PSE_EINVAL;
  const int n_tok = rows * width;
  const int grid = n_tok < kNumSMs * 16 ? n_tok : kNumSMs * 16;
  if (vec_ok) {
    const int per_tok = kv.kv_heads * (kv.head_dim / V16);
    const int threads = per_tok >= 256 ? 256 : ((per_tok + 31) / 32) * 32;
    cudaError_t e = launch_pdl(append_kernel<T, V16>, dim3(grid), dim3(threads), 0, s, st, (T*)kv.k_pool,
                               (T*)kv.v_pool, (int)kv.kv_heads, (int)kv.head_dim, (const T*)k_src, (const T*)v_src,
                               tok_stride, head_stride, slots, base_len, rows, width);
    if (e != cudaSuccess) return (int)e;
  } else {
    const int per_tok = kv.kv_heads * kv.head_dim;
    const int threads = per_tok >= 256 ? 256 : ((per_tok + 31) / 32) * 32;
    append_kernel<T, 1><<<grid, threads, 0, s>>>(st, (T*)kv.k_pool, (T*)kv.v_pool, kv.kv_heads, kv.head_dim,
                                                 (const T*)k_src, (const T*)v_src, tok_stride, head_stride, slots,
                                                 base_len, rows, width);
  }
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

}  // namespace
}  // namespace pse

using namespace pse;

extern "C" int pse_block_init(pse_block_state st, void* stream) {
  if (!state_ok(st)) return PSE_EINVAL;
  int64_t work = st.num_blocks;
  if ((int64_t)st.num_slots * st.max_blocks > work) work = (int64_t)st.num_slots * st.max_blocks;
  block_init_kernel<<<grid_for(work, 256), 256, 0, (cudaStream_t)stream>>>(st);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

extern "C" int pse_block_alloc_one(pse_block_state st, int32_t* out_id, void* stream) {
  if (!state_ok(st) || !out_id) return PSE_EINVAL;
  block_alloc_one_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(st, out_id);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

extern "C" int pse_block_free_one(pse_block_state st, const int32_t* block_id, void* stream) {
  if (!state_ok(st) || !block_id) return PSE_EINVAL;
  block_free_one_kernel<<<1, 1, 0, (cudaStream_t)stream>>>(st, block_id);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

extern "C" int pse_kv_reserve(pse_block_state st, const int32_t* slots, int32_t rows, int32_t width,
                              int32_t* base_len, void* stream) {
  if (!state_ok(st) || rows < 0 || width < 0 || (rows > 0 && (!slots || !base_len))) return PSE_EINVAL;
  if (rows == 0) return PSE_OK;
  reserve_kernel<<<1, kScanThreads, 0, (cudaStream_t)stream>>>(st, slots, rows, width, nullptr, base_len);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

extern "C" int pse_kv_reserve_rows(pse_block_state st, const int32_t* slots, int32_t rows, const int32_t* widths,
                                   int32_t* base_len, void* stream) {
  if (!state_ok(st) || rows < 0 || (rows > 0 && (!slots || !widths || !base_len))) return PSE_EINVAL;
  if (rows == 0) return PSE_OK;
  reserve_kernel<<<1, kScanThreads, 0, (cudaStream_t)stream>>>(st, slots, rows, 0, widths, base_len);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

extern "C" int pse_kv_truncate(pse_block_state st, const int32_t* slots, int32_t rows, const int32_t* new_len,
                               const int32_t* base_len, const int32_t* accepted, void* stream) {
  if (!state_ok(st) || rows < 0 || (rows > 0 && !slots)) return PSE_EINVAL;
  if (!new_len && (!base_len || !accepted)) return PSE_EINVAL;
  if (rows == 0) return PSE_OK;
  free_rows_kernel<<<1, kScanThreads, 0, (cudaStream_t)stream>>>(st, slots, rows, new_len, base_len, accepted, 0);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

extern "C" int pse_kv_release(pse_block_state st, const int32_t* slots, int32_t rows, void* stream) {
  if (!state_ok(st) || rows < 0 || (rows > 0 && !slots)) return PSE_EINVAL;
  if (rows == 0) return PSE_OK;
  free_rows_kernel<<<1, kScanThreads, 0, (cudaStream_t)stream>>>(st, slots, rows, nullptr, nullptr, nullptr, 1);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

extern "C" int pse_kv_append(pse_block_state st, pse_kv_layer kv, const void* k_src, const void* v_src,
                             int64_t tok_stride, int64_t head_stride, const int32_t* slots, const int32_t* base_len,
                             int32_t rows, int32_t width, void* stream) {
  if (!state_ok(st) || !kv.k_pool || !kv.v_pool || kv.kv_heads <= 0 || kv.head_dim <= 0 || rows < 0 || width < 0)
    return PSE_EINVAL;
  if (rows == 0 || width == 0) return PSE_OK;
  if (!k_src || !v_src || !slots || !base_len) return PSE_EINVAL;
  cudaStream_t s = (cudaStream_t)stream;
  if (kv.dtype == PSE_BF16)
    return launch_append<__nv_bfloat16>(st, kv, k_src, v_src, tok_stride, head_stride, slots, base_len, rows, width, s);
  if (kv.dtype == PSE_F32)
    return launch_append<float>(st, kv, k_src, v_src, tok_stride, head_stride, slots, base_len, rows, width, s);
  return PSE_EINVAL;
}

// Token-tree commit: row i keeps n[i] of the tokens its tree calls appended,
// the token at position base_len[i] + src[i*max_n + m] moving to position
// base_len[i] + m (m < n[i]; src increasing with src[m] >= m, so no source is
// overwritten before it is read: each thread walks m in order over its own
// (head, element) slice).
template <typename T>
__global__ void compact_kernel(pse_block_state st, T* __restrict__ k_pool, T* __restrict__ v_pool, int kv_heads,
                               int head_dim, const int32_t* slots, const int32_t* base_len, const int32_t* src,
                               const int32_t* n, int max_n) {
  const int i = blockIdx.x;
  const int slot = slots[i];
  if (slot < 0 || slot >= st.num_slots) {
    if (threadIdx.x == 0) atomicOr(st.status, PSE_STATUS_BAD_BLOCK);
    return;
  }
  const int L = base_len[i], cnt = min(n[i], max_n), len = st.seq_len[slot], nb = st.nblocks[slot];
  const int bs = st.block_size;
  const int32_t* row = st.block_table + (int64_t)slot * st.max_blocks;
  bool bad = false;
  for (int e = threadIdx.x; e < kv_heads * head_dim; e += blockDim.x) {
    const int h = e / head_dim, d = e % head_dim;
    for (int m = 0; m < cnt; ++m) {
      const int from = L + src[(int64_t)i * max_n + m], to = L + m;
      if (from == to) continue;
      if (to < 0 || from < to || from >= len || from / bs >= nb) {
        bad = true;
        break;
      }
      const int bf = row[from / bs], bt = row[to / bs];
      if (bf < 0 || bf >= st.num_blocks || bt < 0 || bt >= st.num_blocks) {
        bad = true;
        break;
      }
      const int64_t of = (((int64_t)bf * kv_heads + h) * bs + from % bs) * head_dim + d;
      const int64_t ot = (((int64_t)bt * kv_heads + h) * bs + to % bs) * head_dim + d;
      k_pool[ot] = k_pool[of];
      v_pool[ot] = v_pool[of];
    }
  }
  if (bad) atomicOr(st.status, PSE_STATUS_BAD_BLOCK);
}

extern "C" int pse_kv_compact(pse_block_state st, pse_kv_layer kv, const int32_t* slots, const int32_t* base_len,
                              const int32_t* src, const int32_t* n, int32_t rows, int32_t max_n, void* stream) {
  if (!state_ok(st) || !kv.k_pool || !kv.v_pool || kv.kv_heads <= 0 || kv.head_dim <= 0 || rows < 0 || max_n < 0)
    return PSE_EINVAL;
  if (rows == 0 || max_n == 0) return PSE_OK;
  if (!slots || !base_len || !src || !n) return PSE_EINVAL;
  cudaStream_t s = (cudaStream_t)stream;
  if (kv.dtype == PSE_BF16)
    compact_kernel<__nv_bfloat16><<<rows, 256, 0, s>>>(st, (__nv_bfloat16*)kv.k_pool, (__nv_bfloat16*)kv.v_pool,
                                                        kv.kv_heads, kv.head_dim, slots, base_len, src, n, max_n);
  else if (kv.dtype == PSE_F32)
    compact_kernel<float><<<rows, 256, 0, s>>>(st, (float*)kv.k_pool, (float*)kv.v_pool, kv.kv_heads, kv.head_dim,
                                               slots, base_len, src, n, max_n);
  else
    return PSE_EINVAL;
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

extern "C" int pse_kv_gather(pse_block_state st, pse_kv_layer kv, const int32_t* slots, int32_t rows, int32_t max_len,
                             void* k_out, void* v_out, void* stream) {
  if (!state_ok(st) || rows < 0 || max_len < 0) return PSE_EINVAL;
  if (rows == 0 || max_len == 0) return PSE_OK;
  if (!slots || !k_out || !v_out) return PSE_EINVAL;
  const int64_t work = (int64_t)rows * kv.kv_heads * max_len * kv.head_dim;
  cudaStream_t s = (cudaStream_t)stream;
  if (kv.dtype == PSE_BF16)
    gather_kernel<__nv_bfloat16><<<grid_for(work, 256), 256, 0, s>>>(
        st, (const __nv_bfloat16*)kv.k_pool, (const __nv_bfloat16*)kv.v_pool, kv.kv_heads, kv.head_dim, slots, rows,
        max_len, (__nv_bfloat16*)k_out, (__nv_bfloat16*)v_out);
  else if (kv.dtype == PSE_F32)
    gather_kernel<float><<<grid_for(work, 256), 256, 0, s>>>(st, (const float*)kv.k_pool, (const float*)kv.v_pool,
                                                             kv.kv_heads, kv.head_dim, slots, rows, max_len,
                                                             (float*)k_out, (float*)v_out);
  else
    return PSE_EINVAL;
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

namespace pse {
bool pdl_enabled() { return g_pdl; }
}  // namespace pse

extern "C" int pse_launch_overlap(int32_t on) {
  g_pdl = on != 0;
  return PSE_OK;
}
