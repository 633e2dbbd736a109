// Paged attention over the device block pool (replaces the gather + masked
// matmul attention of engine/batched_forward.py:37-65 / engine/model.py:99-116).
//
// Work decomposition: one CTA per (row, KV head, query tile, KV split).  The
// query tile holds up to RMAX query rows of the KV head's group (GQA heads x
// the call's W positions, row r = w * group + g); all of them share every K/V
// page the CTA streams, so each page is read from HBM once per tile.  Pages are
// staged into shared memory 128 tokens at a time with 16-byte loads; each of
// the 4 warps owns 32 tokens of a chunk (lane = token) for the Q.K dot
// products, keeps its own online-softmax state per query row, and the warps
// are merged at the end.  With more than one KV split the partial (max, sum,
// unnormalised output) go to a float workspace and a combine kernel merges
// them (flash-decoding).  Causality: query w of row i sits at position
// base_len[i] + w and sees keys 0..base_len[i]+w.

#include <cfloat>
#include <mutex>

#include "common.cuh"

namespace pse {
namespace {

constexpr int kWarps = 4;
constexpr int kThreads = kWarps * 32;
constexpr int kChunk = kWarps * 32;  // tokens staged per iteration

struct AttnArgs {
  const int32_t* block_table;
  const int32_t* nblocks;
  int max_blocks, block_size, num_blocks, num_slots;
  const void* k_pool;
  const void* v_pool;
  int kv_heads, head_dim;
  const void* q;
  int64_t q_tok_stride;
  void* out;
  int64_t out_tok_stride;
  const int32_t* slots;
  const int32_t* base_len;
  int rows, width, q_heads;
  float scale;
  int split_tokens, n_splits, n_qtiles;
  float* ws;  // [n_splits][rows*width][q_heads][head_dim + 2]
  int tree_b, tree_d0;  // token-tree call (key_vis in common.cuh); tree_b == 0: causal
};

template <typename T>
__device__ __forceinline__ int words_per_token(int head_dim) {
  return (head_dim * (int)sizeof(T) + 3) / 4;
}

// Shared-memory row stride (32-bit words) of a staged token: odd, so lane t
// reading token t's word c hits bank (t * stride + c) % 32 without conflicts.
template <typename T>
__device__ __forceinline__ int smem_stride(int head_dim) {
  return words_per_token<T>(head_dim) | 1;
}

template <typename T>
__device__ __forceinline__ float2 word_to_f2(uint32_t w);
template <>
__device__ __forceinline__ float2 word_to_f2<__nv_bfloat16>(uint32_t w) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&w);
  return __bfloat1622float2(b);
}

template <typename T, int MAXD, int RMAX>
__global__ void __launch_bounds__(kThreads) paged_attn_kernel(AttnArgs a) {
  extern __shared__ __align__(16) uint32_t smem[];
  const int HD = a.head_dim;
  const int group = a.q_heads / a.kv_heads;
  const int n_qrows = group * a.width;

  int bid = blockIdx.x;
  const int qtile = bid % a.n_qtiles;
  bid /= a.n_qtiles;
  const int hk = bid % a.kv_heads;
  const int i = bid / a.kv_heads;
  const int split = blockIdx.y;
  const int slot = a.slots[i];
  const int base = a.base_len[i];
  const int r0 = qtile * RMAX;
  const int nr = min(RMAX, n_qrows - r0);
  if (nr <= 0 || slot < 0 || slot >= a.num_slots || base < 0) return;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int stride = smem_stride<T>(HD);
  const int wpt = words_per_token<T>(HD);
  const int HDP = (HD + 3) & ~3;

  float* q_s = reinterpret_cast<float*>(smem);                 // [RMAX][HDP]
  uint32_t* k_s = smem + RMAX * HDP;                           // [kChunk][stride]
  uint32_t* v_s = k_s + kChunk * stride;                       // [kChunk][stride]

  // Query rows of this tile, pre-scaled, as fp32.
  const T* qp = reinterpret_cast<const T*>(a.q);
  for (int e = tid; e < RMAX * HDP; e += kThreads) {
    const int r = e / HDP, d = e % HDP;
    float v = 0.f;
    if (r < nr && d < HD) {
      const int rr = r0 + r, w = rr / group, g = rr % group;
      v = to_f32(qp[((int64_t)i * a.width + w) * a.q_tok_stride + (int64_t)(hk * group + g) * HD + d]) * a.scale;
    }
    q_s[e] = v;
  }

  // Key range of this split, clipped to the last query's causal limit.
  const int w_last = (r0 + nr - 1) / group;
  const int kmax = base + w_last + 1;  // keys [0, kmax) may be visible
  const int k_lo = split * a.split_tokens;
  const int k_hi = min(k_lo + a.split_tokens, kmax);
  const int row_nblocks = a.nblocks[slot];

  KeyVis vis[RMAX];
#pragma unroll
  for (int r = 0; r < RMAX; ++r) vis[r] = r < nr ? key_vis(base, (r0 + r) / group, a.tree_b, a.tree_d0) : kNoKeys;

  float m[RMAX], l[RMAX], o[RMAX][MAXD];
#pragma unroll
  for (int r = 0; r < RMAX; ++r) {
    m[r] = -INFINITY;
    l[r] = 0.f;
#pragma unroll
    for (int c = 0; c < MAXD; ++c) o[r][c] = 0.f;
  }

  const int32_t* table = a.block_table + (int64_t)slot * a.max_blocks;
  const T* kpool = reinterpret_cast<const T*>(a.k_pool);
  const T* vpool = reinterpret_cast<const T*>(a.v_pool);
  const bool vec16 = (HD * (int)sizeof(T)) % 16 == 0;

  for (int c0 = k_lo; c0 < k_hi; c0 += kChunk) {
    __syncthreads();
    // Stage K/V of tokens [c0, c0 + kChunk).
    if (vec16) {
      const int vpt = HD * (int)sizeof(T) / 16;  // 16-byte vectors per token
      for (int e = tid; e < kChunk * vpt; e += kThreads) {
        const int t = e / vpt, vv = e % vpt;
        const int pos = c0 + t;
        uint4 kv4 = make_uint4(0, 0, 0, 0), vv4 = make_uint4(0, 0, 0, 0);
        if (pos < k_hi) {
          const int bi = pos / a.block_size;
          const int blk = bi < row_nblocks ? table[bi] : -1;
          if (blk >= 0 && blk < a.num_blocks) {
            const int64_t off = (((int64_t)blk * a.kv_heads + hk) * a.block_size + pos % a.block_size) * HD;
            kv4 = reinterpret_cast<const uint4*>(kpool + off)[vv];
            vv4 = reinterpret_cast<const uint4*>(vpool + off)[vv];
          }
        }
        uint32_t* kd = k_s + t * stride + vv * 4;
        uint32_t* vd = v_s + t * stride + vv * 4;
        kd[0] = kv4.x; kd[1] = kv4.y; kd[2] = kv4.z; kd[3] = kv4.w;
        vd[0] = vv4.x; vd[1] = vv4.y; vd[2] = vv4.z; vd[3] = vv4.w;
      }
    } else {
      for (int e = tid; e < kChunk * HD; e += kThreads) {
        const int t = e / HD, d = e % HD;
        const int pos = c0 + t;
        T kv = from_f32<T>(0.f), vv = from_f32<T>(0.f);
        if (pos < k_hi) {
          const int bi = pos / a.block_size;
          const int blk = bi < row_nblocks ? table[bi] : -1;
          if (blk >= 0 && blk < a.num_blocks) {
            const int64_t off = (((int64_t)blk * a.kv_heads + hk) * a.block_size + pos % a.block_size) * HD;
            kv = kpool[off + d];
            vv = vpool[off + d];
          }
        }
        reinterpret_cast<T*>(k_s + t * stride)[d] = kv;
        reinterpret_cast<T*>(v_s + t * stride)[d] = vv;
      }
    }
    __syncthreads();

    // Scores: lane owns token c0 + warp*32 + lane.
    const int tloc = warp * 32 + lane;
    const int tok = c0 + tloc;
    float s[RMAX];
#pragma unroll
    for (int r = 0; r < RMAX; ++r) s[r] = 0.f;
    const uint32_t* krow = k_s + tloc * stride;
    if constexpr (sizeof(T) == 2) {
      for (int c = 0; c < wpt; ++c) {
        const float2 kf = word_to_f2<T>(krow[c]);
#pragma unroll
        for (int r = 0; r < RMAX; ++r) {
          const float2 qf = *reinterpret_cast<const float2*>(q_s + r * HDP + 2 * c);
          s[r] = fmaf(qf.x, kf.x, s[r]);
          s[r] = fmaf(qf.y, kf.y, s[r]);
        }
      }
    } else {
      for (int c = 0; c < wpt; ++c) {
        const float kf = __uint_as_float(krow[c]);
#pragma unroll
        for (int r = 0; r < RMAX; ++r) s[r] = fmaf(q_s[r * HDP + c], kf, s[r]);
      }
    }
    float p[RMAX], corr[RMAX];
#pragma unroll
    for (int r = 0; r < RMAX; ++r) {
      const bool ok = tok < k_hi && key_visible(vis[r], tok, a.tree_b);
      const float sv = ok ? s[r] : -INFINITY;
      const float cmax = warp_max(sv);
      const float m_new = fmaxf(m[r], cmax);
      if (m_new == -INFINITY) {
        p[r] = 0.f;
        corr[r] = 1.f;
      } else {
        p[r] = ok ? __expf(sv - m_new) : 0.f;
        corr[r] = __expf(m[r] - m_new);
        m[r] = m_new;
      }
      l[r] = l[r] * corr[r] + warp_sum(p[r]);
#pragma unroll
      for (int c = 0; c < MAXD; ++c) o[r][c] *= corr[r];
    }
    // P.V: lane owns output columns lane + 32c.
    const int jmax = min(32, k_hi - (c0 + warp * 32));
    for (int j = 0; j < jmax; ++j) {
      const T* vrow = reinterpret_cast<const T*>(v_s + (warp * 32 + j) * stride);
      float vv[MAXD];
#pragma unroll
      for (int c = 0; c < MAXD; ++c) {
        const int d = lane + 32 * c;
        vv[c] = d < HD ? to_f32(vrow[d]) : 0.f;
      }
#pragma unroll
      for (int r = 0; r < RMAX; ++r) {
        const float pj = __shfl_sync(0xffffffffu, p[r], j);
#pragma unroll
        for (int c = 0; c < MAXD; ++c) o[r][c] = fmaf(pj, vv[c], o[r][c]);
      }
    }
  }
  __syncthreads();

  // Merge the 4 warps' states (reuse the K/V staging area).
  float* mw = reinterpret_cast<float*>(k_s);        // [kWarps][RMAX]
  float* lw = mw + kWarps * RMAX;                   // [kWarps][RMAX]
  float* ow = lw + kWarps * RMAX;                   // [kWarps][RMAX][32*MAXD]
  if (lane == 0) {
#pragma unroll
    for (int r = 0; r < RMAX; ++r) {
      mw[warp * RMAX + r] = m[r];
      lw[warp * RMAX + r] = l[r];
    }
  }
#pragma unroll
  for (int r = 0; r < RMAX; ++r)
#pragma unroll
    for (int c = 0; c < MAXD; ++c) ow[(warp * RMAX + r) * 32 * MAXD + lane + 32 * c] = o[r][c];
  __syncthreads();

  T* outp = reinterpret_cast<T*>(a.out);
  for (int r = warp; r < nr; r += kWarps) {
    float M = -INFINITY;
#pragma unroll
    for (int w2 = 0; w2 < kWarps; ++w2) M = fmaxf(M, mw[w2 * RMAX + r]);
    float L = 0.f, f[kWarps];
#pragma unroll
    for (int w2 = 0; w2 < kWarps; ++w2) {
      f[w2] = M == -INFINITY ? 0.f : __expf(mw[w2 * RMAX + r] - M);
      L += lw[w2 * RMAX + r] * f[w2];
    }
    const int rr = r0 + r, w = rr / group, g = rr % group, h = hk * group + g;
    const int64_t tokrow = (int64_t)i * a.width + w;
    if (a.n_splits == 1) {
      const float inv = L > 0.f ? 1.f / L : 0.f;
      for (int c = 0; c < MAXD; ++c) {
        const int d = lane + 32 * c;
        if (d >= HD) break;
        float acc = 0.f;
#pragma unroll
        for (int w2 = 0; w2 < kWarps; ++w2) acc += ow[(w2 * RMAX + r) * 32 * MAXD + d] * f[w2];
        outp[tokrow * a.out_tok_stride + (int64_t)h * HD + d] = from_f32<T>(acc * inv);
      }
    } else {
      float* ws = a.ws + (((int64_t)split * a.rows * a.width + tokrow) * a.q_heads + h) * (HD + 2);
      for (int c = 0; c < MAXD; ++c) {
        const int d = lane + 32 * c;
        if (d >= HD) break;
        float acc = 0.f;
#pragma unroll
        for (int w2 = 0; w2 < kWarps; ++w2) acc += ow[(w2 * RMAX + r) * 32 * MAXD + d] * f[w2];
        ws[d] = acc;
      }
      if (lane == 0) {
        ws[HD] = M;
        ws[HD + 1] = L;
      }
    }
  }
}

// Merge of the KV splits: one warp per (token row, query head).
template <typename T>
__global__ void combine_kernel(AttnArgs a) {
  const int HD = a.head_dim;
  const int64_t n_items = (int64_t)a.rows * a.width * a.q_heads;
  const int64_t item = (int64_t)blockIdx.x * (blockDim.x / 32) + (threadIdx.x >> 5);
  if (item >= n_items) return;
  const int lane = threadIdx.x & 31;
  const int h = (int)(item % a.q_heads);
  const int64_t tokrow = item / a.q_heads;
  const int64_t split_stride = (int64_t)a.rows * a.width * a.q_heads * (HD + 2);
  const float* base = a.ws + item * (HD + 2);
  float M = -INFINITY;
  for (int s = 0; s < a.n_splits; ++s) M = fmaxf(M, base[s * split_stride + HD]);
  float L = 0.f;
  for (int s = 0; s < a.n_splits; ++s) {
    const float ms = base[s * split_stride + HD];
    if (ms != -INFINITY) L += base[s * split_stride + HD + 1] * __expf(ms - M);
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  T* outp = reinterpret_cast<T*>(a.out);
  for (int d = lane; d < HD; d += 32) {
    float acc = 0.f;
    for (int s = 0; s < a.n_splits; ++s) {
      const float ms = base[s * split_stride + HD];
      if (ms != -INFINITY) acc += base[s * split_stride + d] * __expf(ms - M);
    }
    outp[tokrow * a.out_tok_stride + (int64_t)h * HD + d] = from_f32<T>(acc * inv);
  }
}

struct Plan {
  int rmax, maxd, n_qtiles, n_splits, split_tokens;
};

// Work items the split plan aims for per SM: a call with fewer (row, KV head,
// query tile) items than this splits each row's keys into more items.
#ifndef PSE_ATTN_ITEMS_PER_SM
#define PSE_ATTN_ITEMS_PER_SM 4
#endif

// The KV split count depends only on the call's shape (not on which kernel
// runs it), so the workspace query and both kernels agree.
Plan make_plan(int rows, int width, int q_heads, int kv_heads, int head_dim, int max_ctx) {
  Plan p;
  const int n_qrows = (q_heads / kv_heads) * width;
  p.rmax = n_qrows <= 1 ? 1 : n_qrows <= 2 ? 2 : n_qrows <= 4 ? 4 : 8;
  p.maxd = head_dim <= 32 ? 1 : head_dim <= 64 ? 2 : head_dim <= 128 ? 4 : 8;
  p.n_qtiles = ceil_div(n_qrows, p.rmax);
  const long base_ctas = (long)rows * kv_heads * ceil_div(n_qrows, 16);
  const int target = PSE_ATTN_ITEMS_PER_SM * kNumSMs;
  int splits = base_ctas >= target ? 1 : (int)((target + base_ctas - 1) / base_ctas);
  const int max_useful = ceil_div(max_ctx > 0 ? max_ctx : 1, 256);
  if (splits > max_useful) splits = max_useful;
  if (splits < 1) splits = 1;
  int st = ceil_div(ceil_div(max_ctx > 0 ? max_ctx : 1, splits), kChunk) * kChunk;
  p.split_tokens = st;
  p.n_splits = ceil_div(max_ctx > 0 ? max_ctx : 1, st);
  return p;
}

template <typename T>
size_t smem_bytes(int rmax, int head_dim) {
  const int stride = ((head_dim * (int)sizeof(T) + 3) / 4) | 1;
  const int hdp = (head_dim + 3) & ~3;
  size_t stage = (size_t)2 * kChunk * stride * 4;
  const int maxd = head_dim <= 32 ? 1 : head_dim <= 64 ? 2 : head_dim <= 128 ? 4 : 8;
  size_t merge = (size_t)(2 * kWarps * rmax + kWarps * rmax * 32 * maxd) * 4;
  return (size_t)rmax * hdp * 4 + (stage > merge ? stage : merge);
}

template <typename T, int MAXD, int RMAX>
int launch_t(const AttnArgs& a, cudaStream_t s) {
  const size_t smem = smem_bytes<T>(RMAX, a.head_dim);
  auto kern = paged_attn_kernel<T, MAXD, RMAX>;
  // Opt in once to the largest dynamic shared memory this instantiation can
  // ask for (head_dim 256), so no attribute call is issued during a capture.
  static const cudaError_t opt_in = cudaFuncSetAttribute(
      kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes<T>(RMAX, 32 * MAXD));
  if (opt_in != cudaSuccess) return (int)opt_in;
  dim3 grid((unsigned)(a.rows * a.kv_heads * a.n_qtiles), (unsigned)a.n_splits);
  kern<<<grid, kThreads, smem, s>>>(a);
  PSE_LAUNCH_CHECK();
  if (a.n_splits > 1) {
    const int64_t items = (int64_t)a.rows * a.width * a.q_heads;
    const int wpb = 8;
    combine_kernel<T><<<(unsigned)((items + wpb - 1) / wpb), wpb * 32, 0, s>>>(a);
    PSE_LAUNCH_CHECK();
  }
  return PSE_OK;
}

template <typename T, int MAXD>
int launch_r(const AttnArgs& a, int rmax, cudaStream_t s) {
  switch (rmax) {
    case 1: return launch_t<T, MAXD, 1>(a, s);
    case 2: return launch_t<T, MAXD, 2>(a, s);
    case 4: return launch_t<T, MAXD, 4>(a, s);
    default: return launch_t<T, MAXD, 8>(a, s);
  }
}

template <typename T>
int launch_d(const AttnArgs& a, const Plan& p, cudaStream_t s) {
  switch (p.maxd) {
    case 1: return launch_r<T, 1>(a, p.rmax, s);
    case 2: return launch_r<T, 2>(a, p.rmax, s);
    case 4: return launch_r<T, 4>(a, p.rmax, s);
    default: return launch_r<T, 8>(a, p.rmax, s);
  }
}

}  // namespace

bool tc_eligible(const pse_block_state& st, const pse_kv_layer& kv, int q_heads, int width);
int tc_attention(const pse_block_state& st, const pse_kv_layer& kv, const void* q, int64_t q_tok_stride, void* out,
                 int64_t out_tok_stride, const int32_t* slots, const int32_t* base_len, int rows, int width,
                 int q_heads, float scale, int split_tokens, int n_splits, void* ws, int* counter,
                 const int32_t* row_order, bool self_reset, int tree_b, int tree_d0, cudaStream_t s);

extern bool g_prefill_pair;
bool prefill_eligible(const pse_block_state& st, const pse_kv_layer& kv, const void* q, int64_t q_tok_stride,
                      const void* out, int64_t out_tok_stride, int q_heads, int width);
int prefill_attention(const pse_block_state& st, const pse_kv_layer& kv, const void* q, int64_t q_tok_stride,
                      void* out, int64_t out_tok_stride, const int32_t* slots, const int32_t* base_len, int rows,
                      int width, int q_heads, float scale, const int32_t* row_order, cudaStream_t s);

}  // namespace pse

using namespace pse;

namespace {
bool g_force_generic = false;
bool g_prefill_off = false;

bool use_prefill(const pse_block_state& st, const pse_kv_layer& kv, const void* q, int64_t q_tok_stride,
                 const void* out, int64_t out_tok_stride, int q_heads, int width) {
  return !g_force_generic && !g_prefill_off &&
         prefill_eligible(st, kv, q, q_tok_stride, out, out_tok_stride, q_heads, width);
}
}  // namespace

/* Test hook: route every call to the generic kernel (1) or let the shape pick (0). */
extern "C" int pse_attention_force_generic(int32_t on) {
  g_force_generic = on != 0;
  return PSE_OK;
}

extern "C" int pse_attention_prefill_select(int32_t mode) {
  if (mode < 0 || mode > 2) return PSE_EINVAL;
  g_prefill_off = mode == 1;
  pse::g_prefill_pair = mode == 0;
  return PSE_OK;
}

// Workspace layout: a 256-byte header (the persistent kernel's work counters,
// zero before a call and left zero by it) followed by the split-KV partials
// [n_splits][rows*width][q_heads][head_dim + 2] floats when the call splits.
constexpr size_t kWsHeader = 256;

extern "C" size_t pse_paged_attention_workspace(int32_t rows, int32_t width, int32_t q_heads, int32_t kv_heads,
                                                int32_t head_dim, int32_t max_ctx) {
  if (rows <= 0 || width <= 0 || q_heads <= 0 || kv_heads <= 0 || head_dim <= 0) return kWsHeader;
  Plan p = make_plan(rows, width, q_heads, kv_heads, head_dim, max_ctx);
  if (p.n_splits <= 1) return kWsHeader;
  return kWsHeader + (size_t)p.n_splits * rows * width * q_heads * (head_dim + 2) * sizeof(float);
}

namespace {
int paged_attention(const pse_block_state& st, const pse_kv_layer& kv, const void* q, int64_t q_tok_stride, void* out,
                    int64_t out_tok_stride, const int32_t* slots, const int32_t* base_len, int32_t rows, int32_t width,
                    int32_t q_heads, float scale, int32_t max_ctx, const int32_t* row_order, void* workspace,
                    size_t workspace_bytes, int tree_b, int tree_d0, void* stream) {
  if (rows < 0 || width < 0 || tree_b < 0 || tree_d0 < 0) return PSE_EINVAL;
  if (rows == 0 || width == 0) return PSE_OK;
  if (!q || !out || !slots || !base_len || !kv.k_pool || !kv.v_pool || !st.block_table || !st.nblocks)
    return PSE_EINVAL;
  if (kv.kv_heads <= 0 || q_heads <= 0 || q_heads % kv.kv_heads != 0) return PSE_EINVAL;
  if (kv.head_dim <= 0 || kv.head_dim > 256 || max_ctx <= 0 || st.block_size <= 0) return PSE_EINVAL;
  Plan p = make_plan(rows, width, q_heads, kv.kv_heads, kv.head_dim, max_ctx);
  if (!workspace ||
      workspace_bytes < pse_paged_attention_workspace(rows, width, q_heads, kv.kv_heads, kv.head_dim, max_ctx))
    return PSE_EWORKSPACE;
  AttnArgs a;
  a.block_table = st.block_table;
  a.nblocks = st.nblocks;
  a.max_blocks = st.max_blocks;
  a.block_size = st.block_size;
  a.num_blocks = st.num_blocks;
  a.num_slots = st.num_slots;
  a.k_pool = kv.k_pool;
  a.v_pool = kv.v_pool;
  a.kv_heads = kv.kv_heads;
  a.head_dim = kv.head_dim;
  a.q = q;
  a.q_tok_stride = q_tok_stride;
  a.out = out;
  a.out_tok_stride = out_tok_stride;
  a.slots = slots;
  a.base_len = base_len;
  a.rows = rows;
  a.width = width;
  a.q_heads = q_heads;
  a.scale = scale;
  a.split_tokens = p.split_tokens;
  a.n_splits = p.n_splits;
  a.n_qtiles = p.n_qtiles;
  a.ws = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(workspace) + kWsHeader);
  a.tree_b = tree_b;
  a.tree_d0 = tree_d0;
  cudaStream_t s = (cudaStream_t)stream;
  // the prompt kernel is causal only: token-tree calls (narrow) never take it
  if (tree_b == 0 && use_prefill(st, kv, q, q_tok_stride, out, out_tok_stride, q_heads, width))
    return prefill_attention(st, kv, q, q_tok_stride, out, out_tok_stride, slots, base_len, rows, width, q_heads,
                             scale, row_order, s);
  if (tc_eligible(st, kv, q_heads, width) && !g_force_generic) {
    int rc = tc_attention(st, kv, q, q_tok_stride, out, out_tok_stride, slots, base_len, rows, width, q_heads, scale,
                          p.split_tokens, p.n_splits, a.ws, reinterpret_cast<int*>(workspace), row_order,
                          /*self_reset=*/true, tree_b, tree_d0, s);
    if (rc) return rc;
    if (p.n_splits > 1) {
      const int64_t items = (int64_t)rows * width * q_heads;
      const int wpb = 8;
      combine_kernel<__nv_bfloat16><<<(unsigned)((items + wpb - 1) / wpb), wpb * 32, 0, s>>>(a);
      PSE_LAUNCH_CHECK();
    }
    return PSE_OK;
  }
  if (kv.dtype == PSE_BF16) return launch_d<__nv_bfloat16>(a, p, s);
  if (kv.dtype == PSE_F32) return launch_d<float>(a, p, s);
  return PSE_EINVAL;
}
}  // namespace

extern "C" int pse_paged_attention(pse_block_state st, pse_kv_layer kv, const void* q, int64_t q_tok_stride, void* out,
                                   int64_t out_tok_stride, const int32_t* slots, const int32_t* base_len, int32_t rows,
                                   int32_t width, int32_t q_heads, float scale, int32_t max_ctx,
                                   const int32_t* row_order, void* workspace, size_t workspace_bytes, void* stream) {
  return paged_attention(st, kv, q, q_tok_stride, out, out_tok_stride, slots, base_len, rows, width, q_heads, scale,
                         max_ctx, row_order, workspace, workspace_bytes, 0, 0, stream);
}

extern "C" int pse_paged_attention_tree(pse_block_state st, pse_kv_layer kv, const void* q, int64_t q_tok_stride,
                                        void* out, int64_t out_tok_stride, const int32_t* slots,
                                        const int32_t* base_len, int32_t rows, int32_t width, int32_t q_heads,
                                        float scale, int32_t max_ctx, const int32_t* row_order, void* workspace,
                                        size_t workspace_bytes, int32_t tree_branches, int32_t tree_depth0,
                                        void* stream) {
  if (tree_branches < 1) return PSE_EINVAL;
  return paged_attention(st, kv, q, q_tok_stride, out, out_tok_stride, slots, base_len, rows, width, q_heads, scale,
                         max_ctx, row_order, workspace, workspace_bytes, tree_branches, tree_depth0, stream);
}

// ---------------------------------------------------------------------------
// Attention without a caller-provided workspace.
//
// Some hosts of this library cannot allocate device memory where they call
// it: a serving runtime in another language that binds only this C ABI and
// has no CUDA allocator of its own, or a process whose device memory belongs
// entirely to another allocator (a framework's caching allocator, a fixed
// pre-reserved pool) that must not be bypassed with cudaMalloc.  For them,
// pse_paged_attention_noalloc takes the split-KV scratch from the fixed array
// below, which is part of the library image: every GPU that loads the library
// holds these PSE_NOALLOC_SCRATCH_BYTES until the process exits.
// ---------------------------------------------------------------------------
namespace {

constexpr size_t kNoallocScratchBytes = PSE_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) float g_noalloc_scratch[kNoallocScratchBytes / sizeof(float)];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device.  In host code the
// array's name is only a host-side stand-in, so the address is looked up once
// per device (with that device current) and cached.
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return PSE_EINVAL;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (!g_noalloc_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return (int)e;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return PSE_OK;
}

}  // namespace

extern "C" int pse_paged_attention_noalloc(pse_block_state st, pse_kv_layer kv, const void* q, int64_t q_tok_stride,
                                           void* out, int64_t out_tok_stride, const int32_t* slots,
                                           const int32_t* base_len, int32_t rows, int32_t width, int32_t q_heads,
                                           float scale, int32_t max_ctx, void* stream) {
  void* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);  // first call on a device: symbol lookup
  if (rc) return rc;
  if (rows < 0 || width < 0) return PSE_EINVAL;
  if (rows == 0 || width == 0) return PSE_OK;
  if (!q || !out || !slots || !base_len || !kv.k_pool || !kv.v_pool || !st.block_table || !st.nblocks)
    return PSE_EINVAL;
  if (kv.kv_heads <= 0 || q_heads <= 0 || q_heads % kv.kv_heads != 0) return PSE_EINVAL;
  if (kv.head_dim <= 0 || kv.head_dim > 256 || max_ctx <= 0 || st.block_size <= 0) return PSE_EINVAL;
  cudaStream_t s = (cudaStream_t)stream;
  // wide (prompt) calls use no split-KV scratch: route them before the size check
  if (use_prefill(st, kv, q, q_tok_stride, out, out_tok_stride, q_heads, width))
    return prefill_attention(st, kv, q, q_tok_stride, out, out_tok_stride, slots, base_len, rows, width, q_heads,
                             scale, nullptr, s);
  const size_t need = pse_paged_attention_workspace(rows, width, q_heads, kv.kv_heads, kv.head_dim, max_ctx);
  if (need > kNoallocScratchBytes) return PSE_ESCRATCH;
  Plan p = make_plan(rows, width, q_heads, kv.kv_heads, kv.head_dim, max_ctx);
  AttnArgs a;
  a.block_table = st.block_table;
  a.nblocks = st.nblocks;
  a.max_blocks = st.max_blocks;
  a.block_size = st.block_size;
  a.num_blocks = st.num_blocks;
  a.num_slots = st.num_slots;
  a.k_pool = kv.k_pool;
  a.v_pool = kv.v_pool;
  a.kv_heads = kv.kv_heads;
  a.head_dim = kv.head_dim;
  a.q = q;
  a.q_tok_stride = q_tok_stride;
  a.out = out;
  a.out_tok_stride = out_tok_stride;
  a.slots = slots;
  a.base_len = base_len;
  a.rows = rows;
  a.width = width;
  a.q_heads = q_heads;
  a.scale = scale;
  a.split_tokens = p.split_tokens;
  a.n_splits = p.n_splits;
  a.n_qtiles = p.n_qtiles;
  // The work counter at the start of the array is zeroed on the stream by every
  // call; every (split, row, head) slot after it is written before the combine
  // reads it, so stale contents from an earlier call never leak in.
  a.ws = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(scratch) + kWsHeader);
  a.tree_b = 0;
  a.tree_d0 = 0;
  if (tc_eligible(st, kv, q_heads, width) && !g_force_generic) {
    rc = tc_attention(st, kv, q, q_tok_stride, out, out_tok_stride, slots, base_len, rows, width, q_heads, scale,
                      p.split_tokens, p.n_splits, a.ws, reinterpret_cast<int*>(scratch), nullptr,
                      /*self_reset=*/false, 0, 0, s);
    if (rc) return rc;
    if (p.n_splits > 1) {
      const int64_t items = (int64_t)rows * width * q_heads;
      const int wpb = 8;
      combine_kernel<__nv_bfloat16><<<(unsigned)((items + wpb - 1) / wpb), wpb * 32, 0, s>>>(a);
      PSE_LAUNCH_CHECK();
    }
    return PSE_OK;
  }
  if (kv.dtype == PSE_BF16) return launch_d<__nv_bfloat16>(a, p, s);
  if (kv.dtype == PSE_F32) return launch_d<float>(a, p, s);
  return PSE_EINVAL;
}
