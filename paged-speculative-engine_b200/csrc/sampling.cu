// Draft sampling and the fused accept / reject / resample kernel.
//
// Replaces the per-row Python loops of engine/speculative.py:97-157 and the
// torch helpers of engine/sampling.py:10-23.  One CTA per request row; the
// vocabulary is streamed with coalesced loads and reduced block-wide.
//
// Arithmetic (shared with the CPU oracle, stated once):
//   s_i = l_i / T (fp32), m = max s_i, w_i = expf(s_i - m) (fp32),
//   Z = sum w_i accumulated in fp64;
//   inverse CDF at uniform u: first i whose fp64 running sum exceeds u * Z,
//   else the last i with w_i > 0;
//   accept test u < min(1, (w_p[x] * Z_q) / (w_q[x] * Z_p)) in fp64, 0 if
//   w_q[x] == 0; residual r_i = max(0, w_p[i] / Z_p - w_q[i] / Z_q) in fp64
//   (as w * (1/Z)), sampled from p instead if sum r_i <= 0.
//   Greedy: argmax with ties to the lowest index.

#include <climits>

#include "common.cuh"

namespace pse {
namespace {

constexpr int kSampleThreads = 512;

// Which accept kernel runs at T > 0 (tests compare the forms): 0 the default
// (cluster-split streaming), 1 the CTA-per-row scalar kernel, 2 the cluster
// kernel holding the row on chip, 3 the CTA-per-row streaming kernel.  Draft
// sampling at T > 0 uses the streaming sampler when this is 0 or 3, the
// scalar kernel otherwise.
int g_accept_kernel = 0;
constexpr int kWarpsPerBlock = kSampleThreads / 32;

// ---------------------------------------------------------------- Philox4x32-10
struct U4 {
  uint32_t x, y, z, w;
};

__device__ __forceinline__ U4 philox4x32_10(U4 c, uint32_t k0, uint32_t k1) {
  const uint32_t M0 = 0xD2511F53u, M1 = 0xCD9E8D57u, W0 = 0x9E3779B9u, W1 = 0xBB67AE85u;
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r) {
      k0 += W0;
      k1 += W1;
    }
    const uint32_t hi0 = __umulhi(M0, c.x), lo0 = M0 * c.x;
    const uint32_t hi1 = __umulhi(M1, c.z), lo1 = M1 * c.z;
    c = U4{hi1 ^ c.y ^ k0, lo1, hi0 ^ c.w ^ k1, lo0};
  }
  return c;
}

__device__ __forceinline__ double words_to_unit(uint32_t hi, uint32_t lo) {
  const unsigned long long bits = ((unsigned long long)hi << 32) | lo;
  return (double)(bits >> 11) * 0x1.0p-53;
}

constexpr uint32_t kStreamTag = 0x53504543u;  // "SPEC"

__global__ void philox_kernel(uint64_t seed, const uint32_t* req_key, const int32_t* step, int rows, int n,
                              double* out) {
  const int pairs = (n + 1) / 2;
  const int64_t total = (int64_t)rows * pairs;
  for (int64_t e = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; e < total; e += (int64_t)gridDim.x * blockDim.x) {
    const int i = (int)(e / pairs), pr = (int)(e % pairs);
    U4 c{(uint32_t)pr, req_key[i], (uint32_t)step[i], kStreamTag};
    U4 w = philox4x32_10(c, (uint32_t)(seed & 0xffffffffu), (uint32_t)(seed >> 32));
    out[(int64_t)i * n + 2 * pr] = words_to_unit(w.x, w.y);
    if (2 * pr + 1 < n) out[(int64_t)i * n + 2 * pr + 1] = words_to_unit(w.z, w.w);
  }
}

// ---------------------------------------------------------------- block reductions
struct Scratch {
  float f[kWarpsPerBlock];
  double d[kWarpsPerBlock];
  int i[kWarpsPerBlock];
  float bf;
  double bd;
  int bi;
  int bi2;
  double run;
};

__device__ __forceinline__ float block_max(float v, Scratch& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max(v);
  if (lane == 0) sh.f[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float x = lane < kWarpsPerBlock ? sh.f[lane] : -INFINITY;
    x = warp_max(x);
    if (lane == 0) sh.bf = x;
  }
  __syncthreads();
  return sh.bf;
}

__device__ __forceinline__ double block_sum_d(double v, Scratch& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum_d(v);
  if (lane == 0) sh.d[warp] = v;
  __syncthreads();
  if (warp == 0) {
    double x = lane < kWarpsPerBlock ? sh.d[lane] : 0.0;
    x = warp_sum_d(x);
    if (lane == 0) sh.bd = x;
  }
  __syncthreads();
  return sh.bd;
}

__device__ __forceinline__ void argmax_combine(float& v, int& i, float ov, int oi) {
  // larger value wins; equal values -> lower index; NaN never wins
  if (ov > v || (ov == v && oi < i) || (v != v && ov == ov)) {
    v = ov;
    i = oi;
  }
}

__device__ __forceinline__ void argmax_step(float x, int e, float& bv, int& bi) {
  if (x > bv || (bi == INT_MAX && x == x)) {
    bv = x;
    bi = e;
  }
}

__device__ int block_argmax(const float* row, int V, Scratch& sh) {
  float bv = -INFINITY;
  int bi = INT_MAX;
  if ((V & 3) == 0 && (reinterpret_cast<uintptr_t>(row) & 15) == 0) {
    // 16-byte loads, four of them in flight per thread, candidates taken in
    // index order
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const int n4 = V >> 2;
    const int bd = blockDim.x;
    int e = threadIdx.x;
    for (; e + 3 * bd < n4; e += 4 * bd) {
      float4 a[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) a[q] = r4[e + q * bd];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int f = 4 * (e + q * bd);
        argmax_step(a[q].x, f, bv, bi);
        argmax_step(a[q].y, f + 1, bv, bi);
        argmax_step(a[q].z, f + 2, bv, bi);
        argmax_step(a[q].w, f + 3, bv, bi);
      }
    }
    for (; e < n4; e += blockDim.x) {
      const float4 a = r4[e];
      argmax_step(a.x, 4 * e, bv, bi);
      argmax_step(a.y, 4 * e + 1, bv, bi);
      argmax_step(a.z, 4 * e + 2, bv, bi);
      argmax_step(a.w, 4 * e + 3, bv, bi);
    }
  } else {
    for (int e = threadIdx.x; e < V; e += blockDim.x) argmax_step(row[e], e, bv, bi);
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    argmax_combine(bv, bi, ov, oi);
  }
  if (lane == 0) {
    sh.f[warp] = bv;
    sh.i[warp] = bi;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float v = sh.f[0];
    int i = sh.i[0];
    for (int w = 1; w < kWarpsPerBlock; ++w) argmax_combine(v, i, sh.f[w], sh.i[w]);
    sh.bi = i == INT_MAX ? 0 : i;
  }
  __syncthreads();
  return sh.bi;
}

// Softmax statistics of one logits row at temperature T: max of l/T and the
// fp64 sum of expf(l/T - max).
struct Stats {
  float m;
  double z;
};

__device__ Stats row_stats(const float* row, int V, float T, Scratch& sh) {
  float mx = -INFINITY;
  for (int e = threadIdx.x; e < V; e += blockDim.x) mx = fmaxf(mx, row[e] / T);
  mx = block_max(mx, sh);
  double z = 0.0;
  for (int e = threadIdx.x; e < V; e += blockDim.x) z += (double)expf(row[e] / T - mx);
  z = block_sum_d(z, sh);
  return Stats{mx, z};
}

// Inverse CDF over weights wf(i), i in [0, V), at threshold t = u * total.
// Warp w owns the contiguous segment [w*seg, (w+1)*seg); segment sums are
// prefixed in order and only the crossing segment is walked, 32 at a time.
template <class WF>
__device__ int block_icdf(const WF& wf, int V, double t, Scratch& sh) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int seg = ((V + kWarpsPerBlock - 1) / kWarpsPerBlock + 31) & ~31;
  const int lo = min(warp * seg, V), hi = min(lo + seg, V);
  double s = 0.0;
  int last = -1;
  for (int e = lo + lane; e < hi; e += 32) {
    const double w = wf(e);
    s += w;
    if (w > 0.0) last = e;
  }
  s = warp_sum_d(s);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
  if (lane == 0) {
    sh.d[warp] = s;
    sh.i[warp] = last;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    double run = 0.0;
    int found = -1, fallback = -1;
    for (int w = 0; w < kWarpsPerBlock; ++w) {
      if (sh.i[w] >= 0) fallback = sh.i[w];
      if (found < 0 && run + sh.d[w] > t) {
        found = w;
        break;
      }
      run += sh.d[w];
    }
    if (found < 0) {
      for (int w = 0; w < kWarpsPerBlock; ++w)
        if (sh.i[w] >= 0) fallback = sh.i[w];
    }
    sh.bi = found;
    sh.bi2 = fallback < 0 ? 0 : fallback;
    sh.run = run;
  }
  __syncthreads();
  const int found = sh.bi;
  if (found >= 0 && warp == found) {
    double run = sh.run;
    int result = -1;
    for (int base = lo; base < hi; base += 32) {
      const int e = base + lane;
      const double w = e < hi ? wf(e) : 0.0;
      const double incl = warp_inclusive_scan_d(w) + run;
      const unsigned hit = __ballot_sync(0xffffffffu, e < hi && incl > t);
      if (hit) {
        result = base + __ffs(hit) - 1;
        break;
      }
      run = __shfl_sync(0xffffffffu, incl, 31);
    }
    if (lane == 0) sh.bi2 = result >= 0 ? result : (sh.i[warp] >= 0 ? sh.i[warp] : sh.bi2);
  }
  __syncthreads();
  const int r = sh.bi2;
  __syncthreads();
  return r;
}

struct SoftmaxWeight {
  const float* row;
  float T, m;
  __device__ double operator()(int e) const { return (double)expf(row[e] / T - m); }
};

struct ResidualWeight {
  const float* p;
  const float* q;
  float T, mp, mq;
  double invp, invq;
  __device__ double operator()(int e) const {
    const double a = (double)expf(p[e] / T - mp) * invp;
    const double b = (double)expf(q[e] / T - mq) * invq;
    const double r = a - b;
    return r > 0.0 ? r : 0.0;
  }
};

// ---------------------------------------------------------------- draft sampling
__global__ void __launch_bounds__(kSampleThreads) sample_kernel(const float* logits, int64_t row_stride,
                                                                const int32_t* index, int V, float T, const double* u,
                                                                int64_t u_stride, int u_col, int32_t* out,
                                                                int64_t out_stride, int32_t* out2, int64_t out2_stride) {
  __shared__ Scratch sh;
  const int i = blockIdx.x;
  const float* row = logits + (int64_t)(index ? index[i] : i) * row_stride;
  int tok;
  if (T <= 0.f) {
    tok = block_argmax(row, V, sh);
  } else {
    const Stats st = row_stats(row, V, T, sh);
    const double t = u[(int64_t)i * u_stride + u_col] * st.z;
    tok = block_icdf(SoftmaxWeight{row, T, st.m}, V, t, sh);
  }
  if (threadIdx.x == 0) {
    out[(int64_t)i * out_stride] = tok;
    if (out2) out2[(int64_t)i * out2_stride] = tok;
  }
}

// ---------------------------------------------------------------- accept / resample
struct AcceptArgs {
  const float* target0;
  int64_t t0_stride;
  const int32_t* t0_index;
  const float* verify;
  int64_t v_row, v_pos;
  const float* draft0;
  int64_t d0_stride;
  const int32_t* d0_index;
  const float* draft_rest;
  int64_t dr_row, dr_pos;
  const int32_t* drafts;
  const double* u;
  int64_t u_stride;
  int k, V;
  float T;
  int32_t* tokens;
  int32_t* n_accepted;
  int32_t* final_token;
};

__device__ __forceinline__ const float* target_row(const AcceptArgs& a, int i, int j) {
  if (j == 0) return a.target0 + (int64_t)(a.t0_index ? a.t0_index[i] : i) * a.t0_stride;
  return a.verify + (int64_t)i * a.v_row + (int64_t)(j - 1) * a.v_pos;
}

__device__ __forceinline__ const float* draft_row(const AcceptArgs& a, int i, int j) {
  if (j == 0) return a.draft0 + (int64_t)(a.d0_index ? a.d0_index[i] : i) * a.d0_stride;
  return a.draft_rest + (int64_t)i * a.dr_row + (int64_t)(j - 1) * a.dr_pos;
}

__global__ void __launch_bounds__(kSampleThreads) accept_kernel(AcceptArgs a) {
  __shared__ Scratch sh;
  const int i = blockIdx.x;
  const int k = a.k, V = a.V;
  int32_t* toks = a.tokens + (int64_t)i * (k + 1);
  const int32_t* drafted = a.drafts + (int64_t)i * k;
  int n_acc = k, fin = -1;

  if (a.T <= 0.f) {
    // engine/speculative.py:146-155
    for (int j = 0; j <= k; ++j) {
      const int best = block_argmax(target_row(a, i, j), V, sh);
      if (j == k) {
        fin = best;
        break;
      }
      if (threadIdx.x == 0) toks[j] = best;
      if (drafted[j] != best) {
        n_acc = j;
        fin = best;
        break;
      }
    }
  } else {
    const double* u = a.u + (int64_t)i * a.u_stride;
    const float T = a.T;
    for (int j = 0; j < k; ++j) {
      // engine/speculative.py:133-142
      const float* p = target_row(a, i, j);
      const float* q = draft_row(a, i, j);
      const int x = drafted[j];
      const bool x_ok = x >= 0 && x < V;
      const Stats sp = row_stats(p, V, T, sh);
      const Stats sq = row_stats(q, V, T, sh);
      const double wpx = x_ok ? (double)expf(p[x] / T - sp.m) : 0.0;
      const double wqx = x_ok ? (double)expf(q[x] / T - sq.m) : 0.0;
      double prob = 0.0;
      if (wqx > 0.0) {
        const double ratio = (wpx * sq.z) / (wqx * sp.z);
        prob = ratio < 1.0 ? ratio : 1.0;
      }
      if (u[k + j] < prob) {
        if (threadIdx.x == 0) toks[j] = x;
        continue;
      }
      // engine/speculative.py:43-50
      const ResidualWeight rw{p, q, T, sp.m, sq.m, 1.0 / sp.z, 1.0 / sq.z};
      double R = 0.0;
      for (int e = threadIdx.x; e < V; e += blockDim.x) R += rw(e);
      R = block_sum_d(R, sh);
      int tok;
      if (R <= 0.0)
        tok = block_icdf(SoftmaxWeight{p, T, sp.m}, V, u[2 * k] * sp.z, sh);
      else
        tok = block_icdf(rw, V, u[2 * k] * R, sh);
      n_acc = j;
      fin = tok;
      break;
    }
    if (fin < 0) {
      // engine/speculative.py:143-144: every draft accepted -> bonus from p_k
      const float* p = target_row(a, i, k);
      const Stats sp = row_stats(p, V, T, sh);
      fin = block_icdf(SoftmaxWeight{p, T, sp.m}, V, u[2 * k] * sp.z, sh);
    }
  }
  if (threadIdx.x == 0) {
    toks[n_acc] = fin;
    for (int j = n_acc + 1; j <= k; ++j) toks[j] = -1;
    a.n_accepted[i] = n_acc;
    a.final_token[i] = fin;
  }
}

// ---------------------------------------------------------------- accept / resample, T > 0, one cluster per row
//
// A thread-block cluster of C CTAs (C = ceil(V / 16384) <= 8) owns one request
// row at a time.  The vocabulary is cut into C x 16 warp segments of 32 lane
// runs of `run_len` consecutive entries (a multiple of 4, at most 32).  A lane keeps its run of
// the current position's target logits in registers and of the draft logits
// in shared memory (16-byte cp.async, no register staging), so every logit is
// read from HBM once and the max / sum / residual passes of the rule run on
// chip.
//
// Cluster reductions: every warp stores its partial (max, sum, last nonzero
// index) straight into the mailbox of every CTA of the cluster (DSMEM
// stores), then one cluster barrier; each warp then reduces the C x 16
// partials from its own mailbox with the same fixed tree, so all CTAs hold
// bit-identical totals, take identical decisions and keep their barriers
// matched.  Mailboxes alternate between two slots: a slot is rewritten only
// two reductions later, after every CTA has passed the barrier that follows
// its reads of it.  Clusters are persistent over rows.
//
// Sums: a lane adds its run in index order; lanes, warps and CTAs combine by
// fixed trees.  The inverse CDF descends warp segment (scan over the C x 16
// segment sums) -> lane (scan over the warp's 32 run sums) -> entry (the
// lane's run, in order).

constexpr int kClThreads = 512;
constexpr int kClWarps = kClThreads / 32;
constexpr int kClRun = 32;                            // max entries per lane per vector
constexpr int kClCtaCap = kClWarps * 32 * kClRun;     // 16384 vocabulary entries per CTA
constexpr int kClMax = 8;                             // portable cluster size
constexpr int kClSegs = kClMax * kClWarps;            // warp segments per cluster (max)
constexpr int kClQStride = kClRun + 4;                // lane stride of the draft run in shared memory

struct Mail {
  float mx[2][kClSegs];     // maxima of s_p, s_q per warp segment
  double sum[2][kClSegs];   // sums of w_p, w_q (or the residual in [1]) per segment
  int last[2][kClSegs];     // last index of nonzero weight per segment
  double xw[2];             // w_p[x], w_q[x] from the lane that holds x
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of `p` (this CTA's shared memory) in the shared memory of cluster rank `rank`.
__device__ __forceinline__ uint32_t peer_addr(const void* p, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_u32(p)), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_peer(uint32_t a, float v) {
  asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}
__device__ __forceinline__ void st_peer(uint32_t a, double v) {
  asm volatile("st.shared::cluster.f64 [%0], %1;" ::"r"(a), "d"(v) : "memory");
}
__device__ __forceinline__ void st_peer(uint32_t a, int v) {
  asm volatile("st.shared::cluster.s32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}

__device__ __forceinline__ int warp_max_i(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = max(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

constexpr int kClG = kClSegs / 32;  // warp segments per lane in the descent (4)

// Exclusive prefix over lanes of per-lane totals, plus `run`.
__device__ __forceinline__ double lane_excl_prefix(double tot, double run) {
  const int lane = threadIdx.x & 31;
  const double incl = warp_inclusive_scan_d(tot);
  const double ex = __shfl_up_sync(0xffffffffu, incl, 1);
  return (lane == 0 ? 0.0 : ex) + run;
}

// Values v[0..G) of each lane, in lane-major order, form one sequence.  Finds
// the first element at which `run + prefix` exceeds t; returns its index
// (lane * G + j) and sets `run` to the prefix before it.  -1 (run unchanged)
// if none.  Uniform over the warp.
template <int G>
__device__ __forceinline__ int group_cross(const double (&v)[G], double t, double& run) {
  double tot = 0.0;
#pragma unroll
  for (int j = 0; j < G; ++j) tot += v[j];
  double acc = lane_excl_prefix(tot, run);
  int jh = -1;
  double before = 0.0;
#pragma unroll
  for (int j = 0; j < G; ++j) {
    if (jh < 0) {
      if (acc + v[j] > t) {
        jh = j;
        before = acc;
      } else {
        acc += v[j];
      }
    }
  }
  const unsigned m = __ballot_sync(0xffffffffu, jh >= 0);
  if (!m) return -1;
  const int l = __ffs(m) - 1;
  run = __shfl_sync(0xffffffffu, before, l);
  return l * G + __shfl_sync(0xffffffffu, jh, l);
}

__device__ __forceinline__ double resid(float wp, float wq, double invp, double invq) {
  // max(0, w_p / Z_p - w_q / Z_q) in fp64, products and difference rounded separately
  const double r = __dsub_rn(__dmul_rn((double)wp, invp), __dmul_rn((double)wq, invq));
  return r > 0.0 ? r : 0.0;
}

template <int C>
__global__ void __launch_bounds__(kClThreads, 1) accept_cluster_kernel(AcceptArgs a, int rows, int run_len) {
  __shared__ Mail box[2];
  extern __shared__ __align__(16) float q_all[];  // [kClThreads][kClQStride] draft runs
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rank = (int)cluster_ctarank();
  const int n_cl = (int)cluster_count_x();
  const int k = a.k, V = a.V;
  const float T = a.T;
  const int seg = 32 * run_len;                  // entries per warp segment
  const int n_seg = C * kClWarps;
  const int g = rank * kClWarps + warp;          // this warp's segment
  const int e_lane = g * seg + lane * run_len;   // first entry of this lane's run
  const int n4 = run_len >> 2;
  float* qs = q_all + threadIdx.x * kClQStride;
  float p[kClRun];
  int ph = 0;
  const uint32_t slot_bytes = sizeof(Mail);

  auto load_p = [&](const float* row) {
#pragma unroll
    for (int c = 0; c < kClRun / 4; ++c) {
      float4 v = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      if (c < n4 && e_lane + 4 * c < V) v = __ldcs(reinterpret_cast<const float4*>(row + e_lane + 4 * c));
      p[4 * c] = v.x;
      p[4 * c + 1] = v.y;
      p[4 * c + 2] = v.z;
      p[4 * c + 3] = v.w;
    }
  };
  auto load_q = [&](const float* row) {
#pragma unroll
    for (int c = 0; c < kClRun / 4; ++c) {
      if (c < n4) {
        const bool ok = e_lane + 4 * c < V;
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(qs + 4 * c)),
                     "l"(ok ? row + e_lane + 4 * c : row), "r"(ok ? 16 : 0)
                     : "memory");
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  for (int i = (int)cluster_id_x(); i < rows; i += n_cl) {
    const double* u = a.u + (int64_t)i * a.u_stride;
    const int32_t* drafted = a.drafts + (int64_t)i * k;
    int32_t* toks = a.tokens + (int64_t)i * (k + 1);
    load_q(draft_row(a, i, 0));
    load_p(target_row(a, i, 0));
    for (int j = 0; j <= k; ++j) {
      const bool bonus = j == k;  // every draft accepted: sample target[k]
      if (j > 0) {
        if (!bonus) load_q(draft_row(a, i, j));
        load_p(target_row(a, i, j));
      }
      // ---- maxima of s = l / T (s kept in place)
      float mp = -INFINITY, mq = -INFINITY;
#pragma unroll
      for (int c = 0; c < kClRun; ++c) {
        if (T != 1.0f) p[c] = p[c] / T;  // l / 1 is l: skip the division
        mp = fmaxf(mp, p[c]);
      }
      if (!bonus) {
        asm volatile("cp.async.wait_group 0;" ::: "memory");
#pragma unroll
        for (int c = 0; c < kClRun / 4; ++c) {
          if (c < n4) {
            float4 v = *reinterpret_cast<float4*>(qs + 4 * c);
            const bool ok = e_lane + 4 * c < V;
            if (T != 1.0f) {
              v.x = v.x / T;
              v.y = v.y / T;
              v.z = v.z / T;
              v.w = v.w / T;
            }
            if (!ok) v.x = v.y = v.z = v.w = -INFINITY;
            *reinterpret_cast<float4*>(qs + 4 * c) = v;
            mq = fmaxf(mq, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
          }
        }
      }
      mp = warp_max(mp);
      mq = warp_max(mq);
      if (lane < C) {
        const uint32_t b = peer_addr(&box[0], lane) + ph * slot_bytes;
        st_peer(b + (uint32_t)offsetof(Mail, mx[0][0]) + 4u * g, mp);
        st_peer(b + (uint32_t)offsetof(Mail, mx[1][0]) + 4u * g, mq);
      }
      cluster_sync_all();
      {
        const Mail& m = box[ph];
        float x0 = -INFINITY, y0 = -INFINITY;
#pragma unroll
        for (int jj = 0; jj < kClG; ++jj) {
          const int sg = kClG * lane + jj;
          if (sg < n_seg) {
            x0 = fmaxf(x0, m.mx[0][sg]);
            y0 = fmaxf(y0, m.mx[1][sg]);
          }
        }
        mp = warp_max(x0);
        mq = warp_max(y0);
      }
      ph ^= 1;
      // ---- weights w = expf(s - m) in place; run sums; last nonzero; w[x]
      const int x = bonus ? -1 : drafted[j];
      const bool x_ok = x >= 0 && x < V;
      double sp = 0.0, sq = 0.0;
      int lp = -1;
#pragma unroll
      for (int c = 0; c < kClRun; ++c) {
        const float wp = expf(p[c] - mp);
        p[c] = wp;
        sp += (double)wp;
        if (wp > 0.f) lp = e_lane + c;
      }
      if (!bonus) {
#pragma unroll
        for (int c = 0; c < kClRun / 4; ++c) {
          if (c < n4) {
            float4 v = *reinterpret_cast<float4*>(qs + 4 * c);
            v.x = expf(v.x - mq);
            v.y = expf(v.y - mq);
            v.z = expf(v.z - mq);
            v.w = expf(v.w - mq);
            *reinterpret_cast<float4*>(qs + 4 * c) = v;
            sq += (double)v.x;
            sq += (double)v.y;
            sq += (double)v.z;
            sq += (double)v.w;
          }
        }
      }
      // lane sums in lane order within the warp (fixed tree)
      const double sp_lane = sp;
      sp = warp_sum_d(sp);
      sq = warp_sum_d(sq);
      lp = warp_max_i(lp);
      const bool x_here = x_ok && x >= e_lane && x < e_lane + run_len;
      if (lane < C) {
        const uint32_t b = peer_addr(&box[0], lane) + ph * slot_bytes;
        st_peer(b + (uint32_t)offsetof(Mail, sum[0][0]) + 8u * g, sp);
        st_peer(b + (uint32_t)offsetof(Mail, sum[1][0]) + 8u * g, sq);
        st_peer(b + (uint32_t)offsetof(Mail, last[0][0]) + 4u * g, lp);
      }
      if (x_here) {
        const int c = x - e_lane;
        float wpx = 0.f;
#pragma unroll
        for (int c2 = 0; c2 < kClRun; ++c2)
          if (c2 == c) wpx = p[c2];
        const float wqx = qs[c];
        for (int r = 0; r < C; ++r) {
          const uint32_t b = peer_addr(&box[0], r) + ph * slot_bytes;
          st_peer(b + (uint32_t)offsetof(Mail, xw[0]), (double)wpx);
          st_peer(b + (uint32_t)offsetof(Mail, xw[1]), (double)wqx);
        }
      }
      cluster_sync_all();
      // segment sums stay in registers for the descent (lane l: segments kClG*l ..)
      double segp[kClG];
      int lastseg[kClG];
      int last_p = -1;
      double wpx = 0.0, wqx = 0.0;
      double Zp = 0.0, Zq = 0.0;
      {
        const Mail& m = box[ph];
#pragma unroll
        for (int jj = 0; jj < kClG; ++jj) {
          const int sg = kClG * lane + jj;
          segp[jj] = sg < n_seg ? m.sum[0][sg] : 0.0;
          lastseg[jj] = sg < n_seg ? m.last[0][sg] : -1;
          Zp += segp[jj];
          Zq += sg < n_seg ? m.sum[1][sg] : 0.0;
          last_p = max(last_p, lastseg[jj]);
        }
        last_p = warp_max_i(last_p);
        if (x_ok) {
          wpx = m.xw[0];
          wqx = m.xw[1];
        }
      }
      ph ^= 1;
      Zp = warp_sum_d(Zp);
      Zq = warp_sum_d(Zq);
      bool use_resid = false;
      double t = 0.0, invp = 0.0, invq = 0.0;
      double sr_lane = 0.0;
      int n_acc = k;
      if (!bonus) {
        // engine/speculative.py:133-142
        double prob = 0.0;
        if (x_ok && wqx > 0.0) {
          const double ratio = __ddiv_rn(__dmul_rn(wpx, Zq), __dmul_rn(wqx, Zp));
          prob = ratio < 1.0 ? ratio : 1.0;
        }
        if (u[k + j] < prob) {
          if (rank == 0 && threadIdx.x == 0) toks[j] = x;
          continue;
        }
        // engine/speculative.py:43-50: residual max(0, p - q), or p if it is empty
        n_acc = j;
        invp = 1.0 / Zp;
        invq = 1.0 / Zq;
        int lr = -1;
#pragma unroll
        for (int c4 = 0; c4 < kClRun / 4; ++c4) {
          if (c4 < n4) {
            const float4 w4 = *reinterpret_cast<const float4*>(qs + 4 * c4);
            const float wq4[4] = {w4.x, w4.y, w4.z, w4.w};
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
              const double r = resid(p[4 * c4 + cc], wq4[cc], invp, invq);
              sr_lane += r;
              if (r > 0.0) lr = e_lane + 4 * c4 + cc;
            }
          }
        }
        const double sr = warp_sum_d(sr_lane);
        lr = warp_max_i(lr);
        if (lane < C) {
          const uint32_t b = peer_addr(&box[0], lane) + ph * slot_bytes;
          st_peer(b + (uint32_t)offsetof(Mail, sum[1][0]) + 8u * g, sr);
          st_peer(b + (uint32_t)offsetof(Mail, last[1][0]) + 4u * g, lr);
        }
        cluster_sync_all();
        double segr[kClG];
        int lastr_seg[kClG];
        int last_r = -1;
        double R = 0.0;
        {
          const Mail& m = box[ph];
#pragma unroll
          for (int jj = 0; jj < kClG; ++jj) {
            const int sg = kClG * lane + jj;
            segr[jj] = sg < n_seg ? m.sum[1][sg] : 0.0;
            lastr_seg[jj] = sg < n_seg ? m.last[1][sg] : -1;
            R += segr[jj];
            last_r = max(last_r, lastr_seg[jj]);
          }
          last_r = warp_max_i(last_r);
        }
        ph ^= 1;
        R = warp_sum_d(R);
        if (R > 0.0) {
          use_resid = true;
          t = u[2 * k] * R;
#pragma unroll
          for (int jj = 0; jj < kClG; ++jj) {  // descend over the residual sums
            segp[jj] = segr[jj];
            lastseg[jj] = lastr_seg[jj];
          }
          last_p = last_r;
        }
      }
      if (!use_resid) t = u[2 * k] * Zp;
      // ---- inverse CDF: warp segment -> lane run -> entry
      double run = 0.0;
      const int g_hit = group_cross<kClG>(segp, t, run);
      int fin = last_p >= 0 ? last_p : 0;  // fallback: last entry of nonzero weight
      const int writer = g_hit >= 0 ? g_hit : 0;  // the segment whose lane 0 writes the row
      if (g_hit >= 0) {
        // the hit segment's last nonzero entry, in case rounding leaves no crossing inside it
        int ls = -1;
#pragma unroll
        for (int jj = 0; jj < kClG; ++jj)
          if (jj == g_hit % kClG) ls = lastseg[jj];
        ls = __shfl_sync(0xffffffffu, ls, g_hit / kClG);
        if (ls >= 0) fin = ls;
      }
      if (g == writer) {
        if (g_hit >= 0) {
          const double mine[1] = {use_resid ? sr_lane : sp_lane};
          const int l_hit = group_cross<1>(mine, t, run);
          int found = -1;
          if (l_hit >= 0 && lane == l_hit) {
            double acc = run;
#pragma unroll
            for (int c = 0; c < kClRun; ++c) {
              if (found < 0 && c < run_len && e_lane + c < V) {
                acc += use_resid ? resid(p[c], qs[c], invp, invq) : (double)p[c];
                if (acc > t) found = e_lane + c;
              }
            }
          }
          found = warp_max_i(found);
          if (found >= 0) fin = found;
        }
        if (lane == 0) {
          toks[n_acc] = fin;
          for (int jj = n_acc + 1; jj <= k; ++jj) toks[jj] = -1;
          a.n_accepted[i] = n_acc;
          a.final_token[i] = fin;
        }
      }
      break;  // the row is finished (rejection or bonus)
    }
  }
  // no CTA leaves while a peer may still store into or read its mailbox
  cluster_sync_all();
}

template <int C>
int launch_accept_cluster(const AcceptArgs& a, int rows, int run_len, cudaStream_t stream) {
  static int max_clusters[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
  const size_t smem = (size_t)kClThreads * kClQStride * sizeof(float);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kClThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (max_clusters[dev] == 0) {
    if (cudaFuncSetAttribute(accept_cluster_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
        cudaSuccess) {
      cudaGetLastError();
      return -1;
    }
    int sms = kNumSMs;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cfg.gridDim = dim3((unsigned)(C * (sms / C)), 1, 1);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, accept_cluster_kernel<C>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      return -1;
    }
    max_clusters[dev] = n;
  }
  const int n_cl = rows < max_clusters[dev] ? rows : max_clusters[dev];
  cfg.gridDim = dim3((unsigned)(C * n_cl), 1, 1);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, accept_cluster_kernel<C>, a, rows, run_len);
  return e == cudaSuccess ? 0 : (int)e;
}

// ---------------------------------------------------------------- accept / resample, T > 0, one CTA per row, L2-resident
//
// One CTA of 1024 threads owns a request row at a time; CTAs are persistent and
// at most ACCEPT_ROWS_IN_FLIGHT rows are worked on at once, so the rows being
// worked on (about 1 MB each at vocab 128k: target + draft) stay in L2.  The
// first pass over a position (maxima) streams from HBM; the exp / sum pass, the
// residual pass and the inverse-CDF walk re-read from L2 (ld.global.cg), so
// each needed logit crosses HBM once.  Reductions are CTA-local.
//
// Layout: warp w owns the vocabulary segment [w*seg, (w+1)*seg), seg a
// multiple of 128; its lanes read it as consecutive 128-entry rows, lane l
// taking entries 4l..4l+3 of each row with one 16-byte load (coalesced).
// Index order inside a segment is (row, lane, component).  Sums: a lane adds
// its entries in index order, warps combine by butterfly, the CTA adds its 32
// warp sums in warp order.  The inverse CDF descends warp segment (in order)
// -> 128-entry row (warp scan of the lanes' 4-entry sums) -> entry.

#ifndef PSE_ACCEPT_ROWS_IN_FLIGHT
#define PSE_ACCEPT_ROWS_IN_FLIGHT 148
#endif

constexpr int kStThreads = 1024;
constexpr int kStWarps = kStThreads / 32;

struct StShared {
  float wm[2][kStWarps];
  double ws[2][kStWarps];
  int wl[2][kStWarps];
  double xw[2];
  float m[2];
  double z[2];
  int last[2];
  double cross_run;
  int cross_warp;
};

__device__ __forceinline__ float4 ld_l2(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ float4 scale_s(float4 v, float T) {
  if (T != 1.0f) {  // l / 1 is l
    v.x = v.x / T;
    v.y = v.y / T;
    v.z = v.z / T;
    v.w = v.w / T;
  }
  return v;
}

__device__ __forceinline__ float4 weights4(float4 l, float T, float m) {
  const float4 sv = scale_s(l, T);
  return make_float4(expf(sv.x - m), expf(sv.y - m), expf(sv.z - m), expf(sv.w - m));
}

// CTA reduction of two per-warp values already stored in sh.ws / sh.wl (lane 0
// of every warp wrote them): ordered sums and max of the last-nonzero indices.
__device__ __forceinline__ void st_reduce_sums(StShared& sh, int n) {
  if (threadIdx.x == 0) {
    for (int v = 0; v < n; ++v) {
      double z = 0.0;
      int last = -1;
      for (int w = 0; w < kStWarps; ++w) {
        z += sh.ws[v][w];
        last = max(last, sh.wl[v][w]);
      }
      sh.z[v] = z;
      sh.last[v] = last;
    }
  }
}

__global__ void __launch_bounds__(kStThreads, 1) accept_stream_kernel(AcceptArgs a, int rows, int seg) {
  __shared__ StShared sh;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int V = a.V, k = a.k;
  const float T = a.T;
  const int e_w = warp * seg;  // this warp's segment
  const int n_c = seg >> 7;    // 128-entry rows in a segment
  for (int i = blockIdx.x; i < rows; i += gridDim.x) {
    const double* u = a.u + (int64_t)i * a.u_stride;
    const int32_t* drafted = a.drafts + (int64_t)i * k;
    int32_t* toks = a.tokens + (int64_t)i * (k + 1);
    for (int j = 0; j <= k; ++j) {
      const bool bonus = j == k;  // every draft accepted: sample target[k]
      const float* P = target_row(a, i, j);
      const float* Q = bonus ? P : draft_row(a, i, j);
      // ---- maxima of s = l / T
      float mp = -INFINITY, mq = -INFINITY;
#pragma unroll 4
      for (int c = 0; c < n_c; ++c) {
        const int e = e_w + c * 128 + lane * 4;
        if (e < V) {
          const float4 sp = scale_s(ld_l2(P + e), T);
          mp = fmaxf(mp, fmaxf(fmaxf(sp.x, sp.y), fmaxf(sp.z, sp.w)));
          if (!bonus) {
            const float4 sq = scale_s(ld_l2(Q + e), T);
            mq = fmaxf(mq, fmaxf(fmaxf(sq.x, sq.y), fmaxf(sq.z, sq.w)));
          }
        }
      }
      mp = warp_max(mp);
      mq = warp_max(mq);
      if (lane == 0) {
        sh.wm[0][warp] = mp;
        sh.wm[1][warp] = mq;
      }
      __syncthreads();
      if (warp == 0) {
        const float x = warp_max(sh.wm[0][lane]);
        const float y = warp_max(sh.wm[1][lane]);
        if (lane == 0) {
          sh.m[0] = x;
          sh.m[1] = y;
        }
      }
      __syncthreads();
      mp = sh.m[0];
      mq = sh.m[1];
      // ---- weights: sums, last nonzero, w[x]
      const int x = bonus ? -1 : drafted[j];
      const bool x_ok = x >= 0 && x < V;
      double zp = 0.0, zq = 0.0;
      int lp = -1;
#pragma unroll 4
      for (int c = 0; c < n_c; ++c) {
        const int e = e_w + c * 128 + lane * 4;
        if (e < V) {
          const float4 wp = weights4(ld_l2(P + e), T, mp);
          zp += (double)wp.x;
          zp += (double)wp.y;
          zp += (double)wp.z;
          zp += (double)wp.w;
          if (wp.w > 0.f) lp = e + 3;
          else if (wp.z > 0.f) lp = e + 2;
          else if (wp.y > 0.f) lp = e + 1;
          else if (wp.x > 0.f) lp = e;
          if (!bonus) {
            const float4 wq = weights4(ld_l2(Q + e), T, mq);
            zq += (double)wq.x;
            zq += (double)wq.y;
            zq += (double)wq.z;
            zq += (double)wq.w;
            if (x_ok && x >= e && x < e + 4) {
              const int q = x - e;
              sh.xw[0] = (double)(q == 0 ? wp.x : q == 1 ? wp.y : q == 2 ? wp.z : wp.w);
              sh.xw[1] = (double)(q == 0 ? wq.x : q == 1 ? wq.y : q == 2 ? wq.z : wq.w);
            }
          }
        }
      }
      zp = warp_sum_d(zp);
      zq = warp_sum_d(zq);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) lp = max(lp, __shfl_xor_sync(0xffffffffu, lp, o));
      if (lane == 0) {
        sh.ws[0][warp] = zp;
        sh.ws[1][warp] = zq;
        sh.wl[0][warp] = lp;
        sh.wl[1][warp] = -1;
      }
      __syncthreads();
      st_reduce_sums(sh, 2);
      __syncthreads();
      const double Zp = sh.z[0], Zq = sh.z[1];
      int n_acc = k;
      bool use_resid = false;
      double t, invp = 0.0, invq = 0.0;
      if (!bonus) {
        // engine/speculative.py:133-142
        const double wpx = x_ok ? sh.xw[0] : 0.0, wqx = x_ok ? sh.xw[1] : 0.0;
        double prob = 0.0;
        if (x_ok && wqx > 0.0) {
          const double ratio = __ddiv_rn(__dmul_rn(wpx, Zq), __dmul_rn(wqx, Zp));
          prob = ratio < 1.0 ? ratio : 1.0;
        }
        if (u[k + j] < prob) {
          if (threadIdx.x == 0) toks[j] = x;
          continue;
        }
        // engine/speculative.py:43-50: residual max(0, p - q), or p if it is empty
        n_acc = j;
        invp = 1.0 / Zp;
        invq = 1.0 / Zq;
        double zr = 0.0;
        int lr = -1;
#pragma unroll 4
        for (int c = 0; c < n_c; ++c) {
          const int e = e_w + c * 128 + lane * 4;
          if (e < V) {
            const float4 wp = weights4(ld_l2(P + e), T, mp);
            const float4 wq = weights4(ld_l2(Q + e), T, mq);
            const double r0 = resid(wp.x, wq.x, invp, invq), r1 = resid(wp.y, wq.y, invp, invq);
            const double r2 = resid(wp.z, wq.z, invp, invq), r3 = resid(wp.w, wq.w, invp, invq);
            zr += r0;
            zr += r1;
            zr += r2;
            zr += r3;
            if (r3 > 0.0) lr = e + 3;
            else if (r2 > 0.0) lr = e + 2;
            else if (r1 > 0.0) lr = e + 1;
            else if (r0 > 0.0) lr = e;
          }
        }
        zr = warp_sum_d(zr);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) lr = max(lr, __shfl_xor_sync(0xffffffffu, lr, o));
        if (lane == 0) {
          sh.ws[1][warp] = zr;  // draft sums are done with: the residual's go here
          sh.wl[1][warp] = lr;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
          double z = 0.0;
          int last = -1;
          for (int w = 0; w < kStWarps; ++w) {
            z += sh.ws[1][w];
            last = max(last, sh.wl[1][w]);
          }
          sh.z[1] = z;
          sh.last[1] = last;
        }
        __syncthreads();
        use_resid = sh.z[1] > 0.0;
      }
      const int v = use_resid ? 1 : 0;
      t = u[2 * k] * sh.z[v];
      // ---- inverse CDF: warp segment -> 128-entry row -> entry
      if (threadIdx.x == 0) {
        double run = 0.0;
        int hit = -1;
        for (int w = 0; w < kStWarps; ++w) {
          if (run + sh.ws[v][w] > t) {
            hit = w;
            break;
          }
          run += sh.ws[v][w];
        }
        sh.cross_warp = hit;
        sh.cross_run = run;
      }
      __syncthreads();
      const int w_hit = sh.cross_warp;
      const int last_all = sh.last[v];
      if (w_hit < 0) {
        if (threadIdx.x == 0) {  // rounding left no crossing: the last entry of nonzero weight
          const int fin = last_all >= 0 ? last_all : 0;
          toks[n_acc] = fin;
          for (int jj = n_acc + 1; jj <= k; ++jj) toks[jj] = -1;
          a.n_accepted[i] = n_acc;
          a.final_token[i] = fin;
        }
      } else if (warp == w_hit) {
        double run = sh.cross_run;
        int found = -1;
        for (int c = 0; c < n_c && found < 0; ++c) {
          const int e = e_w + c * 128 + lane * 4;
          double w4[4] = {0.0, 0.0, 0.0, 0.0};
          if (e < V) {
            const float4 wp = weights4(ld_l2(P + e), T, mp);
            if (use_resid) {
              const float4 wq = weights4(ld_l2(Q + e), T, mq);
              w4[0] = resid(wp.x, wq.x, invp, invq);
              w4[1] = resid(wp.y, wq.y, invp, invq);
              w4[2] = resid(wp.z, wq.z, invp, invq);
              w4[3] = resid(wp.w, wq.w, invp, invq);
            } else {
              w4[0] = wp.x;
              w4[1] = wp.y;
              w4[2] = wp.z;
              w4[3] = wp.w;
            }
          }
          const double mine = ((w4[0] + w4[1]) + w4[2]) + w4[3];
          const double incl = warp_inclusive_scan_d(mine) + run;
          const unsigned hit = __ballot_sync(0xffffffffu, incl > t);
          if (hit) {
            const int l = __ffs(hit) - 1;
            if (lane == l) {
              double acc = incl - mine;
              for (int q = 0; q < 4 && found < 0; ++q) {
                acc += w4[q];
                if (acc > t) found = e + q;
              }
              if (found < 0) {  // rounding: the lane's last entry of nonzero weight
                for (int q = 3; q >= 0 && found < 0; --q)
                  if (w4[q] > 0.0) found = e + q;
              }
            }
            found = __shfl_sync(0xffffffffu, found, l);
            if (found < 0) found = sh.wl[v][warp] >= 0 ? sh.wl[v][warp] : (last_all >= 0 ? last_all : 0);
          }
          run = __shfl_sync(0xffffffffu, incl, 31);
        }
        if (found < 0) found = sh.wl[v][warp] >= 0 ? sh.wl[v][warp] : (last_all >= 0 ? last_all : 0);
        if (lane == 0) {
          toks[n_acc] = found;
          for (int jj = n_acc + 1; jj <= k; ++jj) toks[jj] = -1;
          a.n_accepted[i] = n_acc;
          a.final_token[i] = found;
        }
      }
      __syncthreads();  // sh is rewritten by the next row
      break;            // the row is finished (rejection or bonus)
    }
  }
}

// ---------------------------------------------------------------- accept / resample, T > 0, cluster-split streaming
//
// A cluster of C CTAs (C = min(8, ceil(V / 8192))) owns one request row at a
// time and several clusters share each SM (256-thread CTAs), so the
// reductions and barriers of one cluster overlap the loads of another.  CTA r
// of a cluster owns the vocabulary chunk [r * chunk, (r + 1) * chunk), cut
// into 8 warp segments of `seg` entries (a multiple of 128); a warp reads its
// segment as 128-entry rows, lane l taking entries 4l..4l+3 with one 16-byte
// load, four rows' loads issued before their arithmetic.  Per position:
//   1. one read from HBM (ld.global.cg, cached in L2 only) of the target (P)
//      and draft (Q) logits: maxima of s = l / T and the segment sums of
//      w = expf(s - m), kept against each lane's running maximum and moved to
//      the row's maximum M in fp64 (online softmax); every thread reads the
//      drafted token's two logits itself (one broadcast load per warp) for
//      the accept test, with w = expf(s - M);
//   2. after a rejection, fp64 segment sums of the residual (re-read from L2)
//      with w = expf(s - M);
//   3. inverse CDF: every warp finds the crossing segment from the segment
//      sums (none: the last segment holding a nonzero entry, scanned with no
//      threshold); that segment's warp re-reads and scans it, remembering
//      its last nonzero entry for the no-crossing case.
// The normalisers differ from sums of the expf(s - M) weights only by
// rounding (the weights of one row agree with the fp64-exact ones to an ulp
// either way); draws and accept decisions are those of the fp64 definition
// except where a uniform lies within that rounding of a boundary.
// The clusters in flight are capped so that their rows (2 x V x 4 bytes each)
// stay within kSpL2Budget of L2: every re-read hits L2 (ncu: DRAM reads 1.11x
// the needed bytes at vocab 128256).
//
// Every warp stores its segment's partial into the mailbox of every CTA of
// the cluster (DSMEM) before one cluster barrier; each warp then reduces the
// mailbox with the same fixed tree, so all CTAs hold bit-identical totals,
// take identical decisions and keep their barriers matched.  Mailboxes
// alternate between two slots: a slot is rewritten two reductions later,
// after every CTA has passed the barrier that follows its reads of it.
//
// Sums: a lane adds its entries in index order; lanes combine by butterfly;
// segment sums combine in lane-major order (2 segments per lane).

constexpr int kSpThreads = 256;
constexpr int kSpWarps = kSpThreads / 32;
constexpr int kSpMaxC = 8;                     // portable cluster size
constexpr int kSpSegs = kSpMaxC * kSpWarps;    // warp segments per row, at most
constexpr int kSpG = kSpSegs / 32;             // segments per lane in the descent
constexpr int kSpBatch = 4;                    // 128-entry rows loaded before their arithmetic
constexpr size_t kSpL2Budget = 96u << 20;      // bytes of logits rows in flight

struct SpMail {
  float mx[2][kSpSegs];    // maxima of s_p, s_q per segment
  double sum[3][kSpSegs];  // sums of w_p, w_q, residual per segment
};

__device__ __forceinline__ float4 neg_inf4() { return make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY); }

// Online softmax sums.  A sum z of exp(s_i - m) is kept against a running
// maximum m; when a batch raises the maximum to c, z is multiplied by
// exp(m - c) in fp64 (rare: a handful of times per lane and row for
// unordered logits).  Four weights are added in fp32 and the group in fp64.
template <int B>
__device__ __forceinline__ void online_add(const float4 (&s)[B], float& m, double& z) {
  float c = m;
#pragma unroll
  for (int b = 0; b < B; ++b) c = fmaxf(c, fmaxf(fmaxf(s[b].x, s[b].y), fmaxf(s[b].z, s[b].w)));
  if (c > m) {
    if (z > 0.0) z *= exp((double)m - (double)c);
    m = c;
  }
  if (m == -INFINITY) return;  // nothing but pads so far
#pragma unroll
  for (int b = 0; b < B; ++b) {
    const float4 w = make_float4(expf(s[b].x - m), expf(s[b].y - m), expf(s[b].z - m), expf(s[b].w - m));
    z += (double)((w.x + w.y) + (w.z + w.w));
  }
}

// z (kept against m) moved to the maximum M >= m.
__device__ __forceinline__ double rescaled(double z, float m, float M) {
  return z > 0.0 && m != M ? z * exp((double)m - (double)M) : z;
}

// Lanes' (m, z) pairs combined: every lane gets the warp's maximum and sum.
__device__ __forceinline__ void online_warp(float& m, double& z) {
  const float M = warp_max(m);
  z = warp_sum_d(rescaled(z, m, M));
  m = M;
}

template <int C>
__global__ void __launch_bounds__(kSpThreads, 4) accept_split_kernel(AcceptArgs a, int rows, int seg) {
  __shared__ SpMail box[2];
  constexpr int n_seg = C * kSpWarps;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int rank = (int)cluster_ctarank();
  const int n_cl = (int)cluster_count_x();
  const int k = a.k, V = a.V;
  const float T = a.T;
  const int g = rank * kSpWarps + warp;  // this warp's segment
  const int e0 = g * seg + lane * 4;     // this lane's first entry
  const int n_c = seg >> 7;              // 128-entry rows per segment
  int ph = 0;

  for (int i = (int)cluster_id_x(); i < rows; i += n_cl) {
    const double* u = a.u + (int64_t)i * a.u_stride;
    const int32_t* drafted = a.drafts + (int64_t)i * k;
    int32_t* toks = a.tokens + (int64_t)i * (k + 1);
    for (int j = 0; j <= k; ++j) {
      const bool bonus = j == k;  // every draft accepted: sample target[k]
      const float* P = target_row(a, i, j);
      const float* Q = bonus ? P : draft_row(a, i, j);
      // ---- 1. one pass from HBM: maxima of s = l / T and sums of exp(s - max),
      //      kept against a running maximum and rescaled when it grows; the
      //      drafted token's two logits (one broadcast load per warp)
      const int x = bonus ? -1 : drafted[j];
      const bool x_ok = x >= 0 && x < V;
      float lpx = 0.f, lqx = 0.f;
      if (x_ok) {
        lpx = __ldcg(P + x);
        lqx = __ldcg(Q + x);
      }
      float mp = -INFINITY, mq = -INFINITY;
      double sp = 0.0, sq = 0.0;
      for (int c0 = 0; c0 < n_c; c0 += kSpBatch) {
        float4 sp4[kSpBatch], sq4[kSpBatch];
#pragma unroll
        for (int b = 0; b < kSpBatch; ++b) {
          const int e = e0 + (c0 + b) * 128;
          const bool ok = c0 + b < n_c && e < V;  // -inf pads weigh 0
          sp4[b] = ok ? scale_s(ld_l2(P + e), T) : neg_inf4();
          sq4[b] = ok && !bonus ? scale_s(ld_l2(Q + e), T) : neg_inf4();
        }
        online_add<kSpBatch>(sp4, mp, sp);
        if (!bonus) online_add<kSpBatch>(sq4, mq, sq);
      }
      online_warp(mp, sp);
      online_warp(mq, sq);
      if (lane < C) {
        const uint32_t b = peer_addr(&box[ph], lane);
        st_peer(b + (uint32_t)offsetof(SpMail, mx[0][0]) + 4u * g, mp);
        st_peer(b + (uint32_t)offsetof(SpMail, mx[1][0]) + 4u * g, mq);
        st_peer(b + (uint32_t)offsetof(SpMail, sum[0][0]) + 8u * g, sp);
        st_peer(b + (uint32_t)offsetof(SpMail, sum[1][0]) + 8u * g, sq);
      }
      cluster_sync_all();
      double segv[kSpG];  // segment sums of the distribution the draw descends
      double Zp = 0.0, Zq = 0.0;
      {
        const SpMail& m = box[ph];
        float x0 = -INFINITY, y0 = -INFINITY;
#pragma unroll
        for (int jj = 0; jj < kSpG; ++jj) {
          const int sg = kSpG * lane + jj;
          if (sg < n_seg) {
            x0 = fmaxf(x0, m.mx[0][sg]);
            y0 = fmaxf(y0, m.mx[1][sg]);
          }
        }
        mp = warp_max(x0);
        mq = warp_max(y0);
        // every segment's sum moved to the row's maximum, in fixed order
#pragma unroll
        for (int jj = 0; jj < kSpG; ++jj) {
          const int sg = kSpG * lane + jj;
          segv[jj] = sg < n_seg ? rescaled(m.sum[0][sg], m.mx[0][sg], mp) : 0.0;
          Zp += segv[jj];
          Zq += sg < n_seg ? rescaled(m.sum[1][sg], m.mx[1][sg], mq) : 0.0;
        }
      }
      ph ^= 1;
      Zp = warp_sum_d(Zp);
      Zq = warp_sum_d(Zq);
      int n_acc = k;
      bool use_resid = false;
      double invp = 0.0, invq = 0.0, R = 0.0;
      if (!bonus) {
        // engine/speculative.py:133-142
        double prob = 0.0;
        if (x_ok) {
          const double wpx = (double)expf((T != 1.0f ? lpx / T : lpx) - mp);
          const double wqx = (double)expf((T != 1.0f ? lqx / T : lqx) - mq);
          if (wqx > 0.0) {
            const double ratio = __ddiv_rn(__dmul_rn(wpx, Zq), __dmul_rn(wqx, Zp));
            prob = ratio < 1.0 ? ratio : 1.0;
          }
        }
        if (u[k + j] < prob) {
          if (rank == 0 && threadIdx.x == 0) toks[j] = x;
          continue;
        }
        // engine/speculative.py:43-50: residual max(0, p - q), or p if it is empty
        n_acc = j;
        invp = 1.0 / Zp;
        invq = 1.0 / Zq;
        // ---- 2. residual segment sums
        double sr = 0.0;
        for (int c0 = 0; c0 < n_c; c0 += kSpBatch) {
          float4 lp4[kSpBatch], lq4[kSpBatch];
#pragma unroll
          for (int b = 0; b < kSpBatch; ++b) {
            const int e = e0 + (c0 + b) * 128;
            const bool ok = c0 + b < n_c && e < V;
            lp4[b] = ok ? ld_l2(P + e) : neg_inf4();
            lq4[b] = ok ? ld_l2(Q + e) : neg_inf4();
          }
#pragma unroll
          for (int b = 0; b < kSpBatch; ++b) {
            const float4 wp = weights4(lp4[b], T, mp);
            const float4 wq = weights4(lq4[b], T, mq);
            sr += resid(wp.x, wq.x, invp, invq);
            sr += resid(wp.y, wq.y, invp, invq);
            sr += resid(wp.z, wq.z, invp, invq);
            sr += resid(wp.w, wq.w, invp, invq);
          }
        }
        sr = warp_sum_d(sr);
        if (lane < C) {
          const uint32_t b = peer_addr(&box[ph], lane);
          st_peer(b + (uint32_t)offsetof(SpMail, sum[2][0]) + 8u * g, sr);
        }
        cluster_sync_all();
        double segr[kSpG];
        {
          const SpMail& m = box[ph];
#pragma unroll
          for (int jj = 0; jj < kSpG; ++jj) {
            const int sg = kSpG * lane + jj;
            segr[jj] = sg < n_seg ? m.sum[2][sg] : 0.0;
            R += segr[jj];
          }
        }
        ph ^= 1;
        R = warp_sum_d(R);
        if (R > 0.0) {
          use_resid = true;
#pragma unroll
          for (int jj = 0; jj < kSpG; ++jj) segv[jj] = segr[jj];
        }
      }
      // ---- 3. inverse CDF: segment -> 128-entry row -> entry
      double t = u[2 * k] * (use_resid ? R : Zp);
      double run = 0.0;
      int g_scan = group_cross<kSpG>(segv, t, run);
      if (g_scan < 0) {
        // rounding left no crossing: the last entry of nonzero weight, found
        // in the last segment whose sum is nonzero (sums of nonnegative terms)
        int ls = -1;
#pragma unroll
        for (int jj = 0; jj < kSpG; ++jj)
          if (segv[jj] > 0.0) ls = kSpG * lane + jj;
        g_scan = warp_max_i(ls);
        t = INFINITY;
      }
      if (g == (g_scan >= 0 ? g_scan : 0)) {  // one warp of the cluster finishes the row
        int found = -1, last_nz = -1;
        if (g_scan >= 0) {
          for (int c = 0; c < n_c && found < 0; ++c) {
            const int e = e0 + c * 128;
            double v0 = 0.0, v1 = 0.0, v2 = 0.0, v3 = 0.0;
            if (e < V) {
              const float4 wp = weights4(ld_l2(P + e), T, mp);
              if (use_resid) {
                const float4 wq = weights4(ld_l2(Q + e), T, mq);
                v0 = resid(wp.x, wq.x, invp, invq);
                v1 = resid(wp.y, wq.y, invp, invq);
                v2 = resid(wp.z, wq.z, invp, invq);
                v3 = resid(wp.w, wq.w, invp, invq);
              } else {
                v0 = wp.x;
                v1 = wp.y;
                v2 = wp.z;
                v3 = wp.w;
              }
            }
            const double incl = warp_inclusive_scan_d(((v0 + v1) + v2) + v3);
            const double ex = __shfl_up_sync(0xffffffffu, incl, 1);
            double acc = run + (lane == 0 ? 0.0 : ex);
            int f = -1, lz = -1;
            acc += v0;
            if (v0 > 0.0) {
              lz = e;
              if (acc > t) f = e;
            }
            acc += v1;
            if (v1 > 0.0) {
              lz = e + 1;
              if (f < 0 && acc > t) f = e + 1;
            }
            acc += v2;
            if (v2 > 0.0) {
              lz = e + 2;
              if (f < 0 && acc > t) f = e + 2;
            }
            acc += v3;
            if (v3 > 0.0) {
              lz = e + 3;
              if (f < 0 && acc > t) f = e + 3;
            }
            const unsigned hit = __ballot_sync(0xffffffffu, f >= 0);
            if (hit) found = __shfl_sync(0xffffffffu, f, __ffs(hit) - 1);
            last_nz = max(last_nz, warp_max_i(lz));
            run += __shfl_sync(0xffffffffu, incl, 31);
          }
        }
        // no crossing inside the hit segment (rounding): its last nonzero entry
        const int fin = found >= 0 ? found : (last_nz >= 0 ? last_nz : 0);
        if (lane == 0) {
          toks[n_acc] = fin;
          for (int jj = n_acc + 1; jj <= k; ++jj) toks[jj] = -1;
          a.n_accepted[i] = n_acc;
          a.final_token[i] = fin;
        }
      }
      break;  // the row is finished (rejection or bonus)
    }
  }
  // no CTA leaves while a peer may still store into its mailbox
  cluster_sync_all();
}

template <int C>
int launch_accept_split(const AcceptArgs& a, int rows, int seg, cudaStream_t stream) {
  static int max_clusters[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return -1;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.blockDim = dim3(kSpThreads, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (max_clusters[dev] == 0) {
    int sms = kNumSMs;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cfg.gridDim = dim3((unsigned)(C * (sms / C)), 1, 1);
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, accept_split_kernel<C>, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      return -1;
    }
    max_clusters[dev] = n;
  }
  // rows in flight: every resident cluster, capped so their logits rows stay in L2
  int n_cl = max_clusters[dev];
  const int64_t row_bytes = (int64_t)a.V * 8;  // target + draft row
  const int64_t cap = (int64_t)kSpL2Budget / row_bytes;
  if (n_cl > cap) n_cl = cap < 1 ? 1 : (int)cap;
  if (n_cl > rows) n_cl = rows;
  cfg.gridDim = dim3((unsigned)(C * n_cl), 1, 1);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, accept_split_kernel<C>, a, rows, seg);
  return e == cudaSuccess ? 0 : (int)e;
}

// ---------------------------------------------------------------- draft sampling, T > 0, one CTA per row
//
// The streaming kernel's layout for one logits row: the max pass, one exp /
// sum pass that also leaves each warp segment's sum, then the inverse-CDF
// descent walks only the crossing segment (weights recomputed there).
__global__ void __launch_bounds__(kStThreads, 1) sample_stream_kernel(const float* logits, int64_t row_stride,
                                                                      const int32_t* index, int rows, int V, float T,
                                                                      const double* u, int64_t u_stride, int u_col,
                                                                      int32_t* out, int64_t out_stride,
                                                                      int32_t* out2, int64_t out2_stride, int seg) {
  __shared__ StShared sh;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int e_w = warp * seg;
  const int n_c = seg >> 7;
  for (int i = blockIdx.x; i < rows; i += gridDim.x) {
    const float* P = logits + (int64_t)(index ? index[i] : i) * row_stride;
    float mp = -INFINITY;
#pragma unroll 4
    for (int c = 0; c < n_c; ++c) {
      const int e = e_w + c * 128 + lane * 4;
      if (e < V) {
        const float4 sp = scale_s(ld_l2(P + e), T);
        mp = fmaxf(mp, fmaxf(fmaxf(sp.x, sp.y), fmaxf(sp.z, sp.w)));
      }
    }
    mp = warp_max(mp);
    if (lane == 0) sh.wm[0][warp] = mp;
    __syncthreads();
    if (warp == 0) {
      const float x = warp_max(sh.wm[0][lane]);
      if (lane == 0) sh.m[0] = x;
    }
    __syncthreads();
    mp = sh.m[0];
    double zp = 0.0;
    int lp = -1;
#pragma unroll 4
    for (int c = 0; c < n_c; ++c) {
      const int e = e_w + c * 128 + lane * 4;
      if (e < V) {
        const float4 wp = weights4(ld_l2(P + e), T, mp);
        zp += (double)wp.x;
        zp += (double)wp.y;
        zp += (double)wp.z;
        zp += (double)wp.w;
        if (wp.w > 0.f) lp = e + 3;
        else if (wp.z > 0.f) lp = e + 2;
        else if (wp.y > 0.f) lp = e + 1;
        else if (wp.x > 0.f) lp = e;
      }
    }
    zp = warp_sum_d(zp);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lp = max(lp, __shfl_xor_sync(0xffffffffu, lp, o));
    if (lane == 0) {
      sh.ws[0][warp] = zp;
      sh.wl[0][warp] = lp;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      double z = 0.0;
      int last = -1;
      for (int w = 0; w < kStWarps; ++w) {
        z += sh.ws[0][w];
        last = max(last, sh.wl[0][w]);
      }
      const double t = u[(int64_t)i * u_stride + u_col] * z;
      double run = 0.0;
      int hit = -1;
      for (int w = 0; w < kStWarps; ++w) {
        if (run + sh.ws[0][w] > t) {
          hit = w;
          break;
        }
        run += sh.ws[0][w];
      }
      sh.z[0] = t;
      sh.last[0] = last;
      sh.cross_warp = hit;
      sh.cross_run = run;
    }
    __syncthreads();
    const int w_hit = sh.cross_warp;
    const int last_all = sh.last[0];
    const double t = sh.z[0];
    int tok = -1;
    if (w_hit < 0) {
      tok = last_all >= 0 ? last_all : 0;  // rounding left no crossing: the last entry of nonzero weight
    } else if (warp == w_hit) {
      double run = sh.cross_run;
      int found = -1;
      for (int c = 0; c < n_c && found < 0; ++c) {
        const int e = e_w + c * 128 + lane * 4;
        double w4[4] = {0.0, 0.0, 0.0, 0.0};
        if (e < V) {
          const float4 wp = weights4(ld_l2(P + e), T, mp);
          w4[0] = wp.x;
          w4[1] = wp.y;
          w4[2] = wp.z;
          w4[3] = wp.w;
        }
        const double mine = ((w4[0] + w4[1]) + w4[2]) + w4[3];
        const double incl = warp_inclusive_scan_d(mine) + run;
        const unsigned hit = __ballot_sync(0xffffffffu, incl > t);
        if (hit) {
          const int l = __ffs(hit) - 1;
          if (lane == l) {
            double acc = incl - mine;
            for (int q = 0; q < 4 && found < 0; ++q) {
              acc += w4[q];
              if (acc > t) found = e + q;
            }
            for (int q = 3; q >= 0 && found < 0; --q)
              if (w4[q] > 0.0) found = e + q;
          }
          found = __shfl_sync(0xffffffffu, found, l);
          if (found < 0) found = sh.wl[0][warp] >= 0 ? sh.wl[0][warp] : (last_all >= 0 ? last_all : 0);
        }
        run = __shfl_sync(0xffffffffu, incl, 31);
      }
      tok = found >= 0 ? found : (sh.wl[0][warp] >= 0 ? sh.wl[0][warp] : (last_all >= 0 ? last_all : 0));
    }
    if ((w_hit < 0 && threadIdx.x == 0) || (w_hit >= 0 && warp == w_hit && lane == 0)) {
      out[(int64_t)i * out_stride] = tok;
      if (out2) out2[(int64_t)i * out2_stride] = tok;
    }
    __syncthreads();  // sh is rewritten by the next row
  }
}

// ---------------------------------------------------------------- tree speculation: accept / resample
//
// One CTA per request row over a token tree of b branches x k depths (node
// (j, d) is branch j's token at depth d).  T = 0: the first branch whose
// candidate is the target's argmax, then the greedy linear rule along it.
// T > 0: recursive rejection over the b candidates at depth 0 (round i tests
// candidate i against P_{i-1}, the previous rounds' normalised residual
// max(0, P - Q) / R), then the linear rule (accept_kernel above) along the
// accepted branch.  Uniform layout per row: u[d*b + j] drew node (j, d),
// u[b*k + i] tests candidate i, u[b*k + b + d - 1] tests depth d >= 1,
// u[b*k + b + k - 1] is the final draw.  Arithmetic as stated in the header
// of this file, plus: P_0 = w_p * (1/Z_p), Q = w_q * (1/Z_q), r = max(0, P - Q),
// P_next = r * (1/R) -- each product and difference rounded on its own.

constexpr int kTreeMaxB = 8;

struct TreeArgs {
  const float* p_root;
  int64_t pr_stride;
  const int32_t* pr_index;
  const float* q_root;
  int64_t qr_stride;
  const int32_t* qr_index;
  const float* verify;  // target after node (i, j, d): verify + i * v_req + j * v_branch + d * v_depth
  int64_t v_req, v_branch, v_depth;
  const float* dchain;  // draft after node (i, j, d), d < k-1: dchain + i * dc_req + j * dc_branch + d * dc_depth
  int64_t dc_req, dc_branch, dc_depth;
  const int32_t* chain;  // [rows][b][k]
  const double* u;
  int64_t u_stride;
  int b, k, V;
  float T;
  int32_t* tokens;  // [rows][k+1]
  int32_t* n_accepted;
  int32_t* branch;
  int32_t* final_token;
};

// P_rounds(e): the target's root distribution after `rounds` residual rounds
// (invR[s] == 0 marks a round whose residual was empty: P unchanged).
struct TreeChainP {
  const float* p;
  const float* q;
  float T, mp, mq;
  double invp, invq;
  const double* invR;
  int rounds;
  __device__ __forceinline__ double Q(int e) const { return __dmul_rn((double)expf(q[e] / T - mq), invq); }
  __device__ __forceinline__ double P(int e) const {
    double P = __dmul_rn((double)expf(p[e] / T - mp), invp);
    if (rounds == 0) return P;
    const double qe = Q(e);
    for (int s = 0; s < rounds; ++s) {
      if (invR[s] > 0.0) {
        const double d = __dsub_rn(P, qe);
        P = __dmul_rn(d > 0.0 ? d : 0.0, invR[s]);
      }
    }
    return P;
  }
};

// r_{rounds+1}(e) = max(0, P_rounds(e) - Q(e)): the residual of the next round.
struct TreeResidual {
  TreeChainP c;
  __device__ double operator()(int e) const {
    const double d = __dsub_rn(c.P(e), c.Q(e));
    return d > 0.0 ? d : 0.0;
  }
};

__device__ __forceinline__ const float* tree_node_target(const TreeArgs& a, int i, int j, int d) {
  return a.verify + (int64_t)i * a.v_req + (int64_t)j * a.v_branch + (int64_t)d * a.v_depth;
}
__device__ __forceinline__ const float* tree_node_draft(const TreeArgs& a, int i, int j, int d) {
  return a.dchain + (int64_t)i * a.dc_req + (int64_t)j * a.dc_branch + (int64_t)d * a.dc_depth;
}

__global__ void __launch_bounds__(kSampleThreads) tree_accept_kernel(TreeArgs a) {
  __shared__ Scratch sh;
  const int i = blockIdx.x;
  const int b = a.b, k = a.k, V = a.V;
  const float T = a.T;
  const int32_t* chain = a.chain + (int64_t)i * b * k;
  int32_t* toks = a.tokens + (int64_t)i * (k + 1);
  const float* pr = a.p_root + (int64_t)(a.pr_index ? a.pr_index[i] : i) * a.pr_stride;
  const float* qr = a.q_root + (int64_t)(a.qr_index ? a.qr_index[i] : i) * a.qr_stride;
  int n_acc = 0, fin = -1, jb = 0;

  if (T <= 0.f) {
    const int y0 = block_argmax(pr, V, sh);
    jb = -1;
    for (int j = 0; j < b; ++j)
      if (chain[j * k] == y0) {
        jb = j;
        break;
      }
    if (jb < 0) {
      jb = 0;
      fin = y0;
    } else {
      if (threadIdx.x == 0) toks[0] = y0;
      n_acc = k;
      for (int d = 1; d <= k; ++d) {
        const int y = block_argmax(tree_node_target(a, i, jb, d - 1), V, sh);
        if (d == k) {
          fin = y;
          break;
        }
        if (threadIdx.x == 0) toks[d] = y;
        if (chain[jb * k + d] != y) {
          n_acc = d;
          fin = y;
          break;
        }
      }
    }
  } else {
    const double* u = a.u + (int64_t)i * a.u_stride;
    const int base = b * k;
    const double u_fin = u[base + b + k - 1];
    const Stats sp = row_stats(pr, V, T, sh);
    const Stats sq = row_stats(qr, V, T, sh);
    double invR[kTreeMaxB];
    TreeChainP cp{pr, qr, T, sp.m, sq.m, 1.0 / sp.z, 1.0 / sq.z, invR, 0};
    double last_R = 0.0;
    int last_round = -1;
    jb = -1;
    for (int r = 0; r < b; ++r) {
      // round r + 1: candidate r against P_r (engine/speculative.py:133-142 for r = 0)
      const int x = chain[r * k];
      const bool x_ok = x >= 0 && x < V;
      double prob = 0.0;
      if (x_ok) {
        if (r == 0) {
          const double wpx = (double)expf(pr[x] / T - sp.m), wqx = (double)expf(qr[x] / T - sq.m);
          if (wqx > 0.0) {
            const double ratio = __ddiv_rn(__dmul_rn(wpx, sq.z), __dmul_rn(wqx, sp.z));
            prob = ratio < 1.0 ? ratio : 1.0;
          }
        } else {
          cp.rounds = r;
          const double qx = cp.Q(x);
          if (qx > 0.0) {
            const double ratio = __ddiv_rn(cp.P(x), qx);
            prob = ratio < 1.0 ? ratio : 1.0;
          }
        }
      }
      if (u[base + r] < prob) {
        jb = r;
        break;
      }
      cp.rounds = r;
      const TreeResidual rw{cp};
      double R = 0.0;
      for (int e = threadIdx.x; e < V; e += blockDim.x) R += rw(e);
      R = block_sum_d(R, sh);
      invR[r] = R > 0.0 ? 1.0 / R : 0.0;
      if (R > 0.0) {
        last_R = R;
        last_round = r;
      }
    }
    if (jb < 0) {
      // every candidate rejected: the last non-empty residual, else p
      jb = 0;
      n_acc = 0;
      if (last_round >= 0) {
        cp.rounds = last_round;
        fin = block_icdf(TreeResidual{cp}, V, u_fin * last_R, sh);
      } else {
        fin = block_icdf(SoftmaxWeight{pr, T, sp.m}, V, u_fin * sp.z, sh);
      }
    } else {
      if (threadIdx.x == 0) toks[0] = chain[jb * k];
      n_acc = k;
      for (int d = 1; d < k; ++d) {
        // engine/speculative.py:133-142 along the accepted branch
        const float* p = tree_node_target(a, i, jb, d - 1);
        const float* q = tree_node_draft(a, i, jb, d - 1);
        const int x = chain[jb * k + d];
        const bool x_ok = x >= 0 && x < V;
        const Stats s1 = row_stats(p, V, T, sh);
        const Stats s2 = row_stats(q, V, T, sh);
        const double wpx = x_ok ? (double)expf(p[x] / T - s1.m) : 0.0;
        const double wqx = x_ok ? (double)expf(q[x] / T - s2.m) : 0.0;
        double prob = 0.0;
        if (wqx > 0.0) {
          const double ratio = __ddiv_rn(__dmul_rn(wpx, s2.z), __dmul_rn(wqx, s1.z));
          prob = ratio < 1.0 ? ratio : 1.0;
        }
        if (u[base + b + d - 1] < prob) {
          if (threadIdx.x == 0) toks[d] = x;
          continue;
        }
        // engine/speculative.py:43-50
        const ResidualWeight rw{p, q, T, s1.m, s2.m, 1.0 / s1.z, 1.0 / s2.z};
        double R = 0.0;
        for (int e = threadIdx.x; e < V; e += blockDim.x) R += rw(e);
        R = block_sum_d(R, sh);
        fin = R <= 0.0 ? block_icdf(SoftmaxWeight{p, T, s1.m}, V, u_fin * s1.z, sh)
                       : block_icdf(rw, V, u_fin * R, sh);
        n_acc = d;
        break;
      }
      if (fin < 0) {
        // every depth accepted: the bonus from the target after node (jb, k-1)
        const float* p = tree_node_target(a, i, jb, k - 1);
        const Stats s1 = row_stats(p, V, T, sh);
        fin = block_icdf(SoftmaxWeight{p, T, s1.m}, V, u_fin * s1.z, sh);
      }
    }
  }
  if (threadIdx.x == 0) {
    toks[n_acc] = fin;
    for (int j = n_acc + 1; j <= k; ++j) toks[j] = -1;
    a.n_accepted[i] = n_acc;
    a.branch[i] = jb;
    a.final_token[i] = fin;
  }
}

// The vector kernels read 16-byte vectors: every logits row must start on a
// 16-byte boundary (base pointers aligned, strides and vocab multiples of 4).
bool vec_accept_ok(const AcceptArgs& a) {
  auto al = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  auto m4 = [](int64_t v) { return (v & 3) == 0; };
  if (!m4(a.V)) return false;
  if (!al(a.target0) || !al(a.verify) || !al(a.draft0) || (a.k > 1 && !al(a.draft_rest))) return false;
  return m4(a.t0_stride) && m4(a.v_row) && m4(a.v_pos) && m4(a.d0_stride) && (a.k <= 1 || (m4(a.dr_row) && m4(a.dr_pos)));
}

}  // namespace
}  // namespace pse

using namespace pse;

extern "C" int pse_philox_uniforms(uint64_t seed, const uint32_t* req_key, const int32_t* step, int32_t rows,
                                   int32_t n, double* out, void* stream) {
  if (rows < 0 || n < 0) return PSE_EINVAL;
  if (rows == 0 || n == 0) return PSE_OK;
  if (!req_key || !step || !out) return PSE_EINVAL;
  const int64_t work = (int64_t)rows * ((n + 1) / 2);
  int grid = (int)((work + 255) / 256);
  if (grid > kNumSMs * 16) grid = kNumSMs * 16;
  philox_kernel<<<grid, 256, 0, (cudaStream_t)stream>>>(seed, req_key, step, rows, n, out);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

extern "C" int pse_sample_tokens(const float* logits, int64_t row_stride, const int32_t* index, int32_t rows,
                                 int32_t vocab, float temperature, const double* u, int64_t u_stride, int32_t u_col,
                                 int32_t* out, int64_t out_stride, int32_t* out2, int64_t out2_stride, void* stream) {
  if (rows < 0 || vocab <= 0) return PSE_EINVAL;
  if (rows == 0) return PSE_OK;
  if (!logits || !out || (temperature > 0.f && !u)) return PSE_EINVAL;
  if (temperature > 0.f && (g_accept_kernel == 0 || g_accept_kernel == 3) && vocab % 4 == 0 && row_stride % 4 == 0 &&
      (reinterpret_cast<uintptr_t>(logits) & 15) == 0) {
    const int seg = ((vocab + kStWarps - 1) / kStWarps + 127) & ~127;
    sample_stream_kernel<<<rows, kStThreads, 0, (cudaStream_t)stream>>>(logits, row_stride, index, rows, vocab,
                                                                       temperature, u, u_stride, u_col, out, out_stride,
                                                                       out2, out2_stride, seg);
    PSE_LAUNCH_CHECK();
    return PSE_OK;
  }
  sample_kernel<<<rows, kSampleThreads, 0, (cudaStream_t)stream>>>(logits, row_stride, index, vocab, temperature, u,
                                                                    u_stride, u_col, out, out_stride, out2,
                                                                    out2_stride);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

extern "C" int pse_accept_select(int32_t kernel) {
  if (kernel < 0 || kernel > 3) return PSE_EINVAL;
  g_accept_kernel = kernel;
  return PSE_OK;
}

extern "C" int pse_spec_accept(const float* target0, int64_t t0_stride, const int32_t* t0_index, const float* verify,
                               int64_t v_row, int64_t v_pos, const float* draft0, int64_t d0_stride,
                               const int32_t* d0_index, const float* draft_rest, int64_t dr_row, int64_t dr_pos,
                               const int32_t* drafts, const double* u, int64_t u_stride, int32_t rows, int32_t k,
                               int32_t vocab, float temperature, int32_t* tokens, int32_t* n_accepted,
                               int32_t* final_token, void* stream) {
  if (rows < 0 || k < 1 || vocab <= 0) return PSE_EINVAL;
  if (rows == 0) return PSE_OK;
  if (!target0 || !verify || !drafts || !tokens || !n_accepted || !final_token) return PSE_EINVAL;
  if (temperature > 0.f && (!u || !draft0 || (k > 1 && !draft_rest))) return PSE_EINVAL;
  AcceptArgs a{target0, t0_stride, t0_index, verify, v_row, v_pos, draft0, d0_stride, d0_index, draft_rest,
               dr_row, dr_pos, drafts, u, u_stride, k, vocab, temperature, tokens, n_accepted, final_token};
  const bool vec = temperature > 0.f && vec_accept_ok(a);
  if (vec && g_accept_kernel == 0) {
    // one cluster of C CTAs per row, several clusters per SM
    int C = (vocab + 8191) / 8192;
    if (C > kSpMaxC) C = kSpMaxC;
    const int unit = kSpWarps * 128;
    const int chunk = ((vocab + C - 1) / C + unit - 1) / unit * unit;
    const int seg = chunk / kSpWarps;
    int rc = -1;
    switch (C) {
      case 1: rc = launch_accept_split<1>(a, rows, seg, (cudaStream_t)stream); break;
      case 2: rc = launch_accept_split<2>(a, rows, seg, (cudaStream_t)stream); break;
      case 3: rc = launch_accept_split<3>(a, rows, seg, (cudaStream_t)stream); break;
      case 4: rc = launch_accept_split<4>(a, rows, seg, (cudaStream_t)stream); break;
      case 5: rc = launch_accept_split<5>(a, rows, seg, (cudaStream_t)stream); break;
      case 6: rc = launch_accept_split<6>(a, rows, seg, (cudaStream_t)stream); break;
      case 7: rc = launch_accept_split<7>(a, rows, seg, (cudaStream_t)stream); break;
      default: rc = launch_accept_split<8>(a, rows, seg, (cudaStream_t)stream); break;
    }
    if (rc > 0) return rc;
    if (rc == 0) return PSE_OK;
    // rc < 0: no cluster of this size fits on the device; the streaming kernel below handles it
  }
  if (vec && (g_accept_kernel == 0 || g_accept_kernel == 3)) {
    const int seg = ((vocab + kStWarps - 1) / kStWarps + 127) & ~127;
    int sms = kNumSMs, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int grid = rows < PSE_ACCEPT_ROWS_IN_FLIGHT ? rows : PSE_ACCEPT_ROWS_IN_FLIGHT;
    if (grid > sms) grid = sms;
    accept_stream_kernel<<<grid, kStThreads, 0, (cudaStream_t)stream>>>(a, rows, seg);
    PSE_LAUNCH_CHECK();
    return PSE_OK;
  }
  if (vec && g_accept_kernel == 2 && vocab <= kClMax * kClCtaCap) {
    // one cluster per row with the row held on chip (vocabularies up to 8 x 16384)
    const int C = (vocab + kClCtaCap - 1) / kClCtaCap;
    const int per_lane = (vocab + C * kClThreads - 1) / (C * kClThreads);
    const int run_len = (per_lane + 3) & ~3;  // <= 32
    int rc = -1;
    switch (C) {
      case 1: rc = launch_accept_cluster<1>(a, rows, run_len, (cudaStream_t)stream); break;
      case 2: rc = launch_accept_cluster<2>(a, rows, run_len, (cudaStream_t)stream); break;
      case 3: rc = launch_accept_cluster<3>(a, rows, run_len, (cudaStream_t)stream); break;
      case 4: rc = launch_accept_cluster<4>(a, rows, run_len, (cudaStream_t)stream); break;
      case 5: rc = launch_accept_cluster<5>(a, rows, run_len, (cudaStream_t)stream); break;
      case 6: rc = launch_accept_cluster<6>(a, rows, run_len, (cudaStream_t)stream); break;
      case 7: rc = launch_accept_cluster<7>(a, rows, run_len, (cudaStream_t)stream); break;
      default: rc = launch_accept_cluster<8>(a, rows, run_len, (cudaStream_t)stream); break;
    }
    if (rc > 0) return rc;
    if (rc == 0) return PSE_OK;
    // rc < 0: no cluster of this size fits on the device; the CTA-per-row kernel below handles it
  }
  accept_kernel<<<rows, kSampleThreads, 0, (cudaStream_t)stream>>>(a);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

extern "C" int pse_tree_accept(const float* p_root, int64_t pr_stride, const int32_t* pr_index, const float* q_root,
                               int64_t qr_stride, const int32_t* qr_index, const float* verify, int64_t v_req,
                               int64_t v_branch, int64_t v_depth, const float* dchain, int64_t dc_req,
                               int64_t dc_branch, int64_t dc_depth, const int32_t* chain, const double* u,
                               int64_t u_stride, int32_t rows, int32_t branches, int32_t k, int32_t vocab,
                               float temperature, int32_t* tokens, int32_t* n_accepted, int32_t* branch,
                               int32_t* final_token, void* stream) {
  if (rows < 0 || k < 1 || vocab <= 0 || branches < 1 || branches > kTreeMaxB || branches > vocab) return PSE_EINVAL;
  if (rows == 0) return PSE_OK;
  if (!p_root || !verify || !chain || !tokens || !n_accepted || !branch || !final_token) return PSE_EINVAL;
  if (temperature > 0.f && (!u || !q_root || (k > 1 && !dchain))) return PSE_EINVAL;
  TreeArgs a{p_root,  pr_stride, pr_index, q_root,   qr_stride, qr_index, verify, v_req,  v_branch,
             v_depth, dchain,    dc_req,   dc_branch, dc_depth,  chain,    u,      u_stride, branches,
             k,       vocab,     temperature, tokens, n_accepted, branch, final_token};
  tree_accept_kernel<<<rows, kSampleThreads, 0, (cudaStream_t)stream>>>(a);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}
