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
    // 16-byte loads, four rows of candidates per thread in index order
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const int n4 = V >> 2;
    int e = threadIdx.x;
    for (; e + blockDim.x < n4; e += 2 * blockDim.x) {
      const float4 a = r4[e], b = r4[e + blockDim.x];
      argmax_step(a.x, 4 * e, bv, bi);
      argmax_step(a.y, 4 * e + 1, bv, bi);
      argmax_step(a.z, 4 * e + 2, bv, bi);
      argmax_step(a.w, 4 * e + 3, bv, bi);
      const int f = e + blockDim.x;
      argmax_step(b.x, 4 * f, bv, bi);
      argmax_step(b.y, 4 * f + 1, bv, bi);
      argmax_step(b.z, 4 * f + 2, bv, bi);
      argmax_step(b.w, 4 * f + 3, bv, bi);
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
  sample_kernel<<<rows, kSampleThreads, 0, (cudaStream_t)stream>>>(logits, row_stride, index, vocab, temperature, u,
                                                                    u_stride, u_col, out, out_stride, out2,
                                                                    out2_stride);
  PSE_LAUNCH_CHECK();
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
  accept_kernel<<<rows, kSampleThreads, 0, (cudaStream_t)stream>>>(a);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}
