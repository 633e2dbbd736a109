// Scheduler bookkeeping of one speculative step on the device
// (engine/scheduler.py:107-126): the per-row loop that extends each request's
// token list with the step's accepted tokens, counts them, tests
// `generated >= max_new_tokens`, and trims the overshoot of a finishing
// request.  Each request owns `max_new[o]` int32 slots of an output arena at
// `out_off[o]`; tokens past a request's budget are the overshoot the reference
// trims, so they are never stored.  The finished rows are compacted in row
// order (the order the reference frees and reports them) into `finished`.
#include "common.cuh"

namespace pse {
namespace {

constexpr int kCommitThreads = 1024;

__global__ void __launch_bounds__(kCommitThreads)
    sched_commit_kernel(const int32_t* __restrict__ tokens, int32_t tok_stride, const int32_t* __restrict__ n_acc,
                        const int32_t* __restrict__ ords, int32_t rows, const int64_t* __restrict__ out_off,
                        const int32_t* __restrict__ max_new, int32_t* __restrict__ generated,
                        int32_t* __restrict__ out, int32_t* __restrict__ finished) {
  __shared__ int tmp[33];
  int carry = 0;
  for (int base = 0; base < rows; base += kCommitThreads) {
    const int i = base + threadIdx.x;
    int fin = 0;
    if (i < rows) {
      const int o = ords[i];
      int n = n_acc[i] + 1;  // accepted drafts + the final token
      n = n < 1 ? 1 : (n > tok_stride ? tok_stride : n);
      const int g = generated[o];
      const int budget = max_new[o];
      int32_t* dst = out + out_off[o];
      const int32_t* src = tokens + (int64_t)i * tok_stride;
      for (int j = 0; j < n; ++j)
        if (g + j < budget) dst[g + j] = src[j];
      generated[o] = g + n;
      fin = g + n >= budget;
    }
    int total;
    const int pos = block_exclusive_scan(fin, tmp, &total);
    if (fin) finished[1 + carry + pos] = i;
    carry += total;
  }
  if (threadIdx.x == 0) finished[0] = carry;
}

// ---------------------------------------------------------------- step glue
//
// The integer hand-offs between the step's calls, one launch each instead of
// a handful of small tensor operations.

constexpr int kGlueThreads = 256;

__device__ __forceinline__ int32_t slot_value(const int32_t* v, int32_t slot, int32_t n_slots) {
  return slot >= 0 && slot < n_slots ? v[slot] : 0;
}

// Input of the verify call made from pending rows: row i runs
// [last_token[slot], d_1 .. d_k] from position base[i] - 1.
__global__ void verify_ids_kernel(const int32_t* __restrict__ last_token, int32_t n_slots,
                                  const int32_t* __restrict__ slots, const int32_t* __restrict__ drafts,
                                  const int32_t* __restrict__ base, int32_t rows, int32_t k,
                                  int32_t* __restrict__ ids, int32_t* __restrict__ first_pos) {
  const int w = k + 1;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < rows * w; e += gridDim.x * blockDim.x) {
    const int i = e / w, c = e % w;
    if (c == 0) {
      ids[e] = slot_value(last_token, slots[i], n_slots);
      first_pos[i] = base[i] - 1;
    } else {
      ids[e] = drafts[(int64_t)i * k + c - 1];
    }
  }
}

// Input of the draft's tail call: [d_k, final] when all k drafts were
// accepted, else [final, final]; it runs from base0 + min(n_acc, k - 1), and
// the row's next logits come from hidden row 2 i + (n_acc == k).
__global__ void bonus_ids_kernel(const int32_t* __restrict__ n_acc, const int32_t* __restrict__ drafts,
                                 const int32_t* __restrict__ final_tok, const int32_t* __restrict__ base0,
                                 int32_t rows, int32_t k, int32_t* __restrict__ ids2, int32_t* __restrict__ pos,
                                 int64_t* __restrict__ sel) {
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += gridDim.x * blockDim.x) {
    const int n = n_acc[i];
    const bool full = n == k;
    const int32_t f = final_tok[i];
    ids2[2 * i] = full ? drafts[(int64_t)i * k + k - 1] : f;
    ids2[2 * i + 1] = f;
    pos[i] = base0[i] + (n < k - 1 ? n : k - 1);
    sel[i] = 2 * (int64_t)i + (full ? 1 : 0);
  }
}

// End of the step: each row's final token becomes its slot's last token in
// both caches, and the result pack [tokens | n_acc | status_d | status_t] is
// filled for the one device-to-host copy.
__global__ void step_finish_kernel(const int32_t* __restrict__ final_tok, const int32_t* __restrict__ slots_d,
                                   const int32_t* __restrict__ slots_t, int32_t rows, int32_t* last_d,
                                   int32_t n_slots_d, int32_t* last_t, int32_t n_slots_t,
                                   const int32_t* __restrict__ tokens, int32_t k, const int32_t* __restrict__ n_acc,
                                   const int32_t* status_d, const int32_t* status_t, int32_t* __restrict__ pack) {
  const int nt = rows * (k + 1);
  const int stride = gridDim.x * blockDim.x;
  for (int e = blockIdx.x * blockDim.x + threadIdx.x; e < nt; e += stride) pack[e] = tokens[e];
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < rows; i += stride) {
    pack[nt + i] = n_acc[i];
    const int32_t f = final_tok[i];
    const int32_t sd = slots_d[i], st = slots_t[i];
    if (sd >= 0 && sd < n_slots_d) last_d[sd] = f;
    if (st >= 0 && st < n_slots_t) last_t[st] = f;
  }
  if (blockIdx.x == 0 && threadIdx.x == 0) {
    pack[nt + rows] = *status_d;
    pack[nt + rows + 1] = *status_t;
  }
}

int glue_grid(int64_t n) {
  const int64_t g = (n + kGlueThreads - 1) / kGlueThreads;
  return (int)(g < 1 ? 1 : g > 1184 ? 1184 : g);
}

}  // namespace
}  // namespace pse

extern "C" int pse_step_verify_ids(const int32_t* last_token, int32_t n_slots, const int32_t* slots,
                                   const int32_t* drafts, const int32_t* base, int32_t rows, int32_t k, int32_t* ids,
                                   int32_t* first_pos, void* stream) {
  if (rows < 0 || k < 1 || n_slots < 0 || (int64_t)rows * (k + 1) > (1 << 30)) return PSE_EINVAL;
  if (rows == 0) return PSE_OK;
  if (!last_token || !slots || !drafts || !base || !ids || !first_pos) return PSE_EINVAL;
  pse::verify_ids_kernel<<<pse::glue_grid((int64_t)rows * (k + 1)), pse::kGlueThreads, 0, (cudaStream_t)stream>>>(
      last_token, n_slots, slots, drafts, base, rows, k, ids, first_pos);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

extern "C" int pse_step_bonus_ids(const int32_t* n_acc, const int32_t* drafts, const int32_t* final_tok,
                                  const int32_t* base0, int32_t rows, int32_t k, int32_t* ids2, int32_t* pos,
                                  int64_t* sel, void* stream) {
  if (rows < 0 || k < 1 || rows > (1 << 29)) return PSE_EINVAL;
  if (rows == 0) return PSE_OK;
  if (!n_acc || !drafts || !final_tok || !base0 || !ids2 || !pos || !sel) return PSE_EINVAL;
  pse::bonus_ids_kernel<<<pse::glue_grid(rows), pse::kGlueThreads, 0, (cudaStream_t)stream>>>(
      n_acc, drafts, final_tok, base0, rows, k, ids2, pos, sel);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

extern "C" int pse_step_finish(const int32_t* final_tok, const int32_t* slots_d, const int32_t* slots_t,
                               int32_t rows, int32_t* last_d, int32_t n_slots_d, int32_t* last_t, int32_t n_slots_t,
                               const int32_t* tokens, int32_t k, const int32_t* n_acc, const int32_t* status_d,
                               const int32_t* status_t, int32_t* pack, void* stream) {
  if (rows < 0 || k < 1 || n_slots_d < 0 || n_slots_t < 0 || (int64_t)rows * (k + 2) + 2 > (1 << 30))
    return PSE_EINVAL;
  if (!status_d || !status_t || !pack) return PSE_EINVAL;
  if (rows > 0 && (!final_tok || !slots_d || !slots_t || !last_d || !last_t || !tokens || !n_acc)) return PSE_EINVAL;
  pse::step_finish_kernel<<<pse::glue_grid((int64_t)rows * (k + 1)), pse::kGlueThreads, 0, (cudaStream_t)stream>>>(
      final_tok, slots_d, slots_t, rows, last_d, n_slots_d, last_t, n_slots_t, tokens, k, n_acc, status_d, status_t,
      pack);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}

extern "C" int pse_sched_commit(const int32_t* tokens, int32_t tok_stride, const int32_t* n_acc, const int32_t* ords,
                                int32_t rows, const int64_t* out_off, const int32_t* max_new, int32_t* generated,
                                int32_t* out, int32_t* finished, void* stream) {
  if (rows < 0 || tok_stride < 1) return PSE_EINVAL;
  if (!finished) return PSE_EINVAL;
  if (rows > 0 && (!tokens || !n_acc || !ords || !out_off || !max_new || !generated || !out)) return PSE_EINVAL;
  pse::sched_commit_kernel<<<1, pse::kCommitThreads, 0, (cudaStream_t)stream>>>(
      tokens, tok_stride, n_acc, ords, rows, out_off, max_new, generated, out, finished);
  PSE_LAUNCH_CHECK();
  return PSE_OK;
}
