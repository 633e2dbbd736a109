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

}  // namespace
}  // namespace pse

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
