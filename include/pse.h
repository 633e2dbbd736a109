/*
 * pse.h -- C ABI of libpse.so, the sm_100a kernels of the speculative
 * draft -> verify -> accept/reject -> commit path.
 *
 * Every entry point takes plain device pointers, sizes and a CUDA stream
 * (as void*), launches asynchronously on that stream, allocates nothing and
 * never synchronises.  Return value: 0 on success, a cudaError_t value from
 * the launch, or one of the PSE_EINVAL... codes below for bad arguments
 * (checked on the host before anything is launched).
 *
 * Cache-state errors found on the device (pool exhausted, truncate beyond
 * length, double free) are latched in the state's `status` word instead of
 * trapping; while it is non-zero every state-mutating kernel is a no-op.  The
 * host reads the word at a step boundary and raises the reference's
 * exception (MemoryError / ValueError).
 *
 * Each declaration names the reference interface it replaces
 * (vedantjain09/paged-speculative-engine, engine/...:line).
 */
#ifndef PSE_H_
#define PSE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- return codes (host-side argument checks) ---- */
#define PSE_OK 0
#define PSE_EINVAL 10001       /* bad size / pointer / unsupported combination */
#define PSE_EWORKSPACE 10002   /* workspace smaller than the query function said */
#define PSE_ESCRATCH 10003     /* scratch need exceeds PSE_NOALLOC_SCRATCH_BYTES */

/* ---- device status latch bits ---- */
#define PSE_STATUS_OOM 1              /* pool exhausted (reference: MemoryError) */
#define PSE_STATUS_TABLE_OVERFLOW 2   /* block table too narrow for the row */
#define PSE_STATUS_TRUNCATE_LONG 4    /* truncate beyond length (ValueError) */
#define PSE_STATUS_DOUBLE_FREE 8      /* block freed twice (ValueError) */
#define PSE_STATUS_BAD_BLOCK 16       /* block id out of range */
#define PSE_STATUS_TIMEOUT 32         /* a bounded in-kernel wait expired */

/* ---- element types ---- */
#define PSE_F32 0
#define PSE_BF16 1

/* Device bookkeeping of one paged cache (one model).  All arrays on device. */
typedef struct {
  int32_t *block_table; /* [num_slots, max_blocks] physical block ids, -1 unused */
  int32_t *seq_len;     /* [num_slots] tokens held by the row                   */
  int32_t *nblocks;     /* [num_slots] blocks held by the row                   */
  int32_t *free_stack;  /* [num_blocks] LIFO stack, valid entries [0, *free_top) */
  int32_t *free_top;    /* [1]                                                  */
  uint8_t *block_free;  /* [num_blocks] 1 while the block is on the stack       */
  int32_t *status;      /* [1] error latch (PSE_STATUS_* bits)                  */
  int32_t num_blocks;
  int32_t block_size;
  int32_t max_blocks;
  int32_t num_slots;
} pse_block_state;

/* One layer's K and V pools: [num_blocks, kv_heads, block_size, head_dim]. */
typedef struct {
  void *k_pool;
  void *v_pool;
  int32_t kv_heads;
  int32_t head_dim;
  int32_t dtype; /* PSE_F32 or PSE_BF16 */
} pse_kv_layer;

/* ------------------------------------------------------------------------ */
/* Block pool / free list                                                   */
/* ------------------------------------------------------------------------ */

/* BlockAllocator.__init__ (engine/paged_cache.py:37-39) and PagedKVCache's
 * empty tables (engine/paged_cache.py:89-90): stack = [0..n-1], all tables -1,
 * lengths 0, status 0. */
int pse_block_init(pse_block_state st, void *stream);

/* BlockAllocator.allocate (engine/paged_cache.py:45-48): pops the stack top
 * into *out_id, or writes -1 and latches PSE_STATUS_OOM. */
int pse_block_alloc_one(pse_block_state st, int32_t *out_id, void *stream);

/* BlockAllocator.free (engine/paged_cache.py:50-56): pushes `block_id`
 * (device scalar); latches PSE_STATUS_DOUBLE_FREE / BAD_BLOCK instead. */
int pse_block_free_one(pse_block_state st, const int32_t *block_id, void *stream);

/* The allocation half of PagedKVCache.append (engine/paged_cache.py:116-130)
 * for `rows` rows of one batched forward (engine/batched_forward.py:67-70):
 * every row grows by `width` tokens, missing blocks are popped in row order
 * (exclusive prefix sum over rows), base_len[i] receives the row's length
 * before the call and seq_len advances.  On exhaustion the state is the
 * reference's after its MemoryError (earlier rows complete, the failing row
 * keeps its partial blocks, later rows untouched) and OOM is latched. */
int pse_kv_reserve(pse_block_state st, const int32_t *slots, int32_t rows, int32_t width,
                   int32_t *base_len, void *stream);

/* pse_kv_reserve with a width per row (widths[i] >= 0; a negative one latches
 * PSE_STATUS_BAD_BLOCK and changes nothing): the allocation half of one
 * PagedKVCache.append per row, rows in call order -- what prefilling requests
 * one after another (engine/speculative.py:53-73, engine/scheduler.py:78-90)
 * allocates, in one launch. */
int pse_kv_reserve_rows(pse_block_state st, const int32_t *slots, int32_t rows, const int32_t *widths,
                        int32_t *base_len, void *stream);

/* PagedKVCache.truncate (engine/paged_cache.py:140-154) for many rows in call
 * order, as the commit loop of engine/speculative.py:162-164 runs it.  New
 * length of row i = new_len[i] if new_len != NULL, else base_len[i] +
 * accepted[i].  Trailing blocks are pushed from the table end. */
int pse_kv_truncate(pse_block_state st, const int32_t *slots, int32_t rows, const int32_t *new_len,
                    const int32_t *base_len, const int32_t *accepted, void *stream);

/* PagedKVCache.free_request (engine/paged_cache.py:156-160) for many rows in
 * call order: each row's blocks are pushed in forward table order. */
int pse_kv_release(pse_block_state st, const int32_t *slots, int32_t rows, void *stream);

/* ------------------------------------------------------------------------ */
/* KV append and paged attention                                            */
/* ------------------------------------------------------------------------ */

/* The copy half of PagedKVCache.append (engine/paged_cache.py:131-136): token
 * w of row i, head h, element d is read from k_src/v_src + (i*width + w) *
 * tok_stride + h * head_stride + d and written at position base_len[i] + w of
 * the row.  Sources have the pool's dtype.  Blocks must have been reserved. */
int pse_kv_append(pse_block_state st, pse_kv_layer kv, const void *k_src, const void *v_src,
                  int64_t tok_stride, int64_t head_stride, const int32_t *slots,
                  const int32_t *base_len, int32_t rows, int32_t width, void *stream);

/* PagedKVCache.gather (engine/paged_cache.py:162-198) for one layer: padded
 * [rows, kv_heads, max_len, head_dim] K and V, zeros past each row's length. */
int pse_kv_gather(pse_block_state st, pse_kv_layer kv, const int32_t *slots, int32_t rows,
                  int32_t max_len, void *k_out, void *v_out, void *stream);

/* Attention of engine/model.py:99-116 over the paged state, replacing the
 * gather + masked matmul of engine/batched_forward.py:37-65.  Query w of row
 * i (head h at q + (i*width + w) * q_tok_stride + h*head_dim) sits at position
 * base_len[i] + w and attends to positions 0..base_len[i]+w of the row, whose
 * K/V are already in the pool.  Grouped heads: query head h reads KV head
 * h / (q_heads / kv_heads).  `max_ctx` bounds base_len[i] + width over rows
 * (it sizes the split-KV grid; rows may be shorter).  row_order (nullable) is a
 * permutation of 0..rows-1: the tensor-core kernel hands out rows in that order
 * (longest first keeps the end of the launch from idling on one long row).
 * Output has the pool's
 * dtype.  workspace: pse_paged_attention_workspace() bytes (at least 256: the
 * kernel's work counters, then split-KV partials).  The first 256 bytes must
 * be zero before the first call with a workspace (e.g. one cudaMemsetAsync
 * when it is allocated); every call leaves them zero, so a workspace kept for
 * many calls (or captured in a CUDA graph) needs no per-call clearing.  Calls
 * that share a workspace must not overlap on the GPU. */
int pse_paged_attention(pse_block_state st, pse_kv_layer kv, const void *q, int64_t q_tok_stride,
                        void *out, int64_t out_tok_stride, const int32_t *slots, const int32_t *base_len,
                        int32_t rows, int32_t width, int32_t q_heads, float scale, int32_t max_ctx,
                        const int32_t *row_order, void *workspace, size_t workspace_bytes, void *stream);

size_t pse_paged_attention_workspace(int32_t rows, int32_t width, int32_t q_heads, int32_t kv_heads,
                                     int32_t head_dim, int32_t max_ctx);

/* pse_paged_attention for a token-tree call (no counterpart in the reference:
 * its README lists tree-based speculation as future work).  The call's tokens
 * are tree nodes of `tree_branches` (b) branches in depth-major order, from
 * depth tree_depth0 (d0): query w is node n = d0*b + w, branch n % b at depth
 * n / b, at position L + n of its row (L = base_len[i] - d0*b, the row's
 * length at the tree's root); it attends to positions 0..L-1 and to its own
 * branch's nodes at depths up to its own.  Everything else as
 * pse_paged_attention (same workspace rules); prompt-sized calls do not take
 * the prefill kernel.  tree_branches < 1: PSE_EINVAL. */
int pse_paged_attention_tree(pse_block_state st, pse_kv_layer kv, const void *q, int64_t q_tok_stride,
                             void *out, int64_t out_tok_stride, const int32_t *slots,
                             const int32_t *base_len, int32_t rows, int32_t width, int32_t q_heads,
                             float scale, int32_t max_ctx, const int32_t *row_order, void *workspace,
                             size_t workspace_bytes, int32_t tree_branches, int32_t tree_depth0,
                             void *stream);

/* Token-tree commit for one layer: row i keeps n[i] of the tokens its tree
 * calls appended -- the token at position base_len[i] + src[i*max_n + m] moves
 * to position base_len[i] + m, m < n[i] (src increasing, src[m] >= m).  The
 * caller then truncates the row to base_len[i] + n[i].  No counterpart in the
 * reference. */
int pse_kv_compact(pse_block_state st, pse_kv_layer kv, const int32_t *slots, const int32_t *base_len,
                   const int32_t *src, const int32_t *n, int32_t rows, int32_t max_n, void *stream);

/* pse_paged_attention without a workspace argument, for hosts that cannot
 * allocate device memory where they call this library (a runtime in another
 * language that binds only this C ABI and has no CUDA allocator, or a process
 * whose device memory belongs to another allocator that must not be bypassed).
 * It allocates nothing: the split-KV scratch is a fixed array of
 * PSE_NOALLOC_SCRATCH_BYTES compiled into the library, resident on every GPU
 * that loads it until the process exits.  Calls whose scratch need
 * (pse_paged_attention_workspace) exceeds that return PSE_ESCRATCH without
 * launching (wide prompt-shaped calls, which take the prefill kernel and use
 * no split-KV scratch, are never refused for size).  The first call on each
 * device looks up the array's device address (cudaGetSymbolAddress) with that
 * device current and keeps it for the life of the process; make that first
 * call before any stream capture, and do not keep using the library across a
 * device reset (cudaDeviceReset), after which the kept address is stale.  All calls share the array and it keeps the
 * last call's contents (nothing in it needs to start at zero): calls that
 * overlap on the GPU race, so issue them on one stream or otherwise ordered.
 * No counterpart in the reference. */
#define PSE_NOALLOC_SCRATCH_BYTES (8u << 20)
int pse_paged_attention_noalloc(pse_block_state st, pse_kv_layer kv, const void *q, int64_t q_tok_stride,
                                void *out, int64_t out_tok_stride, const int32_t *slots,
                                const int32_t *base_len, int32_t rows, int32_t width, int32_t q_heads,
                                float scale, int32_t max_ctx, void *stream);

/* bf16 pools with head_dim 64/128 and block_size 16/32/64 run the TMA +
 * tensor-core kernel; every other shape runs the generic CUDA-core kernel.
 * on != 0 forces the generic kernel for every shape (parity tests compare the
 * two); no counterpart in the reference. */
int pse_attention_force_generic(int32_t on);

/* on != 0 (the default): the per-token kernels of the forward (embedding,
 * residual add + norm, bf16 epilogues, K/V append) and the projection GEMM
 * launch with programmatic dependent launch, so each may start while the
 * kernel before it finishes and waits for it before touching memory; 0
 * launches them plainly.  Process-wide; no counterpart in the reference. */
int pse_launch_overlap(int32_t on);

/* on != 0 (the default): pse_gemm_bf16 runs wide problems on two-SM tiles
 * (a cluster of two CTAs, tcgen05.mma.cta_group::2, 256 x 256 outputs) and
 * the rest on single-CTA tiles; 0: single-CTA tiles always (tests compare
 * the two).  No counterpart in the reference. */
int pse_gemm_pair_tiles(int32_t on);

/* Wide calls (at least 64 query rows per row and KV head: prompt prefill, a
 * wide batched append) with bf16 pools, head_dim 64/128, block_size 16..128
 * dividing 128 and 16-byte aligned q / out rows run a tcgen05 kernel (scores
 * and output accumulator in tensor memory, 128 query rows x 128 keys per
 * tile); query tokens at or past the row's length (seq_len) get zero output
 * there.  head_dim 64 runs two query tiles per CTA (one per softmax
 * warpgroup, sharing the K/V tiles).  mode 0: those kernels for wide calls
 * (default); 1: never (the calls take the kernels above); 2: one query tile
 * per CTA at every head_dim.  No counterpart in the reference. */
int pse_attention_prefill_select(int32_t mode);

/* ------------------------------------------------------------------------ */
/* Sampling, accept/resample                                                */
/* ------------------------------------------------------------------------ */

/* Uniform source of the explicit-uniform mode (replaces the torch.Generator
 * draws of engine/sampling.py:16-18 and engine/speculative.py:136):
 * out[i*n + j] = Philox4x32-10 uniform keyed (seed, req_key[i], step[i], j). */
int pse_philox_uniforms(uint64_t seed, const uint32_t *req_key, const int32_t *step, int32_t rows,
                        int32_t n, double *out, void *stream);

/* One draft-round draw per row (engine/speculative.py:99-108 with
 * engine/sampling.py:10-23): logits row of row i = logits + (index ? index[i] :
 * i) * row_stride.  T <= 0: argmax (first maximum).  T > 0: inverse CDF of
 * softmax(l / T) at uniform u[i*u_stride + u_col].  The token goes to
 * out[i*out_stride] and, if out2 != NULL, to out2[i*out2_stride]. */
int pse_sample_tokens(const float *logits, int64_t row_stride, const int32_t *index, int32_t rows,
                      int32_t vocab, float temperature, const double *u, int64_t u_stride,
                      int32_t u_col, int32_t *out, int64_t out_stride, int32_t *out2,
                      int64_t out2_stride, void *stream);

/* Fused accept / reject / residual / bonus of engine/speculative.py:119-157
 * (and _residual_sample, :43-50).  Target position 0 is
 * target0 + (t0_index ? t0_index[i] : i) * t0_stride; positions 1..k are
 * verify + i*v_row + (j-1)*v_pos.  Draft position 0 is draft0 + (d0_index ?
 * d0_index[i] : i) * d0_stride; positions 1..k-1 are draft_rest + i*dr_row +
 * (j-1)*dr_pos (draft logits are unused when T <= 0).  drafts[i*k + j] are
 * the drafted ids, u[i*u_stride + k + j] the accept uniforms and u[i*u_stride
 * + 2k] the residual / bonus uniform.  Writes tokens[i*(k+1) + 0..n] (the
 * accepted drafts then the corrected / bonus token), n_accepted[i] and
 * final_token[i] (= tokens[i*(k+1) + n_accepted[i]]).
 * T <= 0 runs one CTA per row.  T > 0 with 16-byte aligned rows (vocab and
 * strides multiples of 4) runs persistent 1024-thread CTAs, one row each, with
 * the rows in flight kept resident in L2 so every needed logit crosses HBM
 * once; other rows run the CTA-per-row scalar kernel. */
int pse_spec_accept(const float *target0, int64_t t0_stride, const int32_t *t0_index,
                    const float *verify, int64_t v_row, int64_t v_pos,
                    const float *draft0, int64_t d0_stride, const int32_t *d0_index,
                    const float *draft_rest, int64_t dr_row, int64_t dr_pos,
                    const int32_t *drafts, const double *u, int64_t u_stride, int32_t rows,
                    int32_t k, int32_t vocab, float temperature, int32_t *tokens,
                    int32_t *n_accepted, int32_t *final_token, void *stream);

/* Tree speculation: accept / reject / resample over a token tree of
 * `branches` (b <= 8) first-level candidates, each followed by a draft chain:
 * node (j, d), j < b, d < k, is branch j's token at depth d (chain[(i*b + j)*k
 * + d]).  The reference has no counterpart (its README lists tree-based
 * speculation as future work); b = 1 is exactly pse_spec_accept's rule.
 * Target logits at the root: p_root + (pr_index ? pr_index[i] : i) * pr_stride;
 * after node (j, d): verify + i*v_req + j*v_branch + d*v_depth.  Draft logits
 * at the root: q_root (+ qr_index / qr_stride); after node (j, d), d < k-1:
 * dchain + i*dc_req + j*dc_branch + d*dc_depth (draft logits unused at T <= 0).
 * T <= 0: the first branch whose candidate is the target's argmax, then the
 * greedy rule along it.  T > 0: recursive rejection over the b candidates
 * (drawn iid from the draft's root distribution): candidate j is tested
 * against the normalised residual of the rounds before it, so the first token
 * keeps the target's distribution; then the linear rule along the accepted
 * branch.  Uniforms u[i*u_stride + ...]: d*b + j drew node (j, d), b*k + j
 * tests candidate j, b*k + b + d - 1 tests depth d >= 1, b*k + b + k - 1 is
 * the final draw.  Writes tokens[i*(k+1) + 0..n] (accepted nodes, then the
 * corrected / bonus token), n_accepted[i], branch[i] (0 when no candidate was
 * accepted) and final_token[i].  One CTA per row. */
int pse_tree_accept(const float *p_root, int64_t pr_stride, const int32_t *pr_index,
                    const float *q_root, int64_t qr_stride, const int32_t *qr_index,
                    const float *verify, int64_t v_req, int64_t v_branch, int64_t v_depth,
                    const float *dchain, int64_t dc_req, int64_t dc_branch, int64_t dc_depth,
                    const int32_t *chain, const double *u, int64_t u_stride, int32_t rows,
                    int32_t branches, int32_t k, int32_t vocab, float temperature,
                    int32_t *tokens, int32_t *n_accepted, int32_t *branch,
                    int32_t *final_token, void *stream);

/* Which kernel pse_spec_accept runs at T > 0: 0 the default (one cluster of
 * min(8, ceil(vocab / 8192)) CTAs per row, several clusters per SM, the row
 * streamed from HBM once and re-read from L2), 1 the CTA-per-row scalar
 * kernel, 2 one thread-block cluster of ceil(vocab / 16384) CTAs per row with
 * the row held on chip (vocab <= 131072), 3 one streaming CTA per row.  All
 * four give the same tokens; parity tests compare them.  Draft sampling
 * (pse_sample_tokens) at T > 0 runs a streaming CTA per row for 0 and 3 and
 * the scalar kernel otherwise.  Other values: PSE_EINVAL.  No counterpart in
 * the reference. */
int pse_accept_select(int32_t kernel);

/* ------------------------------------------------------------------------ */
/* Model pieces (TinyGPT engine/model.py:121-206; Llama-style variant)       */
/* ------------------------------------------------------------------------ */

/* x[i*width + w, :] = tok_emb[ids[i*width + w]] + pos_emb[base_len[i] + w]
 * (engine/model.py:174-181); pos_emb may be NULL (rotary models).  x is fp32,
 * the tables have `emb_dtype`, `vocab` rows of tok_emb and `n_pos` rows of
 * pos_emb (out-of-range ids / positions contribute zeros). */
int pse_embed(const int32_t *ids, const int32_t *base_len, int32_t rows, int32_t width,
              const void *tok_emb, const void *pos_emb, int32_t d, int32_t emb_dtype, int32_t vocab,
              int32_t n_pos, float *x, void *stream);

/* pse_embed with the position of every token given (positions[i*width + w]),
 * for calls whose tokens are not consecutive positions (token-tree nodes). */
int pse_embed_pos(const int32_t *ids, const int32_t *positions, int32_t rows, int32_t width,
                  const void *tok_emb, const void *pos_emb, int32_t d, int32_t emb_dtype, int32_t vocab,
                  int32_t n_pos, float *x, void *stream);

/* LayerNorm (engine/model.py:124-126, eps 1e-5, biased variance) or RMSNorm
 * (rms != 0, beta ignored) of fp32 rows into out (out_dtype). */
int pse_norm(const float *x, int64_t ldx, const void *gamma, const void *beta, int32_t param_dtype,
             int32_t n_rows, int32_t d, float eps, int32_t rms, void *out, int64_t ldo,
             int32_t out_dtype, void *stream);

/* Residual add fused with the next norm (engine/model.py:139-142 then
 * :124-126 / :155), one warp per row: if y != NULL, x[r] += y[r] (+ bias),
 * written back to x (fp32); then out[r] = LayerNorm(x[r]) (rms == 0; eps,
 * biased variance, gamma / beta) or RMSNorm (rms != 0).  d <= 4096; y, the
 * norm parameters and out share one dtype (y_dtype == param_dtype == out_dtype). */
int pse_add_norm(float *x, int64_t ldx, const void *y, int64_t ldy, const void *bias, int32_t y_dtype,
                 const void *gamma, const void *beta, int32_t param_dtype, int32_t n_rows, int32_t d, float eps,
                 int32_t rms, void *out, int64_t ldo, int32_t out_dtype, void *stream);

/* Elementwise epilogues on [n_rows, n] row-major data:
 * op 0: y = gelu(y + bias)            (engine/model.py:127-129, exact erf GELU)
 * op 1: x(fp32) += y + bias           (residual add, engine/model.py:140-141)
 * op 2: y2[:, :n] = silu(y[:, :n]) * y[:, n:2n]   (SwiGLU)
 * bias may be NULL. y has `dtype`. */
int pse_epilogue(int32_t op, void *y, int64_t ldy, const void *bias, float *x, int64_t ldx, void *y2,
                 int64_t ldy2, int32_t n_rows, int32_t n, int32_t dtype, void *stream);

/* The nn.Linear projections of engine/model.py:73-74, 127-129, 156 on the
 * tcgen05 tensor cores: C[m, n] = A[m, k] . W[n, k]^T (+ bias[n]) (-> GELU if
 * act == 1), A / W / bias bf16, fp32 accumulation, C bf16 (out_f32 == 0) or
 * fp32.  k must be a multiple of 64; leading dimensions multiples of 8
 * elements (4 for fp32 C); base pointers 16-byte aligned.  status (nullable)
 * receives PSE_STATUS_TIMEOUT if a bounded in-kernel wait expires. */
int pse_gemm_bf16(const void *a, int64_t lda, const void *w, int64_t ldw, const void *bias, void *c,
                  int64_t ldc, int32_t m, int32_t n, int32_t k, int32_t act, int32_t out_f32, int32_t *status,
                  void *stream);

/* Rotate-half RoPE in place on the q and k heads of a fused qkv buffer
 * (q heads at column 0, k heads after them), position base_len[i] + w. */
int pse_rope(void *qkv, int64_t ld, int32_t rows, int32_t width, int32_t q_heads, int32_t kv_heads,
             int32_t head_dim, const int32_t *base_len, float theta, int32_t dtype, void *stream);

/* pse_rope with the position of every token given (positions[i*width + w]). */
int pse_rope_pos(void *qkv, int64_t ld, int32_t rows, int32_t width, int32_t q_heads, int32_t kv_heads,
                 int32_t head_dim, const int32_t *positions, float theta, int32_t dtype, void *stream);

/* Scatter rows: dst[index[i] * ld_dst + :n] = src[i * ld_src + :n] (fp32),
 * for index[i] in [0, n_dst_rows). */
int pse_scatter_rows(const float *src, int64_t ld_src, const int32_t *index, int32_t rows, int32_t n,
                     float *dst, int64_t ld_dst, int32_t n_dst_rows, void *stream);

/* ------------------------------------------------------------------------ */
/* Scheduler bookkeeping                                                    */
/* ------------------------------------------------------------------------ */

/* The per-row loop of run_continuous_speculative_batches after a step
 * (engine/scheduler.py:107-126) on the device.  Row i of the step belongs to
 * request ordinal ords[i]; its n_acc[i] + 1 accepted tokens (tokens[i *
 * tok_stride + j], n_acc[i] + 1 <= tok_stride) extend the request's output at
 * out[out_off[o] + generated[o] ...], keeping only the first max_new[o]
 * (the reference trims the overshoot when the request finishes), and
 * generated[o] grows by n_acc[i] + 1.  finished[0] receives the number of rows
 * with generated >= max_new after the step and finished[1..] those rows'
 * indices in row order (the order the reference reports and frees them).
 * Every ords[i] must index out_off / max_new / generated; rows <= 2^30. */
int pse_sched_commit(const int32_t *tokens, int32_t tok_stride, const int32_t *n_acc, const int32_t *ords,
                     int32_t rows, const int64_t *out_off, const int32_t *max_new, int32_t *generated,
                     int32_t *out, int32_t *finished, void *stream);

/* Input of the verify call when every row's final token from the previous
 * step is still pending (its position reserved, its K/V not yet written):
 * ids[i * (k + 1)] = last_token[slots[i]] (0 for a slot outside
 * [0, n_slots)), ids[i * (k + 1) + j] = drafts[i * k + j - 1] for j = 1..k,
 * first_pos[i] = base[i] - 1.  Stands in for the token list of the
 * reference's bonus call (engine/speculative.py:166-177) followed by its
 * width-k verify (engine/speculative.py:115-117), run as one call. */
int pse_step_verify_ids(const int32_t *last_token, int32_t n_slots, const int32_t *slots, const int32_t *drafts,
                        const int32_t *base, int32_t rows, int32_t k, int32_t *ids, int32_t *first_pos,
                        void *stream);

/* Input of the draft's bonus call (engine/speculative.py:166-177), merged
 * with the last draft round's call into one width-2 call: ids2[2 i] =
 * drafts[i * k + k - 1] if n_acc[i] == k else final[i], ids2[2 i + 1] =
 * final[i], pos[i] = base0[i] + min(n_acc[i], k - 1), sel[i] = 2 i + (n_acc[i]
 * == k) (the hidden row whose logits become the row's draft_next_logits). */
int pse_step_bonus_ids(const int32_t *n_acc, const int32_t *drafts, const int32_t *final_tok, const int32_t *base0,
                       int32_t rows, int32_t k, int32_t *ids2, int32_t *pos, int64_t *sel, void *stream);

/* End of a speculative step: final[i] becomes the last token of slot
 * slots_d[i] in the draft cache and of slots_t[i] in the target cache (slots
 * outside [0, n_slots) are skipped), and pack receives [tokens (rows x (k+1))
 * | n_acc (rows) | *status_d | *status_t] for the step's one device-to-host
 * copy (the accepted tokens of engine/speculative.py:159-164 with the
 * caches' error words). */
int pse_step_finish(const int32_t *final_tok, const int32_t *slots_d, const int32_t *slots_t, int32_t rows,
                    int32_t *last_d, int32_t n_slots_d, int32_t *last_t, int32_t n_slots_t, const int32_t *tokens,
                    int32_t k, const int32_t *n_acc, const int32_t *status_d, const int32_t *status_t,
                    int32_t *pack, void *stream);

/* Number of kernels the library registers (load check) and a version tag. */
int pse_version(void);
int pse_warmup(void);

#ifdef __cplusplus
}
#endif

#endif /* PSE_H_ */
