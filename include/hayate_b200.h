/*
 * hayate_b200 -- C ABI of the B200 continuous-batching kernels.
 *
 * Plain C: device pointers, sizes and a CUDA stream passed as void*.  The
 * library allocates nothing: every buffer (including the attention workspace,
 * sized by hy_attention_workspace_size) belongs to the caller.  All calls are
 * asynchronous on the given stream; none synchronises.
 *
 * Return value: HY_OK, or a negative HY_E_* code with a message available from
 * hy_get_last_error() (thread-local).  Device-side problems (an index out of
 * range, a block pool that ran dry, a wait that ran out) do not trap: the
 * kernels OR an HY_DEV_* bit into the caller's device error word `err`
 * (nullable), which the caller reads back when it synchronises.
 *
 * Layouts (all row-major):
 *   qkv           [tokens][ld]: q heads, then k heads, then v heads, 128 each
 *   q, out        [tokens][q_heads][128]
 *   KV cache      [layer][block][2 (K,V)][kv_heads][16][128]
 *   block tables  [rows][bt_pitch] int32 physical block ids in position order
 *   schedule      int32[4][num_seqs]: slot, start, q_len, flags (bit 0: sample)
 * dtype: 0 = bf16, 1 = fp32.  q_heads must be 4 x kv_heads; head_dim is 128; a
 * KV block holds 16 tokens.
 *
 * Each entry point names the reference code (axrshz/hayate) it replaces.
 */
#ifndef HAYATE_B200_H
#define HAYATE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define HY_OK 0
#define HY_E_INVALID (-1)     /* bad argument (null pointer, size, dtype) */
#define HY_E_CUDA (-2)        /* a CUDA call or launch failed */
#define HY_E_UNSUPPORTED (-3) /* geometry the kernels are not built for */

#define HY_DEV_BOUNDS 1       /* device error word bits */
#define HY_DEV_TIMEOUT 2
#define HY_DEV_POOL 4
#define HY_DEV_PLAN 8

#define HY_DTYPE_BF16 0
#define HY_DTYPE_FP32 1

#define HY_ATTN_EARLY 1       /* hy_varlen_attention flag, see there */

/* Library version (major*10000 + minor*100 + patch). */
int hy_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* hy_get_last_error(void);

/* ---------------------------------------------------------------- packing */

/* Fill the free-block stack with every block id; pops then return 0, 1, 2, ...
 * Replaces: per-request Cache() creation, hayate/engine/engine.py:63-67 and
 * hayate/model/cache.py:6-26 (the paged pool supersedes per-request tensors). */
int hy_block_pool_init(int32_t* free_stack, int32_t* free_top, int32_t num_blocks,
                       void* stream);

/* Build one step's flat batch from device-resident request state: allocate the
 * KV blocks the step needs, then write input ids, positions, slot mapping,
 * cu_seqlens_q (num_seqs+1), seq_lens_k and the rows to sample.
 * Replaces: Engine.prefill_batch / decode_batch token tensors and left padding
 * (hayate/engine/engine.py:165-194), position ids and the padding/causal mask
 * (hayate/model/qwen.py:66-106), and the pad-and-stack cache gather
 * (engine.py:80-116). */
int hy_pack_batch(const int32_t* sched, int32_t num_seqs, int32_t num_tokens,
                  const int32_t* req_tokens, int32_t tok_pitch, int32_t max_reqs,
                  int32_t* block_tables, int32_t bt_pitch, int32_t* req_num_blocks,
                  int32_t* free_stack, int32_t* free_top, int32_t num_blocks,
                  int32_t* input_ids, int32_t* positions, int32_t* slot_mapping,
                  int32_t* cu_seqlens_q, int32_t* seq_lens_k, int32_t* sample_rows,
                  int32_t* sample_seq, int32_t* err, void* stream);

/* Return all blocks of the listed slots to the pool.
 * Replaces: dropping a finished request's Cache (engine.py:196-200, cache.py:25-26). */
int hy_free_blocks(const int32_t* slots, int32_t n, int32_t max_reqs, int32_t* block_tables,
                   int32_t bt_pitch, int32_t* req_num_blocks, int32_t* free_stack,
                   int32_t* free_top, int32_t num_blocks, int32_t* err, void* stream);

/* As hy_free_blocks, but slot slots[i] gives back only its blocks from
 * position first_block[i] on; the blocks before it stay allocated for their
 * other owner (a prefix cache holding them for later requests).  No reference
 * counterpart: the reference has no block pool (its README lists prefix
 * caching as future work, README.md:70). */
int hy_free_blocks_from(const int32_t* slots, const int32_t* first_block, int32_t n,
                        int32_t max_reqs, int32_t* block_tables, int32_t bt_pitch,
                        int32_t* req_num_blocks, int32_t* free_stack, int32_t* free_top,
                        int32_t num_blocks, int32_t* err, void* stream);

/* Push n block ids onto the free stack, in order (a prefix cache evicting the
 * blocks it held).  Nothing is pushed, and an error bit is set, if an id is
 * outside [0, num_blocks) or the stack has no room for all of them.  No
 * reference counterpart (see hy_free_blocks_from). */
int hy_push_blocks(const int32_t* block_ids, int32_t n, int32_t* free_stack, int32_t* free_top,
                   int32_t num_blocks, int32_t* err, void* stream);

/* Append each sampled token to its request's token row.
 * Replaces: the device->host .item() and list append of
 * Engine._finalize_generated_token (engine.py:73-78, 178-194). */
int hy_commit_tokens(const int32_t* next_tokens, int32_t n_sample, const int32_t* sample_seq,
                     const int32_t* sched, int32_t num_seqs, int32_t* req_tokens,
                     int32_t tok_pitch, int32_t max_reqs, int32_t* err, void* stream);

/* ------------------------------------------------- QK-norm + RoPE + append */

/* Per-head RMSNorm of q and k, RoPE at `positions`, optional KV append.
 * rope_cos/rope_sin: fp32 [max_pos][64] (first half of the reference tables).
 * q_out [tokens][q_heads][128] and k_out [tokens][kv_heads][128] are nullable;
 * kv_cache_layer (nullable) receives rotated k and raw v at slot_mapping.
 * Every pointer given, and each qkv row (ld), is 16-byte aligned.
 * Replaces: q_norm/k_norm + apply_rope_vectorized + cache torch.cat,
 * hayate/model/attention.py:40-56 and hayate/model/rope.py:31-44. */
int hy_qk_norm_rope(int32_t dtype, const void* qkv, int64_t ld, int32_t num_tokens,
                    int32_t q_heads, int32_t kv_heads, const int32_t* positions,
                    const void* q_norm_w, const void* k_norm_w, const float* rope_cos,
                    const float* rope_sin, int32_t max_pos, float eps, void* q_out,
                    void* k_out, void* kv_cache_layer, const int32_t* slot_mapping,
                    int32_t num_blocks, int32_t* err, void* stream);

/* Scatter k and v ([tokens][kv_heads][128]) into the paged cache at
 * slot_mapping (slot < 0: skipped).  k, v and the cache are 16-byte aligned.
 * Replaces: torch.cat of new K/V onto the cache (hayate/model/attention.py:52-54)
 * and the per-request compaction (hayate/engine/engine.py:118-141). */
int hy_kv_append(int32_t dtype, const void* k, const void* v, int32_t num_tokens,
                 int32_t kv_heads, const int32_t* slot_mapping, void* kv_cache_layer,
                 int32_t num_blocks, int32_t* err, void* stream);

/* ------------------------------------------------------------- attention */

/* Bytes of attention workspace for batches of at most max_seqs sequences and
 * max_tokens query tokens on the current device. */
size_t hy_attention_workspace_size(int32_t max_seqs, int32_t max_tokens, int32_t kv_heads);

/* Split the step's sequences into prefill tiles and decode items; the plan is
 * written into the workspace and reused by every layer's hy_varlen_attention.
 * Replaces: the per-step mask construction, hayate/model/qwen.py:79-106. */
int hy_attention_plan(const int32_t* cu_seqlens_q, const int32_t* seq_lens_k, int32_t num_seqs,
                      int32_t kv_heads, int32_t max_seqs, int32_t max_tokens, void* workspace,
                      size_t workspace_bytes, int32_t* err, void* stream);

/* Causal varlen GQA attention over the paged cache of one layer, chunked
 * prefill and decode in one launch.  seq_bt_row (nullable) maps sequence i to
 * its block-table row.  bf16 runs the TMA + tensor-core kernel (q and the cache
 * 16-byte aligned: both are read by TMA); fp32 a scalar kernel for parity runs.
 * The plan of a prefill-only step with fewer prefill items (64 query tokens x
 * KV head) than SMs cuts long items into key-range pieces; the workspace holds
 * their partial results.  max_seqs/max_tokens must equal those given to
 * hy_attention_plan for the same workspace.  The first bf16 call after a plan
 * caches each decode item's block-table row and first block ids in the
 * workspace for the later calls: block_tables and seq_bt_row must not change
 * between a plan and the last call that uses it.
 * flags: 0, or HY_ATTN_EARLY when the plan, the block tables and the cache
 * (but for the keys and values of this call's query tokens) were written at
 * least two launches before this one on the stream, and the call is not the
 * plan's first.  A decode-only bf16 launch then reads its work items and starts
 * loading the K/V of older blocks before it waits for the kernel just before
 * it (programmatic dependent launch), overlapping that kernel's tail.  An
 * engine step meets this from its second layer on.
 * Replaces: cat + F.scaled_dot_product_attention(attn_mask, enable_gqa=True),
 * hayate/model/attention.py:52-64. */
int hy_varlen_attention(int32_t dtype, const void* q, void* out, int32_t num_tokens,
                        int32_t q_heads, int32_t kv_heads, const void* kv_cache,
                        int32_t num_layers, int32_t num_blocks, int32_t layer,
                        const int32_t* block_tables, int32_t bt_pitch,
                        const int32_t* seq_bt_row, const int32_t* cu_seqlens_q,
                        const int32_t* seq_lens_k, int32_t num_seqs, float scale,
                        int32_t max_seqs, int32_t max_tokens, void* workspace,
                        size_t workspace_bytes, int32_t flags, int32_t* err, void* stream);

/* Plan + bf16 attention in one call, with no caller workspace: for callers
 * that cannot allocate device memory where they call the kernel (a plugin or
 * FFI host that passes only the operation's tensors, a runtime whose memory
 * pool owns all device memory, a latency-critical path that must not call
 * cudaMalloc because it can synchronise the device).  Its scratch is a fixed
 * 12 MiB device array inside the library, held by every GPU that loads it
 * until the process exits; batches above 256 sequences, 8192 query tokens or
 * 8 KV heads are rejected (HY_E_INVALID).  The first call on a device looks up
 * the array's address there; make that first call before any stream capture.
 * All calls share the array, so calls that overlap on the GPU race.  Its plan
 * cuts no prefill item into key-range pieces (their partial results would not
 * fit the array).  No counterpart in the reference: it adds an allocation-free
 * way into hy_varlen_attention's kernels. */
int hy_varlen_attention_noalloc(const void* q, void* out, int32_t num_tokens, int32_t q_heads,
                                int32_t kv_heads, const void* kv_cache, int32_t num_layers,
                                int32_t num_blocks, int32_t layer, const int32_t* block_tables,
                                int32_t bt_pitch, const int32_t* seq_bt_row,
                                const int32_t* cu_seqlens_q, const int32_t* seq_lens_k,
                                int32_t num_seqs, float scale, int32_t* err, void* stream);

/* ------------------------------------------------------- layer elementwise */

/* Residual add + RMSNorm, row-wise over `cols` (<= 4096, a multiple of 8 for
 * bf16 / 4 for fp32): if delta is non-null, x[r] <- round(x[r] + delta[r]) in
 * place; then y[r] = round(RMSNorm(x[r]) * w), fp32 math, as nn.RMSNorm.
 * Replaces: the residual adds and input_layernorm / post_attention_layernorm /
 * final norm, hayate/model/block.py:18-31 and hayate/model/qwen.py:35,122. */
int hy_add_rms_norm(int32_t dtype, void* x, int64_t ldx, const void* delta, int64_t ldd,
                    int32_t rows, int32_t cols, const void* w, float eps, void* y, int64_t ldy,
                    void* stream);

/* As hy_add_rms_norm with the residual's delta given as nparts (1..64) fp32
 * split-K partials of the projection that produced it: part p of row r at
 * parts + p * part_stride + r * ldp (floats).  delta = round(sum of the parts in
 * order), then x[r] <- round(x[r] + delta) and y[r] = round(RMSNorm(x[r]) * w),
 * so the projection's output is rounded once, as its unsplit GEMM rounds it.
 * Lets the caller run a decode-sized projection (few rows, long K) as a batched
 * GEMM over K slices, which fills the GPU where one GEMM of a few rows cannot.
 * Replaces: the o_proj / down_proj outputs' residual adds and the following
 * post_attention_layernorm / input_layernorm, hayate/model/block.py:21-31,
 * hayate/model/attention.py:66 and hayate/model/linear.py:11-14. */
int hy_add_rms_norm_splitk(int32_t dtype, void* x, int64_t ldx, const float* parts,
                           int32_t nparts, int64_t part_stride, int64_t ldp, int32_t rows,
                           int32_t cols, const void* w, float eps, void* y, int64_t ldy,
                           void* stream);

/* hy_add_rms_norm over gathered rows: output row r takes residual row
 * x_rows[r] of x (x has x_nrows rows; x itself is not written), adds delta[r]
 * (model dtype) or round(sum of the nparts fp32 split-K partials of row r,
 * part_stride apart) -- at most one of them, row pitch ldd -- writes the
 * updated residual to row r of x_out (nullable) and y[r] = RMSNorm * w.  A row
 * index outside [0, x_nrows) ORs HY_DEV_BOUNDS into err and leaves row r
 * unwritten.  Lets the last block run its post-attention half and the final
 * norm on the step's sampled tokens only.
 * Replaces: the last block's residual add + post_attention_layernorm
 * (hayate/model/block.py:24-28) and the final norm applied to every position
 * (hayate/model/qwen.py:122-123, whose logits the engine then cuts to the last
 * position, engine.py:163). */
int hy_gather_add_rms_norm(int32_t dtype, const void* x, int64_t ldx, const int32_t* x_rows,
                           int32_t x_nrows, const void* delta, int64_t ldd, const float* parts,
                           int32_t nparts, int64_t part_stride, int32_t rows, int32_t cols,
                           const void* w, float eps, void* x_out, int64_t ldxo, void* y,
                           int64_t ldy, int32_t* err, void* stream);

/* y[r][i] = silu(gu[r][i]) * gu[r][inter + i] with the reference's two rounding
 * points (silu result, product).  `inter` a multiple of 8 (bf16) / 4 (fp32).
 * Replaces: FeedForward's silu(gate) * up, hayate/model/linear.py:11-13. */
int hy_silu_mul(int32_t dtype, const void* gu, int64_t ld, int32_t rows, int32_t inter, void* y,
                int64_t ldy, void* stream);

/* ---------------------------------------------------------------- sampling */

/* out[r] = argmax(logits[r][0:vocab]) with first-index ties (torch.argmax).
 * Replaces: Engine.sample, hayate/engine/engine.py:69-71. */
int hy_argmax(int32_t dtype, const void* logits, int64_t ld, int32_t rows, int32_t vocab,
              int32_t* out, void* stream);

/* Greedy sampling fused into the LM head (bf16 only): out[r] = argmax over
 * v < vocab of bf16(sum_k x[r][k] * w[v][k]), the last-token logits of the
 * sampled rows computed on the tensor cores and reduced in the same kernel, so
 * the rows x vocab logits are never written.  x: rows x hidden (row pitch ldx
 * elements; the final RMSNorm's output), w: the tied embedding, vocab x hidden
 * (pitch ldw); hidden a multiple of 64; x, w 16-byte aligned with pitches a
 * multiple of 8 elements.  Each logit is rounded to bf16 before the comparison,
 * which follows torch.argmax (first index on ties, NaN above every number,
 * -0 == +0); a logit whose fp32 sum lies within rounding distance of a bf16
 * boundary can round the other way than a library GEMM with another summation
 * order.  Any number of rows (launches of up to 256).  workspace:
 * hy_lm_head_argmax_workspace_size() bytes, 16-byte aligned, zeroed once by
 * the caller before its first use; every call leaves it zeroed again, so calls
 * on one stream may share it and calls that may overlap on the GPU may not.
 * Waits that run out set HY_DEV_TIMEOUT in *err (may be null).
 * Replaces: out_head and Engine.sample, hayate/model/qwen.py:122-123 (logits
 * of every position) and hayate/engine/engine.py:69-71 (torch.argmax). */
int64_t hy_lm_head_argmax_workspace_size(void);
int hy_lm_head_argmax(const void* x, int64_t ldx, int32_t rows, const void* w, int64_t ldw,
                      int32_t vocab, int32_t hidden, int32_t* out, void* workspace,
                      int32_t* err, void* stream);

/* ------------------------------------------------------------- diagnostics */

/* Failure-detection self-test (no reference counterpart: the reference has no
 * device waits).  Launches one CTA that waits on an mbarrier nothing arrives
 * on, with a limit of timeout_ms; the wait gives up, ORs HY_DEV_TIMEOUT into
 * *err and the kernel returns, writing *done = 1 (2 if the wait had succeeded).
 * The kernels' own waits use the same bounded wait (limit 2 s). */
int hy_selftest_wait_timeout(int32_t* err, int32_t timeout_ms, int32_t* done, void* stream);

/* Accuracy self-test of the polynomial 2^x the prefill softmax computes part of
 * its weights with (the rest on the hardware exp2 unit): y[i] = 2^x[i] for
 * -126 < x[i] <= 127 with relative error below 1e-4 (2e-4 at -126, whose result
 * is subnormal); 0 for x[i] < -126 and for -inf.  No
 * reference counterpart: the reference takes its softmax from torch SDPA
 * (hayate/model/attention.py:58-64). */
int hy_selftest_exp2_poly(const float* x, float* y, int32_t n, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* HAYATE_B200_H */
