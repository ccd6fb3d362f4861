// Plan layout shared by the attention kernels and the C-ABI layer.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#ifndef HY_ATTN_EARLY
#define HY_ATTN_EARLY 1       /* the public header's attention flag */
#endif

// Tensor maps over the bf16 KV cache viewed as rows of 128 elements (256 B):
//   kgroups: 4-D (64 columns, rows, 2 halves 128 B apart, 2 eight-row groups
//            2 KB apart), box = 64 x 8 x 2 x 2: one (block, K, head) tile landing
//            as four 1 KB swizzle atoms, [key group][half][8 rows][64] (128-byte
//            swizzle), so that a key tile's 8-row groups sit a uniform 2 KB apart
//   tiles:   3-D (64 columns, rows, 2 halves 128 B apart), box = 16 rows x both
//            halves: one (block, K or V, head) tile landing as [half][16 rows][64]
//            (half h at +2 KB h, 128-byte swizzle)
struct KvMaps {
  CUtensorMap kgroups;
  CUtensorMap tiles;
};

// Capacities of one attention workspace.
struct PlanDims {
  int max_pre;       // prefill items (kv_head x 64-token tile, or a key range of one)
  int max_dec;       // decode items (kv_head x block range)
  int max_seqs;
  int kv_heads;
  int max_pre_part;  // partial-result slots of prefill items split over key ranges
                     // (0: the plan splits none)
};

// Device view of a workspace (see attention.cu for the layout).
struct PlanView {
  int* header;        // n_pre, n_dec, split, status, (sequence, KV head) pairs of a
                      // per-CTA decode step (0: decode items split over all warps)
  int4* pre;          // prefill items by sequence (plan scratch)
  int4* pre_sorted;   // the same items, most key tiles first (what the kernel runs)
  int4* dec;          // per decode item: (seq, kv head, first block, end block), then
                      // (query row, key length, splits of its sequence, first item
                      // of its sequence and KV head)
  int4* dec_ids;      // per decode item, 2 x int4: its block-table row and first 4
                      // block ids, cached by the first attention launch on the
                      // plan (the plan writes row -1: not cached yet)
  int2* seqinfo;      // per sequence: first decode item, number of splits
  float* part_o;      // [max_dec][4][128]
  float2* part_ml;    // [max_dec][4]  (running max in log2 units, sum)
  int* counters;      // [max_seqs][kv_heads] finished split items (zeroed by the plan)
  int* grab;          // [64][4] per layer: next decode item, CTAs done, next prefill item
  float4* pre_part_o; // [max_pre_part][32][256]: per piece of a split prefill item, its
                      // unnormalised O as float4 c of row r at [c][r] (rows in the
                      // item's order: sub-tile X row r at 128 X + r)
  float2* pre_part_ml;// [max_pre_part][256] (running max in log2 units, sum) per row
  int* pre_ctr;       // [max_pre_part] finished pieces, at a split item's first slot
                      // (zeroed by the plan and by the merging piece)
  int max_pre, max_dec, max_seqs, max_pre_part;
};

int hy_attn_warp_slots(int dev);
// split_prefill false: a plan on these dimensions splits no prefill item over
// key ranges, and the workspace holds no partial results for them
PlanDims hy_attn_plan_dims(int max_seqs, int max_tokens, int kv_heads, int dev,
                           bool split_prefill = true);
size_t hy_attn_workspace_bytes(const PlanDims& d);

cudaError_t hy_launch_attn_plan(const int32_t* cu_q, const int32_t* seq_lens_k, int S,
                                int kv_heads, const PlanDims& d, void* ws, int32_t* err,
                                int dev, cudaStream_t st);
// The query rows' tensor map (hy_attention_q_map in capi.cu): 4-D (64 columns,
// tokens at q_heads x 256 B, heads at 256 B, 2 halves at 128 B), box 64 x 64 x
// 2 x 2 (one prefill sub-tile's Q, 32 KB, 128-byte swizzle).
int hy_attention_q_map(const void* q, int num_tokens, int q_heads, CUtensorMap* out);
cudaError_t hy_launch_attn_bf16(const KvMaps& maps, const CUtensorMap& qmap, const void* cache,
                                const void* q, void* out, int q_heads,
                                int kv_heads, int layer_row_base, int oob_row, int num_blocks,
                                const int32_t* block_tables, int bt_pitch,
                                const int32_t* seq_bt_row, const int32_t* cu_q,
                                const int32_t* seq_lens_k, int S, float scale,
                                const PlanDims& d, void* ws, int32_t* err, int dev,
                                cudaStream_t st, int flags = 0);
cudaError_t hy_launch_attn_fp32(const float* q, float* out, int T, int q_heads, int kv_heads,
                                const float* cache_layer, int num_blocks,
                                const int32_t* block_tables, int bt_pitch,
                                const int32_t* seq_bt_row, const int32_t* cu_q,
                                const int32_t* seq_lens_k, int S, float scale, int32_t* err,
                                cudaStream_t st);
