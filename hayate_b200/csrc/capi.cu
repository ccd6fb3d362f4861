// C-ABI layer: argument checks, tensor-map cache, error reporting.
#include "hayate_b200.h"
#include "common.cuh"

#include <stdlib.h>
#include "attention.cuh"

#include <mutex>
#include <stdio.h>
#include <string.h>

// Launchers defined in the kernel files.
cudaError_t hy_launch_pool_init(int32_t*, int32_t*, int, cudaStream_t);
cudaError_t hy_launch_pack(const int32_t*, int, int, const int32_t*, int, int, int32_t*, int,
                           int32_t*, int32_t*, int32_t*, int, int32_t*, int32_t*, int32_t*,
                           int32_t*, int32_t*, int32_t*, int32_t*, int32_t*, cudaStream_t);
cudaError_t hy_launch_push(const int32_t*, int, int32_t*, int32_t*, int, int32_t*, cudaStream_t);
cudaError_t hy_launch_free(const int32_t*, const int32_t*, int, int, int32_t*, int, int32_t*,
                           int32_t*, int32_t*, int, int32_t*, cudaStream_t);
cudaError_t hy_launch_commit(const int32_t*, int, const int32_t*, const int32_t*, int, int32_t*,
                             int, int, int32_t*, cudaStream_t);
cudaError_t hy_launch_qk_norm_rope(int, const void*, int, int, int, int, const int32_t*,
                                   const void*, const void*, const float*, const float*, int,
                                   float, void*, void*, void*, const int32_t*, int, int32_t*,
                                   cudaStream_t);
cudaError_t hy_launch_kv_append(int, const void*, const void*, int, int, const int32_t*, void*,
                                int, int32_t*, cudaStream_t);
cudaError_t hy_launch_argmax(int, const void*, long, int, int, int32_t*, cudaStream_t);
cudaError_t hy_launch_add_rms_norm(int, void*, long, const void*, long, int, int, const void*,
                                   float, void*, long, const float*, int, long, cudaStream_t,
                                   const int32_t* = nullptr, int = 0, void* = nullptr, long = 0,
                                   int32_t* = nullptr);
cudaError_t hy_launch_silu_mul(int, const void*, long, int, int, void*, long, cudaStream_t);

namespace {

thread_local char g_last_error[512] = "";

int fail(int code, const char* fmt, const char* detail = nullptr) {
  if (detail) snprintf(g_last_error, sizeof(g_last_error), fmt, detail);
  else snprintf(g_last_error, sizeof(g_last_error), "%s", fmt);
  return code;
}

int cuda_result(cudaError_t e, const char* what) {
  if (e == cudaSuccess) { g_last_error[0] = 0; return HY_OK; }
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s", what, cudaGetErrorString(e));
  return HY_E_CUDA;
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

bool dtype_ok(int32_t dtype) { return dtype == HY_DTYPE_BF16 || dtype == HY_DTYPE_FP32; }

// ---- tensor maps over the bf16 KV cache (one per cache allocation)
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct MapEntry {
  int dev;
  const void* base;
  long rows;
  KvMaps maps;
};

std::mutex g_map_mu;
MapEntry g_maps[32];
int g_nmaps = 0;
EncodeTiledFn g_encode = nullptr;

int get_encoder() {
  if (g_encode) return HY_OK;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &fn, 12000,
                                                   cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr)
    return fail(HY_E_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  g_encode = reinterpret_cast<EncodeTiledFn>(fn);
  return HY_OK;
}

// The cache's tensor maps (KvMaps): rows of 128 bf16 (256 B), 16-row boxes,
// 128-byte swizzle in shared memory.
int kv_map_for(int dev, const void* base, long rows, KvMaps* out) {
  std::lock_guard<std::mutex> lk(g_map_mu);
  for (int i = 0; i < g_nmaps; ++i)
    if (g_maps[i].dev == dev && g_maps[i].base == base && g_maps[i].rows == rows) {
      *out = g_maps[i].maps;
      return HY_OK;
    }
  int rc = get_encoder();
  if (rc) return rc;
  if ((reinterpret_cast<uintptr_t>(base) & 15) != 0)
    return fail(HY_E_INVALID, "kv_cache must be 16-byte aligned");
  KvMaps m;
  // element (x, y, z, w) at x + 128 y + 64 z + 1024 w: column x of half z of
  // row y + 8 w; a box at row y = a block's first row covers its 16 rows, and
  // a y past the end (the zero-fill row) leaves the whole box zero
  cuuint64_t dims4[4] = {64, (cuuint64_t)rows, 2, 2};
  cuuint64_t strides4[3] = {HY_HEAD_DIM * 2, 128, 8 * HY_HEAD_DIM * 2};
  cuuint32_t box4[4] = {64, 8, 2, 2};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = g_encode(&m.kgroups, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base),
                        dims4, strides4, box4, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r == CUDA_SUCCESS) {
    cuuint64_t dims3[3] = {64, (cuuint64_t)rows, 2};
    cuuint64_t strides3[2] = {HY_HEAD_DIM * 2, 128};         // row: 256 B, half: 128 B
    cuuint32_t box3[3] = {64, HY_BLOCK, 2};
    r = g_encode(&m.tiles, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims3,
                 strides3, box3, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                 CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  }
  if (r != CUDA_SUCCESS) {
    char buf[64];
    snprintf(buf, sizeof(buf), "%d", (int)r);
    return fail(HY_E_CUDA, "cuTensorMapEncodeTiled failed (CUresult %s)", buf);
  }
  const int slot = g_nmaps < 32 ? g_nmaps++ : (int)(reinterpret_cast<uintptr_t>(base) >> 8) % 32;
  g_maps[slot] = MapEntry{dev, base, rows, m};
  *out = m;
  return HY_OK;
}

int current_device() {
  int d = 0;
  cudaGetDevice(&d);
  return d;
}

}  // namespace

// Waits on an mbarrier that nothing arrives on: the bounded wait must give up,
// set HY_ERR_TIMEOUT in the error word and let the kernel return.
__global__ void wait_timeout_probe_kernel(int32_t* err, uint64_t timeout_ns, int32_t* done) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) mbar_init(&bar, 1);
  fence_mbar_init();
  __syncthreads();
  const bool ok = mbar_wait(&bar, 0u, err, timeout_ns);
  if (threadIdx.x == 0) *done = ok ? 2 : 1;
}

// The prefill softmax's polynomial 2^x on n inputs (one thread each).
// Elements 2k, 2k + 1 go through the packed form the softmax uses (a last odd
// element through the scalar one).
__global__ void exp2_poly_probe_kernel(const float* __restrict__ x, float* __restrict__ y, int n) {
  const int i = 2 * (blockIdx.x * blockDim.x + threadIdx.x);
  if (i + 1 < n) {
    const float2 r = exp2_poly2(make_float2(x[i], x[i + 1]));
    y[i] = r.x;
    y[i + 1] = r.y;
  } else if (i < n) {
    y[i] = exp2_poly(x[i]);
  }
}

// Shared with other translation units of the library (not part of the C ABI).
int hy_attention_kv_map(int dev, const void* base, long rows, KvMaps* out) {
  return kv_map_for(dev, base, rows, out);
}

// The query rows of one call as a tensor map (encoded per call: the token count
// changes every step, and encoding is host arithmetic).  Element (x, t, h, z) is
// column 64 z + x of head h of token t; tokens past num_tokens read zeros.
int hy_attention_q_map(const void* q, int num_tokens, int q_heads, CUtensorMap* out) {
  int rc = get_encoder();
  if (rc) return rc;
  if ((reinterpret_cast<uintptr_t>(q) & 15) != 0)
    return fail(HY_E_INVALID, "hy_varlen_attention: q must be 16-byte aligned");
  cuuint64_t dims[4] = {64, (cuuint64_t)num_tokens, (cuuint64_t)q_heads, 2};
  cuuint64_t strides[3] = {(cuuint64_t)q_heads * HY_HEAD_DIM * 2, HY_HEAD_DIM * 2, 128};
  cuuint32_t box[4] = {64, 64, 2, 2};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = g_encode(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(q), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[64];
    snprintf(buf, sizeof(buf), "%d", (int)r);
    return fail(HY_E_CUDA, "cuTensorMapEncodeTiled failed on q (CUresult %s)", buf);
  }
  return HY_OK;
}

// A row-major bf16 matrix (rows x cols, row pitch row_bytes) as a 2-D tensor
// map whose box is 64 columns (one 128-byte swizzle row) x box_rows rows, with
// 128-byte swizzle in shared memory; rows past the end read zeros.
int hy_encode_rows_map(const void* base, long cols, long rows, long row_bytes, int box_rows,
                       CUtensorMap* out) {
  int rc = get_encoder();
  if (rc) return rc;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(out, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                        strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[64];
    snprintf(buf, sizeof(buf), "%d", (int)r);
    return fail(HY_E_CUDA, "cuTensorMapEncodeTiled failed on a row-major matrix (CUresult %s)",
                buf);
  }
  return HY_OK;
}

void hy_set_error(const char* msg) { snprintf(g_last_error, sizeof(g_last_error), "%s", msg); }

bool hy_pdl_enabled() {
  static const bool on = [] {
    const char* e = getenv("HY_PDL");
    return !(e != nullptr && e[0] == '0');
  }();
  return on;
}

extern "C" {

int hy_version(void) { return 100; }

const char* hy_get_last_error(void) { return g_last_error; }

int hy_block_pool_init(int32_t* free_stack, int32_t* free_top, int32_t num_blocks, void* stream) {
  if (!free_stack || !free_top || num_blocks <= 0)
    return fail(HY_E_INVALID, "hy_block_pool_init: null pointer or num_blocks <= 0");
  return cuda_result(hy_launch_pool_init(free_stack, free_top, num_blocks, as_stream(stream)),
                     "hy_block_pool_init");
}

int hy_pack_batch(const int32_t* sched, int32_t num_seqs, int32_t num_tokens,
                  const int32_t* req_tokens, int32_t tok_pitch, int32_t max_reqs,
                  int32_t* block_tables, int32_t bt_pitch, int32_t* req_num_blocks,
                  int32_t* free_stack, int32_t* free_top, int32_t num_blocks,
                  int32_t* input_ids, int32_t* positions, int32_t* slot_mapping,
                  int32_t* cu_seqlens_q, int32_t* seq_lens_k, int32_t* sample_rows,
                  int32_t* sample_seq, int32_t* err, void* stream) {
  if (!sched || !req_tokens || !block_tables || !req_num_blocks || !free_stack || !free_top ||
      !input_ids || !positions || !slot_mapping || !cu_seqlens_q || !seq_lens_k ||
      !sample_rows || !sample_seq)
    return fail(HY_E_INVALID, "hy_pack_batch: null pointer");
  if (num_seqs <= 0 || num_tokens < 0 || tok_pitch <= 0 || max_reqs <= 0 || bt_pitch <= 0 ||
      num_blocks <= 0)
    return fail(HY_E_INVALID, "hy_pack_batch: non-positive size");
  return cuda_result(hy_launch_pack(sched, num_seqs, num_tokens, req_tokens, tok_pitch, max_reqs,
                                    block_tables, bt_pitch, req_num_blocks, free_stack, free_top,
                                    num_blocks, input_ids, positions, slot_mapping, cu_seqlens_q,
                                    seq_lens_k, sample_rows, sample_seq, err, as_stream(stream)),
                     "hy_pack_batch");
}

int hy_free_blocks(const int32_t* slots, int32_t n, int32_t max_reqs, int32_t* block_tables,
                   int32_t bt_pitch, int32_t* req_num_blocks, int32_t* free_stack,
                   int32_t* free_top, int32_t num_blocks, int32_t* err, void* stream) {
  if (n == 0) return HY_OK;
  if (!slots || !block_tables || !req_num_blocks || !free_stack || !free_top || n < 0 ||
      max_reqs <= 0 || bt_pitch <= 0 || num_blocks <= 0)
    return fail(HY_E_INVALID, "hy_free_blocks: bad argument");
  return cuda_result(hy_launch_free(slots, nullptr, n, max_reqs, block_tables, bt_pitch,
                                    req_num_blocks, free_stack, free_top, num_blocks, err,
                                    as_stream(stream)),
                     "hy_free_blocks");
}

int hy_free_blocks_from(const int32_t* slots, const int32_t* first_block, int32_t n,
                        int32_t max_reqs, int32_t* block_tables, int32_t bt_pitch,
                        int32_t* req_num_blocks, int32_t* free_stack, int32_t* free_top,
                        int32_t num_blocks, int32_t* err, void* stream) {
  if (n == 0) return HY_OK;
  if (!slots || !first_block || !block_tables || !req_num_blocks || !free_stack || !free_top ||
      n < 0 || max_reqs <= 0 || bt_pitch <= 0 || num_blocks <= 0)
    return fail(HY_E_INVALID, "hy_free_blocks_from: bad argument");
  return cuda_result(hy_launch_free(slots, first_block, n, max_reqs, block_tables, bt_pitch,
                                    req_num_blocks, free_stack, free_top, num_blocks, err,
                                    as_stream(stream)),
                     "hy_free_blocks_from");
}

int hy_push_blocks(const int32_t* block_ids, int32_t n, int32_t* free_stack, int32_t* free_top,
                   int32_t num_blocks, int32_t* err, void* stream) {
  if (n == 0) return HY_OK;
  if (!block_ids || !free_stack || !free_top || n < 0 || num_blocks <= 0)
    return fail(HY_E_INVALID, "hy_push_blocks: bad argument");
  return cuda_result(hy_launch_push(block_ids, n, free_stack, free_top, num_blocks, err,
                                    as_stream(stream)),
                     "hy_push_blocks");
}

int hy_commit_tokens(const int32_t* next_tokens, int32_t n_sample, const int32_t* sample_seq,
                     const int32_t* sched, int32_t num_seqs, int32_t* req_tokens,
                     int32_t tok_pitch, int32_t max_reqs, int32_t* err, void* stream) {
  if (n_sample == 0) return HY_OK;
  if (!next_tokens || !sample_seq || !sched || !req_tokens || n_sample < 0 || num_seqs <= 0 ||
      tok_pitch <= 0 || max_reqs <= 0)
    return fail(HY_E_INVALID, "hy_commit_tokens: bad argument");
  return cuda_result(hy_launch_commit(next_tokens, n_sample, sample_seq, sched, num_seqs,
                                      req_tokens, tok_pitch, max_reqs, err, as_stream(stream)),
                     "hy_commit_tokens");
}

static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int hy_qk_norm_rope(int32_t dtype, const void* qkv, int64_t ld, int32_t num_tokens,
                    int32_t q_heads, int32_t kv_heads, const int32_t* positions,
                    const void* q_norm_w, const void* k_norm_w, const float* rope_cos,
                    const float* rope_sin, int32_t max_pos, float eps, void* q_out,
                    void* k_out, void* kv_cache_layer, const int32_t* slot_mapping,
                    int32_t num_blocks, int32_t* err, void* stream) {
  if (!dtype_ok(dtype)) return fail(HY_E_INVALID, "hy_qk_norm_rope: dtype must be 0 or 1");
  if (num_tokens == 0) return HY_OK;
  if (!qkv || !positions || !q_norm_w || !k_norm_w || !rope_cos || !rope_sin || num_tokens < 0)
    return fail(HY_E_INVALID, "hy_qk_norm_rope: bad argument");
  if (q_heads != HY_GROUP * kv_heads || kv_heads <= 0)
    return fail(HY_E_UNSUPPORTED, "hy_qk_norm_rope: q_heads must be 4 x kv_heads");
  if (ld < (int64_t)(q_heads + 2 * kv_heads) * HY_HEAD_DIM || ld > INT32_MAX)
    return fail(HY_E_INVALID, "hy_qk_norm_rope: ld smaller than one qkv row");
  if (kv_cache_layer && (!slot_mapping || num_blocks <= 0))
    return fail(HY_E_INVALID, "hy_qk_norm_rope: cache given without slot_mapping/num_blocks");
  if (!aligned16(qkv) || ld % (dtype == 0 ? 8 : 4) != 0 || !aligned16(q_norm_w) ||
      !aligned16(k_norm_w) || !aligned16(rope_cos) || !aligned16(rope_sin) || !aligned16(q_out) ||
      !aligned16(k_out) || !aligned16(kv_cache_layer))
    return fail(HY_E_INVALID, "hy_qk_norm_rope: rows and tables must be 16-byte aligned");
  return cuda_result(
      hy_launch_qk_norm_rope(dtype, qkv, (int)ld, num_tokens, q_heads, kv_heads, positions,
                             q_norm_w, k_norm_w, rope_cos, rope_sin, max_pos, eps, q_out, k_out,
                             kv_cache_layer, slot_mapping, num_blocks, err, as_stream(stream)),
      "hy_qk_norm_rope");
}

int hy_kv_append(int32_t dtype, const void* k, const void* v, int32_t num_tokens,
                 int32_t kv_heads, const int32_t* slot_mapping, void* kv_cache_layer,
                 int32_t num_blocks, int32_t* err, void* stream) {
  if (!dtype_ok(dtype)) return fail(HY_E_INVALID, "hy_kv_append: dtype must be 0 or 1");
  if (num_tokens == 0) return HY_OK;
  if (!k || !v || !slot_mapping || !kv_cache_layer || num_tokens < 0 || kv_heads <= 0 ||
      num_blocks <= 0)
    return fail(HY_E_INVALID, "hy_kv_append: bad argument");
  if (!aligned16(k) || !aligned16(v) || !aligned16(kv_cache_layer))
    return fail(HY_E_INVALID, "hy_kv_append: k, v and the cache must be 16-byte aligned");
  return cuda_result(hy_launch_kv_append(dtype, k, v, num_tokens, kv_heads, slot_mapping,
                                         kv_cache_layer, num_blocks, err, as_stream(stream)),
                     "hy_kv_append");
}

size_t hy_attention_workspace_size(int32_t max_seqs, int32_t max_tokens, int32_t kv_heads) {
  if (max_seqs <= 0 || max_tokens <= 0 || kv_heads <= 0) return 0;
  return hy_attn_workspace_bytes(hy_attn_plan_dims(max_seqs, max_tokens, kv_heads,
                                                   current_device()));
}

int hy_attention_plan(const int32_t* cu_seqlens_q, const int32_t* seq_lens_k, int32_t num_seqs,
                      int32_t kv_heads, int32_t max_seqs, int32_t max_tokens, void* workspace,
                      size_t workspace_bytes, int32_t* err, void* stream) {
  if (!cu_seqlens_q || !seq_lens_k || !workspace || num_seqs <= 0 || kv_heads <= 0)
    return fail(HY_E_INVALID, "hy_attention_plan: bad argument");
  if (num_seqs > max_seqs) return fail(HY_E_INVALID, "hy_attention_plan: num_seqs > max_seqs");
  const int dev = current_device();
  const PlanDims d = hy_attn_plan_dims(max_seqs, max_tokens, kv_heads, dev);
  if (workspace_bytes < hy_attn_workspace_bytes(d))
    return fail(HY_E_INVALID, "hy_attention_plan: workspace smaller than hy_attention_workspace_size");
  if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
    return fail(HY_E_INVALID, "hy_attention_plan: workspace must be 256-byte aligned");
  return cuda_result(hy_launch_attn_plan(cu_seqlens_q, seq_lens_k, num_seqs, kv_heads, d,
                                         workspace, err, dev, as_stream(stream)),
                     "hy_attention_plan");
}

int hy_varlen_attention(int32_t dtype, const void* q, void* out, int32_t num_tokens,
                        int32_t q_heads, int32_t kv_heads, const void* kv_cache,
                        int32_t num_layers, int32_t num_blocks, int32_t layer,
                        const int32_t* block_tables, int32_t bt_pitch,
                        const int32_t* seq_bt_row, const int32_t* cu_seqlens_q,
                        const int32_t* seq_lens_k, int32_t num_seqs, float scale,
                        int32_t max_seqs, int32_t max_tokens, void* workspace,
                        size_t workspace_bytes, int32_t flags, int32_t* err, void* stream) {
  if (!dtype_ok(dtype)) return fail(HY_E_INVALID, "hy_varlen_attention: dtype must be 0 or 1");
  if ((flags & ~HY_ATTN_EARLY) != 0) return fail(HY_E_INVALID, "hy_varlen_attention: unknown flags");
  if (!q || !out || !kv_cache || !block_tables || !cu_seqlens_q || !seq_lens_k ||
      num_seqs <= 0 || num_tokens < 0 || num_layers <= 0 || num_blocks <= 0 || layer < 0 ||
      layer >= num_layers || bt_pitch <= 0)
    return fail(HY_E_INVALID, "hy_varlen_attention: bad argument");
  if (q_heads != HY_GROUP * kv_heads || kv_heads <= 0)
    return fail(HY_E_UNSUPPORTED, "hy_varlen_attention: q_heads must be 4 x kv_heads");
  if (num_tokens == 0) return HY_OK;
  const long layer_rows = (long)num_blocks * 2 * kv_heads * HY_BLOCK;
  if (dtype == HY_DTYPE_FP32) {
    const float* base = static_cast<const float*>(kv_cache) + (size_t)layer * layer_rows * HY_HEAD_DIM;
    return cuda_result(hy_launch_attn_fp32(static_cast<const float*>(q), static_cast<float*>(out),
                                           num_tokens, q_heads, kv_heads, base, num_blocks,
                                           block_tables, bt_pitch, seq_bt_row, cu_seqlens_q,
                                           seq_lens_k, num_seqs, scale, err, as_stream(stream)),
                       "hy_varlen_attention(fp32)");
  }
  if (!workspace) return fail(HY_E_INVALID, "hy_varlen_attention: bf16 needs a planned workspace");
  const long rows = layer_rows * num_layers;
  if (rows + HY_BLOCK >= (1L << 31))
    return fail(HY_E_UNSUPPORTED, "hy_varlen_attention: cache exceeds 2^31 rows of 128");
  const int dev = current_device();
  const PlanDims d = hy_attn_plan_dims(max_seqs, max_tokens, kv_heads, dev);
  if (workspace_bytes < hy_attn_workspace_bytes(d))
    return fail(HY_E_INVALID, "hy_varlen_attention: workspace too small for max_seqs/max_tokens");
  KvMaps map;
  int rc = kv_map_for(dev, kv_cache, rows, &map);
  if (rc) return rc;
  CUtensorMap qmap;
  rc = hy_attention_q_map(q, num_tokens, q_heads, &qmap);
  if (rc) return rc;
  return cuda_result(
      hy_launch_attn_bf16(map, qmap, kv_cache, q, out, q_heads, kv_heads, (int)(layer * layer_rows), (int)rows,
                          num_blocks, block_tables, bt_pitch, seq_bt_row, cu_seqlens_q,
                          seq_lens_k, num_seqs, scale, d, workspace, err, dev, as_stream(stream),
                          flags),
      "hy_varlen_attention(bf16)");
}

static bool vec_aligned(const void* p, int64_t ld, int32_t dtype, int32_t n) {
  const int v = dtype == HY_DTYPE_BF16 ? 8 : 4;
  return (reinterpret_cast<uintptr_t>(p) & 15) == 0 && ld % v == 0 && n % v == 0;
}

int hy_add_rms_norm(int32_t dtype, void* x, int64_t ldx, const void* delta, int64_t ldd,
                    int32_t rows, int32_t cols, const void* w, float eps, void* y, int64_t ldy,
                    void* stream) {
  if (!dtype_ok(dtype)) return fail(HY_E_INVALID, "hy_add_rms_norm: dtype must be 0 or 1");
  if (rows == 0) return HY_OK;
  const int maxc = 4096;
  if (!x || !w || !y || rows < 0 || cols <= 0 || cols > maxc || ldx < cols || ldy < cols ||
      (delta && ldd < cols))
    return fail(HY_E_INVALID, "hy_add_rms_norm: bad argument (cols must be in 1..4096)");
  if (!vec_aligned(x, ldx, dtype, cols) || !vec_aligned(y, ldy, dtype, cols) ||
      !vec_aligned(w, cols, dtype, cols) || (delta && !vec_aligned(delta, ldd, dtype, cols)))
    return fail(HY_E_INVALID, "hy_add_rms_norm: rows must be 16-byte aligned vectors");
  return cuda_result(hy_launch_add_rms_norm(dtype, x, (long)ldx, delta, (long)ldd, rows, cols, w,
                                            eps, y, (long)ldy, nullptr, 0, 0, as_stream(stream)),
                     "hy_add_rms_norm");
}

int hy_add_rms_norm_splitk(int32_t dtype, void* x, int64_t ldx, const float* parts,
                           int32_t nparts, int64_t part_stride, int64_t ldp, int32_t rows,
                           int32_t cols, const void* w, float eps, void* y, int64_t ldy,
                           void* stream) {
  if (!dtype_ok(dtype)) return fail(HY_E_INVALID, "hy_add_rms_norm_splitk: dtype must be 0 or 1");
  if (rows == 0) return HY_OK;
  const int maxc = 4096;
  if (!x || !parts || !w || !y || rows < 0 || cols <= 0 || cols > maxc || ldx < cols ||
      ldy < cols || ldp < cols || nparts < 1 || nparts > 64 ||
      (nparts > 1 && part_stride < (int64_t)rows * ldp))
    return fail(HY_E_INVALID, "hy_add_rms_norm_splitk: bad argument (cols must be in 1..4096, "
                              "1..64 parts that do not overlap)");
  if (!vec_aligned(x, ldx, dtype, cols) || !vec_aligned(y, ldy, dtype, cols) ||
      !vec_aligned(w, cols, dtype, cols) || !vec_aligned(parts, ldp, HY_DTYPE_FP32, cols) ||
      (part_stride & 3))
    return fail(HY_E_INVALID, "hy_add_rms_norm_splitk: rows must be 16-byte aligned vectors");
  return cuda_result(hy_launch_add_rms_norm(dtype, x, (long)ldx, nullptr, (long)ldp, rows, cols,
                                            w, eps, y, (long)ldy, parts, nparts,
                                            (long)part_stride, as_stream(stream)),
                     "hy_add_rms_norm_splitk");
}

int hy_gather_add_rms_norm(int32_t dtype, const void* x, int64_t ldx, const int32_t* x_rows,
                           int32_t x_nrows, const void* delta, int64_t ldd, const float* parts,
                           int32_t nparts, int64_t part_stride, int32_t rows, int32_t cols,
                           const void* w, float eps, void* x_out, int64_t ldxo, void* y,
                           int64_t ldy, int32_t* err, void* stream) {
  if (!dtype_ok(dtype)) return fail(HY_E_INVALID, "hy_gather_add_rms_norm: dtype must be 0 or 1");
  if (rows == 0) return HY_OK;
  const int maxc = 4096;
  if (!x || !x_rows || !w || !y || rows < 0 || x_nrows <= 0 || cols <= 0 || cols > maxc ||
      ldx < cols || ldy < cols || (x_out && ldxo < cols) || (delta && parts) ||
      ((delta || parts) && ldd < cols) || (parts && (nparts < 1 || nparts > 64)) ||
      (parts && nparts > 1 && part_stride < (int64_t)rows * ldd))
    return fail(HY_E_INVALID, "hy_gather_add_rms_norm: bad argument (cols must be in 1..4096, "
                              "at most one of delta and parts)");
  if (!vec_aligned(x, ldx, dtype, cols) || !vec_aligned(y, ldy, dtype, cols) ||
      !vec_aligned(w, cols, dtype, cols) || (delta && !vec_aligned(delta, ldd, dtype, cols)) ||
      (x_out && !vec_aligned(x_out, ldxo, dtype, cols)) ||
      (parts && (!vec_aligned(parts, ldd, HY_DTYPE_FP32, cols) || (part_stride & 3))))
    return fail(HY_E_INVALID, "hy_gather_add_rms_norm: rows must be 16-byte aligned vectors");
  return cuda_result(hy_launch_add_rms_norm(dtype, const_cast<void*>(x), (long)ldx, delta,
                                            (long)ldd, rows, cols, w, eps, y, (long)ldy, parts,
                                            parts ? nparts : 0, (long)part_stride,
                                            as_stream(stream), x_rows, x_nrows, x_out, (long)ldxo,
                                            err),
                     "hy_gather_add_rms_norm");
}

int hy_silu_mul(int32_t dtype, const void* gu, int64_t ld, int32_t rows, int32_t inter, void* y,
                int64_t ldy, void* stream) {
  if (!dtype_ok(dtype)) return fail(HY_E_INVALID, "hy_silu_mul: dtype must be 0 or 1");
  if (rows == 0) return HY_OK;
  if (!gu || !y || rows < 0 || inter <= 0 || ld < 2 * (int64_t)inter || ldy < inter)
    return fail(HY_E_INVALID, "hy_silu_mul: bad argument");
  if (!vec_aligned(gu, ld, dtype, inter) || !vec_aligned(y, ldy, dtype, inter))
    return fail(HY_E_INVALID, "hy_silu_mul: rows must be 16-byte aligned vectors");
  return cuda_result(hy_launch_silu_mul(dtype, gu, (long)ld, rows, inter, y, (long)ldy,
                                        as_stream(stream)), "hy_silu_mul");
}

int hy_selftest_wait_timeout(int32_t* err, int32_t timeout_ms, int32_t* done, void* stream) {
  if (!err || !done || timeout_ms <= 0 || timeout_ms > 10000)
    return fail(HY_E_INVALID, "hy_selftest_wait_timeout: bad argument (timeout 1..10000 ms)");
  wait_timeout_probe_kernel<<<1, 32, 0, as_stream(stream)>>>(err, (uint64_t)timeout_ms * 1000000ull,
                                                             done);
  return cuda_result(cudaGetLastError(), "hy_selftest_wait_timeout");
}

int hy_selftest_exp2_poly(const float* x, float* y, int32_t n, void* stream) {
  if (!x || !y || n < 0) return fail(HY_E_INVALID, "hy_selftest_exp2_poly: bad argument");
  if (n == 0) return HY_OK;
  exp2_poly_probe_kernel<<<(n / 2 + 256) / 256, 256, 0, as_stream(stream)>>>(x, y, n);
  return cuda_result(cudaGetLastError(), "hy_selftest_exp2_poly");
}

int hy_argmax(int32_t dtype, const void* logits, int64_t ld, int32_t rows, int32_t vocab,
              int32_t* out, void* stream) {
  if (!dtype_ok(dtype)) return fail(HY_E_INVALID, "hy_argmax: dtype must be 0 or 1");
  if (rows == 0) return HY_OK;
  if (!logits || !out || rows < 0 || vocab <= 0 || ld < vocab)
    return fail(HY_E_INVALID, "hy_argmax: bad argument");
  return cuda_result(hy_launch_argmax(dtype, logits, (long)ld, rows, vocab, out, as_stream(stream)),
                     "hy_argmax");
}

}  // extern "C"
