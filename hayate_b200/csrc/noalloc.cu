// Attention without caller-provided scratch.
//
// hy_varlen_attention needs a workspace (the step plan and the split-K
// partials) that its caller allocates.  Some callers cannot allocate device
// memory where they call the kernel: a plugin or FFI host that hands the
// library only the tensors of the operation, a serving runtime whose memory
// pool already owns all device memory, or a latency-critical path that must
// not call cudaMalloc because it can synchronise the device.  For them,
// hy_varlen_attention_noalloc plans and runs the bf16 kernel with its scratch
// in a fixed array that lives in this file.
//
// The array is HY_NOALLOC_SCRATCH_BYTES (12 MiB) of device memory that every
// GPU loading this library keeps until the process exits.  It fits batches of
// at most 256 sequences, 8192 query tokens and 8 KV heads on a 148-SM B200;
// larger requests are rejected.  All calls share it and it keeps the last
// call's contents, so calls that overlap on the GPU (different streams, or
// several host threads) race and must be serialised by the caller.  Nothing
// in it needs to start at zero: every call's plan kernel rewrites each field
// that the attention kernels of that call later read.
#include "hayate_b200.h"
#include "common.cuh"
#include "attention.cuh"

#include <mutex>
#include <stdio.h>

#define HY_NOALLOC_SCRATCH_BYTES (12u << 20)
#define HY_NOALLOC_MAX_SEQS 256
#define HY_NOALLOC_MAX_TOKENS 8192

// In host code this name is only a stand-in for the device array; its device
// address comes from cudaGetSymbolAddress (see scratch_for).
static __device__ __align__(256) uint8_t g_noalloc_scratch[HY_NOALLOC_SCRATCH_BYTES];

int hy_attention_kv_map(int dev, const void* base, long rows, KvMaps* out);  // capi.cu
void hy_set_error(const char* msg);                                              // capi.cu

namespace {

std::mutex g_mu;
void* g_ptr[64] = {nullptr};

// Device address of the scratch array on the current device, looked up once
// per device with that device current.
void* scratch_for(int dev) {
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_mu);
  if (g_ptr[dev] == nullptr) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      char buf[256];
      snprintf(buf, sizeof(buf), "hy_varlen_attention_noalloc: cudaGetSymbolAddress failed: %s",
               cudaGetErrorString(e));
      hy_set_error(buf);
      return nullptr;
    }
    g_ptr[dev] = p;
  }
  return g_ptr[dev];
}

}  // namespace

extern "C" int hy_varlen_attention_noalloc(
    const void* q, void* out, int32_t num_tokens, int32_t q_heads, int32_t kv_heads,
    const void* kv_cache, int32_t num_layers, int32_t num_blocks, int32_t layer,
    const int32_t* block_tables, int32_t bt_pitch, const int32_t* seq_bt_row,
    const int32_t* cu_seqlens_q, const int32_t* seq_lens_k, int32_t num_seqs, float scale,
    int32_t* err, void* stream) {
  if (!q || !out || !kv_cache || !block_tables || !cu_seqlens_q || !seq_lens_k ||
      num_seqs <= 0 || num_tokens < 0 || num_layers <= 0 || num_blocks <= 0 || layer < 0 ||
      layer >= num_layers || bt_pitch <= 0) {
    hy_set_error("hy_varlen_attention_noalloc: bad argument");
    return HY_E_INVALID;
  }
  if (q_heads != HY_GROUP * kv_heads || kv_heads <= 0) {
    hy_set_error("hy_varlen_attention_noalloc: q_heads must be 4 x kv_heads");
    return HY_E_UNSUPPORTED;
  }
  if (num_seqs > HY_NOALLOC_MAX_SEQS || num_tokens > HY_NOALLOC_MAX_TOKENS || kv_heads > 8) {
    char buf[256];
    snprintf(buf, sizeof(buf),
             "hy_varlen_attention_noalloc: batch of %d sequences / %d tokens / %d KV heads "
             "exceeds the built-in scratch limit (%d sequences, %d tokens, 8 KV heads); use "
             "hy_varlen_attention with a caller-allocated workspace",
             num_seqs, num_tokens, kv_heads, HY_NOALLOC_MAX_SEQS, HY_NOALLOC_MAX_TOKENS);
    hy_set_error(buf);
    return HY_E_INVALID;
  }
  if (num_tokens == 0) return HY_OK;
  const long layer_rows = (long)num_blocks * 2 * kv_heads * HY_BLOCK;
  const long rows = layer_rows * num_layers;
  if (rows + HY_BLOCK >= (1L << 31)) {
    hy_set_error("hy_varlen_attention_noalloc: cache exceeds 2^31 rows of 128");
    return HY_E_UNSUPPORTED;
  }
  int dev = 0;
  cudaGetDevice(&dev);
  // no prefill splits: their partial results would not fit the fixed scratch
  const PlanDims d = hy_attn_plan_dims(num_seqs, num_tokens, kv_heads, dev, false);
  const size_t need = hy_attn_workspace_bytes(d);
  if (need > HY_NOALLOC_SCRATCH_BYTES) {
    char buf[256];
    snprintf(buf, sizeof(buf),
             "hy_varlen_attention_noalloc: this batch needs %zu bytes of scratch on this device, "
             "more than the %u built in", need, HY_NOALLOC_SCRATCH_BYTES);
    hy_set_error(buf);
    return HY_E_INVALID;
  }
  void* ws = scratch_for(dev);
  if (ws == nullptr) return HY_E_CUDA;
  KvMaps map;
  int rc = hy_attention_kv_map(dev, kv_cache, rows, &map);
  if (rc) return rc;
  CUtensorMap qmap;
  rc = hy_attention_q_map(q, num_tokens, q_heads, &qmap);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = hy_launch_attn_plan(cu_seqlens_q, seq_lens_k, num_seqs, kv_heads, d, ws, err,
                                      dev, st);
  if (e == cudaSuccess)
    e = hy_launch_attn_bf16(map, qmap, kv_cache, q, out, q_heads, kv_heads, (int)(layer * layer_rows), (int)rows,
                            num_blocks, block_tables, bt_pitch, seq_bt_row, cu_seqlens_q,
                            seq_lens_k, num_seqs, scale, d, ws, err, dev, st);
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof(buf), "hy_varlen_attention_noalloc: %s", cudaGetErrorString(e));
    hy_set_error(buf);
    return HY_E_CUDA;
  }
  hy_set_error("");
  return HY_OK;
}
