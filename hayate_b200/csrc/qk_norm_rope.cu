// Fused per-head QK-RMSNorm + RoPE, with the KV-cache append folded in.
//
// Reference semantics (hayate/model/attention.py:40-48, rope.py:31-44):
//   y   = round( (f32(x) * rstd) * f32(w) ),  rstd = 1 / sqrt(mean(f32(x)^2) + eps)
//   out = round( f32(y)*cos[pos] + f32(rot(y))*sin[pos] ),  rot(y) = cat(-y2, y1)
// where round() is the model dtype (bf16, or identity for fp32) and every fp32
// product and sum is rounded separately (no fused multiply-add), as the
// reference's separate tensor ops do.  cos/sin are the reference's fp32 tables
// (rope.py:3-13); only their first 64 columns are passed because the reference
// duplicates the angle vector (rope.py:10).
//
// The input is the fused QKV projection row [q heads | k heads | v heads].
// Query heads go to q_out; key heads (after norm+RoPE) and value heads go to the
// paged cache at slot_mapping (replacing the torch.cat of attention.py:52-54 and
// the per-request compaction of engine.py:118-141); k_out is an optional plain
// copy of the rotated keys.
#include "common.cuh"

namespace {

template <typename T> struct Pair;
template <> struct Pair<__nv_bfloat16> {
  using V = __nv_bfloat162;
  static HY_DEVICE float2 load(const __nv_bfloat16* p) {
    return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
  }
  static HY_DEVICE void store(__nv_bfloat16* p, float a, float b) {
    *reinterpret_cast<__nv_bfloat162*>(p) = __floats2bfloat162_rn(a, b);
  }
  static HY_DEVICE float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
};
template <> struct Pair<float> {
  static HY_DEVICE float2 load(const float* p) { return *reinterpret_cast<const float2*>(p); }
  static HY_DEVICE void store(float* p, float a, float b) {
    *reinterpret_cast<float2*>(p) = make_float2(a, b);
  }
  static HY_DEVICE float round(float v) { return v; }
};

// Byte-for-byte location of (slot, kv, head, d) in the paged cache of one layer:
// cache[block][kv][head][token_in_block][d].
template <typename T>
HY_DEVICE T* cache_ptr(T* layer_base, int slot, int kv, int head, int kv_heads) {
  const int blk = slot / HY_BLOCK, j = slot % HY_BLOCK;
  return layer_base + ((((size_t)blk * 2 + kv) * kv_heads + head) * HY_BLOCK + j) * HY_HEAD_DIM;
}

template <typename T>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(
    const T* __restrict__ qkv, int ld, int T_tokens, int q_heads, int kv_heads,
    const int32_t* __restrict__ positions, const T* __restrict__ q_w, const T* __restrict__ k_w,
    const float* __restrict__ rope_cos, const float* __restrict__ rope_sin, int max_pos,
    float eps, T* __restrict__ q_out, T* __restrict__ k_out,
    T* __restrict__ cache, const int32_t* __restrict__ slot_mapping, int num_blocks,
    int32_t* err) {
  using P = Pair<T>;
  const int lane = threadIdx.x & 31;
  const int heads = q_heads + 2 * kv_heads;
  const long total = (long)T_tokens * heads;
  const long nwarps = (long)gridDim.x * (blockDim.x >> 5);
  const int d_lo = 2 * lane, d_hi = 64 + 2 * lane;
  for (long w = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total; w += nwarps) {
    const int t = (int)(w / heads), h = (int)(w % heads);
    const T* src = qkv + (size_t)t * ld + (size_t)h * HY_HEAD_DIM;
    const float2 lo = P::load(src + d_lo);
    const float2 hi = P::load(src + d_hi);
    int slot = -1;
    if (cache != nullptr && h >= q_heads) {
      slot = slot_mapping[t];
      if (slot >= (long)num_blocks * HY_BLOCK) { hy_flag(err, HY_ERR_BOUNDS); slot = -1; }
    }
    if (h >= q_heads + kv_heads) {                     // value head: cache copy only
      if (slot >= 0) {
        T* dst = cache_ptr(cache, slot, 1, h - q_heads - kv_heads, kv_heads);
        P::store(dst + d_lo, lo.x, lo.y);
        P::store(dst + d_hi, hi.x, hi.y);
      }
      continue;
    }
    float ss = __fadd_rn(__fadd_rn(__fmul_rn(lo.x, lo.x), __fmul_rn(lo.y, lo.y)),
                         __fadd_rn(__fmul_rn(hi.x, hi.x), __fmul_rn(hi.y, hi.y)));
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)HY_HEAD_DIM), eps)));
    const T* wv = (h < q_heads) ? q_w : k_w;
    const float2 wlo = P::load(wv + d_lo), whi = P::load(wv + d_hi);
    const float y0 = P::round(__fmul_rn(__fmul_rn(lo.x, rstd), wlo.x));
    const float y1 = P::round(__fmul_rn(__fmul_rn(lo.y, rstd), wlo.y));
    const float y2 = P::round(__fmul_rn(__fmul_rn(hi.x, rstd), whi.x));
    const float y3 = P::round(__fmul_rn(__fmul_rn(hi.y, rstd), whi.y));
    int pos = positions[t];
    if (pos < 0 || pos >= max_pos) { hy_flag(err, HY_ERR_BOUNDS); pos = 0; }
    const float2 c = *reinterpret_cast<const float2*>(rope_cos + (size_t)pos * 64 + d_lo);
    const float2 s = *reinterpret_cast<const float2*>(rope_sin + (size_t)pos * 64 + d_lo);
    // first half: y1*cos + (-y2)*sin ; second half: y2*cos + y1*sin
    const float o0 = __fadd_rn(__fmul_rn(y0, c.x), __fmul_rn(-y2, s.x));
    const float o1 = __fadd_rn(__fmul_rn(y1, c.y), __fmul_rn(-y3, s.y));
    const float o2 = __fadd_rn(__fmul_rn(y2, c.x), __fmul_rn(y0, s.x));
    const float o3 = __fadd_rn(__fmul_rn(y3, c.y), __fmul_rn(y1, s.y));
    if (h < q_heads) {
      if (q_out) {
        T* dst = q_out + ((size_t)t * q_heads + h) * HY_HEAD_DIM;
        P::store(dst + d_lo, o0, o1);
        P::store(dst + d_hi, o2, o3);
      }
    } else {
      const int kh = h - q_heads;
      if (k_out) {
        T* dst = k_out + ((size_t)t * kv_heads + kh) * HY_HEAD_DIM;
        P::store(dst + d_lo, o0, o1);
        P::store(dst + d_hi, o2, o3);
      }
      if (slot >= 0) {
        T* dst = cache_ptr(cache, slot, 0, kh, kv_heads);
        P::store(dst + d_lo, o0, o1);
        P::store(dst + d_hi, o2, o3);
      }
    }
  }
}

// Plain KV append: k, v are [T][kv_heads][128]; one warp moves one head row.
template <typename T>
__global__ void __launch_bounds__(256) kv_append_kernel(
    const T* __restrict__ k, const T* __restrict__ v, int T_tokens, int kv_heads,
    const int32_t* __restrict__ slot_mapping, T* __restrict__ cache, int num_blocks,
    int32_t* err) {
  const int lane = threadIdx.x & 31;
  const long total = (long)T_tokens * kv_heads * 2;
  const long nwarps = (long)gridDim.x * (blockDim.x >> 5);
  constexpr int PER_LANE = HY_HEAD_DIM / 32;       // 4 elements
  for (long w = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total; w += nwarps) {
    const int kv = (int)(w & 1);
    const long th = w >> 1;
    const int t = (int)(th / kv_heads), h = (int)(th % kv_heads);
    const int slot = slot_mapping[t];
    if (slot < 0) continue;
    if (slot >= (long)num_blocks * HY_BLOCK) { hy_flag(err, HY_ERR_BOUNDS); continue; }
    const T* src = (kv ? v : k) + ((size_t)t * kv_heads + h) * HY_HEAD_DIM + lane * PER_LANE;
    T* dst = cache_ptr(cache, slot, kv, h, kv_heads) + lane * PER_LANE;
    if constexpr (sizeof(T) == 2) {
      *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(src);
    } else {
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
    }
  }
}

int grid_for(long warps) {
  long blocks = (warps + 7) / 8;
  if (blocks > 148L * 16) blocks = 148L * 16;
  return blocks > 0 ? (int)blocks : 1;
}

}  // namespace

cudaError_t hy_launch_qk_norm_rope(int dtype, const void* qkv, int ld, int T, int q_heads,
                                   int kv_heads, const int32_t* positions, const void* q_w,
                                   const void* k_w, const float* rope_cos, const float* rope_sin,
                                   int max_pos, float eps, void* q_out, void* k_out, void* cache,
                                   const int32_t* slot_mapping, int num_blocks, int32_t* err,
                                   cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  const int grid = grid_for((long)T * (q_heads + 2 * kv_heads));
  if (dtype == 0) {
    using B = __nv_bfloat16;
    qk_norm_rope_kernel<B><<<grid, 256, 0, st>>>(
        (const B*)qkv, ld, T, q_heads, kv_heads, positions, (const B*)q_w, (const B*)k_w,
        rope_cos, rope_sin, max_pos, eps, (B*)q_out, (B*)k_out, (B*)cache, slot_mapping,
        num_blocks, err);
  } else {
    qk_norm_rope_kernel<float><<<grid, 256, 0, st>>>(
        (const float*)qkv, ld, T, q_heads, kv_heads, positions, (const float*)q_w,
        (const float*)k_w, rope_cos, rope_sin, max_pos, eps, (float*)q_out, (float*)k_out,
        (float*)cache, slot_mapping, num_blocks, err);
  }
  return cudaGetLastError();
}

cudaError_t hy_launch_kv_append(int dtype, const void* k, const void* v, int T, int kv_heads,
                                const int32_t* slot_mapping, void* cache, int num_blocks,
                                int32_t* err, cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  const int grid = grid_for((long)T * kv_heads * 2);
  if (dtype == 0) {
    using B = __nv_bfloat16;
    kv_append_kernel<B><<<grid, 256, 0, st>>>((const B*)k, (const B*)v, T, kv_heads,
                                              slot_mapping, (B*)cache, num_blocks, err);
  } else {
    kv_append_kernel<float><<<grid, 256, 0, st>>>((const float*)k, (const float*)v, T, kv_heads,
                                                  slot_mapping, (float*)cache, num_blocks, err);
  }
  return cudaGetLastError();
}
