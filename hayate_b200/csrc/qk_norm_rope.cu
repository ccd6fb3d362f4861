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

// fp32 path (the parity build of the model): one warp per (token, head), each
// lane holding elements (2 lane, 2 lane + 1) and their RoPE partners 64 apart.
template <typename T>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(
    const T* __restrict__ qkv, int ld, int T_tokens, int q_heads, int kv_heads,
    const int32_t* __restrict__ positions, const T* __restrict__ q_w, const T* __restrict__ k_w,
    const float* __restrict__ rope_cos, const float* __restrict__ rope_sin, int max_pos,
    float eps, T* __restrict__ q_out, T* __restrict__ k_out,
    T* __restrict__ cache, const int32_t* __restrict__ slot_mapping, int num_blocks,
    int32_t* err) {
  hy_grid_wait();
  hy_grid_trigger();
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

// bf16 path of the same operation, laid out for bandwidth: a head row (128
// elements, 256 bytes) is one 16-byte vector per lane of a half-warp, so every
// load and store is a full 16-byte access and a warp moves two rows at once.
// Work unit = (token, group of NPC passes of 16 head rows): pass j of group g
// covers head rows 16 (g NPC + j) + half-warp.  Small batches (decode steps)
// use NPC = 1, so a few tokens still spread over many CTAs; prefill-sized
// batches use NPC = all passes of a token, so one CTA iteration covers the
// whole token with one load of its position, slot and cos/sin rows.  Each CTA
// walks its units one grid stride apart and loads the next unit's head rows,
// position and slot before it computes the current one, so two units' rows are
// in flight per lane (the kernel is bound by bytes in flight, not by issue).
// The RoPE partner of element d (d +- 64) sits 8 lanes away and comes over a
// shuffle.  Rounding points and the order of the products are those of the
// kernel above; only the order of the sum of squares differs (8 in-lane terms,
// then a 16-lane butterfly).
constexpr int QNR_THREADS = 256;
constexpr int QNR_GROUPS = QNR_THREADS / 16;        // head rows per pass

HY_DEVICE void bf16x8_to_f32(const uint4& u, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

HY_DEVICE float2 bf2_to_f2(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
}
HY_DEVICE uint32_t f2_to_bf2(float2 f) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(f.x, f.y);
  return *reinterpret_cast<const uint32_t*>(&h);
}

HY_DEVICE uint4 f32_to_bf16x8(const float (&f)[8]) {
  uint4 u;
  __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
  return u;
}

// One unit's inputs held by a lane: its NPC head-row vectors, the token's
// position and cache slot.
template <int NPC>
struct QnrUnit {
  uint4 raw[NPC];
  int pos, slot;
};

template <int NPC>
HY_DEVICE void qnr_load(QnrUnit<NPC>& u, int t, int g, int T_tokens, int heads, int grp, int d0,
                        const __nv_bfloat16* __restrict__ qkv, int ld,
                        const int32_t* __restrict__ positions,
                        const int32_t* __restrict__ slot_mapping, bool want_slot) {
  u.pos = 0;
  u.slot = -1;
#pragma unroll
  for (int j = 0; j < NPC; ++j) u.raw[j] = make_uint4(0u, 0u, 0u, 0u);
  if (t >= T_tokens) return;
  u.pos = positions[t];
  if (want_slot) u.slot = slot_mapping[t];
#pragma unroll
  for (int j = 0; j < NPC; ++j) {
    const int h = (g * NPC + j) * QNR_GROUPS + grp;
    if (h < heads)
      u.raw[j] = *reinterpret_cast<const uint4*>(qkv + (size_t)t * ld + (size_t)h * HY_HEAD_DIM + d0);
  }
}

template <int NPC>
__global__ void __launch_bounds__(QNR_THREADS, NPC >= 4 ? 2 : 3) qk_norm_rope_bf16_kernel(
    const __nv_bfloat16* __restrict__ qkv, int ld, int T_tokens, int q_heads, int kv_heads,
    const int32_t* __restrict__ positions, const __nv_bfloat16* __restrict__ q_w,
    const __nv_bfloat16* __restrict__ k_w, const float* __restrict__ rope_cos,
    const float* __restrict__ rope_sin, int max_pos, float eps, __nv_bfloat16* __restrict__ q_out,
    __nv_bfloat16* __restrict__ k_out, __nv_bfloat16* __restrict__ cache,
    const int32_t* __restrict__ slot_mapping, int num_blocks, int32_t* err) {
  hy_grid_wait();
  hy_grid_trigger();
  const int grp = threadIdx.x >> 4, l = threadIdx.x & 15;
  const int heads = q_heads + 2 * kv_heads;
  const int npass = (heads + QNR_GROUPS - 1) / QNR_GROUPS;
  const int G = (npass + NPC - 1) / NPC;           // pass groups per token
  const int d0 = l * 8;                    // this lane's 8 elements of a row
  const int c0 = (l & 7) * 8;              // ... and their RoPE table columns
  const bool upper = l >= 8;               // elements 64..127: partner is d - 64
  const bool want_slot = cache != nullptr;
  const long slot_end = (long)num_blocks * HY_BLOCK;
  // unit = t * G + g walks the grid stride as (token, group) pairs, with no
  // division in the loop
  const int dt = (int)(gridDim.x / G), dg = (int)(gridDim.x % G);
  int t = (int)(blockIdx.x / G), g = (int)(blockIdx.x % G);
  QnrUnit<NPC> cur;
  qnr_load(cur, t, g, T_tokens, heads, grp, d0, qkv, ld, positions, slot_mapping, want_slot);
  while (t < T_tokens) {                           // uniform over the CTA
    int tn = t + dt, gn = g + dg;                  // the unit one grid stride on
    if (gn >= G) { gn -= G; ++tn; }
    QnrUnit<NPC> nxt;
    qnr_load(nxt, tn, gn, T_tokens, heads, grp, d0, qkv, ld, positions, slot_mapping, want_slot);
    int pos = cur.pos;
    if (pos < 0 || pos >= max_pos) { hy_flag(err, HY_ERR_BOUNDS); pos = 0; }
    int slot = cur.slot;
    if (slot >= slot_end) { hy_flag(err, HY_ERR_BOUNDS); slot = -1; }
    float cs[8], sn[8];
    {
      const float4* cp = reinterpret_cast<const float4*>(rope_cos + (size_t)pos * 64 + c0);
      const float4* sp = reinterpret_cast<const float4*>(rope_sin + (size_t)pos * 64 + c0);
      const float4 a = cp[0], b = cp[1], e = sp[0], f = sp[1];
      cs[0] = a.x; cs[1] = a.y; cs[2] = a.z; cs[3] = a.w; cs[4] = b.x; cs[5] = b.y; cs[6] = b.z; cs[7] = b.w;
      sn[0] = e.x; sn[1] = e.y; sn[2] = e.z; sn[3] = e.w; sn[4] = f.x; sn[5] = f.y; sn[6] = f.z; sn[7] = f.w;
    }
#pragma unroll
    for (int j = 0; j < NPC; ++j) {
      const int h = (g * NPC + j) * QNR_GROUPS + grp;
      const bool valid = h < heads;                // uniform over each half-warp
      const uint4 raw = cur.raw[j];
      if (valid && h >= q_heads + kv_heads) {      // value head: cache copy only
        if (slot >= 0)
          *reinterpret_cast<uint4*>(cache_ptr(cache, slot, 1, h - q_heads - kv_heads, kv_heads) + d0) = raw;
      }
      // a warp with no query or key row in this pass (both half-warps value
      // heads or past the end) skips the norm; otherwise all its lanes run it
      // for the shuffles
      if (__all_sync(0xffffffffu, !valid || h >= q_heads + kv_heads)) continue;
      // packed f32x2 arithmetic: each lane of a pair rounded as the scalar op
      const uint32_t* xr = &raw.x;
      float2 ss2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 v = bf2_to_f2(xr[q]);
        ss2 = __fadd2_rn(ss2, __fmul2_rn(v, v));
      }
      float ss = __fadd_rn(ss2.x, ss2.y);
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      // mean = ss / 128 exactly (a power of two)
      const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.0f / HY_HEAD_DIM), eps)));
      const float2 rs2 = make_float2(rstd, rstd);
      const uint4 wraw = *reinterpret_cast<const uint4*>(((h < q_heads) ? q_w : k_w) + d0);
      const uint32_t* wr = &wraw.x;
      uint4 yb;                                   // y = bf16((x * rstd) * w)
      uint32_t* yr = &yb.x;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        yr[q] = f2_to_bf2(__fmul2_rn(__fmul2_rn(bf2_to_f2(xr[q]), rs2), bf2_to_f2(wr[q])));
      uint4 pb;
      pb.x = __shfl_xor_sync(0xffffffffu, yb.x, 8);
      pb.y = __shfl_xor_sync(0xffffffffu, yb.y, 8);
      pb.z = __shfl_xor_sync(0xffffffffu, yb.z, 8);
      pb.w = __shfl_xor_sync(0xffffffffu, yb.w, 8);
      const uint32_t* pr = &pb.x;
      uint4 ob;                                   // lower: y*cos + (-y[d+64])*sin; upper: y*cos + y[d-64]*sin
      uint32_t* orr = &ob.x;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 yv = bf2_to_f2(yr[q]);
        float2 pe = bf2_to_f2(pr[q]);
        if (!upper) pe = make_float2(-pe.x, -pe.y);
        const float2 c2 = make_float2(cs[2 * q], cs[2 * q + 1]);
        const float2 s2 = make_float2(sn[2 * q], sn[2 * q + 1]);
        orr[q] = f2_to_bf2(__fadd2_rn(__fmul2_rn(yv, c2), __fmul2_rn(pe, s2)));
      }
      if (!valid || h >= q_heads + kv_heads) continue;
      if (h < q_heads) {
        if (q_out) *reinterpret_cast<uint4*>(q_out + ((size_t)t * q_heads + h) * HY_HEAD_DIM + d0) = ob;
      } else {
        const int kh = h - q_heads;
        if (k_out) *reinterpret_cast<uint4*>(k_out + ((size_t)t * kv_heads + kh) * HY_HEAD_DIM + d0) = ob;
        if (slot >= 0) *reinterpret_cast<uint4*>(cache_ptr(cache, slot, 0, kh, kv_heads) + d0) = ob;
      }
    }
    cur = nxt;
    t = tn;
    g = gn;
  }
}

// The bf16 path for prefill-sized batches: a head row is 8 lanes x 16
// elements (two 16-byte vectors per lane), so the per-row work that does not
// scale with the elements (the reciprocal square root, the reduction, the
// addressing) is spread over 4 rows per warp; the CTA's consumer warps (8 x
// heads threads, rounded up to whole warps, at most 384: 48 head rows) cover
// every head row of one token per iteration.  A producer warp streams the
// CTA's tokens (one grid stride apart) into a QNR_NS-stage shared-memory ring
// by bulk copies: each stage holds a token's whole qkv row and its cos and sin
// table rows (the producer reads 32 tokens' positions at once), so several
// tokens are in flight without holding registers and the consumers make no
// dependent global load.  A thread's head row is the same for every token, so its
// norm weights are loaded once.  The RoPE partner of element d (d +- 64) is 4
// lanes away.  Rounding points are those of the kernel above, except that the
// sum of squares is accumulated with fused multiply-adds (its order already
// differs from the reference's).
constexpr int QNR_LPR = 8;                        // lanes per head row
constexpr int QNR_ROWS_MAX_THREADS = 384;         // consumer threads: up to 48 head rows
constexpr int QNR_NS = 4;                         // ring stages (qkv rows of tokens)

__global__ void __launch_bounds__(QNR_ROWS_MAX_THREADS + 32, 2) qk_norm_rope_rows_kernel(
    const __nv_bfloat16* __restrict__ qkv, int ld, int T_tokens, int q_heads, int kv_heads,
    const int32_t* __restrict__ positions, const __nv_bfloat16* __restrict__ q_w,
    const __nv_bfloat16* __restrict__ k_w, const float* __restrict__ rope_cos,
    const float* __restrict__ rope_sin, int max_pos, float eps, __nv_bfloat16* __restrict__ q_out,
    __nv_bfloat16* __restrict__ k_out, __nv_bfloat16* __restrict__ cache,
    const int32_t* __restrict__ slot_mapping, int num_blocks, int32_t* err) {
  extern __shared__ __align__(128) uint8_t qnr_ring[];
  __shared__ uint64_t full[QNR_NS], empty[QNR_NS];
  const int heads = q_heads + 2 * kv_heads;
  const int row_bytes = heads * HY_HEAD_DIM * 2;
  const int stage_bytes = row_bytes + 2 * 64 * 4;   // qkv row, cos row, sin row
  const int n_cons = (int)blockDim.x - 32;        // consumer threads
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int grid = (int)gridDim.x;
  const int ntok = T_tokens > (int)blockIdx.x ? (T_tokens - (int)blockIdx.x + grid - 1) / grid : 0;
  if (threadIdx.x == 0) {
    for (int s = 0; s < QNR_NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], n_cons / 32);          // one arrival per consumer warp
    }
    fence_mbar_init();
  }
  __syncthreads();
  if ((int)threadIdx.x >= n_cons) {               // the producer warp
    hy_grid_wait();
    hy_grid_trigger();
    int i = 0;
    bool ok = true;
    while (ok && i < ntok) {
      // the positions of the next 32 tokens, one per lane (a bad one flags the
      // error and reads table row 0)
      int pl = 0;
      if (i + lane < ntok) {
        pl = positions[(int)blockIdx.x + (i + lane) * grid];
        if (pl < 0 || pl >= max_pos) { hy_flag(err, HY_ERR_BOUNDS); pl = 0; }
      }
      for (int k = 0; k < 32 && i < ntok; ++k, ++i) {
        const int pos = __shfl_sync(0xffffffffu, pl, k);
        const int s = i % QNR_NS;
        int w_ok = 1;
        if (lane == 0 && i >= QNR_NS) w_ok = mbar_wait(&empty[s], ((i / QNR_NS) - 1) & 1, err);
        if (!__shfl_sync(0xffffffffu, w_ok, 0)) { ok = false; break; }
        if (lane == 0) {
          const int t = (int)blockIdx.x + i * grid;
          uint8_t* st = qnr_ring + s * stage_bytes;
          mbar_arrive_expect_tx(&full[s], stage_bytes);
          bulk_load(st, qkv + (size_t)t * ld, row_bytes, &full[s]);
          bulk_load(st + row_bytes, rope_cos + (size_t)pos * 64, 256, &full[s]);
          bulk_load(st + row_bytes + 256, rope_sin + (size_t)pos * 64, 256, &full[s]);
        }
      }
    }
    // the last copies issued land before the CTA may exit
    if (lane == 0)
      for (int j = i > QNR_NS ? i - QNR_NS : 0; j < i; ++j)
        mbar_wait(&full[j % QNR_NS], (j / QNR_NS) & 1, nullptr);
    return;
  }
  const int h = threadIdx.x / QNR_LPR, l = threadIdx.x % QNR_LPR;
  const bool valid = h < heads;
  const bool is_v = valid && h >= q_heads + kv_heads;
  const bool is_q = h < q_heads;
  const bool normed = valid && !is_v;
  // a warp (4 rows) with no query or key row skips the norm and the shuffles
  const bool warp_norm = __any_sync(0xffffffffu, normed);
  const int d0 = l * 16;                          // this lane's 16 elements
  const int c0 = (l & 3) * 16;                    // ... and their RoPE table columns
  const bool upper = l >= 4;                      // elements 64..127: partner is d - 64
  float2 wf[8];                                   // the row's norm weights, as pairs
  {
    const __nv_bfloat16* wsrc = (is_q ? q_w : k_w) + d0;
    const uint4 wa = normed ? *reinterpret_cast<const uint4*>(wsrc) : make_uint4(0u, 0u, 0u, 0u);
    const uint4 wb = normed ? *reinterpret_cast<const uint4*>(wsrc + 8) : make_uint4(0u, 0u, 0u, 0u);
    const uint32_t* a = &wa.x;
    const uint32_t* b = &wb.x;
#pragma unroll
    for (int q = 0; q < 4; ++q) { wf[q] = bf2_to_f2(a[q]); wf[4 + q] = bf2_to_f2(b[q]); }
  }
  hy_grid_wait();
  hy_grid_trigger();
  const bool want_slot = cache != nullptr && valid && h >= q_heads;
  const long slot_end = (long)num_blocks * HY_BLOCK;
  int t = (int)blockIdx.x;
  int slot_n = (ntok > 0 && want_slot) ? slot_mapping[t] : -1;   // the next token's slot
  for (int i = 0; i < ntok; ++i, t += grid) {
    const int s = i % QNR_NS;
    int slot = slot_n;
    if (i + 1 < ntok && want_slot) slot_n = slot_mapping[t + grid];
    if (slot >= slot_end) { hy_flag(err, HY_ERR_BOUNDS); slot = -1; }
    const bool w_ok = mbar_wait(&full[s], (i / QNR_NS) & 1, err);
    if (__any_sync(0xffffffffu, !w_ok)) break;
    const uint8_t* st = qnr_ring + s * stage_bytes;
    uint4 ca = make_uint4(0u, 0u, 0u, 0u), cb = ca;
    if (valid) {
      const uint4* p = reinterpret_cast<const uint4*>(st + h * HY_HEAD_DIM * 2 + d0 * 2);
      ca = p[0];
      cb = p[1];
    }
    // this lane's 16 cos and sin columns stay in the stage until the RoPE
    const float4* cp = reinterpret_cast<const float4*>(st + row_bytes) + c0 / 4;
    const float4* sp = reinterpret_cast<const float4*>(st + row_bytes + 256) + c0 / 4;
    if (is_v && slot >= 0) {                      // value head: cache copy only
      uint4* dst = reinterpret_cast<uint4*>(cache_ptr(cache, slot, 1, h - q_heads - kv_heads, kv_heads) + d0);
      dst[0] = ca;
      dst[1] = cb;
    }
    if (warp_norm) {
      uint32_t xr[8] = {ca.x, ca.y, ca.z, ca.w, cb.x, cb.y, cb.z, cb.w};
      float2 ss2 = make_float2(0.f, 0.f);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float2 v = bf2_to_f2(xr[q]);
        ss2 = __ffma2_rn(v, v, ss2);
      }
      float ss = __fadd_rn(ss2.x, ss2.y);
#pragma unroll
      for (int o = 4; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
      // mean = ss / 128 exactly (a power of two)
      const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fmul_rn(ss, 1.0f / HY_HEAD_DIM), eps)));
      const float2 rs2 = make_float2(rstd, rstd);
      uint32_t yr[8];                             // y = bf16((x * rstd) * w)
#pragma unroll
      for (int q = 0; q < 8; ++q) yr[q] = f2_to_bf2(__fmul2_rn(__fmul2_rn(bf2_to_f2(xr[q]), rs2), wf[q]));
      uint32_t pr[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) pr[q] = __shfl_xor_sync(0xffffffffu, yr[q], 4);
      if (normed) {
        uint32_t orr[8];                          // lower: y*cos + (-y[d+64])*sin; upper: y*cos + y[d-64]*sin
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float4 c4 = cp[k], s4 = sp[k];
          const float2 cc[2] = {make_float2(c4.x, c4.y), make_float2(c4.z, c4.w)};
          const float2 sv[2] = {upper ? make_float2(s4.x, s4.y) : make_float2(-s4.x, -s4.y),
                                upper ? make_float2(s4.z, s4.w) : make_float2(-s4.z, -s4.w)};
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int q = 2 * k + e;
            orr[q] = f2_to_bf2(__fadd2_rn(__fmul2_rn(bf2_to_f2(yr[q]), cc[e]),
                                          __fmul2_rn(bf2_to_f2(pr[q]), sv[e])));
          }
        }
        const uint4 oa = make_uint4(orr[0], orr[1], orr[2], orr[3]);
        const uint4 ob = make_uint4(orr[4], orr[5], orr[6], orr[7]);
        if (is_q) {
          if (q_out) {
            uint4* dst = reinterpret_cast<uint4*>(q_out + ((size_t)t * q_heads + h) * HY_HEAD_DIM + d0);
            dst[0] = oa;
            dst[1] = ob;
          }
        } else {
          const int kh = h - q_heads;
          if (k_out) {
            uint4* dst = reinterpret_cast<uint4*>(k_out + ((size_t)t * kv_heads + kh) * HY_HEAD_DIM + d0);
            dst[0] = oa;
            dst[1] = ob;
          }
          if (slot >= 0) {
            uint4* dst = reinterpret_cast<uint4*>(cache_ptr(cache, slot, 0, kh, kv_heads) + d0);
            dst[0] = oa;
            dst[1] = ob;
          }
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);        // the stage is free once every warp is done with it
  }
}

// Plain KV append: k, v are [T][kv_heads][128].  A head row is one 16-byte
// vector per lane of a lane group (16 lanes for bf16, 32 for fp32); item
// i = token * 2 * kv_heads + row (K rows, then V rows); KVA_UNROLL items'
// loads are in flight per lane before the stores.
#ifndef HY_KVA_UNROLL
#define HY_KVA_UNROLL 4
#endif
constexpr int KVA_THREADS = 256;
constexpr int KVA_UNROLL = HY_KVA_UNROLL;

template <typename T>
__global__ void __launch_bounds__(KVA_THREADS) kv_append_kernel(
    const T* __restrict__ k, const T* __restrict__ v, int T_tokens, int kv_heads,
    const int32_t* __restrict__ slot_mapping, T* __restrict__ cache, int num_blocks,
    int32_t* err) {
  hy_grid_wait();
  hy_grid_trigger();
  constexpr int E = 16 / (int)sizeof(T);           // elements per lane
  constexpr int LPR = HY_HEAD_DIM / E;             // lanes per row
  constexpr int G = KVA_THREADS / LPR;             // rows per CTA pass
  const int grp = threadIdx.x / LPR, l = threadIdx.x % LPR;
  const int R = 2 * kv_heads;
  const long total = (long)T_tokens * R;
  const long stride = (long)gridDim.x * G;
  for (long base = (long)blockIdx.x * G + grp; base < total; base += stride * KVA_UNROLL) {
    uint4 val[KVA_UNROLL];
    T* dst[KVA_UNROLL];
#pragma unroll
    for (int u = 0; u < KVA_UNROLL; ++u) {
      const long i = base + u * stride;
      dst[u] = nullptr;
      if (i < total) {                            // the row's load does not wait for its slot
        const int t = (int)(i / R), r = (int)(i % R);
        const int kv = r >= kv_heads, h = kv ? r - kv_heads : r;
        val[u] = *reinterpret_cast<const uint4*>((kv ? v : k) + ((size_t)t * kv_heads + h) * HY_HEAD_DIM + l * E);
        const int slot = slot_mapping[t];
        if (slot >= (long)num_blocks * HY_BLOCK) hy_flag(err, HY_ERR_BOUNDS);
        else if (slot >= 0) dst[u] = cache_ptr(cache, slot, kv, h, kv_heads) + l * E;
      }
    }
#pragma unroll
    for (int u = 0; u < KVA_UNROLL; ++u)
      if (dst[u] != nullptr) *reinterpret_cast<uint4*>(dst[u]) = val[u];
  }
}

// min(units, 148 SMs x resident CTAs of the kernel), the occupancy asked once
// per pass-group size
template <typename K>
int qnr_grid(K kernel, int npc, long units) {
  static int occ[5] = {0, 0, 0, 0, 0};
  if (occ[npc] == 0) {
    int n = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kernel, QNR_THREADS, 0);
    occ[npc] = n > 0 ? n : 1;
  }
  const long cap = 148L * occ[npc];
  return (int)(units < cap ? (units > 0 ? units : 1) : cap);
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
  if (dtype == 0) {
    using B = __nv_bfloat16;
    const int heads = q_heads + 2 * kv_heads;
    const int npass = (heads + QNR_GROUPS - 1) / QNR_GROUPS;
    // prefill-sized batches: a token per CTA iteration, 8 lanes per head row
    // (a CTA of 8 x heads threads)
    if ((long)T * npass > 148L * 8 && heads * QNR_LPR <= QNR_ROWS_MAX_THREADS &&
        ld % 8 == 0 && (reinterpret_cast<uintptr_t>(qkv) & 15) == 0) {
      // consumers (8 x heads threads in whole warps) + the producer warp
      const int threads = (heads * QNR_LPR + 31) / 32 * 32 + 32;
      const int smem = QNR_NS * (heads * HY_HEAD_DIM * 2 + 2 * 64 * 4);
      // per device: the shared-memory attribute once, the occupancy per shape
      static bool attr[64] = {};
      static int occ_rows[64] = {}, occ_key[64] = {};
      int dev = 0;
      cudaGetDevice(&dev);
      if (dev < 0 || dev >= 64) dev = 0;
      if (!attr[dev]) {
        cudaError_t e = cudaFuncSetAttribute(qk_norm_rope_rows_kernel,
                                             cudaFuncAttributeMaxDynamicSharedMemorySize, 64 * 1024);
        if (e != cudaSuccess) return e;
        attr[dev] = true;
      }
      if (occ_key[dev] != threads * 65536 + smem) {
        int n = 0;
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, qk_norm_rope_rows_kernel, threads, smem);
        occ_rows[dev] = n > 0 ? n : 1;
        occ_key[dev] = threads * 65536 + smem;
      }
      const long cap = 148L * occ_rows[dev];
      const int grid = (int)(T < cap ? T : cap);
      return hy_launch(qk_norm_rope_rows_kernel, dim3(grid), dim3(threads), smem, st, (const B*)qkv,
                       (int)ld, T, q_heads, kv_heads, positions, (const B*)q_w, (const B*)k_w,
                       rope_cos, rope_sin, max_pos, eps, (B*)q_out, (B*)k_out, (B*)cache,
                       slot_mapping, num_blocks, err);
    }
    // decode-sized batches: one pass of 16 head rows per unit while that still
    // leaves units for fewer than 8 CTAs per SM; otherwise up to 4 passes
    const int npc = (long)T * npass <= 148L * 8 ? 1 : (npass < 4 ? npass : 4);
    const long units = (long)T * ((npass + npc - 1) / npc);
    // as many CTAs as are resident at once (each walks its units), at most one per unit
#define HY_QNR_LAUNCH(N)                                                                      \
  hy_launch(qk_norm_rope_bf16_kernel<N>, dim3(qnr_grid(qk_norm_rope_bf16_kernel<N>, N, units)), \
            dim3(QNR_THREADS), 0, st, (const B*)qkv, (int)ld, T, q_heads, kv_heads, positions, \
            (const B*)q_w, (const B*)k_w, rope_cos, rope_sin, max_pos, eps, (B*)q_out,         \
            (B*)k_out, (B*)cache, slot_mapping, num_blocks, err)
    switch (npc) {
      case 1: return HY_QNR_LAUNCH(1);
      case 2: return HY_QNR_LAUNCH(2);
      case 3: return HY_QNR_LAUNCH(3);
      default: return HY_QNR_LAUNCH(4);
    }
#undef HY_QNR_LAUNCH
  } else {
    const int grid = grid_for((long)T * (q_heads + 2 * kv_heads));
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
  const long rows = (long)T * kv_heads * 2;
  const int per_cta = KVA_THREADS / (HY_HEAD_DIM / (dtype == 0 ? 8 : 4));
  long blocks = (rows + (long)per_cta * KVA_UNROLL - 1) / ((long)per_cta * KVA_UNROLL);
  const int grid = (int)(blocks < 148L * 8 ? (blocks > 0 ? blocks : 1) : 148L * 8);
  if (dtype == 0) {
    using B = __nv_bfloat16;
    return hy_launch(kv_append_kernel<B>, dim3(grid), dim3(KVA_THREADS), 0, st, (const B*)k,
                     (const B*)v, T, kv_heads, slot_mapping, (B*)cache, num_blocks, err);
  } else {
    kv_append_kernel<float><<<grid, KVA_THREADS, 0, st>>>((const float*)k, (const float*)v, T, kv_heads,
                                                  slot_mapping, (float*)cache, num_blocks, err);
  }
  return cudaGetLastError();
}
