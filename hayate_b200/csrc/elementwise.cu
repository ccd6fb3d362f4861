// Row-wise residual-add + RMSNorm and SiLU(gate)*up around the cuBLAS GEMMs.
//
// Add+RMSNorm replaces the residual adds and nn.RMSNorm of a block
// (hayate/model/block.py:18-31, qwen.py:35,122):
//   x = round(delta + x);  y = round( (f32(x) * rstd) * f32(w) ),
//   rstd = 1 / sqrt(mean(f32(x)^2) + eps)
// SiLU*up replaces FeedForward's activation (hayate/model/linear.py:11-13):
//   y = round( f32(round(silu(f32(g)))) * f32(u) ),  silu(g) = g / (1 + exp(-g))
// with round() the model dtype, i.e. the rounding points of the reference's
// separate torch ops.  16-byte vector loads.
#include "common.cuh"

namespace {

template <typename T> struct Vec;   // 16 bytes of T
template <> struct Vec<__nv_bfloat16> {
  static constexpr int N = 8;
  static HY_DEVICE void load(const __nv_bfloat16* p, float (&f)[8]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __bfloat1622float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
  static HY_DEVICE void store(__nv_bfloat16* p, const float (&f)[8]) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  }
  static HY_DEVICE float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
};
template <> struct Vec<float> {
  static constexpr int N = 4;
  static HY_DEVICE void load(const float* p, float (&f)[4]) {
    const float4 u = *reinterpret_cast<const float4*>(p);
    f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w;
  }
  static HY_DEVICE void store(float* p, const float (&f)[4]) {
    *reinterpret_cast<float4*>(p) = make_float4(f[0], f[1], f[2], f[3]);
  }
  static HY_DEVICE float round(float v) { return v; }
};

// One CTA per row, RN_THREADS threads, up to 32 elements per thread in 16-byte
// vectors: rows of at most 128 x 32 = 4096 elements.  The weight
// vectors are loaded together with the row, so a row costs one memory round
// trip plus a CTA reduction.
constexpr int RN_THREADS = 128;
// The split-K variant runs decode-sized batches (a few rows): 384 threads give
// one 16-byte slot per thread at hidden size 2560, so each thread's partial
// loads are one short batch.
constexpr int RN_PARTS_THREADS = 384;

// x <- round(x + delta) (when delta is given: the residual add of block.py:24,30),
// y <- RMSNorm(x) * w.  With split-K partials instead of delta, delta is first
// round(sum of the nparts fp32 partials, in order), i.e. the projection's
// output as its GEMM would have rounded it.
// GATHER: output row r takes residual row x_rows[r] of x (a step's sampled
// tokens); the updated residual goes to row r of x_out (nullable) instead of
// back into x, and a row index outside [0, x_nrows) sets HY_ERR_BOUNDS and
// leaves the output row unwritten.
template <typename T, bool PARTS, bool GATHER, int THREADS>
__global__ void __launch_bounds__(THREADS) add_rms_norm_kernel(
    T* __restrict__ x, long ldx, const T* __restrict__ delta, long ldd, int cols,
    const T* __restrict__ w, float eps, T* __restrict__ y, long ldy,
    const float* __restrict__ parts, int nparts, long pstride,
    const int32_t* __restrict__ x_rows, int x_nrows, T* __restrict__ x_out, long ldxo,
    int32_t* err) {
  using V = Vec<T>;
  constexpr int N = V::N;
  constexpr int RN_VEC = (4096 / N + THREADS - 1) / THREADS;   // 16-byte slots per thread
  __shared__ float red[THREADS / 32];
  const long r = blockIdx.x;
  const int nvec = cols / N;
  // rows and weights stay as their 16-byte vectors (the stored residual is in
  // the model dtype anyway) and are unpacked where used: fewer registers, more
  // rows in flight per SM
  uint4 xv[RN_VEC], wv[RN_VEC];
#pragma unroll
  for (int k = 0; k < RN_VEC; ++k) {          // the weights are no earlier kernel's output
    const int vi = threadIdx.x + THREADS * k;
    if (vi < nvec) wv[k] = *reinterpret_cast<const uint4*>(w + vi * N);
  }
  hy_grid_wait();
  hy_grid_trigger();
  T* xr = x + r * ldx;                        // residual row read
  T* xw = xr;                                 // residual row written (nullable)
  if constexpr (GATHER) {
    const int src = x_rows[r];                // the same for the whole CTA
    if (src < 0 || src >= x_nrows) {
      if (threadIdx.x == 0) hy_flag(err, HY_ERR_BOUNDS);
      return;
    }
    xr = x + (long)src * ldx;
    xw = x_out ? x_out + r * ldxo : nullptr;
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < RN_VEC; ++k) {
    const int vi = threadIdx.x + THREADS * k;
    if (vi < nvec) {
      float v[N];
      V::load(xr + vi * N, v);
      if (!PARTS && delta != nullptr) {
        float dv[N];
        V::load(delta + r * ldd + vi * N, dv);
#pragma unroll
        for (int e = 0; e < N; ++e) v[e] = V::round(__fadd_rn(dv[e], v[e]));
        if (xw) V::store(xw + vi * N, v);
      } else if (GATHER && !PARTS) {
        if (xw) V::store(xw + vi * N, v);
      } else if (PARTS) {
        // the loads of the first PMAX partials are all issued before the sum
        // uses any of them (one L2 round trip, not one per partial)
        constexpr int PMAX = 8;
        float dv[N];
        const float* pp = parts + r * ldd + vi * N;
        float4 pb[PMAX][N / 4];
#pragma unroll
        for (int p = 0; p < PMAX; ++p)
          if (p < nparts)
#pragma unroll
            for (int e = 0; e < N / 4; ++e)
              pb[p][e] = __ldcg(reinterpret_cast<const float4*>(pp + p * pstride + 4 * e));
#pragma unroll
        for (int e = 0; e < N / 4; ++e) {
          dv[4 * e] = pb[0][e].x; dv[4 * e + 1] = pb[0][e].y;
          dv[4 * e + 2] = pb[0][e].z; dv[4 * e + 3] = pb[0][e].w;
        }
#pragma unroll
        for (int p = 1; p < PMAX; ++p)
          if (p < nparts)
#pragma unroll
            for (int e = 0; e < N / 4; ++e) {
              dv[4 * e] = __fadd_rn(dv[4 * e], pb[p][e].x);
              dv[4 * e + 1] = __fadd_rn(dv[4 * e + 1], pb[p][e].y);
              dv[4 * e + 2] = __fadd_rn(dv[4 * e + 2], pb[p][e].z);
              dv[4 * e + 3] = __fadd_rn(dv[4 * e + 3], pb[p][e].w);
            }
        for (int p = PMAX; p < nparts; ++p) {
#pragma unroll
          for (int e = 0; e < N; e += 4) {
            const float4 a = __ldcg(reinterpret_cast<const float4*>(pp + p * pstride + e));
            dv[e] = __fadd_rn(dv[e], a.x);
            dv[e + 1] = __fadd_rn(dv[e + 1], a.y);
            dv[e + 2] = __fadd_rn(dv[e + 2], a.z);
            dv[e + 3] = __fadd_rn(dv[e + 3], a.w);
          }
        }
#pragma unroll
        for (int e = 0; e < N; ++e) v[e] = V::round(__fadd_rn(V::round(dv[e]), v[e]));
        if (xw) V::store(xw + vi * N, v);
      }
#pragma unroll
      for (int e = 0; e < N; ++e) ss = __fadd_rn(ss, __fmul_rn(v[e], v[e]));
      V::store(reinterpret_cast<T*>(&xv[k]), v);          // exact: v is in T already
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < THREADS / 32; ++i) tot = __fadd_rn(tot, red[i]);
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)cols), eps)));
  T* yr = y + r * ldy;
#pragma unroll
  for (int k = 0; k < RN_VEC; ++k) {
    const int vi = threadIdx.x + THREADS * k;
    if (vi < nvec) {
      float v[N], g[N], o[N];
      V::load(reinterpret_cast<const T*>(&xv[k]), v);
      V::load(reinterpret_cast<const T*>(&wv[k]), g);
#pragma unroll
      for (int e = 0; e < N; ++e) o[e] = __fmul_rn(__fmul_rn(v[e], rstd), g[e]);
      V::store(yr + vi * N, o);
    }
  }
}

// Prefill-sized bf16 residual add + RMSNorm, streamed: a persistent grid whose
// warps take one row at a time (row r of warp gw = gw + k x all warps).  A
// warp's rows arrive in its two-stage shared-memory ring by bulk copies (x and
// delta, 2 x cols x 2 bytes), issued two rows ahead, so every warp keeps a
// row in flight while it works on another and no registers hold the loads.
// The sum x + delta is rounded, written to x and kept in the ring (over the x
// row) for the second pass after the warp's sum of squares; the weights sit in
// shared memory, loaded once per CTA.  Rounding points are those of
// add_rms_norm_kernel, with packed f32x2 arithmetic (each lane rounded as the
// scalar operation); only the order of the sum of squares differs.
constexpr int RNB_WARPS = 8;
constexpr int RNB_STAGES = 2;
constexpr int RNB_MIN_ROWS = 256;                 // fewer rows: one CTA per row
constexpr int RNB_MAX_SMEM = 200 * 1024;

HY_DEVICE float2 bf2_to_f2(uint32_t u) {
  return __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u));
}
HY_DEVICE uint32_t f2_to_bf2(float2 f) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(f.x, f.y);
  return *reinterpret_cast<const uint32_t*>(&h);
}

template <bool DELTA>
__global__ void __launch_bounds__(RNB_WARPS * 32) add_rms_norm_bulk_kernel(
    __nv_bfloat16* __restrict__ x, long ldx, const __nv_bfloat16* __restrict__ delta, long ldd,
    int rows, int cols, const __nv_bfloat16* __restrict__ w, float eps,
    __nv_bfloat16* __restrict__ y, long ldy, int32_t* err) {
  extern __shared__ __align__(128) uint8_t rnb_smem[];
  __shared__ uint64_t bars[RNB_WARPS][RNB_STAGES];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row_bytes = cols * 2;
  const int stage_bytes = row_bytes * (DELTA ? 2 : 1);
  const int nvec = cols / 8;
  uint4* ws = reinterpret_cast<uint4*>(rnb_smem);                 // the weights
  uint8_t* ring = rnb_smem + row_bytes + (size_t)warp * RNB_STAGES * stage_bytes;
  if (lane == 0) {
    for (int s = 0; s < RNB_STAGES; ++s) mbar_init(&bars[warp][s], 1);
    fence_mbar_init();
  }
  for (int i = threadIdx.x; i < nvec; i += RNB_WARPS * 32)        // no earlier kernel's output
    ws[i] = reinterpret_cast<const uint4*>(w)[i];
  __syncthreads();
  hy_grid_wait();
  hy_grid_trigger();
  const int gw = (int)blockIdx.x * RNB_WARPS + warp, GW = (int)gridDim.x * RNB_WARPS;
  auto issue = [&](int s, int r) {                // lane 0
    uint8_t* st = ring + s * stage_bytes;
    mbar_arrive_expect_tx(&bars[warp][s], stage_bytes);
    bulk_load(st, x + (size_t)r * ldx, row_bytes, &bars[warp][s]);
    if (DELTA) bulk_load(st + row_bytes, delta + (size_t)r * ldd, row_bytes, &bars[warp][s]);
  };
  uint32_t pend = 0;                              // stages with a copy in flight
  if (lane == 0)
    for (int s = 0; s < RNB_STAGES; ++s)
      if (gw + s * GW < rows) issue(s, gw + s * GW);
  for (int s = 0; s < RNB_STAGES; ++s)
    if (gw + s * GW < rows) pend |= 1u << s;
  uint32_t phase = 0;
  bool ok = true;
  for (int i = 0, r = gw; r < rows; ++i, r += GW) {
    const int s = i % RNB_STAGES;
    if (!mbar_wait(&bars[warp][s], (phase >> s) & 1u, err)) { ok = false; break; }
    phase ^= 1u << s;
    pend &= ~(1u << s);
    uint4* xs = reinterpret_cast<uint4*>(ring + s * stage_bytes);
    const uint4* ds = reinterpret_cast<const uint4*>(ring + s * stage_bytes + row_bytes);
    uint4* xg = reinterpret_cast<uint4*>(x + (size_t)r * ldx);
    float2 ss2 = make_float2(0.f, 0.f);
    for (int vi = lane; vi < nvec; vi += 32) {
      uint4 xv = xs[vi];
      if (DELTA) {
        const uint4 dv = ds[vi];
        const uint32_t* xa = &xv.x;
        const uint32_t* da = &dv.x;
        uint4 o;
        uint32_t* oa = &o.x;
#pragma unroll
        for (int q = 0; q < 4; ++q) oa[q] = f2_to_bf2(__fadd2_rn(bf2_to_f2(da[q]), bf2_to_f2(xa[q])));
        xv = o;
        xg[vi] = xv;
        xs[vi] = xv;
      }
      const uint32_t* va = &xv.x;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float2 v = bf2_to_f2(va[q]);
        ss2 = __fadd2_rn(ss2, __fmul2_rn(v, v));
      }
    }
    float ss = __fadd_rn(ss2.x, ss2.y);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)cols), eps)));
    const float2 rs2 = make_float2(rstd, rstd);
    uint4* yg = reinterpret_cast<uint4*>(y + (size_t)r * ldy);
    for (int vi = lane; vi < nvec; vi += 32) {
      const uint4 xv = xs[vi], wv = ws[vi];
      const uint32_t* va = &xv.x;
      const uint32_t* wa = &wv.x;
      uint4 o;
      uint32_t* oa = &o.x;
#pragma unroll
      for (int q = 0; q < 4; ++q)
        oa[q] = f2_to_bf2(__fmul2_rn(__fmul2_rn(bf2_to_f2(va[q]), rs2), bf2_to_f2(wa[q])));
      yg[vi] = o;
    }
    fence_proxy_async();                          // this lane's ring writes before the next copy
    __syncwarp();
    const int rn = r + RNB_STAGES * GW;
    if (rn < rows) {
      if (lane == 0) issue(s, rn);
      pend |= 1u << s;
    }
  }
  if (!ok) {                                      // let the copies in flight land before exit
    for (int s = 0; s < RNB_STAGES; ++s)
      if ((pend >> s) & 1u) mbar_wait(&bars[warp][s], (phase >> s) & 1u, nullptr);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) silu_mul_kernel(
    const T* __restrict__ gu, long ld, int rows, int inter, T* __restrict__ y, long ldy) {
  using V = Vec<T>;
  constexpr int N = V::N;
  hy_grid_wait();
  hy_grid_trigger();
  const int nvec = inter / N;
  const long total = (long)rows * nvec;
  const long stride = (long)gridDim.x * blockDim.x;
  for (long i = (long)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const long r = i / nvec;
    const int c = (int)(i % nvec) * N;
    float g[N], u[N], o[N];
    V::load(gu + r * ld + c, g);
    V::load(gu + r * ld + inter + c, u);
#pragma unroll
    for (int e = 0; e < N; ++e) {
      float s;
      if constexpr (N == 8) {
        // bf16: SiLU is rounded to bf16 right away, so the fast exp and divide
        // (errors near 1e-7 relative) leave it within one bf16 ulp
        s = V::round(__fdividef(g[e], 1.0f + __expf(-g[e])));
      } else {
        s = V::round(__fdiv_rn(g[e], __fadd_rn(1.0f, expf(-g[e]))));
      }
      o[e] = __fmul_rn(s, u[e]);
    }
    V::store(y + r * ldy + c, o);
  }
}

}  // namespace

template <typename T, bool GATHER>
static cudaError_t launch_add_rms_norm(void* x, long ldx, const void* delta, long ldd, int rows,
                                       int cols, const void* w, float eps, void* y, long ldy,
                                       const float* parts, int nparts, long pstride,
                                       const int32_t* x_rows, int x_nrows, void* x_out,
                                       long ldxo, int32_t* err, cudaStream_t st) {
  if (parts)
    return hy_launch(add_rms_norm_kernel<T, true, GATHER, RN_PARTS_THREADS>, dim3(rows),
                     dim3(RN_PARTS_THREADS), 0, st, (T*)x, ldx, (const T*)delta, ldd, cols,
                     (const T*)w, eps, (T*)y, ldy, parts, nparts, pstride, x_rows, x_nrows,
                     (T*)x_out, ldxo, err);
  return hy_launch(add_rms_norm_kernel<T, false, GATHER, RN_THREADS>, dim3(rows),
                   dim3(RN_THREADS), 0, st, (T*)x, ldx, (const T*)delta, ldd, cols, (const T*)w,
                   eps, (T*)y, ldy, parts, nparts, pstride, x_rows, x_nrows, (T*)x_out, ldxo, err);
}

// delta (model dtype) or parts (fp32, nparts x rows, pstride apart) -- at most
// one of them -- with row pitch ldd.  With x_rows, output row r reads residual
// row x_rows[r] (< x_nrows) and writes the updated residual to x_out.
// The streamed kernel for a prefill-sized bf16 add + RMSNorm (rows and row
// pitches 16-byte aligned, which the C ABI checks).
static cudaError_t launch_add_rms_norm_bulk(void* x, long ldx, const void* delta, long ldd,
                                            int rows, int cols, const void* w, float eps, void* y,
                                            long ldy, int32_t* err, cudaStream_t st) {
  using B = __nv_bfloat16;
  const int row_bytes = cols * 2;
  const int smem = row_bytes + RNB_WARPS * RNB_STAGES * row_bytes * (delta ? 2 : 1);
  // per device: the shared-memory attribute once, the occupancy per ring size
  static bool attr[64][2] = {};
  static int occ[64][2] = {}, occ_smem[64][2] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) dev = 0;
  const int k = delta ? 1 : 0;
  auto kern = delta ? add_rms_norm_bulk_kernel<true> : add_rms_norm_bulk_kernel<false>;
  if (!attr[dev][k]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         RNB_MAX_SMEM + 4096);
    if (e != cudaSuccess) return e;
    attr[dev][k] = true;
  }
  if (occ_smem[dev][k] != smem) {
    int n = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, RNB_WARPS * 32, smem);
    occ[dev][k] = n > 0 ? n : 1;
    occ_smem[dev][k] = smem;
  }
  const long warps = 148L * occ[dev][k] * RNB_WARPS;
  const long want = (rows + 1) / 2;               // two rows per warp at least
  const long ctas = ((want < warps ? want : warps) + RNB_WARPS - 1) / RNB_WARPS;
  return hy_launch(kern, dim3((unsigned)ctas), dim3(RNB_WARPS * 32), smem, st, (B*)x, ldx,
                   (const B*)delta, ldd, rows, cols, (const B*)w, eps, (B*)y, ldy, err);
}

cudaError_t hy_launch_add_rms_norm(int dtype, void* x, long ldx, const void* delta, long ldd,
                                   int rows, int cols, const void* w, float eps, void* y,
                                   long ldy, const float* parts, int nparts, long pstride,
                                   cudaStream_t st, const int32_t* x_rows, int x_nrows,
                                   void* x_out, long ldxo, int32_t* err) {
  if (rows <= 0) return cudaSuccess;
  using B = __nv_bfloat16;
  if (dtype == 0 && !x_rows && !parts && rows >= RNB_MIN_ROWS && cols % 8 == 0 &&
      cols * 2 + RNB_WARPS * RNB_STAGES * cols * 2 * (delta ? 2 : 1) <= RNB_MAX_SMEM)
    return launch_add_rms_norm_bulk(x, ldx, delta, ldd, rows, cols, w, eps, y, ldy, err, st);
  if (x_rows)
    return dtype == 0 ? launch_add_rms_norm<B, true>(x, ldx, delta, ldd, rows, cols, w, eps, y,
                                                     ldy, parts, nparts, pstride, x_rows,
                                                     x_nrows, x_out, ldxo, err, st)
                      : launch_add_rms_norm<float, true>(x, ldx, delta, ldd, rows, cols, w, eps,
                                                         y, ldy, parts, nparts, pstride, x_rows,
                                                         x_nrows, x_out, ldxo, err, st);
  return dtype == 0 ? launch_add_rms_norm<B, false>(x, ldx, delta, ldd, rows, cols, w, eps, y,
                                                    ldy, parts, nparts, pstride, nullptr, 0,
                                                    nullptr, 0, nullptr, st)
                    : launch_add_rms_norm<float, false>(x, ldx, delta, ldd, rows, cols, w, eps, y,
                                                        ldy, parts, nparts, pstride, nullptr, 0,
                                                        nullptr, 0, nullptr, st);
}

cudaError_t hy_launch_silu_mul(int dtype, const void* gu, long ld, int rows, int inter, void* y,
                               long ldy, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  const long vecs = (long)rows * inter / (dtype == 0 ? 8 : 4);
  long blocks = (vecs + 255) / 256;
  if (blocks > 148L * 32) blocks = 148L * 32;
  if (dtype == 0)
    return hy_launch(silu_mul_kernel<__nv_bfloat16>, dim3((int)blocks), dim3(256), 0, st,
                     (const __nv_bfloat16*)gu, ld, rows, inter, (__nv_bfloat16*)y, ldy);
  return hy_launch(silu_mul_kernel<float>, dim3((int)blocks), dim3(256), 0, st, (const float*)gu,
                   ld, rows, inter, (float*)y, ldy);
}
