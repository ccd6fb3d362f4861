// Greedy sampling on the GPU: row-wise argmax over the vocabulary.
//
// Replaces Engine.sample (hayate/engine/engine.py:69-71), torch.argmax over the
// last dimension.  Ties resolve to the lowest index, as torch.argmax does; a
// NaN counts as larger than every number (torch propagates NaN the same way),
// the first NaN winning; -0 and +0 are equal.
#include "common.cuh"

#include <cooperative_groups.h>

namespace cg = cooperative_groups;

namespace {

constexpr int AM_THREADS = 256;
#ifndef HY_AM_UNROLL
#define HY_AM_UNROLL 2
#endif
constexpr int AM_UNROLL = HY_AM_UNROLL;   // 16-byte vectors per thread per batch
constexpr int AM_MAX_CLUSTER = 8;         // portable cluster size

// (v, i) beats (a, j): NaN beats every number (torch.argmax propagates NaN),
// otherwise the larger value; equal values (-0 == +0, NaN and NaN) go to the
// lower index.
HY_DEVICE bool better(float av, int ai, float bv, int bi) {
  const bool an = isnan(av), bn = isnan(bv);
  if (an || bn) return bn && (!an || bi < ai);
  return bv > av || (bv == av && bi < ai);
}

// Reduce (value, index) over the CTA; the result is valid in thread 0.
HY_DEVICE void cta_best(float& bv, int& bi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(bv, bi, ov, oi)) { bv = ov; bi = oi; }
  }
  __shared__ float sv[AM_THREADS / 32];
  __shared__ int si[AM_THREADS / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { sv[warp] = bv; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    bv = lane < AM_THREADS / 32 ? sv[lane] : -INFINITY;
    bi = lane < AM_THREADS / 32 ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(bv, bi, ov, oi)) { bv = ov; bi = oi; }
    }
  }
}

template <typename T> struct Scan;

// bf16: 16-byte vectors of 8 elements.  A batch of AM_UNROLL vectors is reduced
// with packed bf16x2 maxima that propagate NaN, and the stream keeps only the
// thread's best value and the first batch that reached it (a thread's batches
// come in increasing index order, so a strictly better batch maximum keeps
// first-index ties).  That one batch is read again at the end (from L1/L2) and
// searched for the first element holding the value, so the stream itself has
// no data-dependent branch.
template <> struct Scan<__nv_bfloat16> {
  static constexpr int N = 8;
  static HY_DEVICE void load_batch(const __nv_bfloat16* x, int base, int v1, uint4 (&w)[AM_UNROLL]) {
#pragma unroll
    for (int u = 0; u < AM_UNROLL; ++u) {
      const int vi = base + u * AM_THREADS;
      // -inf pairs (0xff80) for vectors past the chunk: they never win
      w[u] = vi < v1 ? __ldg(reinterpret_cast<const uint4*>(x) + vi)
                     : make_uint4(0xff80ff80u, 0xff80ff80u, 0xff80ff80u, 0xff80ff80u);
    }
  }
  static HY_DEVICE void run(const __nv_bfloat16* x, int v0, int v1, float& bv, int& bi) {
    int best_base = -1;
    for (int base = v0 + threadIdx.x; base < v1; base += AM_THREADS * AM_UNROLL) {
      uint4 w[AM_UNROLL];
      load_batch(x, base, v1, w);
      __nv_bfloat162 m = *reinterpret_cast<const __nv_bfloat162*>(&w[0].x);
#pragma unroll
      for (int u = 0; u < AM_UNROLL; ++u) {
        const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&w[u]);
#pragma unroll
        for (int q = 0; q < 4; ++q) m = __hmax2_nan(m, h[q]);
      }
      const float m0 = __low2float(m), m1 = __high2float(m);
      const float bm = (isnan(m0) || m1 != m1) ? NAN : fmaxf(m0, m1);
      // the thread's first batch, or a strictly better value (NaN beats numbers)
      const bool take = best_base < 0 || (isnan(bm) ? !isnan(bv) : bm > bv);
      bv = take ? bm : bv;
      best_base = take ? base : best_base;
    }
    if (best_base < 0) return;
    uint4 w[AM_UNROLL];
    load_batch(x, best_base, v1, w);
    bool found = false;
#pragma unroll
    for (int u = 0; u < AM_UNROLL; ++u) {
      const __nv_bfloat16* e8 = reinterpret_cast<const __nv_bfloat16*>(&w[u]);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float f = __bfloat162float(e8[e]);
        const bool hit = isnan(bv) ? isnan(f) : (f == bv);
        if (!found && hit) {
          found = true;
          bi = (best_base + u * AM_THREADS) * 8 + e;
        }
      }
    }
  }
};

template <> struct Scan<float> {
  static constexpr int N = 4;
  static HY_DEVICE void run(const float* x, int v0, int v1, float& bv, int& bi) {
    for (int vi = v0 + threadIdx.x; vi < v1; vi += AM_THREADS) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(x) + vi);
      const float e4[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (better(bv, bi, e4[e], vi * 4 + e)) { bv = e4[e]; bi = vi * 4 + e; }
    }
  }
};

// A row is split over the C CTAs of one thread-block cluster (C = 1..8, chosen
// on the host so that rows x C CTAs fill the SMs): CTA r scans the contiguous
// chunk r of the row, then rank 0 merges the C partial results it reads from the
// other CTAs' shared memory (distributed shared memory), so no global workspace
// and no second launch are needed.  Chunks are whole 16-byte vectors; the row's
// tail and unaligned rows take the scalar loop.
template <typename T>
__global__ void __launch_bounds__(AM_THREADS) argmax_kernel(
    const T* __restrict__ logits, long ld, int V, int32_t* __restrict__ out) {
  using S = Scan<T>;
  constexpr int N = S::N;
  hy_grid_wait();
  hy_grid_trigger();
  cg::cluster_group cluster = cg::this_cluster();
  const int C = (int)cluster.num_blocks();
  const int rank = (int)cluster.block_rank();
  const int row = blockIdx.x / C;
  const T* x = logits + (size_t)row * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  const bool vec_ok = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  const int nvec = V / N;
  const int per = (nvec + C - 1) / C;                 // vectors per CTA
  const int v0 = min(nvec, rank * per), v1 = min(nvec, v0 + per);
  if (vec_ok) {
    S::run(x, v0, v1, bv, bi);
  } else {
    for (int i = v0 * N + threadIdx.x; i < v1 * N; i += AM_THREADS) {
      const float v = ElemTraits<T>::to_f(x[i]);
      if (better(bv, bi, v, i)) { bv = v; bi = i; }
    }
  }
  if (rank == C - 1)                                  // elements past the last whole vector
    for (int i = nvec * N + threadIdx.x; i < V; i += AM_THREADS) {
      const float v = ElemTraits<T>::to_f(x[i]);
      if (better(bv, bi, v, i)) { bv = v; bi = i; }
    }
  cta_best(bv, bi);
  __shared__ float best_v;
  __shared__ int best_i;
  if (threadIdx.x == 0) { best_v = bv; best_i = bi; }
  cluster.sync();                                     // partials visible cluster-wide
  if (rank == 0 && threadIdx.x < 32) {
    const int lane = threadIdx.x;
    float v = -INFINITY;
    int i = 0x7fffffff;
    if (lane < C) {
      v = *cluster.map_shared_rank(&best_v, lane);
      i = *cluster.map_shared_rank(&best_i, lane);
    }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {                 // C <= 8
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, i, o);
      if (better(v, i, ov, oi)) { v = ov; i = oi; }
    }
    if (lane == 0) out[row] = i == 0x7fffffff ? 0 : i;
  }
  cluster.sync();                                     // keep shared memory alive for rank 0
}

}  // namespace

cudaError_t hy_launch_argmax(int dtype, const void* logits, long ld, int rows, int V,
                             int32_t* out, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  // cluster size: as many CTAs per row as keep the whole grid resident at once
  // (a second, partial wave would run on a few SMs alone), at most 8
  static int occ[2] = {0, 0};
  const int k = dtype == 0 ? 0 : 1;
  if (occ[k] == 0) {
    int n = 0;
    if (dtype == 0)
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, argmax_kernel<__nv_bfloat16>, AM_THREADS, 0);
    else
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, argmax_kernel<float>, AM_THREADS, 0);
    occ[k] = n > 0 ? n : 1;
  }
  const int want = (148 * occ[k]) / rows;
  const int C = want < 1 ? 1 : (want > AM_MAX_CLUSTER ? AM_MAX_CLUSTER : want);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(rows * C));
  cfg.blockDim = dim3(AM_THREADS);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = hy_pdl_enabled() ? 2 : 1;
  if (dtype == 0)
    return cudaLaunchKernelEx(&cfg, argmax_kernel<__nv_bfloat16>,
                              static_cast<const __nv_bfloat16*>(logits), ld, V, out);
  return cudaLaunchKernelEx(&cfg, argmax_kernel<float>, static_cast<const float*>(logits), ld, V,
                            out);
}
