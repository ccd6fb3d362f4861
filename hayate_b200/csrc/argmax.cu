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
constexpr int AM_UNROLL = 4;
constexpr int AM_MAX_CLUSTER = 8;         // portable cluster size

// Elements are compared through order-preserving unsigned keys: a float's bit
// pattern with the sign bit flipped (non-negative) or all bits flipped
// (negative), -0 taken as +0, and every NaN mapped to the largest key, so that
// NaN beats every number as in torch.argmax.  A thread scans its elements in increasing index
// order and replaces its best only on a strictly larger key, keeping the first
// index of a tie; the merges across threads compare (key, index).
HY_DEVICE uint32_t key_f32(float f) {
  uint32_t b = __float_as_uint(f);
  if ((b & 0x7fffffffu) > 0x7f800000u) return 0xffffffffu;
  if ((b & 0x7fffffffu) == 0u) b = 0u;
  return b ^ ((b & 0x80000000u) ? 0xffffffffu : 0x80000000u);
}

// Keys of the two bf16 in a 32-bit word, as two 16-bit lanes.
HY_DEVICE uint32_t key2_bf16(uint32_t w) {
  w &= ~(__vcmpeq2(w & 0x7fff7fffu, 0u) & 0x80008000u);               // -0 -> +0
  const uint32_t neg = ((w >> 15) & 0x00010001u) * 0xffffu;           // 0xffff where negative
  const uint32_t k = w ^ (neg | 0x80008000u);
  return k | __vcmpgtu2(w & 0x7fff7fffu, 0x7f807f80u);               // NaN -> 0xffff
}

HY_DEVICE bool better(uint32_t ak, int ai, uint32_t bk, int bi) {
  return bk > ak || (bk == ak && bi < ai);
}

// Reduce (key, index) over the CTA; the result is valid in thread 0.
HY_DEVICE void cta_best(uint32_t& bk, int& bi) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const uint32_t ok = __shfl_xor_sync(0xffffffffu, bk, o);
    const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (better(bk, bi, ok, oi)) { bk = ok; bi = oi; }
  }
  __shared__ uint32_t sk[AM_THREADS / 32];
  __shared__ int si[AM_THREADS / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) { sk[warp] = bk; si[warp] = bi; }
  __syncthreads();
  if (warp == 0) {
    bk = lane < AM_THREADS / 32 ? sk[lane] : 0u;
    bi = lane < AM_THREADS / 32 ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint32_t ok = __shfl_xor_sync(0xffffffffu, bk, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(bk, bi, ok, oi)) { bk = ok; bi = oi; }
    }
  }
}

template <typename T> struct Scan;

// bf16: 16-byte vectors of 8 elements; a batch of AM_UNROLL vectors is reduced
// with packed 16-bit maxima and searched for its first maximum only when it
// beats the thread's best.
template <> struct Scan<__nv_bfloat16> {
  static constexpr int N = 8;
  static HY_DEVICE void run(const __nv_bfloat16* x, int v0, int v1, uint32_t& bk, int& bi) {
    for (int base = v0 + threadIdx.x; base < v1; base += AM_THREADS * AM_UNROLL) {
      uint4 w[AM_UNROLL];
#pragma unroll
      for (int u = 0; u < AM_UNROLL; ++u) {
        const int vi = base + u * AM_THREADS;
        w[u] = vi < v1 ? __ldg(reinterpret_cast<const uint4*>(x) + vi) : make_uint4(0u, 0u, 0u, 0u);
      }
      uint32_t k[AM_UNROLL][4];
      uint32_t m = 0u;
#pragma unroll
      for (int u = 0; u < AM_UNROLL; ++u) {
        const bool valid = base + u * AM_THREADS < v1;
        k[u][0] = valid ? key2_bf16(w[u].x) : 0u;
        k[u][1] = valid ? key2_bf16(w[u].y) : 0u;
        k[u][2] = valid ? key2_bf16(w[u].z) : 0u;
        k[u][3] = valid ? key2_bf16(w[u].w) : 0u;
        m = __vmaxu2(m, __vmaxu2(__vmaxu2(k[u][0], k[u][1]), __vmaxu2(k[u][2], k[u][3])));
      }
      const uint32_t bm = max(m & 0xffffu, m >> 16);
      if (bm > bk) {                                  // first element of the batch with key bm
        bool found = false;
#pragma unroll
        for (int u = 0; u < AM_UNROLL; ++u)
#pragma unroll
          for (int e = 0; e < 8; ++e) {
            const uint32_t ke = (k[u][e >> 1] >> (16 * (e & 1))) & 0xffffu;
            if (!found && ke == bm) {
              found = true;
              bk = bm;
              bi = (base + u * AM_THREADS) * 8 + e;
            }
          }
      }
    }
  }
};

template <> struct Scan<float> {
  static constexpr int N = 4;
  static HY_DEVICE void run(const float* x, int v0, int v1, uint32_t& bk, int& bi) {
    for (int vi = v0 + threadIdx.x; vi < v1; vi += AM_THREADS) {
      const float4 f = __ldg(reinterpret_cast<const float4*>(x) + vi);
      const float e4[4] = {f.x, f.y, f.z, f.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t k = key_f32(e4[e]);
        if (k > bk) { bk = k; bi = vi * 4 + e; }
      }
    }
  }
};

HY_DEVICE uint32_t key_of(float v) { return key_f32(v); }
HY_DEVICE uint32_t key_of(__nv_bfloat16 v) {
  return key2_bf16((uint32_t)__bfloat16_as_ushort(v)) & 0xffffu;
}

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
  cg::cluster_group cluster = cg::this_cluster();
  const int C = (int)cluster.num_blocks();
  const int rank = (int)cluster.block_rank();
  const int row = blockIdx.x / C;
  const T* x = logits + (size_t)row * ld;
  uint32_t bk = 0u;                                   // below every element's key
  int bi = 0x7fffffff;
  const bool vec_ok = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  const int nvec = V / N;
  const int per = (nvec + C - 1) / C;                 // vectors per CTA
  const int v0 = min(nvec, rank * per), v1 = min(nvec, v0 + per);
  if (vec_ok) {
    S::run(x, v0, v1, bk, bi);
  } else {
    for (int i = v0 * N + threadIdx.x; i < v1 * N; i += AM_THREADS) {
      const uint32_t k = key_of(x[i]);
      if (k > bk) { bk = k; bi = i; }
    }
  }
  if (rank == C - 1)                                  // elements past the last whole vector
    for (int i = nvec * N + threadIdx.x; i < V; i += AM_THREADS) {
      const uint32_t k = key_of(x[i]);
      if (k > bk) { bk = k; bi = i; }
    }
  cta_best(bk, bi);
  __shared__ uint32_t best_k;
  __shared__ int best_i;
  if (threadIdx.x == 0) { best_k = bk; best_i = bi; }
  cluster.sync();                                     // partials visible cluster-wide
  if (rank == 0 && threadIdx.x < 32) {
    const int lane = threadIdx.x;
    uint32_t k = 0u;
    int i = 0x7fffffff;
    if (lane < C) {
      k = *cluster.map_shared_rank(&best_k, lane);
      i = *cluster.map_shared_rank(&best_i, lane);
    }
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) {                 // C <= 8
      const uint32_t ok = __shfl_xor_sync(0xffffffffu, k, o);
      const int oi = __shfl_xor_sync(0xffffffffu, i, o);
      if (better(k, i, ok, oi)) { k = ok; i = oi; }
    }
    if (lane == 0) out[row] = i == 0x7fffffff ? 0 : i;
  }
  cluster.sync();                                     // keep shared memory alive for rank 0
}

}  // namespace

cudaError_t hy_launch_argmax(int dtype, const void* logits, long ld, int rows, int V,
                             int32_t* out, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  // cluster size: enough CTAs for about 8 per SM over the whole grid
  const int want = (148 * 8) / rows;
  int C = 1;
  while (C * 2 <= want && C * 2 <= AM_MAX_CLUSTER) C *= 2;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(rows * C));
  cfg.blockDim = dim3(AM_THREADS);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (dtype == 0)
    return cudaLaunchKernelEx(&cfg, argmax_kernel<__nv_bfloat16>,
                              static_cast<const __nv_bfloat16*>(logits), ld, V, out);
  return cudaLaunchKernelEx(&cfg, argmax_kernel<float>, static_cast<const float*>(logits), ld, V,
                            out);
}
