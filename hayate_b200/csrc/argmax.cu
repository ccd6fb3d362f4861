// Greedy sampling on the GPU: row-wise argmax over the vocabulary.
//
// Replaces Engine.sample (hayate/engine/engine.py:69-71), torch.argmax over the
// last dimension.  Ties resolve to the lowest index, as torch.argmax does; a
// NaN counts as larger than every number (torch propagates NaN the same way),
// the first NaN winning.
#include "common.cuh"

namespace {

constexpr int AM_THREADS = 1024;

// true if (bv, bi) should replace (av, ai)
HY_DEVICE bool better(float av, int ai, float bv, int bi) {
  const bool an = isnan(av), bn = isnan(bv);
  if (an || bn) return bn && (!an || bi < ai);
  return bv > av || (bv == av && bi < ai);
}

template <typename T> struct Vec16;
template <> struct Vec16<__nv_bfloat16> {
  static constexpr int N = 8;
  static HY_DEVICE void load(const __nv_bfloat16* p, float (&f)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __bfloat1622float2(h[i]);
      f[2 * i] = t.x;
      f[2 * i + 1] = t.y;
    }
  }
};
template <> struct Vec16<float> {
  static constexpr int N = 4;
  static HY_DEVICE void load(const float* p, float (&f)[4]) {
    const float4 u = __ldg(reinterpret_cast<const float4*>(p));
    f[0] = u.x; f[1] = u.y; f[2] = u.z; f[3] = u.w;
  }
};

template <typename T>
__global__ void __launch_bounds__(AM_THREADS) argmax_kernel(
    const T* __restrict__ logits, long ld, int V, int32_t* __restrict__ out) {
  using VV = Vec16<T>;
  constexpr int N = VV::N;
  constexpr int UNROLL = 4;
  const int row = blockIdx.x;
  const T* x = logits + (size_t)row * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  // Each thread scans 16-byte vectors i = tid, tid + T, ... in increasing index
  // order (UNROLL loads in flight), keeping the first best it sees.
  const bool vec_ok = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
  const int nvec = vec_ok ? V / N : 0;
  for (int base = threadIdx.x; base < nvec; base += AM_THREADS * UNROLL) {
    float f[UNROLL][N];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int vi = base + u * AM_THREADS;
      if (vi < nvec) VV::load(x + (size_t)vi * N, f[u]);
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int vi = base + u * AM_THREADS;
      if (vi < nvec) {
#pragma unroll
        for (int e = 0; e < N; ++e)
          if (better(bv, bi, f[u][e], vi * N + e)) { bv = f[u][e]; bi = vi * N + e; }
      }
    }
  }
  for (int i = nvec * N + threadIdx.x; i < V; i += AM_THREADS) {   // tail / unaligned rows
    const float v = ElemTraits<T>::to_f(x[i]);
    if (better(bv, bi, v, i)) { bv = v; bi = i; }
  }
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
    if (lane == 0) out[row] = bi == 0x7fffffff ? 0 : bi;
  }
}

}  // namespace

cudaError_t hy_launch_argmax(int dtype, const void* logits, long ld, int rows, int V,
                             int32_t* out, cudaStream_t st) {
  if (rows <= 0) return cudaSuccess;
  if (dtype == 0)
    argmax_kernel<__nv_bfloat16><<<rows, AM_THREADS, 0, st>>>(
        static_cast<const __nv_bfloat16*>(logits), ld, V, out);
  else
    argmax_kernel<float><<<rows, AM_THREADS, 0, st>>>(static_cast<const float*>(logits), ld, V, out);
  return cudaGetLastError();
}
