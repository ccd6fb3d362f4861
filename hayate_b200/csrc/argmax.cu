// Greedy sampling on the GPU: row-wise argmax over the vocabulary.
//
// Replaces Engine.sample (hayate/engine/engine.py:69-71), torch.argmax over the
// last dimension.  Ties resolve to the lowest index, as torch.argmax does; a
// NaN counts as larger than every number (torch propagates NaN the same way),
// the first NaN winning.
#include "common.cuh"

namespace {

constexpr int AM_THREADS = 512;

// true if (bv, bi) should replace (av, ai)
HY_DEVICE bool better(float av, int ai, float bv, int bi) {
  const bool an = isnan(av), bn = isnan(bv);
  if (an || bn) return bn && (!an || bi < ai);
  return bv > av || (bv == av && bi < ai);
}

template <typename T>
__global__ void __launch_bounds__(AM_THREADS) argmax_kernel(
    const T* __restrict__ logits, long ld, int V, int32_t* __restrict__ out) {
  const int row = blockIdx.x;
  const T* x = logits + (size_t)row * ld;
  float bv = -INFINITY;
  int bi = 0x7fffffff;
  // Each thread scans a strided subset in increasing index order.
  for (int i = threadIdx.x; i < V; i += AM_THREADS) {
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
