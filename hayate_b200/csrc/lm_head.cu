// Greedy sampling fused into the LM head: the sampled rows' last-token logits,
// x (rows x hidden bf16, the final RMSNorm's output) times the tied embedding
// W (vocab x hidden bf16), are computed tile by tile on the tensor cores and
// reduced to their argmax in the epilogue, so the (rows x vocab) logits never
// reach global memory.
//
// Replaces out_head and Engine.sample (hayate/model/qwen.py:122-123 and
// hayate/engine/engine.py:69-71: torch.argmax of the bf16 logits[:, -1, :]).
// Each logit is the fp32 dot product rounded to bf16, as a bf16 out_head
// produces it, and the comparison follows torch.argmax: the larger value, ties
// to the lower index, NaN above every number (the first NaN wins), -0 == +0.
//
// One persistent CTA per SM (while there are tiles), 6 warps:
//   warp 0      one lane issues the TMA loads: per 64-wide hidden chunk, the
//               x rows as one or two boxes (M tiles of up to 128 rows) and 208
//               rows of W (a vocab tile) into a ring of stages, W with an L2
//               evict-first hint (it streams through once) and x evict-last
//               (every tile reads it again);
//   warp 1      allocates the TMEM columns; one lane issues the tcgen05 MMAs
//               (M = 128 rows of x, N = 208 vocab columns, fp32 accumulators
//               in TMEM), double-buffered across vocab tiles when x fits one
//               M tile;
//   warps 2-5   the epilogue: thread r owns row r of each M tile (TMEM lane
//               r), reads its 208 accumulators, rounds them to bf16 and keeps
//               its best (value, index) across the CTA's tiles.
// A stage holds only the x rows that exist (rounded up to 8), followed by its
// W rows: an M = 128 MMA over a shorter x box reads the stage's next bytes as
// its remaining rows, whose sums are never read, so small batches leave room
// for more stages (7 at 16 rows, 5 at 128, 3 at 256) and more W in flight.
// The CTAs' row bests meet in a 64-bit atomicMax over (order key of the bf16
// value << 32 | ~index); the last CTA to finish writes the tokens and returns
// the workspace to zero, so each call leaves it as it found it.
#include "hayate_b200.h"
#include "common.cuh"

#include <mutex>
#include <stdio.h>

int hy_encode_rows_map(const void* base, long cols, long rows, long row_bytes, int box_rows,
                       CUtensorMap* out);   // capi.cu
void hy_set_error(const char* msg);        // capi.cu

namespace {

constexpr int LM_N = 208;                   // vocab columns per tile (13 x 16): 731 tiles of a
                                            // 151936 vocabulary, 4.94 per SM of 148
constexpr int LM_KC = 64;                   // hidden elements per chunk: one 128-byte row
constexpr int LM_B_BYTES = LM_N * 128;      // one vocab tile of W per chunk (26 KB)
constexpr int LM_MAX_STAGES = 8;
constexpr int LM_RING = 5 * (128 * 128 + LM_B_BYTES);   // 210 KB: 3 stages at 256 rows
constexpr int LM_SMEM = 1024 + LM_RING;
constexpr int LM_THREADS = 192;            // warps 2-5 (the epilogue) read TMEM lane quarters
                                            // 2, 3, 0, 1
constexpr int LM_TMEM_COLS = 512;           // two 256-column accumulator buffers
constexpr int LM_MAX_ROWS = 256;            // rows of x per launch (two M tiles)

struct LmArgs {
  int rows;                                 // rows of x in this launch (1..256)
  int mt;                                   // M tiles: 1 or 2
  int arows0, arows1;                       // x rows loaded per chunk for M tile 0, 1
                                            // (multiples of 8; arows1 = 0 for one tile)
  int ns;                                   // ring stages
  int vocab;
  int nk;                                   // hidden / 64
  int ntiles;                               // ceil(vocab / LM_N)
  unsigned long long* keys;                 // [LM_MAX_ROWS], zero between calls
  int* done;                                // CTAs finished, zero between calls
  int32_t* out;
  int32_t* err;
};

struct LmShared {
  uint64_t full[LM_MAX_STAGES];
  uint64_t free_[LM_MAX_STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];
  uint64_t drain;
  uint32_t tmem_base;
  int last;
};

// Order key of a bf16 value (held exactly in a float): unsigned comparison of
// keys is torch's comparison of values, NaN above +inf, -0 equal to +0.
HY_DEVICE uint32_t order_key(float v) {
  uint32_t h = __float_as_uint(v) >> 16;
  if (v != v) return 0xFFFFu;
  if ((h & 0x7FFFu) == 0) h = 0;
  return (h & 0x8000u) ? (~h & 0xFFFFu) : (h | 0x8000u);
}

HY_DEVICE uint64_t l2_stream_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 2-D tiled tensor load with an L2 cache policy (no multicast).
HY_DEVICE void tma_load_2d_hint(void* dst, const CUtensorMap* map, int32_t x, int32_t y,
                                uint64_t* bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;"
      :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y),
         "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__global__ void __launch_bounds__(LM_THREADS, 1) lm_head_argmax_kernel(
    const __grid_constant__ CUtensorMap xmap0, const __grid_constant__ CUtensorMap xmap1,
    const __grid_constant__ CUtensorMap wmap, LmArgs a) {
  __shared__ LmShared sh;
  extern __shared__ uint8_t dyn_smem[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int mt = a.mt, ns = a.ns;
  const int nbuf = mt == 1 ? 2 : 1;         // accumulator buffers of mt x 256 columns
  // stage: [x rows of M tile 0][x rows of M tile 1][W rows], each 1 KB-aligned
  const uint32_t a1_off = (uint32_t)a.arows0 * 128u;
  const uint32_t w_off = (uint32_t)(a.arows0 + a.arows1) * 128u;
  const uint32_t stage_bytes = w_off + (uint32_t)LM_B_BYTES;
  // vocab tiles of this CTA: blockIdx.x, + gridDim.x, ... (the grid has at most ntiles CTAs)
  const int my_tiles = (a.ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x;
  if (threadIdx.x == 0) {
    prefetch_tmap(&xmap0);
    if (mt == 2) prefetch_tmap(&xmap1);
    prefetch_tmap(&wmap);
    for (int s = 0; s < LM_MAX_STAGES; ++s) {
      mbar_init(&sh.full[s], 1);
      mbar_init(&sh.free_[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh.acc_full[b], 1);
      mbar_init(&sh.acc_empty[b], 128);     // every epilogue thread
    }
    mbar_init(&sh.drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&sh.tmem_base, LM_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      // W depends on no earlier kernel: the first stages' W boxes go out before
      // the wait for the kernel that wrote x
      const uint64_t pol_w = l2_stream_policy(), pol_x = l2_keep_policy();
      const uint32_t total = (uint32_t)(my_tiles * a.nk);
      const uint32_t pre = min((uint32_t)ns, total);
      for (uint32_t c = 0; c < pre; ++c) {
        const int tile = (int)blockIdx.x + (int)(c / a.nk) * (int)gridDim.x, kc = (int)(c % a.nk);
        uint8_t* st = ring + c * stage_bytes;
        mbar_arrive_expect_tx(&sh.full[c], stage_bytes);
        tma_load_2d_hint(st + w_off, &wmap, kc * LM_KC, tile * LM_N, &sh.full[c], pol_w);
      }
      hy_grid_wait();
      for (uint32_t c = 0; c < pre; ++c) {
        const int kc = (int)(c % a.nk);
        uint8_t* st = ring + c * stage_bytes;
        tma_load_2d_hint(st, &xmap0, kc * LM_KC, 0, &sh.full[c], pol_x);
        if (mt == 2) tma_load_2d_hint(st + a1_off, &xmap1, kc * LM_KC, 128, &sh.full[c], pol_x);
      }
      uint32_t c = pre;
      for (; c < total; ++c) {
        const uint32_t s = c % ns, use = c / ns;
        if (!mbar_wait(&sh.free_[s], (use & 1) ^ 1, a.err)) {
          ok = false;
          break;
        }
        const int tile = (int)blockIdx.x + (int)(c / a.nk) * (int)gridDim.x, kc = (int)(c % a.nk);
        uint8_t* st = ring + s * stage_bytes;
        mbar_arrive_expect_tx(&sh.full[s], stage_bytes);
        tma_load_2d_hint(st + w_off, &wmap, kc * LM_KC, tile * LM_N, &sh.full[s], pol_w);
        tma_load_2d_hint(st, &xmap0, kc * LM_KC, 0, &sh.full[s], pol_x);
        if (mt == 2) tma_load_2d_hint(st + a1_off, &xmap1, kc * LM_KC, 128, &sh.full[s], pol_x);
      }
      if (!ok)                                // the copies in flight land before the CTA ends
        for (uint32_t d = c > (uint32_t)ns ? c - ns : 0; d < c; ++d)
          mbar_wait(&sh.full[d % ns], (d / ns) & 1, nullptr);
    } else {
      hy_grid_wait();
    }
  } else if (warp == 1) {
    hy_grid_wait();
    if (lane == 0) {
      const uint32_t idesc = tc_idesc_bf16(128, LM_N, false);
      const uint32_t sbase = smem_u32(ring);
      uint32_t c = 0;
      for (int j = 0; j < my_tiles && ok; ++j) {
        const int b = j % nbuf;
        const uint32_t u = (uint32_t)(j / nbuf);
        ok = mbar_wait(&sh.acc_empty[b], (u & 1) ^ 1, a.err);   // the epilogue read buffer b
        if (!ok) break;
        tc_fence_after();
        for (int kc = 0; kc < a.nk; ++kc, ++c) {
          const uint32_t s = c % ns, use = c / ns;
          ok = mbar_wait(&sh.full[s], use & 1, a.err);
          if (!ok) break;
          tc_fence_after();
          const uint32_t st = sbase + s * stage_bytes;
          // K-major operands, 8-row groups 1 KB apart; a 16-element K step is
          // 32 bytes into the 128-byte swizzled row.  A reads 128 rows from its
          // tile's start: past the loaded x rows, the stage's next bytes (its
          // sums for those rows are never read)
          const uint64_t dB = tc_desc_sw128(st + w_off, 16, 1024);
          for (int m = 0; m < mt; ++m) {
            const uint64_t dA = tc_desc_sw128(st + (m ? a1_off : 0u), 16, 1024);
#pragma unroll
            for (int kk = 0; kk < LM_KC / 16; ++kk)
              tc_mma_bf16(tmem + (uint32_t)((b * mt + m) * 256), dA + (uint64_t)(kk * 2),
                          dB + (uint64_t)(kk * 2), idesc, (kc | kk) != 0);
          }
          tc_commit(&sh.free_[s]);
        }
        if (!ok) break;
        tc_commit(&sh.acc_full[b]);
      }
      if (!ok) {                              // let every issued MMA finish
        tc_commit(&sh.drain);
        mbar_wait(&sh.drain, 0, nullptr);
      }
    }
    __syncwarp();
  } else {
    hy_grid_wait();
    const int q = warp & 3;                   // TMEM lane quarter this warp may read
    const int r = 32 * q + lane;              // row within an M tile
    const uint32_t lane_off = (uint32_t)(32 * q) << 16;
    float bv[2] = {0.f, 0.f};
    int bi[2] = {-1, -1};
    for (int j = 0; j < my_tiles; ++j) {
      const int b = j % nbuf;
      const uint32_t u = (uint32_t)(j / nbuf);
      ok = __all_sync(0xffffffffu, mbar_wait(&sh.acc_full[b], u & 1, a.err));
      if (!ok) break;
      tc_fence_after();
      const int v0 = ((int)blockIdx.x + j * (int)gridDim.x) * LM_N;
      const int nvalid = min(LM_N, a.vocab - v0);
#pragma unroll
      for (int m = 0; m < 2; ++m) {
        if (m >= mt) break;
        if (m * 128 + 32 * q >= a.rows) continue;   // this warp's rows are all past the end
        const uint32_t tb = tmem + lane_off + (uint32_t)((b * mt + m) * 256);
        float best = bv[m];
        int bidx = bi[m];
#pragma unroll 1
        for (int c0 = 0; c0 < LM_N; c0 += 64) {   // columns past 208 of the last pair unused
          float v[64];
          tmem_ld32(tb + c0, *reinterpret_cast<float(*)[32]>(&v[0]));
          tmem_ld32(tb + c0 + 32, *reinterpret_cast<float(*)[32]>(&v[32]));
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 64; i += 2) {
            const __nv_bfloat162 h = __floats2bfloat162_rn(v[i], v[i + 1]);
            const float f0 = __low2float(h), f1 = __high2float(h);
            const int col = c0 + i;
            if (col < nvalid && (bidx < 0 || f0 > best || (f0 != f0 && best == best))) {
              best = f0;
              bidx = v0 + col;
            }
            if (col + 1 < nvalid && (f1 > best || (f1 != f1 && best == best))) {
              best = f1;
              bidx = v0 + col + 1;
            }
          }
        }
        bv[m] = best;
        bi[m] = bidx;
      }
      tc_fence_before();
      mbar_arrive(&sh.acc_empty[b]);
    }
#pragma unroll
    for (int m = 0; m < 2; ++m) {
      const int row = m * 128 + r;
      if (m >= mt) break;
      if (row < a.rows && bi[m] >= 0)
        atomicMax(&a.keys[row], ((unsigned long long)order_key(bv[m]) << 32) |
                                    (unsigned long long)(0xFFFFFFFFu - (uint32_t)bi[m]));
    }
  }

  // every CTA counts itself done (also after a wait ran out), so the last one
  // always turns the keys into tokens and zeroes the workspace
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    sh.last = atomicAdd(a.done, 1) == (int)gridDim.x - 1;
  }
  __syncthreads();
  if (sh.last) {
    __threadfence();
    for (int row = threadIdx.x; row < a.rows; row += blockDim.x) {
      const unsigned long long k = atomicExch(&a.keys[row], 0ull);
      a.out[row] = k ? (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull)) : 0;
    }
    if (threadIdx.x == 0) atomicExch(a.done, 0);
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, LM_TMEM_COLS);
  }
}

int g_sms[64] = {0};
bool g_attr[64] = {false};

struct WMapEntry {
  int dev;
  const void* base;
  long vocab, hidden, ldw;
  CUtensorMap map;
};
std::mutex g_wmu;
WMapEntry g_wmaps[16];
int g_nw = 0;

// W's tensor map, encoded once per (device, weight allocation, shape).
int w_map_for(int dev, const void* w, long vocab, long hidden, long ldw, CUtensorMap* out) {
  std::lock_guard<std::mutex> lk(g_wmu);
  for (int i = 0; i < g_nw; ++i) {
    const WMapEntry& e = g_wmaps[i];
    if (e.dev == dev && e.base == w && e.vocab == vocab && e.hidden == hidden && e.ldw == ldw) {
      *out = e.map;
      return HY_OK;
    }
  }
  CUtensorMap m;
  const int rc = hy_encode_rows_map(w, hidden, vocab, ldw * 2, LM_N, &m);
  if (rc) return rc;
  const int slot = g_nw < 16 ? g_nw++ : (int)((reinterpret_cast<uintptr_t>(w) >> 8) % 16);
  g_wmaps[slot] = WMapEntry{dev, w, vocab, hidden, ldw, m};
  *out = m;
  return HY_OK;
}

int fail(int code, const char* msg) {
  hy_set_error(msg);
  return code;
}

}  // namespace

extern "C" int64_t hy_lm_head_argmax_workspace_size(void) {
  return 4096;   // LM_MAX_ROWS keys of 8 bytes, the CTA counter, padding
}

extern "C" int hy_lm_head_argmax(const void* x, int64_t ldx, int32_t rows, const void* w,
                                 int64_t ldw, int32_t vocab, int32_t hidden, int32_t* out,
                                 void* workspace, int32_t* err, void* stream) {
  if (rows == 0) {
    hy_set_error("");
    return HY_OK;
  }
  if (!x || !w || !out || !workspace || rows < 0 || vocab <= 0 || hidden <= 0 || ldx < hidden ||
      ldw < hidden)
    return fail(HY_E_INVALID, "hy_lm_head_argmax: bad argument");
  if (hidden % LM_KC != 0)
    return fail(HY_E_UNSUPPORTED, "hy_lm_head_argmax: hidden must be a multiple of 64");
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(w) & 15) ||
      (ldx * 2) % 16 || (ldw * 2) % 16 || (reinterpret_cast<uintptr_t>(workspace) & 15))
    return fail(HY_E_INVALID,
                "hy_lm_head_argmax: x, w and workspace must be 16-byte aligned, with row "
                "pitches a multiple of 16 bytes");
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64) return fail(HY_E_UNSUPPORTED, "hy_lm_head_argmax: device id >= 64");
  if (!g_attr[dev]) {
    cudaError_t e = cudaFuncSetAttribute(lm_head_argmax_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, LM_SMEM);
    if (e != cudaSuccess) return fail(HY_E_CUDA, "hy_lm_head_argmax: cudaFuncSetAttribute failed");
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_sms[dev] = n > 0 ? n : 148;
    g_attr[dev] = true;
  }
  CUtensorMap wmap;
  int rc = w_map_for(dev, w, vocab, hidden, ldw, &wmap);
  if (rc) return rc;
  LmArgs a;
  a.vocab = vocab;
  a.nk = hidden / LM_KC;
  a.ntiles = (vocab + LM_N - 1) / LM_N;
  a.keys = static_cast<unsigned long long*>(workspace);
  a.done = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + LM_MAX_ROWS * 8);
  a.err = err;
  const int grid = a.ntiles < g_sms[dev] ? a.ntiles : g_sms[dev];
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // launches of up to 256 rows each, one after another on the stream (each
  // leaves the workspace at zero for the next)
  for (int r0 = 0; r0 < rows; r0 += LM_MAX_ROWS) {
    a.rows = rows - r0 < LM_MAX_ROWS ? rows - r0 : LM_MAX_ROWS;
    a.mt = a.rows > 128 ? 2 : 1;
    a.arows0 = a.mt == 2 ? 128 : (a.rows + 7) / 8 * 8;
    a.arows1 = a.mt == 2 ? (a.rows - 128 + 7) / 8 * 8 : 0;
    const int stage_bytes = (a.arows0 + a.arows1) * 128 + LM_B_BYTES;
    a.ns = LM_RING / stage_bytes < LM_MAX_STAGES ? LM_RING / stage_bytes : LM_MAX_STAGES;
    a.out = out + r0;
    const __nv_bfloat16* xr = static_cast<const __nv_bfloat16*>(x) + (size_t)r0 * ldx;
    CUtensorMap xmap0, xmap1;
    rc = hy_encode_rows_map(xr, hidden, a.rows, ldx * 2, a.arows0, &xmap0);
    if (rc) return rc;
    xmap1 = xmap0;
    if (a.mt == 2) {
      rc = hy_encode_rows_map(xr, hidden, a.rows, ldx * 2, a.arows1, &xmap1);
      if (rc) return rc;
    }
    cudaError_t e = hy_launch(lm_head_argmax_kernel, dim3(grid), dim3(LM_THREADS),
                              (size_t)LM_SMEM, st, xmap0, xmap1, wmap, a);
    if (e != cudaSuccess) {
      char buf[256];
      snprintf(buf, sizeof(buf), "hy_lm_head_argmax: %s", cudaGetErrorString(e));
      return fail(HY_E_CUDA, buf);
    }
  }
  hy_set_error("");
  return HY_OK;
}
