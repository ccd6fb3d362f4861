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
// Vocab tiles of 208 columns (731 tiles of a 151936 vocabulary) are dealt to
// persistent owners in turn.  An owner is one CTA for up to 128 rows, and a
// pair of CTAs (a cluster of two, cta_group::2, one M = 256 MMA) for 129-256
// rows: each CTA of a pair loads its own 128 rows of x and half of every W
// tile and holds its rows' accumulators, so a stage costs 29 KB per CTA
// instead of the 58 KB of both M tiles in one CTA, and seven stages fit.
// 6 warps per CTA:
//   warp 0      one lane issues the TMA loads: per 64-wide hidden chunk, the
//               CTA's x rows and its W rows of the tile into a ring of stages,
//               W with an L2 evict-first hint (it streams through once) and x
//               evict-last (every tile reads it again);
//   warp 1      allocates the TMEM columns; one lane (of a pair's even CTA)
//               issues the tcgen05 MMAs (N = 208 vocab columns, fp32
//               accumulators in TMEM, two buffers so the epilogue of one tile
//               overlaps the MMAs of the next);
//   warps 2-5   the epilogue: thread r owns row r of the CTA's M tile (TMEM
//               lane r), reads its 208 accumulators, rounds them to bf16 and
//               keeps its best (value, index) across the owner's tiles.
// A single CTA's stage holds only the x rows that exist (rounded up to 8),
// followed by its W rows: an M = 128 MMA over a shorter x box reads the
// stage's next bytes as its remaining rows, whose sums are never read, so
// small batches leave room for more stages (7 at 16 rows, 5 at 128) and more W
// in flight.  The CTAs' row bests meet in a 64-bit atomicMax over (order key
// of the bf16 value << 32 | ~index); the last CTA to finish writes the tokens
// and returns the workspace to zero, so each call leaves it as it found it.
// No TMA load here carries a multicast qualifier: each CTA loads its own tiles.
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
constexpr int LM_MAX_STAGES = 8;
constexpr int LM_RING = 5 * (128 * 128 + LM_N * 128);   // 210 KB
constexpr int LM_SMEM = 1024 + LM_RING;
constexpr int LM_THREADS = 192;            // warps 2-5 (the epilogue) read TMEM lane quarters
                                            // 2, 3, 0, 1
constexpr int LM_TMEM_COLS = 512;           // two 256-column accumulator buffers
constexpr int LM_MAX_ROWS = 256;            // rows of x per launch

struct LmArgs {
  int rows;                                 // rows of x in this launch (1..256)
  int arows;                                // x rows a CTA loads per chunk (multiple of 8;
                                            // 128 in a pair)
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
  uint64_t full[LM_MAX_STAGES];             // pair: the even CTA's count both CTAs' bytes
  uint64_t free_[LM_MAX_STAGES];
  uint64_t acc_full[2];
  uint64_t acc_empty[2];                    // pair: the even CTA's count both CTAs' epilogues
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

// 2-D tiled tensor load into this CTA's shared memory with an L2 cache policy,
// completion counted on `bar` (a shared::cluster address: this CTA's barrier,
// or with PAIR the even CTA's).  No multicast.
template <bool PAIR>
HY_DEVICE void tma_load_2d_hint(void* dst, const CUtensorMap* map, int32_t x, int32_t y,
                                uint32_t bar, uint64_t policy) {
  if (PAIR)
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;"
        :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar),
           "l"(policy)
        : "memory");
  else
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;"
        :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar),
           "l"(policy)
        : "memory");
}

// ---- CTA pairs (cluster of two): the even CTA's thread issues M = 256 MMAs
// whose A rows 0-127 and 128-255 come from the two CTAs' shared memory, whose
// B rows (vocab columns) are split in halves between them (same offsets), and
// whose D rows land in each CTA's own TMEM at the same address.
HY_DEVICE uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
HY_DEVICE void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}
// The shared::cluster address of this CTA's `smem_addr` as seen in CTA `rank`.
HY_DEVICE uint32_t smem_in_cta(uint32_t smem_addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr), "r"(rank));
  return r;
}
HY_DEVICE void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" :: "r"(cluster_addr) : "memory");
}

template <bool PAIR>
HY_DEVICE void tmem_alloc_g(uint32_t* dst, uint32_t ncols) {
  if (PAIR) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 :: "r"(smem_u32(dst)), "r"(ncols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  } else {
    tmem_alloc(dst, ncols);
    tmem_relinquish();
  }
}
template <bool PAIR>
HY_DEVICE void tmem_dealloc_g(uint32_t taddr, uint32_t ncols) {
  if (PAIR)
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" :: "r"(taddr),
                 "r"(ncols) : "memory");
  else
    tmem_dealloc(taddr, ncols);
}
template <bool PAIR>
HY_DEVICE void mma_g(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                     uint32_t accumulate) {
  if (PAIR)
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
  else
    tc_mma_bf16(d_tmem, a_desc, b_desc, idesc, accumulate);
}
// Arrive on `bar` (in both CTAs of a pair) once every tcgen05 op this thread
// issued has completed.
template <bool PAIR>
HY_DEVICE void commit_g(uint64_t* bar) {
  if (PAIR)
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" :: "r"(smem_u32(bar)), "h"((uint16_t)3) : "memory");
  else
    tc_commit(bar);
}
template <bool PAIR>
HY_DEVICE void commit_local_g(uint64_t* bar) {
  if (PAIR)
    asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(smem_u32(bar)) : "memory");
  else
    tc_commit(bar);
}

template <bool PAIR>
__global__ void __launch_bounds__(LM_THREADS, 1) lm_head_argmax_kernel(
    const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap wmap, LmArgs a) {
  __shared__ LmShared sh;
  extern __shared__ uint8_t dyn_smem[];
  uint8_t* ring = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dyn_smem) + 1023) &
                                             ~uintptr_t(1023));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = PAIR ? cluster_rank() : 0u;
  const bool leader = rank == 0;
  const int ns = a.ns;
  // stage: [x rows][W rows], 1 KB-aligned; a pair's two CTAs have the same
  // layout, so one descriptor names both halves of an operand
  const uint32_t w_off = (uint32_t)a.arows * 128u;
  const int w_rows = PAIR ? LM_N / 2 : LM_N;
  const uint32_t stage_bytes = w_off + (uint32_t)w_rows * 128u;
  // bytes of one stage's loads (both CTAs' with a pair: they count at the leader)
  const uint32_t stage_tx = PAIR ? 2 * stage_bytes : stage_bytes;
  // vocab tiles of this owner (CTA or pair): unit, unit + nunits, ...
  const int unit = PAIR ? (int)blockIdx.x >> 1 : (int)blockIdx.x;
  const int nunits = PAIR ? (int)gridDim.x >> 1 : (int)gridDim.x;
  const int my_tiles = (a.ntiles - unit + nunits - 1) / nunits;
  if (threadIdx.x == 0) {
    prefetch_tmap(&xmap);
    prefetch_tmap(&wmap);
    for (int s = 0; s < LM_MAX_STAGES; ++s) {
      mbar_init(&sh.full[s], 1);              // the leader's producer
      mbar_init(&sh.free_[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&sh.acc_full[b], 1);
      mbar_init(&sh.acc_empty[b], PAIR ? 8 : 4);   // one arrival per epilogue warp
    }
    mbar_init(&sh.drain, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc_g<PAIR>(&sh.tmem_base, LM_TMEM_COLS);
  tc_fence_before();
  if (PAIR) cluster_sync();                   // both CTAs' barriers initialised
  else __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  bool ok = true;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = l2_stream_policy(), pol_x = l2_keep_policy();
      const uint32_t total = (uint32_t)(my_tiles * a.nk);
      const uint32_t pre = min((uint32_t)ns, total);
      const int xrow = 128 * (int)rank;
      const int wrow = (LM_N / 2) * (int)rank;
      // W depends on no earlier kernel: the first stages' W boxes go out before
      // the wait for the kernel that wrote x
      for (uint32_t c = 0; c < pre; ++c) {
        const int tile = unit + (int)(c / a.nk) * nunits, kc = (int)(c % a.nk);
        const uint32_t full = PAIR ? smem_in_cta(smem_u32(&sh.full[c]), 0) : smem_u32(&sh.full[c]);
        if (leader) mbar_arrive_expect_tx(&sh.full[c], stage_tx);
        tma_load_2d_hint<PAIR>(ring + c * stage_bytes + w_off, &wmap, kc * LM_KC,
                               tile * LM_N + wrow, full, pol_w);
      }
      hy_grid_wait();
      for (uint32_t c = 0; c < pre; ++c) {
        const uint32_t full = PAIR ? smem_in_cta(smem_u32(&sh.full[c]), 0) : smem_u32(&sh.full[c]);
        tma_load_2d_hint<PAIR>(ring + c * stage_bytes, &xmap, (int)(c % a.nk) * LM_KC, xrow, full,
                               pol_x);
      }
      uint32_t c = pre;
      for (; c < total; ++c) {
        const uint32_t s = c % ns, use = c / ns;
        if (!mbar_wait(&sh.free_[s], (use & 1) ^ 1, a.err)) {
          ok = false;
          break;
        }
        const int tile = unit + (int)(c / a.nk) * nunits, kc = (int)(c % a.nk);
        uint8_t* st = ring + s * stage_bytes;
        const uint32_t full = PAIR ? smem_in_cta(smem_u32(&sh.full[s]), 0) : smem_u32(&sh.full[s]);
        if (leader) mbar_arrive_expect_tx(&sh.full[s], stage_tx);
        tma_load_2d_hint<PAIR>(st + w_off, &wmap, kc * LM_KC, tile * LM_N + wrow, full, pol_w);
        tma_load_2d_hint<PAIR>(st, &xmap, kc * LM_KC, xrow, full, pol_x);
      }
      // the copies in flight land before the CTA ends (a pair's all count at
      // the leader, which waits for them; the final cluster barrier keeps the
      // odd CTA until then)
      if (!ok && leader)
        for (uint32_t d = c > (uint32_t)ns ? c - ns : 0; d < c; ++d)
          mbar_wait(&sh.full[d % ns], (d / ns) & 1, nullptr);
    } else {
      hy_grid_wait();
    }
  } else if (warp == 1) {
    hy_grid_wait();
    if (lane == 0 && leader) {
      const uint32_t idesc = tc_idesc_bf16(PAIR ? 256 : 128, LM_N, false);
      const uint32_t sbase = smem_u32(ring);
      uint32_t c = 0;
      for (int j = 0; j < my_tiles && ok; ++j) {
        const int b = j & 1;
        const uint32_t u = (uint32_t)(j >> 1);
        ok = mbar_wait(&sh.acc_empty[b], (u & 1) ^ 1, a.err);   // the epilogues read buffer b
        if (!ok) break;
        tc_fence_after();
        for (int kc = 0; kc < a.nk; ++kc, ++c) {
          const uint32_t s = c % ns, use = c / ns;
          ok = mbar_wait(&sh.full[s], use & 1, a.err);
          if (!ok) break;
          tc_fence_after();
          const uint32_t st = sbase + s * stage_bytes;
          // K-major operands, 8-row groups 1 KB apart; a 16-element K step is
          // 32 bytes into the 128-byte swizzled row.  A reads 128 rows from the
          // stage's start: past the loaded x rows, the stage's next bytes (their
          // sums are never read)
          const uint64_t dA = tc_desc_sw128(st, 16, 1024);
          const uint64_t dB = tc_desc_sw128(st + w_off, 16, 1024);
#pragma unroll
          for (int kk = 0; kk < LM_KC / 16; ++kk)
            mma_g<PAIR>(tmem + (uint32_t)(b * 256), dA + (uint64_t)(kk * 2),
                        dB + (uint64_t)(kk * 2), idesc, (kc | kk) != 0);
          commit_g<PAIR>(&sh.free_[s]);
        }
        if (!ok) break;
        commit_g<PAIR>(&sh.acc_full[b]);
      }
      if (!ok) {                              // let every issued MMA finish
        commit_local_g<PAIR>(&sh.drain);
        mbar_wait(&sh.drain, 0, nullptr);
      }
    }
    __syncwarp();
  } else {
    hy_grid_wait();
    const int q = warp & 3;                   // TMEM lane quarter this warp may read
    const int row = (int)rank * 128 + 32 * q + lane;
    const bool live = (int)rank * 128 + 32 * q < a.rows;   // warp-uniform: any row to keep
    const uint32_t lane_off = (uint32_t)(32 * q) << 16;
    const uint32_t empty0 = PAIR ? smem_in_cta(smem_u32(&sh.acc_empty[0]), 0)
                                 : smem_u32(&sh.acc_empty[0]);
    float best = 0.f;
    int bidx = -1;
    for (int j = 0; j < my_tiles; ++j) {
      const int b = j & 1;
      const uint32_t u = (uint32_t)(j >> 1);
      ok = __all_sync(0xffffffffu, mbar_wait(&sh.acc_full[b], u & 1, a.err));
      if (!ok) break;
      tc_fence_after();
      const int v0 = (unit + j * nunits) * LM_N;
      const int nvalid = min(LM_N, a.vocab - v0);
      if (live) {
        const uint32_t tb = tmem + lane_off + (uint32_t)(b * 256);
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
      }
      // the warp's reads of buffer b are complete: one arrival (at the leader)
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(empty0 + (uint32_t)(b * 8));
    }
    if (row < a.rows && bidx >= 0)
      atomicMax(&a.keys[row], ((unsigned long long)order_key(best) << 32) |
                                  (unsigned long long)(0xFFFFFFFFu - (uint32_t)bidx));
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
    for (int r = threadIdx.x; r < a.rows; r += blockDim.x) {
      const unsigned long long k = atomicExch(&a.keys[r], 0ull);
      a.out[r] = k ? (int32_t)(0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull)) : 0;
    }
    if (threadIdx.x == 0) atomicExch(a.done, 0);
  }
  if (PAIR) cluster_sync();                   // both CTAs are done with TMEM and the ring
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_g<PAIR>(tmem, LM_TMEM_COLS);
  }
}

std::mutex g_setup_mu;                      // guards the per-device set-up below
int g_sms[64] = {0};
int g_pairs[64] = {0};                      // co-resident CTA pairs (clusters of two)
bool g_attr[64] = {false};

struct WMapEntry {
  int dev;
  const void* base;
  long vocab, hidden, ldw;
  int box_rows;
  CUtensorMap map;
};
std::mutex g_wmu;
WMapEntry g_wmaps[16];
int g_nw = 0;

// W's tensor map, encoded once per (device, weight allocation, shape, box).
int w_map_for(int dev, const void* w, long vocab, long hidden, long ldw, int box_rows,
              CUtensorMap* out) {
  std::lock_guard<std::mutex> lk(g_wmu);
  for (int i = 0; i < g_nw; ++i) {
    const WMapEntry& e = g_wmaps[i];
    if (e.dev == dev && e.base == w && e.vocab == vocab && e.hidden == hidden && e.ldw == ldw &&
        e.box_rows == box_rows) {
      *out = e.map;
      return HY_OK;
    }
  }
  CUtensorMap m;
  const int rc = hy_encode_rows_map(w, hidden, vocab, ldw * 2, box_rows, &m);
  if (rc) return rc;
  const int slot = g_nw < 16 ? g_nw++ : (int)((reinterpret_cast<uintptr_t>(w) >> 8) % 16);
  g_wmaps[slot] = WMapEntry{dev, w, vocab, hidden, ldw, box_rows, m};
  *out = m;
  return HY_OK;
}

int fail(int code, const char* msg) {
  hy_set_error(msg);
  return code;
}

cudaError_t launch(bool pair, int grid, cudaStream_t st, const CUtensorMap& xmap,
                   const CUtensorMap& wmap, const LmArgs& a) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(LM_THREADS);
  cfg.dynamicSmemBytes = LM_SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  int n = 0;
  if (pair) {
    attr[n].id = cudaLaunchAttributeClusterDimension;
    attr[n].val.clusterDim.x = 2;
    attr[n].val.clusterDim.y = 1;
    attr[n].val.clusterDim.z = 1;
    ++n;
  }
  if (hy_pdl_enabled()) {
    attr[n].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[n].val.programmaticStreamSerializationAllowed = 1;
    ++n;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return pair ? cudaLaunchKernelEx(&cfg, lm_head_argmax_kernel<true>, xmap, wmap, a)
              : cudaLaunchKernelEx(&cfg, lm_head_argmax_kernel<false>, xmap, wmap, a);
}

// Per device, once: shared-memory attributes, SM count, co-resident pairs (the
// tiles are dealt to owners in advance, so every pair must be resident at once).
cudaError_t setup(int dev) {
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (g_attr[dev]) return cudaSuccess;
  cudaError_t e = cudaFuncSetAttribute(lm_head_argmax_kernel<false>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, LM_SMEM);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(lm_head_argmax_kernel<true>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, LM_SMEM);
  if (e != cudaSuccess) return e;
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  g_sms[dev] = n > 0 ? n : 148;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * (g_sms[dev] / 2));
  cfg.blockDim = dim3(LM_THREADS);
  cfg.dynamicSmemBytes = LM_SMEM;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int clusters = 0;
  e = cudaOccupancyMaxActiveClusters(&clusters, lm_head_argmax_kernel<true>, &cfg);
  if (e != cudaSuccess) return e;
  g_pairs[dev] = clusters > 0 ? clusters : 1;
  g_attr[dev] = true;
  return cudaSuccess;
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
  cudaError_t e = setup(dev);
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof(buf), "hy_lm_head_argmax: set-up failed: %s", cudaGetErrorString(e));
    return fail(HY_E_CUDA, buf);
  }
  LmArgs a;
  a.vocab = vocab;
  a.nk = hidden / LM_KC;
  a.ntiles = (vocab + LM_N - 1) / LM_N;
  a.keys = static_cast<unsigned long long*>(workspace);
  a.done = reinterpret_cast<int*>(static_cast<uint8_t*>(workspace) + LM_MAX_ROWS * 8);
  a.err = err;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // launches of up to 256 rows each, one after another on the stream (each
  // leaves the workspace at zero for the next)
  for (int r0 = 0; r0 < rows; r0 += LM_MAX_ROWS) {
    a.rows = rows - r0 < LM_MAX_ROWS ? rows - r0 : LM_MAX_ROWS;
    a.out = out + r0;
    // more than 128 rows: CTA pairs, each CTA with its 128 rows (the odd one's
    // box reads zeros past the last row) and half of every W tile
    const bool pair = a.rows > 128;
    a.arows = pair ? 128 : (a.rows + 7) / 8 * 8;
    const int w_rows = pair ? LM_N / 2 : LM_N;
    const int stage_bytes = (a.arows + w_rows) * 128;
    a.ns = LM_RING / stage_bytes < LM_MAX_STAGES ? LM_RING / stage_bytes : LM_MAX_STAGES;
    CUtensorMap xmap, wmap;
    int rc = hy_encode_rows_map(static_cast<const __nv_bfloat16*>(x) + (size_t)r0 * ldx, hidden,
                                a.rows, ldx * 2, a.arows, &xmap);
    if (rc == HY_OK) rc = w_map_for(dev, w, vocab, hidden, ldw, w_rows, &wmap);
    if (rc) return rc;
    const int owners_max = pair ? g_pairs[dev] : g_sms[dev];
    const int owners = a.ntiles < owners_max ? a.ntiles : owners_max;
    e = launch(pair, pair ? 2 * owners : owners, st, xmap, wmap, a);
    if (e != cudaSuccess) {
      char buf[256];
      snprintf(buf, sizeof(buf), "hy_lm_head_argmax: %s", cudaGetErrorString(e));
      return fail(HY_E_CUDA, buf);
    }
  }
  hy_set_error("");
  return HY_OK;
}
