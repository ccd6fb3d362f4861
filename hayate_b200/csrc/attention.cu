// Varlen paged GQA attention: chunked-prefill and decode sequences in one launch.
//
// Replaces the reference's per-layer cache concat + masked SDPA
// (hayate/model/attention.py:52-64) and the additive mask / position logic it
// depends on (hayate/model/qwen.py:66-106).  Semantics: the j-th query token of
// sequence i sits at position prefix_i + j (prefix_i = seq_len_k_i - q_len_i) and
// attends to keys [0, prefix_i + j] of its own sequence -- the reference's causal
// mask with cache-padding and left-padding columns removed.  The softmax scale is
// 1/sqrt(128) (the SDPA default the reference uses).
//
// Memory: q/out are [tokens][q_heads][128]; the cache of one layer is
// [block][2 (K,V)][kv_heads][16][128], all layers back to back.  Block tables are
// rows of physical block ids (row i = sequence i, or seq_bt_row[i]).
//
// Work is planned on the device (plan_kernel) once per step and reused by every
// layer:
//   * prefill items -- (seq, kv_head, 64-token tile): one CTA, warp-specialised:
//     two M=128 tcgen05 tiles (two query heads x 64 tokens each) share every
//     64-key K/V tile, staged by TMA in 4-slot rings by two load warps (two of
//     the tile's four blocks each: one warp issues too few boxes); one MMA warp
//     per tile issues its S = Q K^T and O += P V with S, P and O in TMEM; two
//     softmax warpgroups run one thread per query row;
//   * decode items  -- (seq, kv_head, block range): one warp with its own TMA
//     ring of K/V block tiles, mma.sync for QK^T and PV, an online softmax;
//     for a sequence split over several items, the last item to finish (an
//     atomic count per sequence and KV head) merges the partials.
// The main kernel is persistent (grid = SMs x resident CTAs): CTAs pull prefill
// items (heaviest first) and then decode items (per warp) from per-layer atomic
// counters, so its launch shape does not depend on the batch and a whole step
// can be captured in a CUDA graph.
#include "common.cuh"
#include "attention.cuh"

#include <math.h>

namespace {

#ifndef HY_ATT_WARPS
#define HY_ATT_WARPS 8
#endif
#ifndef HY_DEC_STAGES
#define HY_DEC_STAGES 3
#endif
constexpr int ATT_WARPS = HY_ATT_WARPS;                          // 8 decode / softmax warps
constexpr int TC_MMA_WARP = ATT_WARPS;                           // prefill: tcgen05 issue, tile 0
constexpr int TC_LOAD_WARP = ATT_WARPS + 1;                      // prefill: TMA issue, blocks 0-1
constexpr int TC_LOAD_WARP2 = ATT_WARPS + 3;                     // prefill: TMA issue, blocks 2-3
constexpr int TC_MMA_WARP1 = ATT_WARPS + 2;                      // prefill: tcgen05 issue, tile 1
constexpr int ATT_THREADS = (ATT_WARPS + 4) * 32;                // 384
constexpr int DEC_STAGES = HY_DEC_STAGES;                        // TMA ring per decode warp
constexpr int DEC_TILE_BYTES = 2 * HY_BLOCK * HY_HEAD_DIM * 2;   // K+V of one block: 8 KB
constexpr int DEC_WARP_BYTES = DEC_STAGES * DEC_TILE_BYTES;      // 24 KB
constexpr int PRE_QROWS = 64;                                    // query tokens per prefill item
// tcgen05 prefill: sub-tile X (0, 1) = 128 rows r: query head 4g + 2X + r / 64,
// token t0 + r % 64; KV tiles of 64 keys (4 blocks) in rings of TC_NS slots.
// A K slot holds each block's 4 KB tile as one 4-D TMA box lands it
// ([block][8-key group][half][8 keys][64]: the K-major operand of S = Q K^T,
// its 8-key groups 2 KB apart, column half h at +1 KB h); a V slot holds each
// block's tile as one 3-D box lands it ([block][half][16 keys][64], the MN-major
// operand of P V).
constexpr int TC_KEYS = 64;
constexpr int TC_NS = 4;                                         // K and V ring slots
constexpr int TC_KV_BYTES = TC_KEYS * HY_HEAD_DIM * 2;          // K or V of one tile: 16 KB
constexpr int TC_Q_BYTES = 128 * HY_HEAD_DIM * 2;                // Q of one sub-tile: 32 KB
constexpr int TC_K_OFF = 2 * TC_Q_BYTES;                         // K ring
constexpr int TC_V_OFF = TC_K_OFF + TC_NS * TC_KV_BYTES;         // V ring
constexpr int TC_SMEM = TC_V_OFF + TC_NS * TC_KV_BYTES;          // 192 KB
// TMEM columns: two S buffers per sub-tile, S_X[b] at 64 (2X + b), P_X[b] (bf16
// pairs) written over the first 32 columns of S_X[b]; O_X at 256 + 128 X.
constexpr uint32_t TC_TMEM_COLS = 512;
constexpr uint32_t TM_O = 256;
HY_DEVICE uint32_t tm_s(int X, uint32_t b) { return 64u * (2u * X + b); }
constexpr int SMEM_PAYLOAD = ATT_WARPS * DEC_WARP_BYTES > TC_SMEM ? ATT_WARPS * DEC_WARP_BYTES
                                                                   : TC_SMEM;
constexpr int SMEM_BYTES = SMEM_PAYLOAD + 1024;                  // + alignment slack
#ifndef HY_MIN_SPLIT
#define HY_MIN_SPLIT 4
#endif
#ifndef HY_ITEMS_PER_WARP
#define HY_ITEMS_PER_WARP 3
#endif
constexpr int MIN_SPLIT = HY_MIN_SPLIT;                          // blocks per decode item, at least
constexpr int ITEMS_PER_WARP = HY_ITEMS_PER_WARP;                // decode items aimed at per warp
// Per-CTA decode: a step of decode sequences only, whose (sequence, KV head)
// pairs fit one per CTA and whose contexts are at most GROUP_MAX_BLOCKS blocks,
// gives each pair to one CTA; its decode warps split the pair's blocks and
// merge their partials in shared memory.
#ifndef HY_GROUP_MAX_BLOCKS
#define HY_GROUP_MAX_BLOCKS 128
#endif
constexpr int GROUP_MAX_BLOCKS = HY_GROUP_MAX_BLOCKS;
constexpr int MERGE_BAR = 1;                                     // named barrier of the decode warps
constexpr int PRE_LOAD_BAR = 2;                                  // named barrier of the two prefill
                                                                 // load warps
constexpr int GRAB_INTS = 4;                                     // per layer: decode item, CTAs
                                                                 // done, prefill item, spare
// a split-K merge stages the partials of MERGE_CHUNK splits at a time (2 KB of O
// and 32 B of (m, l) each, then their weights) in the merging warp's TMA ring
constexpr int MERGE_CHUNK = 8;                                   // = 32 lanes / 4 heads
constexpr int MERGE_O_BYTES = MERGE_CHUNK * HY_GROUP * HY_HEAD_DIM * 4;
constexpr int MERGE_ML_BYTES = MERGE_CHUNK * HY_GROUP * 8;
static_assert(MERGE_O_BYTES + MERGE_ML_BYTES + MERGE_CHUNK * HY_GROUP * 4 <= DEC_WARP_BYTES,
              "merge staging must fit a decode warp's ring");
constexpr float NEG_INF = -INFINITY;
// Split prefill items: a step with fewer prefill items (64 query tokens x one
// KV head) than SMs cuts the long ones into pieces over equal key-tile ranges,
// at least PRE_SPLIT_MIN tiles each, so that the pieces fill the idle SMs;
// each piece leaves its unnormalised O, running max and sum in the workspace
// and the last piece to finish merges them.  Without this such a step waits
// for its longest items (one 512-token chunk after 3584 cached tokens: 64
// items of 57-64 key tiles, 84 SMs idle: 80.0 us uncut, 57.6 us cut).  A
// step with at least as many items as SMs, or with decode work for the idle
// SMs, is not cut: a piece costs a second Q load, a 128 KB partial and its
// share of the merge (~25k cycles per cut item, measured), more than the
// balance gains there (4 chunks of 512: 80.6 us uncut, 93.0 us cut to the
// tiles per SM; one chunk beside 256 decode sequences: 704 us uncut, 732 us
// cut).
#ifndef HY_PRE_SPLIT_MIN
#define HY_PRE_SPLIT_MIN 16
#endif
constexpr int PRE_SPLIT_MIN = HY_PRE_SPLIT_MIN;                  // key tiles
constexpr int PRE_MAX_PIECES = 31;
constexpr int PRE_PART_F4 = 32 * 256;                            // float4 of O per piece

// key tiles of the prefill item at query offset t0 of a sequence of q query
// tokens and kv keys
HY_DEVICE int pre_item_tiles(int kv, int q, int t0) {
  return (kv - q + t0 + min(PRE_QROWS, q - t0) + TC_KEYS - 1) / TC_KEYS;
}
HY_DEVICE int pre_pieces(int nt, int cap) {
  return nt > cap ? min(PRE_MAX_PIECES, (nt + cap - 1) / cap) : 1;
}
// An item's w field: 0 for a whole item, else (pieces << 26) | (piece << 20) |
// the first partial slot of the item (its pieces use consecutive slots).
HY_DEVICE int pre_piece_code(int ns, int sp, int slot) { return (ns << 26) | (sp << 20) | slot; }
HY_DEVICE int pre_code_pieces(int w) { return (w >> 26) & 31; }
HY_DEVICE int pre_code_piece(int w) { return (w >> 20) & 63; }
HY_DEVICE int pre_code_slot(int w) { return w & 0xFFFFF; }
// key tiles [lo, hi) that the item (w) of nt key tiles covers
HY_DEVICE void pre_piece_range(int w, int nt, int& lo, int& hi) {
  if (w == 0) { lo = 0; hi = nt; return; }
  const int ns = pre_code_pieces(w), sp = pre_code_piece(w);
  lo = sp * nt / ns;
  hi = (sp + 1) * nt / ns;
}
#ifndef HY_EXP2_POLY_EVERY
#define HY_EXP2_POLY_EVERY 0
#endif
// prefill softmax: 1 in EXP2_POLY_EVERY pairs of weights by exp2_poly (0: none).
// Off: with the row max and sum as independent chains the exp2 unit is not
// the limit, and the polynomial's extra instructions cost issue slots (4
// prefill chunks of 512 / 16 chunks, one box: 83.3 / 300.7 us with none,
// 82.9 / 299.3 with 1 in 8, 85.0 / 307.2 with 1 in 4, 93.0 / 334.1 with 1 in 2).
constexpr int EXP2_POLY_EVERY = HY_EXP2_POLY_EVERY;
// Lazy rescaling: the running max is only raised when a new score exceeds it
// by more than 2^RESCALE_LOG2; until then probabilities may exceed 1 by up to
// that factor, which fp32 accumulators and bf16 P carry without loss of
// relative precision.  Output = O / l is unchanged (both use the same max).
constexpr float RESCALE_LOG2 = 8.0f;

struct Shared {
  uint64_t dec_bar[ATT_WARPS][DEC_STAGES];
  // tcgen05 prefill.  Ring barriers complete once per use of their slot, the
  // per-sub-tile ones once per key tile.
  uint64_t tc_full[TC_NS];   // K and V tiles landed (TMA transaction bytes)
  uint64_t tc_free[TC_NS];   // both PV MMAs of the slot's tile are done (2 commits): with
                             // them the S MMAs that read its K (issued earlier by the
                             // same threads) are done too
  uint64_t tc_sfull[2][2];   // S_X[b] = Q_X K^T complete (once per use of buffer b)
  uint64_t tc_pfull[2][2];   // P_X[b] written over S_X[b] by the 4 softmax warps of X
  uint64_t tc_odone[2];      // O_X += P_X V complete (once per key tile)
  uint64_t tc_drain[2];      // error path: all MMAs an issuing warp issued are complete
  uint64_t tc_qfull;         // the item's Q landed (TMA transaction bytes, once per item)
  uint32_t tmem_base;        // TMEM columns from tcgen05.alloc
  int pre_item;              // prefill item handed to this CTA
  int pre_last;              // this CTA's piece of a split prefill item finished last
  int pre_prefetch;          // the next item's key tiles its Q and loads were issued
                             // for by the current item's load warps (-1: none)
};

HY_DEVICE uint8_t* payload_base(uint8_t* dyn) {
  const uint32_t a = smem_u32(dyn);
  return dyn + (((a + 1023u) & ~1023u) - a);
}

// ------------------------------------------------------------------ plan kernel
constexpr int PLAN_THREADS = 1024;

__device__ int plan_scan(int v, int* ws, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) ws[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = ws[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    ws[lane] = w;
  }
  __syncthreads();
  const int before = warp ? ws[warp - 1] : 0;
  total = ws[31];
  __syncthreads();
  return before + x - v;
}

// a * b / c for non-negative ints, in 32-bit arithmetic when the product fits
HY_DEVICE int mul_div(int a, int b, int c) {
  const long long p = (long long)a * b;
  return p <= 0x7fffffffLL ? (int)((unsigned)p / (unsigned)c) : (int)(p / c);
}

__global__ void __launch_bounds__(PLAN_THREADS) plan_kernel(
    const int32_t* __restrict__ cu_q, const int32_t* __restrict__ seq_lens_k, int S,
    int kv_heads, int warp_slots, PlanView v, int32_t* err) {
  hy_grid_wait();
  hy_grid_trigger();
  __shared__ int ws[32];
  __shared__ int s_total, s_cpre, s_cdec, s_cpart, s_bad, s_maxblk, s_anypre, s_ptiles, s_pitems;
  if (threadIdx.x == 0) {
    s_total = 0; s_cpre = 0; s_cdec = 0; s_cpart = 0; s_bad = 0; s_maxblk = 0; s_anypre = 0;
    s_ptiles = 0; s_pitems = 0;
  }
  __syncthreads();
  // Pass 1: KV blocks over all decode sequences, the longest, any prefill, and
  // the prefill items and their key tiles (per KV head).
  int part = 0, mxb = 0, pre = 0, ptiles = 0, pitems = 0;
  for (int i = threadIdx.x; i < S; i += PLAN_THREADS) {
    const int q = cu_q[i + 1] - cu_q[i], kv = seq_lens_k[i];
    if (q == 1) {
      const int nb = (kv + HY_BLOCK - 1) / HY_BLOCK;
      part += nb;
      mxb = max(mxb, nb);
    } else if (q > 1) {
      pre = 1;
      if (kv >= q)
        for (int t0 = 0; t0 < q; t0 += PRE_QROWS) {
          ptiles += pre_item_tiles(kv, q, t0);
          ++pitems;
        }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    part += __shfl_xor_sync(0xffffffffu, part, o);
    mxb = max(mxb, __shfl_xor_sync(0xffffffffu, mxb, o));
    pre |= __shfl_xor_sync(0xffffffffu, pre, o);
    ptiles += __shfl_xor_sync(0xffffffffu, ptiles, o);
    pitems += __shfl_xor_sync(0xffffffffu, pitems, o);
  }
  if ((threadIdx.x & 31) == 0) {                // 32 shared atomics, not 1024
    atomicAdd(&s_total, part);
    atomicMax(&s_maxblk, mxb);
    atomicOr(&s_anypre, pre);
    atomicAdd(&s_ptiles, ptiles);
    atomicAdd(&s_pitems, pitems);
  }
  __syncthreads();
  // Prefill pieces, only when the n items are fewer than the SMs and the
  // step's decode work would not fill the idle SMs anyway (a decode block of
  // one KV head, 8 KB of K/V at an SM's share of HBM bandwidth, takes about a
  // fifth of a key tile's ~1 us on the tensor cores; the decode work must be
  // at most a quarter of the prefill tiles).  An item of nt key tiles is cut
  // into ceil(nt / cap) pieces, cap >= tiles / (SMs - n), so the pieces, at
  // most tiles / cap + n, are at most the SMs: the workspace's slots.
  const int n_sm = warp_slots / ATT_WARPS;
  const long tiles_all = (long)s_ptiles * kv_heads;
  const long n_items = (long)s_pitems * kv_heads;
  const long dec_tiles = (long)s_total * kv_heads / 5;
  const int cap = v.max_pre_part >= n_sm && n_items > 0 && n_items < n_sm &&
                          4 * dec_tiles <= tiles_all
                      ? (int)max((long)PRE_SPLIT_MIN,
                                 (tiles_all + (n_sm - n_items) - 1) / (n_sm - n_items))
                      : 0x7fffffff;
  const long target = (long)ITEMS_PER_WARP * warp_slots;
  const long want = ((long)kv_heads * s_total + target - 1) / target;
  const int split = (int)max((long)MIN_SPLIT, want);
  // per-CTA decode (see GROUP_MAX_BLOCKS): one item per warp, at most a CTA's warps
  const bool group = !s_anypre && (long)S * kv_heads <= warp_slots / ATT_WARPS &&
                     s_maxblk <= GROUP_MAX_BLOCKS;

  // Pass 2: item counts, offsets, items.
  for (int base = 0; base < S; base += PLAN_THREADS) {
    const int i = base + threadIdx.x;
    int npre = 0, ndec = 0, ns = 0, ntile = 0, nblk = 0, row = 0, kv = 0, q = 0;
    int npart = 0, ph = 0, psl = 0;             // pieces and partial slots per KV head
    if (i < S) {
      row = cu_q[i];
      q = cu_q[i + 1] - row;
      kv = seq_lens_k[i];
      if (q < 0 || kv < q) atomicOr(&s_bad, HY_ERR_BOUNDS);
      else if (q == 1) {
        nblk = (kv + HY_BLOCK - 1) / HY_BLOCK;
        ns = group ? max(1, min(ATT_WARPS, nblk)) : (nblk + split - 1) / split;
        ndec = kv_heads * ns;
      } else if (q > 1) {
        ntile = (q + PRE_QROWS - 1) / PRE_QROWS;
        for (int t = 0; t < ntile; ++t) {
          const int n = pre_pieces(pre_item_tiles(kv, q, t * PRE_QROWS), cap);
          ph += n;
          if (n > 1) psl += n;
        }
        npre = kv_heads * ph;
        npart = kv_heads * psl;
      }
    }
    int tpre, tdec, tpart;
    const int opre = plan_scan(npre, ws, tpre);
    const int odec = plan_scan(ndec, ws, tdec);
    const int opart = plan_scan(npart, ws, tpart);
    const int cpre = s_cpre, cdec = s_cdec, cpart = s_cpart;
    if (i < S && i < v.max_seqs)
      for (int g = 0; g < kv_heads; ++g) v.counters[i * kv_heads + g] = 0;
    bool wr = false;
    int p0 = 0, d0 = 0, s0 = 0;
    if (i < S) {
      p0 = cpre + opre;
      d0 = cdec + odec;
      s0 = cpart + opart;
      if (p0 + npre > v.max_pre || d0 + ndec > v.max_dec || i >= v.max_seqs ||
          s0 + npart > v.max_pre_part) {
        atomicOr(&s_bad, HY_ERR_PLAN);
      } else {
        v.seqinfo[i] = make_int2(d0, ns);
        wr = true;
      }
    }
    // The warp writes the items of its sequences together, one sequence at a
    // time (item k of a sequence: head k / n, split or tile k % n).
    const int lane = threadIdx.x & 31;
    unsigned todo = __ballot_sync(0xffffffffu, wr);
    while (todo) {
      const int j = __ffs(todo) - 1;
      todo &= todo - 1;
      const int ji = __shfl_sync(0xffffffffu, i, j);
      const int jp0 = __shfl_sync(0xffffffffu, p0, j), jd0 = __shfl_sync(0xffffffffu, d0, j);
      const int jns = __shfl_sync(0xffffffffu, ns, j), jnb = __shfl_sync(0xffffffffu, nblk, j);
      const int jrow = __shfl_sync(0xffffffffu, row, j), jkv = __shfl_sync(0xffffffffu, kv, j);
      const int jnt = __shfl_sync(0xffffffffu, ntile, j), jq = __shfl_sync(0xffffffffu, q, j);
      const int jph = __shfl_sync(0xffffffffu, ph, j), jpsl = __shfl_sync(0xffffffffu, psl, j);
      const int js0 = __shfl_sync(0xffffffffu, s0, j);
      for (int k = lane; k < kv_heads * jns; k += 32) {   // splits differ by at most one block
        const int g = k / jns, sp = k - g * jns;
        const int lo = mul_div(sp, jnb, jns), hi = mul_div(sp + 1, jnb, jns);
        v.dec[2 * (jd0 + k)] = make_int4(ji, g, lo, hi);
        v.dec[2 * (jd0 + k) + 1] = make_int4(jrow, jkv, jns, jd0 + g * jns);
        v.dec_ids[2 * (jd0 + k)] = make_int4(-1, 0, 0, 0);
      }
      // (KV head g, query tile t): its pieces follow those of head g's earlier
      // query tiles; a cut item's pieces take consecutive partial slots
      for (int k = lane; k < kv_heads * jnt; k += 32) {
        const int g = k / jnt, t = k - g * jnt;
        int pos = jp0 + g * jph, slot = js0 + g * jpsl;
        for (int u = 0; u < t; ++u) {
          const int n = pre_pieces(pre_item_tiles(jkv, jq, u * PRE_QROWS), cap);
          pos += n;
          if (n > 1) slot += n;
        }
        const int n = pre_pieces(pre_item_tiles(jkv, jq, t * PRE_QROWS), cap);
        for (int sp = 0; sp < n; ++sp)
          v.pre[pos + sp] = make_int4(ji, g, t * PRE_QROWS, n > 1 ? pre_piece_code(n, sp, slot) : 0);
        if (n > 1) v.pre_ctr[slot] = 0;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) { s_cpre += tpre; s_cdec += tdec; s_cpart += tpart; }
    __syncthreads();
  }
  if (threadIdx.x < 64 * GRAB_INTS) v.grab[threadIdx.x] = 0;
  // Prefill items ordered by their key tiles, most first (a counting sort over
  // PLAN_THREADS cost bins), so that CTAs pulling them in order start the
  // longest ones first whatever the order of the sequences in the batch.
  __syncthreads();                              // the items above are written
  const int np = s_bad ? 0 : min(s_cpre, v.max_pre);
  __shared__ int bins[PLAN_THREADS];
  auto cost_bin = [&](int4 it) {                // bin 0 = most key tiles
    const int q = cu_q[it.x + 1] - cu_q[it.x], kv = seq_lens_k[it.x];
    int lo, hi;
    pre_piece_range(it.w, pre_item_tiles(kv, q, it.z), lo, hi);
    return PLAN_THREADS - 1 - min(max(hi - lo, 0), PLAN_THREADS - 1);
  };
  bins[threadIdx.x] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < np; i += PLAN_THREADS) atomicAdd(&bins[cost_bin(v.pre[i])], 1);
  __syncthreads();
  int nbin_total;
  const int start = plan_scan(bins[threadIdx.x], ws, nbin_total);
  __syncthreads();
  bins[threadIdx.x] = start;
  __syncthreads();
  for (int i = threadIdx.x; i < np; i += PLAN_THREADS) {
    const int4 it = v.pre[i];
    v.pre_sorted[atomicAdd(&bins[cost_bin(it)], 1)] = it;
  }
  if (threadIdx.x == 0) {
    const bool bad = s_bad != 0;
    v.header[0] = bad ? 0 : min(s_cpre, v.max_pre);
    v.header[1] = bad ? 0 : min(s_cdec, v.max_dec);
    v.header[2] = split;
    v.header[3] = s_bad;
    v.header[4] = group && !bad ? S * kv_heads : 0;   // per-CTA decode: its pair count
    if (bad) hy_flag(err, s_bad);
  }
}

// ------------------------------------------------------------------ decode item
struct MainArgs {
  const __nv_bfloat16* cache;   // the whole cache: tensor-map row r starts at cache + 128 r
  const __nv_bfloat16* q;
  __nv_bfloat16* out;
  int q_heads, kv_heads;
  int layer;              // layer index (selects the work counters)
  int layer_row_base;     // first tensor-map row of this layer
  int oob_row;            // a row past the end of the map: loads there read zeros
  int num_blocks;
  const int32_t* block_tables;
  int bt_pitch;
  const int32_t* seq_bt_row;
  const int32_t* cu_q;
  const int32_t* seq_lens_k;
  float scale_log2;
  int32_t* err;
  int early;              // HY_ATTN_EARLY: start decode K/V loads before the grid wait
};

// Tensor-map row of (block, K or V, kv head).
HY_DEVICE int kv_row(const MainArgs& a, int blk, int kv, int g) {
  return a.layer_row_base + ((blk * 2 + kv) * a.kv_heads + g) * HY_BLOCK;
}

// Issue the K and V tiles of physical block blk (KV head g) into ring stage s
// (one lane).
HY_DEVICE void dec_issue(const CUtensorMap* tiles, const MainArgs& a, uint8_t* ring,
                         uint64_t* bars, int s, int blk, int g) {
  int rk, rv;
  if (blk < 0 || blk >= a.num_blocks) {
    hy_flag(a.err, HY_ERR_BOUNDS);
    rk = rv = a.oob_row;
  } else {
    rk = kv_row(a, blk, 0, g);
    rv = kv_row(a, blk, 1, g);
  }
  uint8_t* st = ring + s * DEC_TILE_BYTES;
  fence_proxy_async();
  mbar_arrive_expect_tx(&bars[s], DEC_TILE_BYTES);
  tma_load_3d(st, tiles, 0, rk, 0, &bars[s]);            // K: both halves, one box
  tma_load_3d(st + 4096, tiles, 0, rv, 0, &bars[s]);     // V
}

// A decode item's plan record (item, sequence fields) and its cached block ids.
struct DecRec {
  int4 it, info, c0, c1;
};

HY_DEVICE void dec_load_rec(const PlanView& v, int item, uint64_t keep, DecRec& r) {
  r.it = ld_keep(&v.dec[2 * item], keep);
  r.info = ld_keep(&v.dec[2 * item + 1], keep);
  r.c0 = ld_keep(&v.dec_ids[2 * item], keep);
  r.c1 = ld_keep(&v.dec_ids[2 * item + 1], keep);
}

// Before the grid wait (HY_ATTN_EARLY): load the item's record and, if its
// block ids are cached, start the ring's first loads of blocks that hold no
// key of the step's query token (the kernel just before wrote only that key's
// K/V).  Returns the stages issued.
HY_DEVICE uint32_t decode_item_early(const CUtensorMap* tiles, const MainArgs& a,
                                     const PlanView& v, int item, uint8_t* ring, uint64_t* bars,
                                     DecRec& r) {
  dec_load_rec(v, item, l2_keep_policy(), r);
  if (r.c0.x < 0) return 0u;                    // ids not cached yet (warp-uniform)
  const int g = r.it.y, b0 = r.it.z, n = r.it.w - r.it.z;
  const int newest = (r.info.y - 1) / HY_BLOCK;   // the block of the query token's key
  const int ids[DEC_STAGES] = {r.c0.y, r.c0.z, r.c0.w};
  uint32_t mask = 0u;
#pragma unroll
  for (int s = 0; s < DEC_STAGES; ++s)
    if (s < n && b0 + s < newest) mask |= 1u << s;
  if ((threadIdx.x & 31) == 0) {
#pragma unroll
    for (int s = 0; s < DEC_STAGES; ++s)
      if ((mask >> s) & 1u) dec_issue(tiles, a, ring, bars, s, ids[s], g);
  }
  return mask;
}

// The attention of one decode item over its block range: on return lane
// (r, c) = (lane / 4, lane % 4) with r < 4 holds query head 4g + r's unnormalised
// output in o[j][0..1] (dims 8j + 2c, 8j + 2c + 1), and every lane of row r its
// running max m (scaled log2 units) and sum l.  Returns false if a wait ran out.
struct DecodeItemInfo {
  int seq, g, tok, ns, first;
};

// have_pre: pre is the record decode_item_early loaded, which issued the
// stages in pre_issued.
__device__ bool decode_item_core(const CUtensorMap* tiles, const MainArgs& a, const PlanView& v,
                                 int item, uint8_t* ring, uint64_t* bars, uint32_t& phase,
                                 float (&o)[16][4], float& m, float& l, DecodeItemInfo& di,
                                 DecRec pre, bool have_pre, uint32_t pre_issued) {
  const int lane = threadIdx.x & 31;
  const uint64_t keep = l2_keep_policy();
  DecRec rec = pre;
  if (!have_pre) dec_load_rec(v, item, keep, rec);   // one 32-byte record + the id cache
  const int4 it = rec.it, info = rec.info, c0 = rec.c0, c1 = rec.c1;
  const int seq = it.x, g = it.y, b0 = it.z, b1 = it.w;
  const int tok = info.x, kv_len = info.y;
  di.seq = seq; di.g = g; di.tok = tok; di.ns = info.z; di.first = info.w;
  const int n = b1 - b0;
  auto issue = [&](int s, int blk) { dec_issue(tiles, a, ring, bars, s, blk, g); };

  // The block-table row and the ids of the ring's first blocks and the one
  // after: cached with the item by the plan's first attention launch (block
  // tables do not change while a plan is in use), else loaded (one id per
  // lane, together) and cached for the later layers.
  static_assert(DEC_STAGES == 3, "the item cache holds DEC_STAGES + 1 = 4 block ids");
  int bt_row;
  int first_ids[DEC_STAGES + 1];
  if (c0.x >= 0) {                                // warp-uniform
    bt_row = c0.x;
    first_ids[0] = c0.y; first_ids[1] = c0.z; first_ids[2] = c0.w; first_ids[3] = c1.x;
  } else {
    bt_row = a.seq_bt_row ? ld_keep(a.seq_bt_row + seq, keep) : seq;
    const int32_t* bt0 = a.block_tables + (size_t)bt_row * a.bt_pitch;
    const int idl = (lane <= DEC_STAGES && lane < n) ? ld_keep(bt0 + b0 + lane, keep) : 0;
#pragma unroll
    for (int s = 0; s <= DEC_STAGES; ++s) first_ids[s] = __shfl_sync(0xffffffffu, idl, s);
    if (lane == 0) {
      v.dec_ids[2 * item + 1] = make_int4(first_ids[3], 0, 0, 0);
      v.dec_ids[2 * item] = make_int4(bt_row, first_ids[0], first_ids[1], first_ids[2]);
    }
  }
  const int32_t* bt = a.block_tables + (size_t)bt_row * a.bt_pitch;
  if (lane == 0) {
#pragma unroll
    for (int s = 0; s < DEC_STAGES; ++s)
      if (s < n && !((pre_issued >> s) & 1u)) issue(s, first_ids[s]);
  }
  int next_id = (lane == 0 && DEC_STAGES < n) ? first_ids[DEC_STAGES] : 0;

  // Query fragments: rows 0..3 are the group's 4 heads; rows 4..15 are zero.
  const int r = lane >> 2, c = 2 * (lane & 3);
  uint32_t qa[8][2];
  {
    const __nv_bfloat16* qp = a.q + ((size_t)tok * a.q_heads + g * HY_GROUP) * HY_HEAD_DIM;
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      if (r < HY_GROUP) {
        qa[kk][0] = *reinterpret_cast<const uint32_t*>(qp + r * HY_HEAD_DIM + 16 * kk + c);
        qa[kk][1] = *reinterpret_cast<const uint32_t*>(qp + r * HY_HEAD_DIM + 16 * kk + c + 8);
      } else {
        qa[kk][0] = qa[kk][1] = 0u;
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  m = NEG_INF;
  l = 0.f;

  // Per-lane ldmatrix coordinates.
  const int mi = lane >> 3, ri = lane & 7;
  const int k_key = ri + 8 * (mi >> 1), k_dsub = 8 * (mi & 1);   // K: non-transposed
  const int v_key = ri + 8 * (mi & 1), v_dsub = 8 * (mi >> 1);   // V: transposed

  bool ok = true;
  for (int i = 0; i < n; ++i) {
    const int s = i % DEC_STAGES;
    const bool w_ok = mbar_wait(&bars[s], (phase >> s) & 1u, a.err);
    if (__any_sync(0xffffffffu, !w_ok)) { ok = false; break; }
    phase ^= (1u << s);
    const uint32_t kb = smem_u32(ring + s * DEC_TILE_BYTES);
    const uint32_t vb = kb + 4096;

    float sacc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const int d = 16 * kk + k_dsub;
      uint32_t b[4];
      ldmatrix_x4(b, kb + (d >> 6) * 2048 + swz128(k_key, d & 63));
      const uint32_t af[4] = {qa[kk][0], 0u, qa[kk][1], 0u};
      mma_bf16_16816(sacc[0], af, b[0], b[1]);
      mma_bf16_16816(sacc[1], af, b[2], b[3]);
    }
    const int kbase = (b0 + i) * HY_BLOCK;
    const bool tail = kbase + HY_BLOCK > kv_len;            // only the last block is partial
    float p[2][2];
    float mx = NEG_INF;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        float x = sacc[nt][e] * a.scale_log2;
        if (tail && kbase + nt * 8 + c + e >= kv_len) x = NEG_INF;
        p[nt][e] = x;
        mx = fmaxf(mx, x);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const bool grow = mx > m + RESCALE_LOG2;                // true on the first block
    if (__any_sync(0xffffffffu, grow)) {
      const float m_new = grow ? mx : m;
      const float alpha = exp2f(m - m_new);                 // 0 when m was -inf
      l *= alpha;
#pragma unroll
      for (int j = 0; j < 16; ++j) { o[j][0] *= alpha; o[j][1] *= alpha; }
      m = m_new;
    }
    const float m_use = (m == NEG_INF) ? 0.f : m;
#pragma unroll
    for (int nt = 0; nt < 2; ++nt)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        p[nt][e] = exp2f(p[nt][e] - m_use);
        l += p[nt][e];
      }
    const uint32_t pa[4] = {pack_bf16(p[0][0], p[0][1]), 0u, pack_bf16(p[1][0], p[1][1]), 0u};
#pragma unroll
    for (int j2 = 0; j2 < 8; ++j2) {
      const int d = 16 * j2 + v_dsub;
      uint32_t b[4];
      ldmatrix_x4_trans(b, vb + (d >> 6) * 2048 + swz128(v_key, d & 63));
      mma_bf16_16816(o[2 * j2], pa, b[0], b[1]);
      mma_bf16_16816(o[2 * j2 + 1], pa, b[2], b[3]);
    }
    __syncwarp();
    if (i + DEC_STAGES < n && lane == 0) {
      issue(s, next_id);
      next_id = (i + DEC_STAGES + 1 < n) ? ld_keep(bt + b0 + i + DEC_STAGES + 1, keep) : 0;
    }
  }
  if (!ok) {
    // Let the copies still in flight land before the CTA can exit.
    for (int s = 0; s < DEC_STAGES; ++s) mbar_wait(&bars[s], (phase >> s) & 1u, nullptr);
    return false;
  }
  l += __shfl_xor_sync(0xffffffffu, l, 1);
  l += __shfl_xor_sync(0xffffffffu, l, 2);
  return true;
}

// One decode item whose split-K partners may run on other SMs: a sole item
// writes its output; otherwise the partial goes to the workspace and the last
// of the (seq, head)'s items to finish (an atomic count) merges all of them.
__device__ bool decode_item(const CUtensorMap* tiles, const MainArgs& a, const PlanView& v,
                            int item, uint8_t* ring, uint64_t* bars, uint32_t& phase,
                            DecRec pre, bool have_pre, uint32_t pre_issued) {
  const int lane = threadIdx.x & 31;
  float o[16][4];
  float m, l;
  DecodeItemInfo di;
  if (!decode_item_core(tiles, a, v, item, ring, bars, phase, o, m, l, di, pre, have_pre,
                        pre_issued))
    return false;
  const int seq = di.seq, g = di.g, tok = di.tok, ns = di.ns, first = di.first;
  const int r = lane >> 2, c = 2 * (lane & 3);
  if (r < HY_GROUP) {
    if (ns <= 1) {
      const float inv = 1.f / l;
      __nv_bfloat16* op = a.out + ((size_t)tok * a.q_heads + g * HY_GROUP + r) * HY_HEAD_DIM;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        *reinterpret_cast<uint32_t*>(op + 8 * j + c) = pack_bf16(o[j][0] * inv, o[j][1] * inv);
    } else {
      float* po = v.part_o + ((size_t)item * HY_GROUP + r) * HY_HEAD_DIM;
#pragma unroll
      for (int j = 0; j < 16; ++j)
        *reinterpret_cast<float2*>(po + 8 * j + c) = make_float2(o[j][0], o[j][1]);
      if ((lane & 3) == 0) v.part_ml[(size_t)item * HY_GROUP + r] = make_float2(m, l);
    }
  }
  if (ns > 1) {
    // The last of the sequence's split items to finish merges all partials.
    __threadfence();
    __syncwarp();
    int last = 0;
    if (lane == 0) last = atomicAdd(&v.counters[seq * a.kv_heads + g], 1) == ns - 1;
    if (__shfl_sync(0xffffffffu, last, 0)) {
      __threadfence();
      // Other SMs wrote the partials during this launch, so they are read
      // through L2: MERGE_CHUNK splits at a time are staged into this warp's
      // idle TMA ring by cp.async (one L2 round trip per chunk).  Lane
      // (s, h) = (lane / 4, lane % 4) then weighs split s of head h, and every
      // lane accumulates d = 4*lane..4*lane+3 of all 4 heads from shared memory.
      float M[HY_GROUP], L[HY_GROUP];
      float4 acc[HY_GROUP];
#pragma unroll
      for (int rr = 0; rr < HY_GROUP; ++rr) {
        M[rr] = NEG_INF;
        L[rr] = 0.f;
        acc[rr] = make_float4(0.f, 0.f, 0.f, 0.f);
      }
      const float* s_o = reinterpret_cast<const float*>(ring);
      const float2* s_ml = reinterpret_cast<const float2*>(ring + MERGE_O_BYTES);
      float* s_w = reinterpret_cast<float*>(ring + MERGE_O_BYTES + MERGE_ML_BYTES);
      for (int s0 = 0; s0 < ns; s0 += MERGE_CHUNK) {
        const int nsl = min(MERGE_CHUNK, ns - s0);
        const uint8_t* g_o =
            reinterpret_cast<const uint8_t*>(v.part_o + (size_t)(first + s0) * HY_GROUP * HY_HEAD_DIM);
        const uint8_t* g_ml =
            reinterpret_cast<const uint8_t*>(v.part_ml + (size_t)(first + s0) * HY_GROUP);
        const int bytes_o = nsl * HY_GROUP * HY_HEAD_DIM * (int)sizeof(float);
        const int bytes_ml = nsl * HY_GROUP * (int)sizeof(float2);
        __syncwarp();                                   // the previous chunk is read
        for (int off = lane * 16; off < bytes_o; off += 512) cp_async16(ring + off, g_o + off);
        for (int off = lane * 16; off < bytes_ml; off += 512)
          cp_async16(ring + MERGE_O_BYTES + off, g_ml + off);
        cp_async_wait_all();
        __syncwarp();
        const int sl = lane >> 2, h = lane & 3;
        const float2 ml = sl < nsl ? s_ml[sl * HY_GROUP + h] : make_float2(NEG_INF, 0.f);
        float mx = ml.x;                                // max over the chunk's splits of head h
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 4));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 8));
        mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 16));
        float m_old = M[0];
#pragma unroll
        for (int rr = 1; rr < HY_GROUP; ++rr) if (h == rr) m_old = M[rr];
        const float m_new = fmaxf(m_old, mx);
        const float w = sl < nsl ? exp2f(ml.x - m_new) : 0.f;
        float lw = w * ml.y;                            // sum over the chunk of w * l, head h
        lw += __shfl_xor_sync(0xffffffffu, lw, 4);
        lw += __shfl_xor_sync(0xffffffffu, lw, 8);
        lw += __shfl_xor_sync(0xffffffffu, lw, 16);
        s_w[lane] = w;                                  // weight of split sl, head h
        const float sc = exp2f(m_old - m_new);          // 0 when m_old was -inf
#pragma unroll
        for (int rr = 0; rr < HY_GROUP; ++rr) {
          const float scr = __shfl_sync(0xffffffffu, sc, rr);
          M[rr] = __shfl_sync(0xffffffffu, m_new, rr);
          L[rr] = L[rr] * scr + __shfl_sync(0xffffffffu, lw, rr);
          acc[rr].x *= scr; acc[rr].y *= scr; acc[rr].z *= scr; acc[rr].w *= scr;
        }
        __syncwarp();
#pragma unroll 1
        for (int k = 0; k < nsl; ++k) {
#pragma unroll
          for (int rr = 0; rr < HY_GROUP; ++rr) {
            const float wk = s_w[k * HY_GROUP + rr];
            const float4 po =
                *reinterpret_cast<const float4*>(s_o + (k * HY_GROUP + rr) * HY_HEAD_DIM + 4 * lane);
            acc[rr].x += wk * po.x; acc[rr].y += wk * po.y;
            acc[rr].z += wk * po.z; acc[rr].w += wk * po.w;
          }
        }
      }
#pragma unroll
      for (int rr = 0; rr < HY_GROUP; ++rr) {
        const float inv = 1.f / L[rr];
        __nv_bfloat16* op =
            a.out + ((size_t)tok * a.q_heads + g * HY_GROUP + rr) * HY_HEAD_DIM + 4 * lane;
        uint2 pk;
        pk.x = pack_bf16(acc[rr].x * inv, acc[rr].y * inv);
        pk.y = pack_bf16(acc[rr].z * inv, acc[rr].w * inv);
        *reinterpret_cast<uint2*>(op) = pk;
      }
      if (lane == 0) v.counters[seq * a.kv_heads + g] = 0;   // ready for the next layer
    }
  }
  return true;
}

// Per-CTA decode of one (sequence, KV head) pair: warp w < ns runs the pair's
// item w; the partials meet in shared memory (each warp's own TMA ring, idle
// once its item is done) and the CTA's decode warps merge them, one output
// pair of head dimensions per thread.  No workspace round trip, fence or
// atomic count.  All ATT_WARPS decode warps of the CTA call this.
__device__ bool decode_pair_cta(const CUtensorMap* tiles, const MainArgs& a, const PlanView& v,
                                int pair, uint8_t* payload, uint64_t (*bars)[DEC_STAGES],
                                uint32_t& phase, DecRec pre, bool have_pre,
                                uint32_t pre_issued) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int seq = pair / a.kv_heads, g = pair - seq * a.kv_heads;
  const int2 si = v.seqinfo[seq];               // first decode item of the sequence, items per head
  const int ns = si.y, first = si.x + g * ns;
  uint8_t* ring = payload + warp * DEC_WARP_BYTES;
  float* part_o = reinterpret_cast<float*>(ring);                        // [4][128]
  float2* part_ml = reinterpret_cast<float2*>(ring + HY_GROUP * HY_HEAD_DIM * 4);
  bool ok = true;
  if (warp < ns) {
    float o[16][4];
    float m, l;
    DecodeItemInfo di;
    ok = decode_item_core(tiles, a, v, first + warp, ring, bars[warp], phase, o, m, l, di, pre,
                          have_pre, pre_issued);
    const int r = lane >> 2, c = 2 * (lane & 3);
    if (ok && r < HY_GROUP) {
      if (ns == 1) {                            // the only split: final output
        const float inv = 1.f / l;
        __nv_bfloat16* op =
            a.out + ((size_t)di.tok * a.q_heads + g * HY_GROUP + r) * HY_HEAD_DIM;
#pragma unroll
        for (int j = 0; j < 16; ++j)
          *reinterpret_cast<uint32_t*>(op + 8 * j + c) = pack_bf16(o[j][0] * inv, o[j][1] * inv);
      } else {
#pragma unroll
        for (int j = 0; j < 16; ++j)
          *reinterpret_cast<float2*>(part_o + r * HY_HEAD_DIM + 8 * j + c) =
              make_float2(o[j][0], o[j][1]);
        if ((lane & 3) == 0) part_ml[r] = make_float2(m, l);
      }
    }
  }
  if (named_sync_or(MERGE_BAR, ATT_WARPS * 32, !ok)) return false;
  if (ns <= 1) return true;
  const int t = threadIdx.x, r = t >> 6, d = 2 * (t & 63);
  const int tok = v.dec[2 * first + 1].x;
  float M = NEG_INF;
  for (int w = 0; w < ns; ++w)
    M = fmaxf(M, reinterpret_cast<const float2*>(payload + w * DEC_WARP_BYTES +
                                                 HY_GROUP * HY_HEAD_DIM * 4)[r].x);
  float L = 0.f, a0 = 0.f, a1 = 0.f;
  for (int w = 0; w < ns; ++w) {
    const uint8_t* rw = payload + w * DEC_WARP_BYTES;
    const float2 ml = reinterpret_cast<const float2*>(rw + HY_GROUP * HY_HEAD_DIM * 4)[r];
    const float2 po = *reinterpret_cast<const float2*>(
        reinterpret_cast<const float*>(rw) + r * HY_HEAD_DIM + d);
    const float wt = ex2_ftz(ml.x - M);
    L = fmaf(wt, ml.y, L);
    a0 = fmaf(wt, po.x, a0);
    a1 = fmaf(wt, po.y, a1);
  }
  const float inv = 1.f / L;
  *reinterpret_cast<uint32_t*>(a.out + ((size_t)tok * a.q_heads + g * HY_GROUP + r) * HY_HEAD_DIM +
                               d) = pack_bf16(a0 * inv, a1 * inv);
  return true;
}

// The end of one piece of a split prefill item, run by all ATT_WARPS * 32
// softmax threads (thread rr holds row rr of the item's 256 rows): the row's
// unnormalised O (TMEM column base tO) and (m, l) go to the piece's partial
// slot; the piece that finishes last (counted at the item's first slot)
// merges every piece's partials into the output row op (nullptr: a padding row)
// and resets the count.  Piece s weighs 2^(m_s - M), M the largest m_s.
// Returns whether every thread's waits succeeded.
__device__ bool prefill_piece_finish(const PlanView& v, int w, int rr, uint32_t tO, float m,
                                     float l, bool ok, __nv_bfloat16* op, Shared& sh) {
  const int ns = pre_code_pieces(w), sp = pre_code_piece(w), slot = pre_code_slot(w);
  const bool all_ok = !named_sync_or(MERGE_BAR, ATT_WARPS * 32, !ok);
  if (all_ok) {
    float4* po = v.pre_part_o + (size_t)(slot + sp) * PRE_PART_F4 + rr;
#pragma unroll 1
    for (int cc = 0; cc < 4; ++cc) {
      float o[32];
      tmem_ld32(tO + 32 * cc, o);
      tmem_wait_ld();
#pragma unroll
      for (int k = 0; k < 8; ++k)
        __stcg(po + (cc * 8 + k) * 256,
               make_float4(o[4 * k], o[4 * k + 1], o[4 * k + 2], o[4 * k + 3]));
    }
    __stcg(v.pre_part_ml + (size_t)(slot + sp) * 256 + rr, make_float2(m, l));
    __threadfence();                            // this row's partial, before the count
  }
  named_sync(MERGE_BAR, ATT_WARPS * 32);
  if (threadIdx.x == 0) sh.pre_last = all_ok && atomicAdd(&v.pre_ctr[slot], 1) == ns - 1;
  named_sync(MERGE_BAR, ATT_WARPS * 32);
  if (!sh.pre_last) return all_ok;
  __threadfence();                              // the other pieces' partials, after the count
  const float2* ml = v.pre_part_ml + (size_t)slot * 256 + rr;
  float M = NEG_INF;
#pragma unroll 4
  for (int s = 0; s < ns; ++s) M = fmaxf(M, __ldcg(ml + s * 256).x);
  float L = 0.f;
#pragma unroll 4
  for (int s = 0; s < ns; ++s) {
    const float2 e = __ldcg(ml + s * 256);
    L += e.y * (M == NEG_INF ? 0.f : ex2_ftz(e.x - M));
  }
  const float inv = 1.f / L;
#pragma unroll 1
  for (int cc = 0; cc < 4; ++cc) {
    float acc[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) acc[k] = 0.f;
    // two pieces per round: their 16 loads are in flight together
#pragma unroll 1
    for (int s = 0; s < ns; s += 2) {
      const int s1 = min(s + 1, ns - 1);
      const float w0 = M == NEG_INF ? 0.f : ex2_ftz(__ldcg(ml + s * 256).x - M);
      const float w1 = (s1 == s || M == NEG_INF) ? 0.f : ex2_ftz(__ldcg(ml + s1 * 256).x - M);
      const float4* p0 = v.pre_part_o + (size_t)(slot + s) * PRE_PART_F4 + cc * 8 * 256 + rr;
      const float4* p1 = v.pre_part_o + (size_t)(slot + s1) * PRE_PART_F4 + cc * 8 * 256 + rr;
      float4 f0[8], f1[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        f0[k] = __ldcg(p0 + k * 256);
        f1[k] = __ldcg(p1 + k * 256);
      }
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        acc[4 * k] += w0 * f0[k].x + w1 * f1[k].x;
        acc[4 * k + 1] += w0 * f0[k].y + w1 * f1[k].y;
        acc[4 * k + 2] += w0 * f0[k].z + w1 * f1[k].z;
        acc[4 * k + 3] += w0 * f0[k].w + w1 * f1[k].w;
      }
    }
    if (op) {
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        uint4 pk4;
        pk4.x = pack_bf16(acc[8 * q4 + 0] * inv, acc[8 * q4 + 1] * inv);
        pk4.y = pack_bf16(acc[8 * q4 + 2] * inv, acc[8 * q4 + 3] * inv);
        pk4.z = pack_bf16(acc[8 * q4 + 4] * inv, acc[8 * q4 + 5] * inv);
        pk4.w = pack_bf16(acc[8 * q4 + 6] * inv, acc[8 * q4 + 7] * inv);
        *reinterpret_cast<uint4*>(op + 32 * cc + 8 * q4) = pk4;
      }
    }
  }
  if (threadIdx.x == 0) v.pre_ctr[slot] = 0;   // for the next launch on this plan
  return all_ok;
}

// ------------------------------------------------------------------ prefill item
// Geometry of the prefill item (or piece) at run-order index `item`.
struct PreItem {
  int seq, g, t0, row0, nrows, prefix, kv_len, tlo, thi, nblk, w;
};
HY_DEVICE PreItem pre_item_geom(const MainArgs& a, const PlanView& v, int item) {
  const int4 it = v.pre_sorted[item];
  PreItem p;
  p.seq = it.x;
  p.g = it.y;
  p.t0 = it.z;
  p.w = it.w;
  p.row0 = a.cu_q[p.seq];
  const int q_len = a.cu_q[p.seq + 1] - p.row0;
  p.kv_len = a.seq_lens_k[p.seq];
  p.prefix = p.kv_len - q_len;
  p.nrows = min(PRE_QROWS, q_len - p.t0);
  const int kv_end = p.prefix + p.t0 + p.nrows;
  pre_piece_range(p.w, (kv_end + TC_KEYS - 1) / TC_KEYS, p.tlo, p.thi);
  p.nblk = (kv_end + HY_BLOCK - 1) / HY_BLOCK;
  return p;
}
HY_DEVICE const int32_t* pre_block_table(const MainArgs& a, int seq) {
  const int row = a.seq_bt_row ? a.seq_bt_row[seq] : seq;
  return a.block_tables + (size_t)row * a.bt_pitch;
}
// Q of item p: one 32 KB box per sub-tile X (64 columns x 64 tokens x query
// heads 4g + 2X, 4g + 2X + 1 x both column halves), landing as the K-major
// operand [half][128 rows][64] with row = 64 (head - 4g - 2X) + token, counted
// on tc_qfull.  Rows past the chunk read later tokens (or zeros past the last
// token): their scores are computed but never stored.  One thread.
HY_DEVICE void pre_issue_q(const CUtensorMap* qmap, const PreItem& p, uint8_t* payload,
                           Shared& sh) {
  mbar_arrive_expect_tx(&sh.tc_qfull, 2 * TC_Q_BYTES);
  for (int X = 0; X < 2; ++X)
    tma_load_4d(payload + X * TC_Q_BYTES, qmap, 0, p.row0 + p.t0, p.g * HY_GROUP + 2 * X, 0,
                &sh.tc_qfull);
}
// One load warp's (lw) share of key tile kt of item p, ring counter c: lane 0
// waits for the slot and posts the warp's byte count; lanes 0-3 issue one 4 KB
// box each (K of blocks 2 lw, 2 lw + 1, then their V; `id` is the lane's block
// id).  Returns false (warp-uniform) if the wait ran out.
HY_DEVICE bool pre_issue_tile(const CUtensorMap* kgroups, const CUtensorMap* tiles,
                              const MainArgs& a, int g, int lw, int lane, uint32_t c, int id,
                              uint8_t* payload, Shared& sh) {
  const uint32_t slot = c % TC_NS, use = c / TC_NS;
  bool w_ok = true;
  if (lane == 0) w_ok = mbar_wait(&sh.tc_free[slot], (use & 1) ^ 1, a.err);
  if (!__shfl_sync(0xffffffffu, w_ok ? 1 : 0, 0)) return false;
  uint64_t* full = &sh.tc_full[slot];
  if (lane == 0) mbar_arrive_expect_tx(full, TC_KV_BYTES);
  if (lane < 4) {
    const int kv = (lane >> 1) & 1, jb = 2 * lw + (lane & 1);
    int r = a.oob_row;                          // past the end: zero fill
    if (id >= a.num_blocks) hy_flag(a.err, HY_ERR_BOUNDS);
    else if (id >= 0) r = kv_row(a, id, kv, g);
    if (kv)
      tma_load_3d(payload + TC_V_OFF + slot * TC_KV_BYTES + jb * 4096, tiles, 0, r, 0, full);
    else
      tma_load_4d(payload + TC_K_OFF + slot * TC_KV_BYTES + jb * 4096, kgroups, 0, r, 0, 0,
                  full);
  }
  return true;
}

// tcgen05, warp-specialised.  Item = (seq, kv head g, 64-token tile t0): two
// M=128 sub-tiles X of the same tokens (query heads 4g+2X, 4g+2X+1), which see
// the same keys and masks, so each 64-key K/V tile is loaded once for both.
//   warps 0-3 / 4-7  softmax of sub-tile 0 / 1: thread = row = TMEM lane, so a
//                    row's max and sum stay in one thread.  Per key tile: S_X[b]
//                    from TMEM, causal mask, online softmax with lazy rescaling
//                    of O_X, P_X (bf16 pairs) written back over S_X[b];
//   warp 8 / 10,     one per sub-tile: issues S_X(t) = Q_X K_t^T into buffer
//   lane 0           b = t % 2, then O_X += P_X(t-1) V_{t-1} (A operand read from
//                    TMEM), each followed by tcgen05.commit to the barrier its
//                    consumer waits on;
//   warps 9, 11      warp 9 first loads the item's Q (one 32 KB TMA box per
//                    sub-tile, waited for by the MMA warps on tc_qfull, once
//                    per item); both load K_t and V_t (4 TMA boxes each: one
//                    whole 4 KB block tile per box) into ring slot c % TC_NS
//                    once the MMAs of the slot's previous use are done, each
//                    warp two of the tile's four blocks.
// The item may cover a key-tile range [tlo, thi) only (a piece of a cut item:
// see prefill_piece_finish); the key tiles below are those of the range.
// Once their own loads are issued, the load warps take the CTA's next item
// from the counter and issue its Q (after the S MMAs of this item's last tile)
// and its first TC_NS key tiles (as this item's P V MMAs free the slots), so
// that the next item's first MMA needs no load latency after this item's
// epilogue; the next call skips what was issued (pf).
// With two S buffers the MMA warp issues S(t+1) while the softmax works on
// S(t), so the softmax never waits for its scores once the pipeline is full.
// S(t) may overwrite buffer b only after PV(t-2) has read P(t-2) from it: the
// issuing thread issued PV(t-2) before S(t), and tcgen05.mma operations of one
// thread execute in issue order (as the K-step accumulation into one D relies
// on).  The softmax writes P(t) over S(t) after reading S(t), which completed
// after PV(t-2); it need not wait for PV(t-1) (the other buffer) except to
// rescale O.
// c = c0 + t counts key tiles over all items of the launch; each barrier
// completes exactly once per tile (odone), per use of its buffer (sfull, pfull:
// every second tile) or per use of its slot (ring barriers), and no role can
// run a full phase ahead of the role that waits on it, so a wait is always on
// the current or the previous phase (the load warps, which can get ahead of
// the S MMAs of a short item, wait for its S phases in order).  Returns false if a wait ran out; the
// roles then drain their own asynchronous work before the item ends.
__device__ bool prefill_item_tc(const CUtensorMap* kgroups, const CUtensorMap* tiles,
                                const CUtensorMap* qmap, const MainArgs& a, const PlanView& v,
                                int item, uint8_t* payload, Shared& sh, uint32_t tmem,
                                uint32_t& ctr, uint32_t qpar, int pf, int* next_ctr,
                                int n_pre) {
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const PreItem P = pre_item_geom(a, v, item);
  const int seq = P.seq, g = P.g, t0 = P.t0, row0 = P.row0, nrows = P.nrows;
  const int kv_len = P.kv_len, prefix = P.prefix, tlo = P.tlo;
  const int ntiles = P.thi - P.tlo;             // key tiles of this item (or piece)
  const uint32_t sbase = smem_u32(payload);
  const uint32_t c0 = ctr;
  ctr += ntiles;
  bool ok = true;

  if (warp == TC_LOAD_WARP || warp == TC_LOAD_WARP2) {
    // Two load warps, lw = 0, 1, each for blocks 2 lw and 2 lw + 1 of every key
    // tile, one wait and one arm per tile (a load warp's wait, arm and first
    // box are serial round trips of ~150-270 cycles each, so the tile's supply
    // rate is set by how many of them a warp makes per tile).  pf >= 0: the
    // previous item's load warps already issued this item's Q and its first pf
    // key tiles; -1: Q first.
    const int lw = warp == TC_LOAD_WARP2;
    if (pf < 0 && lw == 0 && lane == 0) pre_issue_q(qmap, P, payload, sh);
    const int first = max(pf, 0);
    const int32_t* bt = pre_block_table(a, seq);
    int ids = -1;                               // lane i: block 32 (kt / 8) + i of the sequence
    int issued = first;                         // tiles whose loads were issued
    for (int t = first; t < ntiles && ok; ++t) {
      const int kt = tlo + t;                   // key tile of the sequence
      if (t == first || (kt & 7) == 0) {
        const int b = 4 * (kt & ~7) + lane;
        ids = (b < P.nblk && b < a.bt_pitch) ? bt[b] : -1;
      }
      const int id = __shfl_sync(0xffffffffu, ids, (4 * kt + 2 * lw + (lane & 1)) & 31);
      if (!pre_issue_tile(kgroups, tiles, a, g, lw, lane, c0 + t, id, payload, sh)) {
        ok = false;
        break;
      }
      issued = t + 1;
    }
    if (!ok && lane == 0) {                     // loads still in flight must land first
      for (int t = max(0, issued - TC_NS); t < issued; ++t) {
        const uint32_t c = c0 + t;
        mbar_wait(&sh.tc_full[c % TC_NS], (c / TC_NS) & 1, nullptr);
      }
    }
    // Q has landed before the item ends (the next item's Q reuses the region)
    if (lw == 0 && lane == 0) mbar_wait(&sh.tc_qfull, qpar, nullptr);
    // The CTA's next item, taken now (this item's loads are all issued, a few
    // tiles before its end): its Q, once both sub-tiles' S of this item's last
    // tile completed, and its first key tiles, as this item's P V MMAs free
    // the ring slots, load while this item's last tiles and epilogue run.
    // Both load warps always reach the two barriers below.
    // Load warp 0 decides for both: it takes the item and waits for the S MMAs.
    named_sync(PRE_LOAD_BAR, 64);
    if (lw == 0 && lane == 0) {
      int nx = ok ? atomicAdd(next_ctr, 1) : 0x7fffffff;
      bool go = nx < n_pre;
      if (go) {
        // S of this item's last tile cl, after S of tile cl - 2 (the same S
        // buffer): waiting in order keeps each parity wait on the barrier's
        // current or previous phase (a short item whose tiles were all loaded
        // ahead gets here before its first S, two phases behind; phases before
        // cl - 2 completed before the load of tile cl was issued, or belong to
        // the previous item)
        const uint32_t cl = c0 + ntiles - 1;
        for (uint32_t c = ntiles >= 3 ? cl - 2 : cl; go && c <= cl; c += 2)
          go = mbar_wait(&sh.tc_sfull[0][c & 1], (c >> 1) & 1, a.err) &&
               mbar_wait(&sh.tc_sfull[1][c & 1], (c >> 1) & 1, a.err);
        if (!go) {                              // the CTA stops after this item
          ok = false;
          nx = 0x7fffffff;
        }
      }
      sh.pre_item = nx;
      sh.pre_prefetch = go ? 0 : -1;
    }
    named_sync(PRE_LOAD_BAR, 64);
    if (sh.pre_prefetch == 0) {
      const PreItem N = pre_item_geom(a, v, sh.pre_item);
      if (lw == 0 && lane == 0) pre_issue_q(qmap, N, payload, sh);
      const int32_t* nbt = pre_block_table(a, N.seq);
      const int want = min(TC_NS, N.thi - N.tlo);
      int pfn = 0;
      bool p_ok = true;
      for (; pfn < want; ++pfn) {
        const int b = 4 * (N.tlo + pfn) + 2 * lw + (lane & 1);
        const int id = (lane < 4 && b < N.nblk && b < a.bt_pitch) ? nbt[b] : -1;
        if (!pre_issue_tile(kgroups, tiles, a, N.g, lw, lane, c0 + ntiles + pfn, id, payload,
                            sh)) {
          p_ok = false;
          break;
        }
      }
      // both warps issued `want` tiles unless a wait ran out in either: then the
      // CTA stops after this item, and each warp's look-ahead loads land first
      const bool any_fail = named_sync_or(PRE_LOAD_BAR, 64, !p_ok);
      if (any_fail) {
        ok = false;
        if (lane == 0)
          for (int t = 0; t < pfn; ++t) {
            const uint32_t c = c0 + ntiles + t;
            mbar_wait(&sh.tc_full[c % TC_NS], (c / TC_NS) & 1, nullptr);
          }
        if (lw == 0 && lane == 0) mbar_wait(&sh.tc_qfull, qpar ^ 1u, nullptr);
      }
      if (lw == 0 && lane == 0) sh.pre_prefetch = any_fail ? -1 : want;
    }
  } else if (warp == TC_MMA_WARP || warp == TC_MMA_WARP1) {
    // one MMA warp per sub-tile X: its lane 0 issues S_X(t), then O_X += P_X(t-1)
    // V_{t-1}; both warps commit to the slot's free barrier after P V (count 2)
    const int X = warp == TC_MMA_WARP ? 0 : 1;
    if (lane == 0) {
      constexpr uint32_t ID_S = tc_idesc_bf16(128, TC_KEYS, false);
      constexpr uint32_t ID_O = tc_idesc_bf16(128, HY_HEAD_DIM, true);
      const uint64_t dQ = tc_desc_sw128(sbase + X * TC_Q_BYTES, 16, 1024);
      ok = mbar_wait(&sh.tc_qfull, qpar, a.err);                // Q_X landed
      tc_fence_after();
      for (int t = 0; t <= ntiles && ok; ++t) {
        if (t < ntiles) {                       // S_X(t) = Q_X K_t^T into buffer c % 2
          const uint32_t c = c0 + t, slot = c % TC_NS;
          ok = mbar_wait(&sh.tc_full[slot], (c / TC_NS) & 1, a.err);   // K and V landed
          if (!ok) break;
          tc_fence_after();
          // K slot: 8-key groups 2 KB apart (SBO), column half h at +1 KB
          const uint64_t dK = tc_desc_sw128(sbase + TC_K_OFF + slot * TC_KV_BYTES, 16, 2048);
#pragma unroll
          for (int kk = 0; kk < HY_HEAD_DIM / 16; ++kk)
            tc_mma_bf16(tmem + tm_s(X, c & 1),
                        dQ + (uint64_t)((((kk >> 2) * (TC_Q_BYTES / 2)) + (kk & 3) * 32) >> 4),
                        dK + (uint64_t)((((kk >> 2) * 1024) + (kk & 3) * 32) >> 4), ID_S,
                        kk > 0);
          tc_commit(&sh.tc_sfull[X][c & 1]);
        }
        if (t > 0) {                            // O_X += P_X(t-1) V_{t-1}
          const uint32_t c = c0 + t - 1, slot = c % TC_NS;
          // V_{t-1} landed with K_{t-1}, waited for before S(t-1)
          ok = mbar_wait(&sh.tc_pfull[X][c & 1], (c >> 1) & 1, a.err);
          if (!ok) break;
          tc_fence_after();
          // V slot: block kk's tile at kk x 4 KB, its column halves 2 KB apart (LBO),
          // 8-key groups 1 KB apart (SBO)
          const uint64_t dV = tc_desc_sw128(sbase + TC_V_OFF + slot * TC_KV_BYTES, 2048, 1024);
#pragma unroll
          for (int kk = 0; kk < TC_KEYS / 16; ++kk)
            tc_mma_bf16_ta(tmem + TM_O + 128 * X, tmem + tm_s(X, c & 1) + 8 * kk,
                           dV + (uint64_t)((kk * 4096) >> 4), ID_O, (t > 1 || kk > 0));
          tc_commit(&sh.tc_odone[X]);
          tc_commit(&sh.tc_free[slot]);
        }
      }
      if (!ok) {                                // let every issued MMA finish
        tc_commit(&sh.tc_drain[X]);
        mbar_wait(&sh.tc_drain[X], 0, nullptr);
      }
    }
    __syncwarp();
  } else {                                      // softmax warpgroups
    const int X = warp >> 2, r = (warp & 3) * 32 + lane, j = r & 63;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const uint32_t tO = tmem + lane_base + TM_O + 128 * X;
    const int lim = prefix + t0 + j;            // last key row r may see
    const float sl2 = a.scale_log2;
    float m = NEG_INF, l = 0.f;                 // m in scaled log2 units
    for (int t = 0; t < ntiles && ok; ++t) {
      const uint32_t c = c0 + t;
      const uint32_t tS = tmem + lane_base + tm_s(X, c & 1);
      // waits are made warp-uniform: tcgen05.ld/st below are warp-collective
      ok = __all_sync(0xffffffffu, mbar_wait(&sh.tc_sfull[X][c & 1], (c >> 1) & 1, a.err));
      if (!ok) break;
      tc_fence_after();
      float s[64];
      tmem_ld32(tS, *reinterpret_cast<float(*)[32]>(&s[0]));
      tmem_ld32(tS + 32, *reinterpret_cast<float(*)[32]>(&s[32]));
      tmem_wait_ld();
      const int kb = (tlo + t) * TC_KEYS;
      if (kb + TC_KEYS - 1 > prefix + t0) {     // the tile reaches the diagonal or the end
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (kb + i > lim || kb + i >= kv_len) s[i] = NEG_INF;
      }
      // row max and row sum as 8 independent chains (a 64-long chain of
      // dependent max or add instructions would expose its latency); the max
      // takes two new scores per three-input instruction
      float mxs[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) mxs[k] = fmax3f(s[k], s[8 + k], s[16 + k]);
#pragma unroll
      for (int i = 24; i < 56; i += 16)
#pragma unroll
        for (int k = 0; k < 8; ++k) mxs[k] = fmax3f(mxs[k], s[i + k], s[i + 8 + k]);
      float mx = fmax3f(fmax3f(mxs[0], mxs[1], mxs[2]), fmax3f(mxs[3], mxs[4], mxs[5]),
                        fmax3f(mxs[6], mxs[7], s[56]));
#pragma unroll
      for (int k = 57; k < 64; k += 2) mx = fmax3f(mx, s[k], k + 1 < 64 ? s[k + 1] : s[k]);
      mx *= sl2;
      const bool grow = mx > m + RESCALE_LOG2;
      if (__any_sync(0xffffffffu, grow)) {
        const float mnew = grow ? mx : m;
        const float alpha = ex2_ftz(m - mnew);  // 0 when m was -inf
        l *= alpha;
        m = mnew;
        if (t > 0) {                            // O holds tiles < t: wait for PV(t-1)
          ok = __all_sync(0xffffffffu, mbar_wait(&sh.tc_odone[X], (c & 1) ^ 1, a.err));
          tc_fence_after();
#pragma unroll 1
          for (int cc = 0; cc < 4; ++cc) {
            float o[32];
            tmem_ld32(tO + 32 * cc, o);
            tmem_wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const float2 r2 = __fmul2_rn(make_float2(o[2 * i], o[2 * i + 1]), make_float2(alpha, alpha));
              o[2 * i] = r2.x;
              o[2 * i + 1] = r2.y;
            }
            tmem_st32(tO + 32 * cc, o);
          }
          tmem_wait_st();
        }
      }
      const float mneg = (m == NEG_INF) ? 0.f : -m;
      const float2 sl2v = make_float2(sl2, sl2), mnegv = make_float2(mneg, mneg);
      uint32_t pk[32];
      // ls[k] sums elements 8 j + 2 k (.x) and 8 j + 2 k + 1 (.y): the 8
      // chains of scalar sums, two per packed add
      float2 ls[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                      make_float2(0.f, 0.f)};
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        // every EXP2_POLY_EVERY-th pair of weights on the FMA pipe, the rest on
        // the exp2 unit: the two units then share the tile's 64 exponentials
        const bool poly = EXP2_POLY_EVERY > 0 && (i % EXP2_POLY_EVERY) == EXP2_POLY_EVERY - 1;
        const float2 x = __ffma2_rn(make_float2(s[2 * i], s[2 * i + 1]), sl2v, mnegv);
        const float2 pp = poly ? exp2_poly2(x) : make_float2(ex2_ftz(x.x), ex2_ftz(x.y));
        const float p0 = pp.x, p1 = pp.y;
        ls[i & 3] = __fadd2_rn(ls[i & 3], make_float2(p0, p1));
        pk[i] = pack_bf16(p0, p1);
      }
      l += ((ls[0].x + ls[0].y) + (ls[1].x + ls[1].y)) + ((ls[2].x + ls[2].y) + (ls[3].x + ls[3].y));
      tmem_st32u(tS, pk);                       // P(t) over the first 32 columns of S(t)
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&sh.tc_pfull[X][c & 1]);
    }
    if (ok) {                                   // epilogue: O_X complete
      const uint32_t c = c0 + ntiles - 1;
      ok = __all_sync(0xffffffffu, mbar_wait(&sh.tc_odone[X], c & 1, a.err));
      tc_fence_after();
    }
    // tcgen05.ld is warp-collective: every lane loads, only real rows store
    const bool store = ok && j < nrows;
    __nv_bfloat16* op = a.out + ((size_t)(row0 + t0 + j) * a.q_heads + g * HY_GROUP + 2 * X +
                                 (r >> 6)) * HY_HEAD_DIM;
    if (P.w != 0) {                             // a piece: every softmax thread takes part
      ok = prefill_piece_finish(v, P.w, X * 128 + r, tO, m, l, ok, store ? op : nullptr, sh);
    } else if (ok) {                            // O_X / l -> out
      const float inv = 1.f / l;
#pragma unroll 1
      for (int cc = 0; cc < 4; ++cc) {
        float o[32];
        tmem_ld32(tO + 32 * cc, o);
        tmem_wait_ld();
        if (store) {
#pragma unroll
          for (int q4 = 0; q4 < 4; ++q4) {
            uint4 pk4;
            pk4.x = pack_bf16(o[8 * q4 + 0] * inv, o[8 * q4 + 1] * inv);
            pk4.y = pack_bf16(o[8 * q4 + 2] * inv, o[8 * q4 + 3] * inv);
            pk4.z = pack_bf16(o[8 * q4 + 4] * inv, o[8 * q4 + 5] * inv);
            pk4.w = pack_bf16(o[8 * q4 + 6] * inv, o[8 * q4 + 7] * inv);
            *reinterpret_cast<uint4*>(op + 32 * cc + 8 * q4) = pk4;
          }
        }
      }
    }
  }
  tc_fence_before();
  if (__syncthreads_or(!ok)) ok = false;
  return ok;
}

__global__ void __launch_bounds__(ATT_THREADS, 1) attn_main_kernel(
    const __grid_constant__ CUtensorMap kv_kgroups, const __grid_constant__ CUtensorMap kv_tiles,
    const __grid_constant__ CUtensorMap q_map, MainArgs a, PlanView v) {
  __shared__ Shared sh;
  extern __shared__ uint8_t dyn_smem[];
  uint8_t* payload = payload_base(dyn_smem);
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    prefetch_tmap(&kv_kgroups);
    prefetch_tmap(&kv_tiles);
    prefetch_tmap(&q_map);
    for (int w = 0; w < ATT_WARPS; ++w)
      for (int s = 0; s < DEC_STAGES; ++s) mbar_init(&sh.dec_bar[w][s], 1);
    for (int s = 0; s < TC_NS; ++s) {
      mbar_init(&sh.tc_full[s], 2);             // one arrival per load warp
      mbar_init(&sh.tc_free[s], 2);             // one commit per MMA warp
    }
    for (int x = 0; x < 2; ++x) {
      for (int b = 0; b < 2; ++b) {
        mbar_init(&sh.tc_sfull[x][b], 1);
        mbar_init(&sh.tc_pfull[x][b], 4);       // one arrival per softmax warp
      }
      mbar_init(&sh.tc_odone[x], 1);
    }
    mbar_init(&sh.tc_drain[0], 1);
    mbar_init(&sh.tc_drain[1], 1);
    mbar_init(&sh.tc_qfull, 1);
    fence_mbar_init();
  }
  // set-up that reads nothing an earlier kernel wrote runs before the wait: the
  // barriers above, the tensor-map prefetch and the TMEM columns of the
  // tcgen05 prefill items (every CTA allocates; one CTA per SM holds them)
  if (warp == 0) {
    tmem_alloc(&sh.tmem_base, TC_TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sh.tmem_base;
  const int lane = threadIdx.x & 31;
  const int nw = (int)gridDim.x * ATT_WARPS;
  // HY_ATTN_EARLY: the plan, the block tables and the item id cache were
  // written at least two launches back, so a decode-only launch reads its
  // items and starts the K/V loads of their older blocks now, while the kernel
  // before it (which wrote only the query tokens and their keys) still runs.
  DecRec pre_rec = {};
  uint32_t pre_issued = 0u;
  bool have_pre = false;
  if (a.early && warp < ATT_WARPS) {
    const uint64_t keep0 = l2_keep_policy();
    const int e_pre = ld_keep(v.header, keep0), e_dec = ld_keep(v.header + 1, keep0);
    const int e_pairs = ld_keep(v.header + 4, keep0);
    int item = -1;
    if (e_pairs > 0) {
      if ((int)blockIdx.x < e_pairs) {
        const int seq = (int)blockIdx.x / a.kv_heads, g = (int)blockIdx.x - seq * a.kv_heads;
        const int2 si = v.seqinfo[seq];
        if (warp < si.y) item = si.x + g * si.y + warp;
      }
    } else if (e_pre == 0 && e_dec <= nw) {
      const int it = warp * (int)gridDim.x + (int)blockIdx.x;
      if (it < e_dec) item = it;
    }
    if (item >= 0) {
      pre_issued = decode_item_early(&kv_tiles, a, v, item, payload + warp * DEC_WARP_BYTES,
                                     sh.dec_bar[warp], pre_rec);
      have_pre = true;
    }
  }
  hy_grid_wait();
  hy_grid_trigger();
  const uint64_t keep = l2_keep_policy();
  const int n_pre = ld_keep(v.header, keep), n_dec = ld_keep(v.header + 1, keep);
  const int n_pairs = ld_keep(v.header + 4, keep);    // per-CTA decode when > 0
  const bool use_tmem = (int)blockIdx.x < n_pre;      // the first n_pre CTAs take prefill items
  uint32_t dec_phase = 0, tile_ctr = 0;
  bool ok = true;
  int* grab = v.grab + GRAB_INTS * (a.layer & 63);
  // prefill items: CTA-wide, in the plan's order (most key tiles first); the
  // load warps take each next item from the counter once the current item's
  // loads are issued, and start its loads
  if (use_tmem) {
    if (threadIdx.x == 0) {
      sh.pre_item = atomicAdd(&grab[2], 1);
      sh.pre_prefetch = -1;
    }
    __syncthreads();
    uint32_t n = 0;
    for (; ok; ++n) {
      const int k = sh.pre_item, pf = sh.pre_prefetch;
      __syncthreads();                          // read before the load warps write the next
      if (k >= n_pre) break;
      ok = prefill_item_tc(&kv_kgroups, &kv_tiles, &q_map, a, v, k, payload, sh, tmem, tile_ctr,
                           n & 1, pf, &grab[2], n_pre);
    }
    // a CTA stopped by a wait that ran out: loads issued ahead for an item it
    // will not run land before the shared memory is reused
    if (!ok && (warp == TC_LOAD_WARP || warp == TC_LOAD_WARP2) && lane == 0) {
      const int pf = sh.pre_prefetch;
      for (int t = 0; t < pf; ++t) {
        const uint32_t c = tile_ctr + t;
        mbar_wait(&sh.tc_full[c % TC_NS], (c / TC_NS) & 1, nullptr);
      }
      if (pf >= 0 && warp == TC_LOAD_WARP) mbar_wait(&sh.tc_qfull, n & 1, nullptr);
    }
  }
  // decode items (warps 0..ATT_WARPS-1): each warp takes the next one from this
  // layer's counter, so warps that finish early keep pulling work.  A launch
  // whose decode items fit one round of warps (and has no prefill items)
  // assigns them statically and skips the counters' round trips; item i goes
  // to CTA i % grid, so that a small batch spreads its TMA boxes over every
  // SM (an SM's TMA unit takes a 2 KB box about every 100 cycles).
  if (n_pairs > 0) {                            // one (sequence, KV head) pair per CTA
    if (warp < ATT_WARPS && (int)blockIdx.x < n_pairs)
      ok = decode_pair_cta(&kv_tiles, a, v, blockIdx.x, payload, sh.dec_bar, dec_phase, pre_rec,
                           have_pre, pre_issued);
  } else if (n_pre == 0 && n_dec <= nw) {
    const int item = warp * (int)gridDim.x + (int)blockIdx.x;
    if (warp < ATT_WARPS && item < n_dec && ok)
      ok = decode_item(&kv_tiles, a, v, item, payload + warp * DEC_WARP_BYTES, sh.dec_bar[warp],
                       dec_phase, pre_rec, have_pre, pre_issued);
  } else {
    while (ok && warp < ATT_WARPS) {
      int item = 0;
      if (lane == 0) item = atomicAdd(&grab[0], 1);
      item = __shfl_sync(0xffffffffu, item, 0);
      if (item >= n_dec) break;
      ok = decode_item(&kv_tiles, a, v, item, payload + warp * DEC_WARP_BYTES, sh.dec_bar[warp],
                       dec_phase, pre_rec, false, 0u);
    }
    __syncthreads();
    if (threadIdx.x == 0) {                     // the last CTA out resets the counters
      __threadfence();
      if (atomicAdd(&grab[1], 1) == (int)gridDim.x - 1) {
        atomicExch(&grab[0], 0);
        atomicExch(&grab[2], 0);
        atomicExch(&grab[1], 0);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, TC_TMEM_COLS);
  }
}

// ------------------------------------------------------------------ fp32 path
// Scalar fp32 attention for the parity build of the model: one warp per
// (query token, query head), every key visited in order.
__global__ void __launch_bounds__(256) attn_fp32_kernel(
    const float* __restrict__ q, float* __restrict__ out, int T, int q_heads, int kv_heads,
    const float* __restrict__ cache_layer, int num_blocks, const int32_t* __restrict__ block_tables,
    int bt_pitch, const int32_t* __restrict__ seq_bt_row, const int32_t* __restrict__ cu_q,
    const int32_t* __restrict__ seq_lens_k, int S, float scale, int32_t* err) {
  const int lane = threadIdx.x & 31;
  const long total = (long)T * q_heads;
  const long nwarps = (long)gridDim.x * (blockDim.x >> 5);
  for (long w = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < total; w += nwarps) {
    const int row = (int)(w / q_heads), hq = (int)(w % q_heads);
    const int g = hq / HY_GROUP;
    int lo = 0, hi = S;                     // seq = last i with cu_q[i] <= row
    while (hi - lo > 1) {
      const int mid = (lo + hi) >> 1;
      if (cu_q[mid] <= row) lo = mid; else hi = mid;
    }
    const int seq = lo;
    const int q_len = cu_q[seq + 1] - cu_q[seq];
    const int prefix = seq_lens_k[seq] - q_len;
    const int key_end = prefix + (row - cu_q[seq]) + 1;
    const int bt_row = seq_bt_row ? seq_bt_row[seq] : seq;
    const int32_t* bt = block_tables + (size_t)bt_row * bt_pitch;
    const float4 qv = *reinterpret_cast<const float4*>(q + ((size_t)row * q_heads + hq) * HY_HEAD_DIM + 4 * lane);
    float m = NEG_INF, l = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int key = 0; key < key_end; ++key) {
      const int blk = bt[key / HY_BLOCK];
      if (blk < 0 || blk >= num_blocks) { hy_flag(err, HY_ERR_BOUNDS); break; }
      const size_t kofs = ((((size_t)blk * 2 + 0) * kv_heads + g) * HY_BLOCK + key % HY_BLOCK) * HY_HEAD_DIM;
      const size_t vofs = kofs + (size_t)kv_heads * HY_BLOCK * HY_HEAD_DIM;
      const float4 kv4 = *reinterpret_cast<const float4*>(cache_layer + kofs + 4 * lane);
      float s = qv.x * kv4.x + qv.y * kv4.y + qv.z * kv4.z + qv.w * kv4.w;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      s *= scale;
      const float m_new = fmaxf(m, s);
      const float alpha = expf(m - m_new);
      const float p = expf(s - m_new);
      l = l * alpha + p;
      const float4 vv = *reinterpret_cast<const float4*>(cache_layer + vofs + 4 * lane);
      acc.x = acc.x * alpha + p * vv.x;
      acc.y = acc.y * alpha + p * vv.y;
      acc.z = acc.z * alpha + p * vv.z;
      acc.w = acc.w * alpha + p * vv.w;
      m = m_new;
    }
    const float inv = 1.f / l;
    *reinterpret_cast<float4*>(out + ((size_t)row * q_heads + hq) * HY_HEAD_DIM + 4 * lane) =
        make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
  }
}

int g_num_sms[64] = {0};
int g_ctas_per_sm[64] = {0};

int device_sms(int dev) {
  if (dev < 0 || dev >= 64) return 148;
  if (g_num_sms[dev] == 0) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    g_num_sms[dev] = n > 0 ? n : 148;
  }
  return g_num_sms[dev];
}

}  // namespace

// ------------------------------------------------------------------ host side
int hy_attn_warp_slots(int dev) { return device_sms(dev) * ATT_WARPS; }

PlanDims hy_attn_plan_dims(int max_seqs, int max_tokens, int kv_heads, int dev,
                           bool split_prefill) {
  PlanDims d;
  d.max_seqs = max_seqs;
  // a step's split pieces are at most the SMs (see plan_kernel)
  d.max_pre_part = split_prefill ? device_sms(dev) : 0;
  d.max_pre = kv_heads * (max_tokens / PRE_QROWS + max_seqs) + d.max_pre_part;
  d.max_dec = kv_heads * max_seqs + ITEMS_PER_WARP * hy_attn_warp_slots(dev);
  d.kv_heads = kv_heads;
  return d;
}

static size_t align256(size_t x) { return (x + 255) & ~(size_t)255; }

size_t hy_attn_workspace_bytes(const PlanDims& d) {
  size_t off = 256;                                         // header
  off = align256(off + (size_t)d.max_pre * sizeof(int4));
  off = align256(off + (size_t)d.max_pre * sizeof(int4));  // sorted prefill items
  off = align256(off + (size_t)d.max_dec * 2 * sizeof(int4));
  off = align256(off + (size_t)d.max_dec * 2 * sizeof(int4));   // cached block ids
  off = align256(off + (size_t)d.max_seqs * sizeof(int2));
  off = align256(off + (size_t)d.max_dec * HY_GROUP * HY_HEAD_DIM * sizeof(float));
  off = align256(off + (size_t)d.max_dec * HY_GROUP * sizeof(float2));
  off = align256(off + (size_t)d.max_seqs * d.kv_heads * sizeof(int));
  off = align256(off + 64 * GRAB_INTS * sizeof(int));
  off = align256(off + (size_t)d.max_pre_part * PRE_PART_F4 * sizeof(float4));
  off = align256(off + (size_t)d.max_pre_part * 256 * sizeof(float2));
  off = align256(off + (size_t)d.max_pre_part * sizeof(int));
  return off;
}

static PlanView make_view(void* ws, const PlanDims& d) {
  PlanView v;
  uint8_t* p = static_cast<uint8_t*>(ws);
  size_t off = 0;
  v.header = reinterpret_cast<int*>(p);
  off = 256;
  v.pre = reinterpret_cast<int4*>(p + off);
  off = align256(off + (size_t)d.max_pre * sizeof(int4));
  v.pre_sorted = reinterpret_cast<int4*>(p + off);
  off = align256(off + (size_t)d.max_pre * sizeof(int4));
  v.dec = reinterpret_cast<int4*>(p + off);
  off = align256(off + (size_t)d.max_dec * 2 * sizeof(int4));
  v.dec_ids = reinterpret_cast<int4*>(p + off);
  off = align256(off + (size_t)d.max_dec * 2 * sizeof(int4));
  v.seqinfo = reinterpret_cast<int2*>(p + off);
  off = align256(off + (size_t)d.max_seqs * sizeof(int2));
  v.part_o = reinterpret_cast<float*>(p + off);
  off = align256(off + (size_t)d.max_dec * HY_GROUP * HY_HEAD_DIM * sizeof(float));
  v.part_ml = reinterpret_cast<float2*>(p + off);
  off = align256(off + (size_t)d.max_dec * HY_GROUP * sizeof(float2));
  v.counters = reinterpret_cast<int*>(p + off);
  off = align256(off + (size_t)d.max_seqs * d.kv_heads * sizeof(int));
  v.grab = reinterpret_cast<int*>(p + off);
  off = align256(off + 64 * GRAB_INTS * sizeof(int));
  v.pre_part_o = reinterpret_cast<float4*>(p + off);
  off = align256(off + (size_t)d.max_pre_part * PRE_PART_F4 * sizeof(float4));
  v.pre_part_ml = reinterpret_cast<float2*>(p + off);
  off = align256(off + (size_t)d.max_pre_part * 256 * sizeof(float2));
  v.pre_ctr = reinterpret_cast<int*>(p + off);
  v.max_pre = d.max_pre;
  v.max_dec = d.max_dec;
  v.max_seqs = d.max_seqs;
  v.max_pre_part = d.max_pre_part;
  return v;
}

cudaError_t hy_launch_attn_plan(const int32_t* cu_q, const int32_t* seq_lens_k, int S,
                                int kv_heads, const PlanDims& d, void* ws, int32_t* err,
                                int dev, cudaStream_t st) {
  return hy_launch(plan_kernel, dim3(1), dim3(PLAN_THREADS), 0, st, cu_q, seq_lens_k, S,
                   kv_heads, hy_attn_warp_slots(dev), make_view(ws, d), err);
}

cudaError_t hy_launch_attn_bf16(const KvMaps& maps, const CUtensorMap& qmap, const void* cache,
                                const void* q, void* out, int q_heads,
                                int kv_heads, int layer_row_base, int oob_row, int num_blocks,
                                const int32_t* block_tables, int bt_pitch,
                                const int32_t* seq_bt_row, const int32_t* cu_q,
                                const int32_t* seq_lens_k, int S, float scale,
                                const PlanDims& d, void* ws, int32_t* err, int dev,
                                cudaStream_t st, int flags) {
  static bool attr_set[64] = {false};
  if (dev >= 0 && dev < 64 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(attn_main_kernel,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    if (e != cudaSuccess) return e;
    int occ = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, attn_main_kernel, ATT_THREADS, SMEM_BYTES);
    g_ctas_per_sm[dev] = occ > 0 ? occ : 1;
    attr_set[dev] = true;
  }
  MainArgs a;
  a.cache = static_cast<const __nv_bfloat16*>(cache);
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.out = static_cast<__nv_bfloat16*>(out);
  a.q_heads = q_heads;
  a.kv_heads = kv_heads;
  a.layer_row_base = layer_row_base;
  a.layer = layer_row_base / (num_blocks * 2 * kv_heads * HY_BLOCK);
  a.oob_row = oob_row;
  a.num_blocks = num_blocks;
  a.block_tables = block_tables;
  a.bt_pitch = bt_pitch;
  a.seq_bt_row = seq_bt_row;
  a.cu_q = cu_q;
  a.seq_lens_k = seq_lens_k;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.err = err;
  a.early = (flags & HY_ATTN_EARLY) != 0;
  const PlanView v = make_view(ws, d);
  const int grid = device_sms(dev) * g_ctas_per_sm[dev < 64 && dev >= 0 ? dev : 0];
  return hy_launch(attn_main_kernel, dim3(grid), dim3(ATT_THREADS), SMEM_BYTES, st, maps.kgroups,
                   maps.tiles, qmap, a, v);
}

cudaError_t hy_launch_attn_fp32(const float* q, float* out, int T, int q_heads, int kv_heads,
                                const float* cache_layer, int num_blocks,
                                const int32_t* block_tables, int bt_pitch,
                                const int32_t* seq_bt_row, const int32_t* cu_q,
                                const int32_t* seq_lens_k, int S, float scale, int32_t* err,
                                cudaStream_t st) {
  if (T <= 0) return cudaSuccess;
  long warps = (long)T * q_heads;
  long blocks = (warps + 7) / 8;
  if (blocks > 148L * 32) blocks = 148L * 32;
  attn_fp32_kernel<<<(int)blocks, 256, 0, st>>>(q, out, T, q_heads, kv_heads, cache_layer,
                                                num_blocks, block_tables, bt_pitch, seq_bt_row,
                                                cu_q, seq_lens_k, S, scale, err);
  return cudaGetLastError();
}
