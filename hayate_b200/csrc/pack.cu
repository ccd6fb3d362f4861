// Ragged-batch packing on the GPU.
//
// Replaces the reference's host-side batch building: left-padded prompt
// tensors and decode token tensors (hayate/engine/engine.py:165-194), the
// position ids and padding masks (hayate/model/qwen.py:66-106) and the
// per-request contiguous cache bookkeeping (engine.py:80-141, cache.py:6-26).
//
// Per-request state lives on the device:
//   req_tokens[slot][tok_pitch]   prompt + generated token ids
//   block_tables[slot][bt_pitch]  physical KV block ids, in position order
//   req_nblk[slot]                blocks currently owned by the slot
//   free_stack[0, *free_top)      free physical blocks; pops take the top
// A step's schedule is four int32 rows of length S: slot, start (tokens whose
// KV is already cached), q_len (tokens this step), flags (bit 0: sample a
// token from the last row).  The pack kernel allocates the blocks the step
// needs and emits the flat batch: input ids, positions, slot mapping,
// cu_seqlens_q, seq_lens_k and the rows to sample.
#include "common.cuh"

namespace {

constexpr int PACK_THREADS = 1024;
constexpr int PACK_SMEM_SEQS = 4096;          // sequences whose offsets fit in shared memory

// Exclusive scan over one CTA of PACK_THREADS threads; returns the prefix for
// this thread and writes the CTA total to `total`.
__device__ int cta_exclusive_scan(int v, int* warp_sums, int& total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int w = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      int y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_sums[lane] = w;          // inclusive prefix of warp totals
  }
  __syncthreads();
  const int before = (warp == 0) ? 0 : warp_sums[warp - 1];
  total = warp_sums[31];
  __syncthreads();                // warp_sums is reused by the next call
  return before + x - v;
}

__global__ void __launch_bounds__(PACK_THREADS) pack_kernel(
    const int32_t* __restrict__ sched, int S, int T,
    const int32_t* __restrict__ req_tokens, int tok_pitch, int max_reqs,
    int32_t* __restrict__ block_tables, int bt_pitch, int32_t* __restrict__ req_nblk,
    int32_t* __restrict__ free_stack, int32_t* __restrict__ free_top, int num_blocks,
    int32_t* __restrict__ input_ids, int32_t* __restrict__ positions,
    int32_t* __restrict__ slot_mapping, int32_t* __restrict__ cu_q,
    int32_t* __restrict__ seq_lens_k, int32_t* __restrict__ sample_rows,
    int32_t* __restrict__ sample_seq, int32_t* err) {
  __shared__ int warp_sums[32];
  __shared__ int s_top0, s_carry_q, s_carry_n, s_carry_s, s_bad;
  __shared__ int s_cu[PACK_SMEM_SEQS + 1];      // cu_seqlens_q, for token -> sequence
  hy_grid_wait();
  hy_grid_trigger();
  const int32_t* s_slot = sched;
  const int32_t* s_start = sched + S;
  const int32_t* s_qlen = sched + 2 * S;
  const int32_t* s_flags = sched + 3 * S;

  if (threadIdx.x == 0) {
    s_top0 = *free_top;
    s_carry_q = s_carry_n = s_carry_s = 0;
    s_bad = 0;
  }
  __syncthreads();
  const int top0 = s_top0;

  // Phase A: prefix sums, block allocation, per-sequence metadata.
  for (int base = 0; base < S; base += PACK_THREADS) {
    const int i = base + threadIdx.x;
    const bool live = i < S;
    int slot = 0, start = 0, q = 0, flags = 0, need = 0, nb = 0;
    bool ok = live;
    if (live) {
      slot = s_slot[i]; start = s_start[i]; q = s_qlen[i]; flags = s_flags[i];
      const int end = start + q;
      const int nblk_end = (end + HY_BLOCK - 1) / HY_BLOCK;
      if (slot < 0 || slot >= max_reqs || start < 0 || q < 0 || end > tok_pitch ||
          nblk_end > bt_pitch) {
        ok = false;
      } else {
        nb = req_nblk[slot];
        if (nb < 0 || nb > bt_pitch) ok = false;
        else need = max(0, nblk_end - nb);
      }
      if (!ok) { atomicOr(&s_bad, 1); q = 0; need = 0; flags = 0; }
    }
    int tq, tn, ts;
    const int oq = cta_exclusive_scan(live ? q : 0, warp_sums, tq);
    const int on = cta_exclusive_scan(need, warp_sums, tn);
    const int sample = (live && (flags & 1) && q > 0) ? 1 : 0;
    const int os = cta_exclusive_scan(sample, warp_sums, ts);
    const int cq = s_carry_q, cn = s_carry_n, cs = s_carry_s;
    if (live) {
      cu_q[i] = cq + oq;
      if (S <= PACK_SMEM_SEQS) s_cu[i] = cq + oq;
      seq_lens_k[i] = start + q;
      for (int j = 0; j < need; ++j) {
        const int k = cn + on + j;          // k-th pop of this step
        int blk = -1;
        if (k < top0) blk = free_stack[top0 - 1 - k];
        if (blk < 0 || blk >= num_blocks) { atomicOr(&s_bad, 4); blk = 0; }
        block_tables[(size_t)slot * bt_pitch + nb + j] = blk;
      }
      if (need > 0) req_nblk[slot] = nb + need;
      if (sample) {
        sample_rows[cs + os] = cq + oq + q - 1;
        sample_seq[cs + os] = i;
      }
    }
    __syncthreads();
    if (threadIdx.x == 0) { s_carry_q += tq; s_carry_n += tn; s_carry_s += ts; }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    cu_q[S] = s_carry_q;
    if (S <= PACK_SMEM_SEQS) s_cu[S] = s_carry_q;
    if (s_carry_q != T) s_bad |= 1;
    if (s_carry_n > top0) s_bad |= 4;
    *free_top = max(0, top0 - s_carry_n);
  }
  __syncthreads();

  // Phase B: per-token rows.  With the sequences' row offsets staged in shared
  // memory a thread takes a token and finds its sequence by binary search, so
  // all of the step's token loads are independent; batches of more than
  // PACK_SMEM_SEQS sequences take one warp per sequence instead.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (S <= PACK_SMEM_SEQS) {
    for (int r = threadIdx.x; r < T; r += PACK_THREADS) {
      if (r >= s_cu[S]) { atomicOr(&s_bad, 1); continue; }
      int lo = 0, hi = S;                       // last i with s_cu[i] <= r
      while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (s_cu[mid] <= r) lo = mid; else hi = mid;
      }
      const int slot = s_slot[lo];
      if (slot < 0 || slot >= max_reqs) continue;
      const int pos = s_start[lo] + (r - s_cu[lo]);
      input_ids[r] = req_tokens[(size_t)slot * tok_pitch + pos];
      positions[r] = pos;
      slot_mapping[r] = block_tables[(size_t)slot * bt_pitch + pos / HY_BLOCK] * HY_BLOCK +
                        (pos % HY_BLOCK);
    }
  } else {
    for (int i = warp; i < S; i += PACK_THREADS / 32) {
      const int slot = s_slot[i], start = s_start[i];
      const int q = cu_q[i + 1] - cu_q[i];
      const int row0 = cu_q[i];
      if (slot < 0 || slot >= max_reqs) continue;
      const int32_t* toks = req_tokens + (size_t)slot * tok_pitch;
      const int32_t* bt = block_tables + (size_t)slot * bt_pitch;
      for (int j = lane; j < q; j += 32) {
        const int pos = start + j;
        const int r = row0 + j;
        if (r >= T) { atomicOr(&s_bad, 1); continue; }
        input_ids[r] = toks[pos];
        positions[r] = pos;
        slot_mapping[r] = bt[pos / HY_BLOCK] * HY_BLOCK + (pos % HY_BLOCK);
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && s_bad) {
    hy_flag(err, (s_bad & 1) ? HY_ERR_BOUNDS : 0);
    hy_flag(err, (s_bad & 4) ? HY_ERR_POOL : 0);
  }
}

// Return the blocks of the listed slots to the free stack, slot by slot in
// list order and block by block in position order: all of them, or (first
// given) those from position first[i] on -- the blocks before it stay with
// their other owner (a prefix cache).
__global__ void __launch_bounds__(PACK_THREADS) free_kernel(
    const int32_t* __restrict__ slots, const int32_t* __restrict__ first, int n, int max_reqs,
    int32_t* __restrict__ block_tables, int bt_pitch, int32_t* __restrict__ req_nblk,
    int32_t* __restrict__ free_stack, int32_t* __restrict__ free_top, int num_blocks,
    int32_t* err) {
  __shared__ int warp_sums[32];
  __shared__ int s_top, s_bad;
  if (threadIdx.x == 0) { s_top = *free_top; s_bad = 0; }
  __syncthreads();
  for (int base = 0; base < n; base += PACK_THREADS) {
    const int i = base + threadIdx.x;
    int slot = -1, nb = 0, f = 0;
    if (i < n) {
      slot = slots[i];
      if (slot < 0 || slot >= max_reqs) { atomicOr(&s_bad, 1); slot = -1; }
      else {
        const int have = req_nblk[slot];
        f = first ? first[i] : 0;
        if (have < 0 || have > bt_pitch || f < 0 || f > have) { atomicOr(&s_bad, 1); f = 0; }
        else nb = have - f;
      }
    }
    int tot;
    const int off = cta_exclusive_scan(nb, warp_sums, tot);
    const int top = s_top;
    if (slot >= 0) {
      for (int j = 0; j < nb; ++j) {
        const int dst = top + off + j;
        if (dst < num_blocks) free_stack[dst] = block_tables[(size_t)slot * bt_pitch + f + j];
        else atomicOr(&s_bad, 4);
      }
      req_nblk[slot] = 0;
    }
    __syncthreads();
    if (threadIdx.x == 0) s_top = min(num_blocks, top + tot);
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    *free_top = s_top;
    if (s_bad & 1) hy_flag(err, HY_ERR_BOUNDS);
    if (s_bad & 4) hy_flag(err, HY_ERR_POOL);
  }
}

// Push a list of block ids (in list order) onto the free stack.  All ids are
// checked first: one outside [0, num_blocks) or a stack without room for all
// of them pushes nothing and sets the error bit.
__global__ void __launch_bounds__(PACK_THREADS) push_kernel(
    const int32_t* __restrict__ ids, int n, int32_t* __restrict__ free_stack,
    int32_t* __restrict__ free_top, int num_blocks, int32_t* err) {
  __shared__ int s_bad;
  if (threadIdx.x == 0) s_bad = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < n; i += PACK_THREADS)
    if (ids[i] < 0 || ids[i] >= num_blocks) atomicOr(&s_bad, 1);
  __syncthreads();
  const int top = *free_top;
  if (!s_bad && top + n > num_blocks) s_bad = 4;   // read by thread 0 only below
  __syncthreads();
  if (s_bad == 0)
    for (int i = threadIdx.x; i < n; i += PACK_THREADS) free_stack[top + i] = ids[i];
  __syncthreads();
  if (threadIdx.x == 0) {
    if (s_bad == 0) *free_top = top + n;
    else hy_flag(err, (s_bad & 1) ? HY_ERR_BOUNDS : HY_ERR_POOL);
  }
}

// Write each sampled token after the last token of its sequence.
__global__ void commit_kernel(const int32_t* __restrict__ next_tokens, int n_sample,
                              const int32_t* __restrict__ sample_seq,
                              const int32_t* __restrict__ sched, int S,
                              int32_t* __restrict__ req_tokens, int tok_pitch, int max_reqs,
                              int32_t* err) {
  hy_grid_wait();
  hy_grid_trigger();
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= n_sample) return;
  const int i = sample_seq[k];
  if (i < 0 || i >= S) { hy_flag(err, HY_ERR_BOUNDS); return; }
  const int slot = sched[i], pos = sched[S + i] + sched[2 * S + i];
  if (slot < 0 || slot >= max_reqs || pos < 0 || pos >= tok_pitch) {
    hy_flag(err, HY_ERR_BOUNDS);
    return;
  }
  req_tokens[(size_t)slot * tok_pitch + pos] = next_tokens[k];
}

__global__ void pool_init_kernel(int32_t* free_stack, int32_t* free_top, int num_blocks) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < num_blocks) free_stack[i] = num_blocks - 1 - i;
  if (i == 0) *free_top = num_blocks;
}

}  // namespace

// ------------------------------------------------------------------ launchers
cudaError_t hy_launch_pool_init(int32_t* free_stack, int32_t* free_top, int num_blocks,
                                cudaStream_t st) {
  const int threads = 256;
  const int blocks = (num_blocks + threads - 1) / threads;
  pool_init_kernel<<<blocks > 0 ? blocks : 1, threads, 0, st>>>(free_stack, free_top, num_blocks);
  return cudaGetLastError();
}

cudaError_t hy_launch_pack(const int32_t* sched, int S, int T, const int32_t* req_tokens,
                           int tok_pitch, int max_reqs, int32_t* block_tables, int bt_pitch,
                           int32_t* req_nblk, int32_t* free_stack, int32_t* free_top,
                           int num_blocks, int32_t* input_ids, int32_t* positions,
                           int32_t* slot_mapping, int32_t* cu_q, int32_t* seq_lens_k,
                           int32_t* sample_rows, int32_t* sample_seq, int32_t* err,
                           cudaStream_t st) {
  return hy_launch(pack_kernel, dim3(1), dim3(PACK_THREADS), 0, st, sched, S, T, req_tokens,
                   tok_pitch, max_reqs, block_tables, bt_pitch, req_nblk, free_stack, free_top,
                   num_blocks, input_ids, positions, slot_mapping, cu_q, seq_lens_k, sample_rows,
                   sample_seq, err);
}

cudaError_t hy_launch_free(const int32_t* slots, const int32_t* first, int n, int max_reqs,
                           int32_t* block_tables, int bt_pitch, int32_t* req_nblk,
                           int32_t* free_stack, int32_t* free_top, int num_blocks, int32_t* err,
                           cudaStream_t st) {
  free_kernel<<<1, PACK_THREADS, 0, st>>>(slots, first, n, max_reqs, block_tables, bt_pitch,
                                          req_nblk, free_stack, free_top, num_blocks, err);
  return cudaGetLastError();
}

cudaError_t hy_launch_push(const int32_t* ids, int n, int32_t* free_stack, int32_t* free_top,
                           int num_blocks, int32_t* err, cudaStream_t st) {
  push_kernel<<<1, PACK_THREADS, 0, st>>>(ids, n, free_stack, free_top, num_blocks, err);
  return cudaGetLastError();
}

cudaError_t hy_launch_commit(const int32_t* next_tokens, int n_sample, const int32_t* sample_seq,
                             const int32_t* sched, int S, int32_t* req_tokens, int tok_pitch,
                             int max_reqs, int32_t* err, cudaStream_t st) {
  if (n_sample <= 0) return cudaSuccess;
  const int threads = 128;
  return hy_launch(commit_kernel, dim3((n_sample + threads - 1) / threads), dim3(threads), 0, st,
                   next_tokens, n_sample, sample_seq, sched, S, req_tokens, tok_pitch, max_reqs,
                   err);
}
