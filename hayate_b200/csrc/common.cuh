// Shared device helpers for the hayate_b200 kernels (sm_100a only).
//
// * a device-side error word: kernels OR a bit into it instead of trapping;
// * bounded mbarrier waits (a wait that runs out sets HY_ERR_TIMEOUT and
//   returns false, so a kernel never spins forever);
// * TMA tensor loads without multicast, and the warp-level mma.sync/ldmatrix
//   wrappers used by the decode path.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda.h>
#include <stdint.h>

// Bits of the device error word.
#define HY_ERR_BOUNDS   1   // an index (slot, block, position, token) was out of range
#define HY_ERR_TIMEOUT  2   // an mbarrier wait ran out
#define HY_ERR_POOL     4   // the block pool had too few free blocks
#define HY_ERR_PLAN     8   // the attention plan did not fit its workspace

// Fixed geometry the kernels are specialised for.
#define HY_HEAD_DIM   128
#define HY_GROUP      4     // query heads per KV head
#define HY_BLOCK      16    // tokens per KV block

#define HY_DEVICE __device__ __forceinline__

HY_DEVICE void hy_flag(int32_t* err, int bit) {
  if (err) atomicOr(err, bit);
}

HY_DEVICE uint64_t hy_globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

HY_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------- L2 residency of small tables
// Loads with an L2 evict-last policy: the small per-step tables a kernel reads
// once per layer (plan records, block tables) then stay in L2 while each layer
// streams ~200 MB of weights through it, so the next layer's reads hit L2.
HY_DEVICE uint64_t l2_keep_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
HY_DEVICE int ld_keep(const int* a, uint64_t pol) {
  int v;
  asm volatile("ld.global.L2::cache_hint.b32 %0, [%1], %2;" : "=r"(v) : "l"(a), "l"(pol));
  return v;
}
HY_DEVICE int4 ld_keep(const int4* a, uint64_t pol) {
  int4 v;
  asm volatile("ld.global.L2::cache_hint.v4.b32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(a), "l"(pol));
  return v;
}

// 16-byte global -> shared copy through L2 (cp.async.cg), completed by cp_async_wait_all
HY_DEVICE void cp_async16(void* smem, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" :: "r"(smem_u32(smem)), "l"(gmem)
               : "memory");
}
HY_DEVICE void cp_async_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

// ------------------------------------------------- programmatic dependent launch
// Kernels of the step are launched with hy_launch: with programmatic stream
// serialisation a kernel's CTAs may start while the previous kernel on the
// stream is still running.  Such a kernel does its set-up first and calls
// hy_grid_wait() before it reads anything an earlier kernel wrote (the wait
// returns once the previous grid has completed and its writes are visible; it
// is a no-op for a kernel launched without the attribute).  hy_grid_trigger()
// lets the next kernel's CTAs start early.
HY_DEVICE void hy_grid_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
HY_DEVICE void hy_grid_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

bool hy_pdl_enabled();   // false when the environment sets HY_PDL=0

template <typename... KArgs, typename... Args>
inline cudaError_t hy_launch(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                             cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = hy_pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// ---------------------------------------------------------------- mbarrier
HY_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(bar)), "r"(count) : "memory");
}

HY_DEVICE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
               :: "r"(smem_u32(bar)), "r"(bytes) : "memory");
}

HY_DEVICE void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(bar)) : "memory");
}

HY_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Gives up after
// ~timeout_ns of wall time: sets HY_ERR_TIMEOUT and returns false.
constexpr uint64_t HY_WAIT_TIMEOUT_NS = 2000000000ull;   // 2 s

HY_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, int32_t* err,
                         uint64_t timeout_ns = HY_WAIT_TIMEOUT_NS) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = hy_globaltimer();
  uint32_t n = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++n & 63) == 0 && hy_globaltimer() - t0 > timeout_ns) {
      hy_flag(err, HY_ERR_TIMEOUT);
      return false;
    }
  }
}

// Named barrier over the first `n` threads (ids 1..15; id 0 is __syncthreads).
HY_DEVICE void named_sync(uint32_t id, uint32_t n) {
  asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(n) : "memory");
}
// Named barrier that also ORs a predicate over its `n` threads.
HY_DEVICE bool named_sync_or(uint32_t id, uint32_t n, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r) : "r"((uint32_t)pred), "r"(id), "r"(n) : "memory");
  return r != 0;
}

HY_DEVICE void fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

HY_DEVICE void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// ---------------------------------------------------------------- TMA
// Untiled bulk copy global -> this CTA's shared memory, completion counted on
// `bar` (both addresses 16-byte aligned, bytes a multiple of 16; no multicast).
HY_DEVICE void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      :: "r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// 2-D tiled tensor load into shared memory, completion counted on `bar`.
// No multicast: every CTA loads its own tiles.
HY_DEVICE void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];"
      :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y),
         "r"(smem_u32(bar))
      : "memory");
}

HY_DEVICE void tma_load_3d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z,
                           uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];"
      :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z),
         "r"(smem_u32(bar))
      : "memory");
}

HY_DEVICE void tma_load_4d(void* dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z,
                           int32_t w, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];"
      :: "r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z),
         "r"(w), "r"(smem_u32(bar))
      : "memory");
}

HY_DEVICE void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" :: "l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---------------------------------------------------------------- mma.sync
HY_DEVICE void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}

HY_DEVICE void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]) : "r"(addr));
}

// D = A(16x16 bf16, row) * B(16x8 bf16, col) + D, fp32 accumulate.
HY_DEVICE void mma_bf16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// 2^x with the hardware approximation (PTX ex2.approx.ftz.f32): relative error
// near 2^-22, subnormal results flushed to zero, 2^-inf = 0.  Softmax weights
// are rounded to bf16 or summed in fp32, so neither matters there.
HY_DEVICE float ex2_ftz(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x on the FMA and integer pipes, for softmax weights the exp2 unit cannot
// keep up with: Cody-Waite range reduction to f = x - round(x) in [-0.5, 0.5]
// (round(x) by the 1.5 * 2^23 addition), a degree-3 polynomial for 2^f whose
// coefficients minimise the largest relative error on that interval (fitted by
// linear programming over 4001 points: 7.5e-5, i.e. 2^-13.7), then 2^round(x)
// added to the exponent bits.  Valid for x <= 127; results below 2^-126 are
// returned as 0 (x = -inf gives 0).  Used where the weight is rounded to bf16
// (2^-9 relative) or summed in fp32.
HY_DEVICE float exp2_poly(float x) {
  const float xc = fmaxf(x, -126.0f);
  const float t = __fadd_rn(xc, 12582912.0f);          // 1.5 * 2^23: round(xc) in the low bits
  const float f = __fsub_rn(xc, __fsub_rn(t, 12582912.0f));
  float p = fmaf(0.05517166853f, f, 0.24261112511f);
  p = fmaf(p, f, 0.69326096773f);
  p = fmaf(p, f, 0.99992805719f);
  const int e = __float_as_int(t) - 0x4B400000;         // round(xc) as an integer
  const float y = __int_as_float(__float_as_int(p) + (e << 23));
  return x < -126.0f ? 0.0f : y;
}

// exp2_poly on a pair with packed f32x2 arithmetic (each lane rounded as the
// scalar operation, so each result equals exp2_poly of its input); the
// exponent goes in with one shift-add per lane: (round(x) << 23) is the low
// bits of t shifted, since 1.5 * 2^23's own bits vanish in the shift.
HY_DEVICE float2 exp2_poly2(float2 x) {
  const float2 xc = make_float2(fmaxf(x.x, -126.0f), fmaxf(x.y, -126.0f));
  const float2 big = make_float2(12582912.0f, 12582912.0f);
  const float2 t = __fadd2_rn(xc, big);
  const float2 j = __fadd2_rn(t, make_float2(-12582912.0f, -12582912.0f));   // round(xc)
  const float2 f = __ffma2_rn(j, make_float2(-1.0f, -1.0f), xc);              // xc - j, exact
  float2 p = __ffma2_rn(make_float2(0.05517166853f, 0.05517166853f), f,
                        make_float2(0.24261112511f, 0.24261112511f));
  p = __ffma2_rn(p, f, make_float2(0.69326096773f, 0.69326096773f));
  p = __ffma2_rn(p, f, make_float2(0.99992805719f, 0.99992805719f));
  const float y0 = __int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23));
  const float y1 = __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23));
  return make_float2(x.x < -126.0f ? 0.0f : y0, x.y < -126.0f ? 0.0f : y1);
}

// max(a, b, c) in one instruction (sm_100's three-input max).
HY_DEVICE float fmax3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

HY_DEVICE uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// Byte offset of element (row, d) inside a [rows][64] bf16 tile region laid
// out by a TMA load with CU_TENSOR_MAP_SWIZZLE_128B (region base 1024-aligned).
HY_DEVICE uint32_t swz128(uint32_t row, uint32_t col64) {
  return row * 128u + ((((col64 >> 3) ^ (row & 7u)) << 4) | ((col64 & 7u) << 1));
}

template <typename T> struct ElemTraits;
template <> struct ElemTraits<float> {
  static HY_DEVICE float to_f(float v) { return v; }
  static HY_DEVICE float from_f(float v) { return v; }
};
template <> struct ElemTraits<__nv_bfloat16> {
  static HY_DEVICE float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static HY_DEVICE __nv_bfloat16 from_f(float v) { return __float2bfloat16_rn(v); }
};

// ---------------------------------------------------------------- tcgen05
// Tensor memory (TMEM) allocation: one full warp allocates `ncols` (a power of
// two >= 32) columns of all 128 lanes and writes the base address to smem.
HY_DEVICE void tmem_alloc(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               :: "r"(smem_u32(smem_dst)), "r"(ncols) : "memory");
}
HY_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
HY_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(taddr), "r"(ncols)
               : "memory");
}
HY_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
HY_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive on `bar` once every tcgen05 op this thread issued so far has completed.
HY_DEVICE void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(smem_u32(bar)) : "memory");
}

// D[tmem] (+)= A[smem] * B[smem], bf16 inputs, fp32 accumulators; one thread issues.
HY_DEVICE void tc_mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]: A (M x K bf16, K-major) is read from TMEM,
// row m in lane m, elements (2i, 2i+1) of the row packed in column a_tmem + i.
HY_DEVICE void tc_mma_bf16_ta(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      :: "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}

// Instruction descriptor of kind::f16 with bf16 A/B, fp32 D, A K-major; B K-major
// or MN-major; shape M x N.
HY_DEVICE constexpr uint32_t tc_idesc_bf16(int M, int N, bool b_mn_major) {
  return (1u << 4)                                   // D format: f32
         | (1u << 7)                                 // A format: bf16
         | (1u << 10)                                // B format: bf16
         | ((b_mn_major ? 1u : 0u) << 16)            // B major-ness
         | ((uint32_t)(N >> 3) << 17)                // N / 8
         | ((uint32_t)(M >> 4) << 24);               // M / 16
}

// Shared-memory matrix descriptor for a 128-byte-swizzled canonical layout
// (the layout a SWIZZLE_128B TMA box produces: 8-row x 128 B atoms).
HY_DEVICE uint64_t tc_desc_sw128(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = (uint64_t)((smem_addr & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;                            // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                            // layout: SWIZZLE_128B
  return d;
}

// 32 consecutive fp32 columns of this thread's TMEM lane (warp-collective).
HY_DEVICE void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

HY_DEVICE void tmem_st32u(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      :: "r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]),
         "r"(v[7]), "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]),
         "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]),
         "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
         "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

HY_DEVICE void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};"
      :: "r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])),
         "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])),
         "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
         "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
         "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
         "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])),
         "r"(__float_as_uint(v[17])), "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])),
         "r"(__float_as_uint(v[20])), "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])),
         "r"(__float_as_uint(v[23])), "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])),
         "r"(__float_as_uint(v[26])), "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])),
         "r"(__float_as_uint(v[29])), "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

HY_DEVICE void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
HY_DEVICE void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
