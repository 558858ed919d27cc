// tkv_ptx.cuh -- thin inline-PTX wrappers for sm_100a used by the tiered
// kernels: mbarriers with bounded waits, TMA tile loads and 1-D bulk copies
// (never with cluster multicast), ldmatrix / movmatrix / mma.sync, tcgen05
// (TMEM allocation, MMA, commit, TMEM loads) and the MUFU exp2 / log2.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

namespace tkv {

// A bounded pipeline wait gives up after this long (globaltimer ns) and the
// kernel records TKV_DEVERR_TIMEOUT instead of spinning forever.
constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

// bar.sync on a named barrier (ids 1..15; 0 is __syncthreads) for a subset
// of the CTA's warps; `threads` is a multiple of 32.
__device__ __forceinline__ void named_barrier(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// System-scope release store / acquire load (flags another GPU reads or
// writes through an IPC mapping).
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// System-scope relaxed 64-bit accesses, two words per instruction: each
// 8-byte element is one single-copy-atomic access, so a word written by
// another GPU is seen whole or not at all (epoch-tagged exchange words).
__device__ __forceinline__ void st_relaxed_sys_v2(uint64_t* p, uint64_t a, uint64_t b) {
  asm volatile("st.relaxed.sys.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(a), "l"(b)
               : "memory");
}
__device__ __forceinline__ void st_relaxed_sys(uint64_t* p, uint64_t a) {
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(a) : "memory");
}
__device__ __forceinline__ void ld_relaxed_sys_v2(const uint64_t* p, uint64_t& a, uint64_t& b) {
  asm volatile("ld.relaxed.sys.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p)
               : "memory");
}
__device__ __forceinline__ uint64_t ld_relaxed_sys(const uint64_t* p) {
  uint64_t a;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(a) : "l"(p) : "memory");
  return a;
}

// GPU-scope fetch-and-add with acquire-release semantics (merge tickets):
// the release covers the stores of the whole CTA when a CTA barrier precedes
// it, the acquire covers every store released by earlier increments.
__device__ __forceinline__ uint32_t atom_add_acq_rel_gpu(uint32_t* p, uint32_t v) {
  uint32_t old;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;"
               : "=r"(old)
               : "l"(p), "r"(v)
               : "memory");
  return old;
}

// Programmatic dependent launch (sm_90+): let the next kernel of the stream
// be scheduled now (its CTAs take SM slots as this grid's CTAs exit), and wait
// until the previous kernel of the stream has completed and its memory is
// visible.  Both are no-ops for a launch without the programmatic attribute.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity to complete; false on timeout.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer() - t0 > kWaitTimeoutNs) return false;
  }
}

// ---- TMA / bulk copies (none multicast across a cluster) ----------------------
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int32_t x,
                                            int32_t y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int32_t x,
                                            int32_t y, int32_t z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, int32_t x,
                                            int32_t y, int32_t z, int32_t w, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// L2 prefetches of a tensor tile or a byte range: hints that move data into
// L2 and change no value a later load returns.
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap* map, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void tma_prefetch_3d(const CUtensorMap* map, int32_t x, int32_t y,
                                                int32_t z) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(z)
               : "memory");
}
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- shared-memory loads ------------------------------------------------------
// These are plain (non-volatile) asm so the compiler may schedule them freely,
// e.g. issue every fragment load of a tile before its first MMA instead of
// in program order.  They declare no memory dependency, so a caller must tie
// their addresses to whatever makes the data valid (see wait_token / after)
// and keep their results alive across a stage release (see hold).
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
      : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
      : "r"(addr));
}

__device__ __forceinline__ uint32_t lds32(uint32_t addr) {
  uint32_t v;
  asm("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "r"(addr));
  return v;
}

// An opaque zero produced in program order (volatile) after everything before
// it, e.g. an mbarrier wait; `after(addr, token)` makes an address depend on
// it, so loads through that address cannot be hoisted above the wait.
__device__ __forceinline__ uint32_t wait_token() {
  uint32_t t;
  asm volatile("mov.u32 %0, 0;" : "=r"(t)::"memory");
  return t;
}
__device__ __forceinline__ uint32_t after(uint32_t x, uint32_t token) {
  asm("add.u32 %0, %0, %1;" : "+r"(x) : "r"(token));
  return x;
}
// Keeps a register's producer (a load) ahead of the next volatile asm, e.g.
// the mbarrier arrive that hands a stage back to the producer.
__device__ __forceinline__ void hold(uint32_t x) { asm volatile("" ::"r"(x)); }
__device__ __forceinline__ void hold(float x) { asm volatile("" ::"f"(x)); }

// ---- tensor-core fragments ----------------------------------------------------
// D[16x8] += A[16x16] (row) * B[16x8] (col), fp16 inputs, fp32 accumulate.
__device__ __forceinline__ void mma_16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                          uint32_t a3, uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, "
      "{%8, %9}, {%0, %1, %2, %3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Transposes the 8x8 b16 matrix held one row-pair per thread.
__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// ---- scalar helpers -------------------------------------------------------------
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// exp2 on the FMA and ALU pipes (Cody-Waite range reduction, as in
// FlashAttention-4's software exponential): x = j + f with j = rint(x) taken
// from the low mantissa bits of x + 1.5 * 2^23, 2^f for f in [-0.5, 0.5] from
// a degree-4 polynomial, 2^j added to its exponent field.  The coefficients
// are a least-squares fit of 2^f weighted toward minimax relative error
// (Lawson iterations on 400 Chebyshev nodes); evaluated in float32 Horner form
// the relative error stays below 3e-6.  x is clamped at -126, so x = -inf
// gives 2^-126-scale values (below 1.2e-38) rather than 0, and the exponent
// arithmetic never leaves the positive normal / subnormal encodings.
constexpr float kExp2Poly0 = 0.9999992847442627f;
constexpr float kExp2Poly1 = 0.6931217908859253f;
constexpr float kExp2Poly2 = 0.240247443318367f;
constexpr float kExp2Poly3 = 0.05591785907745361f;
constexpr float kExp2Poly4 = 0.009570101276040077f;
__device__ __forceinline__ float ex2_fma(float x) {
  x = fmaxf(x, -126.f);
  const float t = x + 12582912.f;  // 1.5 * 2^23: t's low mantissa bits hold rint(x)
  const float f = x - (t - 12582912.f);
  float p = fmaf(kExp2Poly4, f, kExp2Poly3);
  p = fmaf(p, f, kExp2Poly2);
  p = fmaf(p, f, kExp2Poly1);
  p = fmaf(p, f, kExp2Poly0);
  // (bits(t) << 23) == rint(x) << 23: the 1.5 * 2^23 offset shifts out
  return __int_as_float(__float_as_int(p) + (__float_as_int(t) << 23));
}

__device__ __forceinline__ float lg2(float x) {
  float y;
  asm("lg2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ uint32_t hsub2_u32(uint32_t a, uint32_t b) {
  __half2 r = __hsub2(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// Byte-level swizzle of TMA SWIZZLE_{32,64,128}B boxes: 16-byte chunk bits
// [4, 4+log2(M+1)) of an offset are XOR-ed with bits [7, ...).  `off` is the
// byte offset from a buffer aligned to 1024 bytes.
template <int M>
__device__ __forceinline__ uint32_t swz(uint32_t off) {
  return off ^ (((off >> 7) & M) << 4);
}

// ---- tcgen05: tensor memory and the 5th-generation tensor cores ------------------
// Tensor memory (TMEM) is 128 lanes x 512 columns of 32-bit cells per SM; an
// address holds the lane in bits [16, 32) and the column in [0, 16).  Warp w
// of a CTA may read lanes [32 (w % 4), 32 (w % 4) + 32) only.

// Allocates `cols` columns (a power of two >= 32) for the CTA; executed by one
// whole warp, which must also free them.  The base address lands in *dst.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major operand stored the way a TMA
// SWIZZLE_128B box lands: rows of 128 bytes (64 fp16 of K), 16-byte chunks
// XOR-ed with the row index mod 8, groups of 8 rows 1024 bytes apart (the
// stride byte offset).  The leading byte offset is unused for this layout
// (encoded as 1); bits 46-48 carry the descriptor version 1; bits 61-63 the
// layout type 2 (128-byte swizzle).  K steps of 16 elements inside the
// 128-byte row advance the start address by 32 bytes.
__device__ __forceinline__ uint64_t umma_desc_k_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Instruction descriptor of kind::f16 with fp16 A and B (both K-major) and an
// fp32 accumulator: bits 4-5 accumulator format (1 = f32), 7-9 / 10-12 the A /
// B formats (0 = f16), 15 / 16 the majors (0 = K), 17-22 N / 8, 24-28 M / 16.
__host__ __device__ constexpr uint32_t umma_idesc_f16_f32(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T; issued by a single thread.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The mbarrier receives one arrival once every tcgen05 operation this thread
// issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 consecutive columns of this thread's TMEM lane (32x32b shape, x32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, "
      "%11, %12, %13, %14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, "
      "%28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

}  // namespace tkv
