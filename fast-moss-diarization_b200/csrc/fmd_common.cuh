// Shared device helpers for the sm_100a decoder kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define FMD_DEV __device__ __forceinline__
#define FMD_HD __host__ __device__ __forceinline__

namespace fmd {

constexpr int kHeadDim = 128;     // only head_dim 128 is supported
constexpr int kPageTokens = 64;   // KV page: 64 positions of one (layer, k|v, kv head)
constexpr int kQ8Block = 32;      // GGML Q8_0 block length along the input axis

// ---- activation dtype traits ------------------------------------------------
template <typename T> struct Act;
template <> struct Act<__nv_bfloat16> {
  static constexpr bool kIsBf16 = true;
  static FMD_DEV float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static FMD_DEV __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
  static FMD_DEV uint32_t pack2(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static FMD_DEV float2 unpack2(uint32_t u) {
    // bf16 -> f32 is a 16-bit shift: exact.
    return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xffff0000u));
  }
};
template <> struct Act<__half> {
  static constexpr bool kIsBf16 = false;
  static FMD_DEV float to_f(__half x) { return __half2float(x); }
  static FMD_DEV __half from_f(float x) { return __float2half_rn(x); }
  static FMD_DEV uint32_t pack2(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  static FMD_DEV float2 unpack2(uint32_t u) {
    __half2 v = *reinterpret_cast<__half2*>(&u);
    return __half22float2(v);
  }
};

// Round an f32 through the activation dtype (the reference stores every op
// result in the activation dtype).
template <typename T> FMD_DEV float rnd(float x) { return Act<T>::to_f(Act<T>::from_f(x)); }

// ---- warp reductions ---------------------------------------------------------
FMD_DEV float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
FMD_DEV float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ---- tensor-core MMA (m16n8k16, f32 accumulate) -------------------------------
template <typename T> FMD_DEV void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1);
template <> FMD_DEV void mma16816<__nv_bfloat16>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <> FMD_DEV void mma16816<__half>(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// ---- shared-memory / async-copy helpers ------------------------------------------
FMD_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

// 16-byte async copy global->shared; `bytes` < 16 zero-fills the rest (0 = all zero).
FMD_DEV void cp_async16(void* smem, const void* gmem, int bytes = 16) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(smem)), "l"(gmem), "r"(bytes));
}
// 4-byte async copy global->shared (through L1: .ca is the only mode for 4 bytes).
FMD_DEV void cp_async4(void* smem, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(smem_u32(smem)), "l"(gmem));
}
FMD_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N> FMD_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N)); }

FMD_DEV void ldmatrix_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}
FMD_DEV void ldmatrix_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

// 16-byte streaming load that bypasses L1 allocation (weights are read once).
FMD_DEV int4 ld_stream16(const void* p) {
  int4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// f16 bits -> f32 (exact).
FMD_DEV float h2f_bits(uint16_t b) { return __half2float(__ushort_as_half(b)); }

// Programmatic dependent launch. griddep_wait returns once the preceding
// grid has completed and its writes are visible; a kernel touches data of
// the kernel right before it only after the wait. Every kernel lets the next
// one be scheduled (griddep_launch) only after its own wait: a kernel that
// starts therefore finds every grid before its predecessor completed, and
// may read their results (the step's plan, the page table, KV rows of
// earlier steps) and prefetch weights before its own wait. Both are no-ops
// for a kernel launched without the attribute.
FMD_DEV void griddep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
FMD_DEV void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

}  // namespace fmd

// ---- mbarrier + TMA (sm_90+/sm_100a) ------------------------------------------------
namespace fmd {

FMD_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Make barrier initialisation visible to the async (TMA) proxy.
FMD_DEV void fence_barrier_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
FMD_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
FMD_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Nanosecond wall clock of the GPU.
FMD_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
  return t;
}
// Wall-time cap of every bounded wait: far beyond any wait of a healthy
// launch (a whole decode step takes a few ms), short enough that a wait
// which can never complete surfaces as FMD_ETIMEDOUT within about a second.
constexpr uint64_t kWaitNsCap = 500ull * 1000 * 1000;
// Bounded wait: returns false if the phase did not complete within `limit`
// polls or kWaitNsCap of wall time, whichever comes first.
FMD_DEV bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, uint32_t limit) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t i = 1; i < limit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 63) == 0 && globaltimer_ns() - t0 > kWaitNsCap) return false;
  }
  return false;
}
// Which kernel's wait gave up, recorded next to the status word (status[1],
// first writer wins) so that the host can name it.
enum TimeoutSite {
  kSiteGemv = 1,
  kSiteLmHead = 2,
  kSiteAttnDecode = 3,
  kSiteAttnPrefill = 4,
  kSiteGemmTc = 5,
  kSiteLayerTail = 6,
  kSiteWaitProbe = 7,
  kSiteProjTc = 8,
};
FMD_DEV void report_timeout(int* status, int site) {
  atomicExch(status, -110);  // FMD_ETIMEDOUT
  atomicCAS(status + 1, 0, site);
}
// 2D tiled TMA load global -> shared, completion counted on `bar` (no multicast).
FMD_DEV void tma_load_2d(void* dst, const void* tmap, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::
          "r"(smem_u32(dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
FMD_DEV void prefetch_tmap(const void* tmap) { asm volatile("prefetch.tensormap [%0];\n" ::"l"(tmap) : "memory"); }
// Plain arrival (no transaction bytes).
FMD_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
// 1D bulk copy global -> shared (16-byte aligned, size a multiple of 16), completion on `bar`.
FMD_DEV void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// Named barrier over `nthreads` threads (a subset of the CTA).
FMD_DEV void named_sync(int id, int nthreads) { asm volatile("bar.sync %0, %1;\n" ::"r"(id), "r"(nthreads) : "memory"); }

// ---- tcgen05 (5th-generation tensor cores, accumulators in tensor memory) ----------
// Tensor memory: 512 columns x 128 lanes of 32 bits per SM. A warp may only
// touch the 32 lanes of its quarter (warp id % 4).

// Allocates `ncols` (a power of two >= 32) columns; the base address is
// written to *dst (shared memory). Executed by one whole warp.
FMD_DEV void tmem_alloc(uint32_t* dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(dst)), "r"(ncols)
               : "memory");
}
FMD_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory"); }
FMD_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}
// Order tcgen05 operations around a thread synchronisation (barrier,
// mbarrier wait): "before" ahead of the signal, "after" behind the wait.
FMD_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
FMD_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }

// Shared-memory matrix descriptor of a K-major operand tile stored with the
// 128-byte swizzle (rows of 128 bytes, 8-row atoms 1024 bytes apart, the tile
// 1024-byte aligned): start address >> 4 in bits 0-13, leading byte offset
// (unused by swizzled K-major layouts, 16 bytes) in 16-29, stride byte offset
// 1024 >> 4 in 32-45, descriptor version 1 in 46-47, swizzle mode 2
// (128-byte) in 61-63. Advancing along K inside the 128-byte row adds the
// byte offset to the start address; the swizzle applies to absolute address
// bits, hence the alignment.
FMD_DEV uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}
// Instruction descriptor of kind::f16 with f32 accumulation, A and B both
// K-major and both f16 (bf16 = false) or both bf16: D format in bits 4-5,
// A / B format in 7-9 / 10-12, N >> 3 in 17-22, M >> 4 in 24-28.
FMD_HD constexpr uint32_t umma_idesc_f16(bool bf16, int M, int N) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}
// D[tmem] (+)= A[smem] x B[smem]^T, one instruction of K = 16; issued by one thread.
FMD_DEV void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, bool accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate)
      : "memory");
}
// True in exactly one lane of the calling (converged) warp. The MMA-issuing
// warps run their whole issue loop as a warp (waits, descriptors, branches
// uniform) and let the elected lane issue tcgen05.mma and tcgen05.commit.
// In this library's kernels that form was faster than a lone thread of a
// diverged warp running the loop (prefill attention 161 -> 143 us per
// captured launch, the tensor-core lm_head 119 -> 107 us); the cost of an
// issue depends on the code around it (fmd_debug_mma_issue measures both
// forms on a bare loop).
FMD_DEV bool elect_one() {
  uint32_t pred;
  asm volatile("{\n .reg .pred e;\n elect.sync _|e, 0xffffffff;\n selp.u32 %0, 1, 0, e;\n}\n" : "=r"(pred));
  return pred != 0;
}
// Bounded wait of a whole warp, with one outcome for all its lanes.
FMD_DEV bool mbar_wait_warp(uint64_t* bar, uint32_t parity, uint32_t limit) {
  return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, limit));
}
// Arrive once on `bar` when every MMA this thread issued so far has completed.
FMD_DEV void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
               : "memory");
}
// 32 consecutive columns of this warp's 32 lanes: register i = column i of the
// thread's lane. Followed by tmem_ld_wait() before the registers are read.
FMD_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}
FMD_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }
// 16 consecutive columns of this warp's 32 lanes (as tmem_ld32).
FMD_DEV void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
// Store 32 consecutive columns of this warp's 32 lanes (register i -> column
// i of the thread's lane); tmem_st_wait() orders it before later tcgen05 work.
FMD_DEV void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
FMD_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory"); }

}  // namespace fmd
