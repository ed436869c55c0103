// ptx.cuh -- thin inline-PTX wrappers for the sm_100a features the kernels use:
// mbarriers, TMA (tiled tensor loads and 1-D bulk copies), and the tcgen05 family
// (TMEM allocation, MMA issue/commit, TMEM loads/stores, fences).
//
// Every wait is bounded: a wait that does not complete within the kernel's time budget
// records an error code in the caller's error word and returns false, so a kernel never
// spins forever on the GPU.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace lmoe {

// ---------------------------------------------------------------------------------------
// error reporting
// ---------------------------------------------------------------------------------------
// Error word layout (uint32): 0 = ok, otherwise (code << 24) | (site & 0xffffff).
enum DevErr : uint32_t {
  kErrTimeout = 1u,     // a bounded wait gave up
  kErrBadArg = 2u,      // the kernel found an argument outside its supported range
};

__device__ __forceinline__ void report_error(uint32_t* err, uint32_t code, uint32_t site) {
  if (err) atomicCAS(err, 0u, (code << 24) | (site & 0xffffffu));
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Budget of one bounded wait.  The hot-path kernels finish in milliseconds; two seconds
// without progress means something is wrong.
constexpr uint64_t kWaitBudgetNs = 2000000000ull;

// ---------------------------------------------------------------------------------------
// shared memory addresses and mbarriers
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
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

// Non-blocking test: has the phase with the given parity completed?  (try_wait may
// suspend the thread for a while; a thread that serves several queues polls with this.)
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  On timeout the error
// word receives kErrTimeout|site, *abort is raised for the rest of the CTA, and false is
// returned.  A raised *abort makes every later wait give up immediately.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* err,
                                          volatile int* abort, uint32_t site) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (((++spins) & 63u) == 0u) {
      if (abort && *abort) return false;
      if (globaltimer_ns() - t0 > kWaitBudgetNs) {
        report_error(err, kErrTimeout, site);
        if (abort) *abort = 1;
        return false;
      }
    }
  }
}

// A progress counter in shared memory, for threads that must not wait on mbarriers
// themselves: on B200 an mbarrier wait in a thread that issues tcgen05.mma costs ~270
// cycles even when the phase has long completed, a plain shared-memory load ~40.  A helper
// thread waits on the mbarrier (acquire) and publishes the count with a release store; the
// issuing thread polls it with acquire loads.
__device__ __forceinline__ uint32_t ld_acquire_shared(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_shared(uint32_t* p, uint32_t v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}
// Bounded wait until *ctr > target (same error / abort contract as mbar_wait).
__device__ __forceinline__ bool counter_wait(const uint32_t* ctr, uint32_t target, uint32_t* err,
                                             volatile int* abort, uint32_t site) {
  if (ld_acquire_shared(ctr) > target) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (ld_acquire_shared(ctr) > target) return true;
    if (((++spins) & 255u) == 0u) {
      if (abort && *abort) return false;
      if (globaltimer_ns() - t0 > kWaitBudgetNs) {
        report_error(err, kErrTimeout, site);
        if (abort) *abort = 1;
        return false;
      }
    }
  }
}

// Four counters (16-byte aligned, one per writing warp) read with one relaxed vector load;
// returns the smallest.
__device__ __forceinline__ uint32_t min4_relaxed_shared(const uint32_t* p) {
  uint32_t a, b, c, d;
  asm volatile("ld.relaxed.cta.shared::cta.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(a), "=r"(b), "=r"(c), "=r"(d)
               : "r"(smem_u32(p))
               : "memory");
  return min(min(a, b), min(c, d));
}
__device__ __forceinline__ void fence_acq_rel_cta() { asm volatile("fence.acq_rel.cta;" ::: "memory"); }

// Bounded wait until all four counters at p exceed target (acquire: relaxed polls, then one
// fence once they do).  *seen receives the smallest value read.  Same error / abort
// contract as mbar_wait.
__device__ __forceinline__ bool counter4_wait(const uint32_t* p, uint32_t target, uint32_t* seen, uint32_t* err,
                                              volatile int* abort, uint32_t site) {
  uint32_t m = min4_relaxed_shared(p);
  if (m <= target) {
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (true) {
      m = min4_relaxed_shared(p);
      if (m > target) break;
      if (((++spins) & 255u) == 0u) {
        if (abort && *abort) return false;
        if (globaltimer_ns() - t0 > kWaitBudgetNs) {
          report_error(err, kErrTimeout, site);
          if (abort) *abort = 1;
          return false;
        }
      }
    }
  }
  fence_acq_rel_cta();
  if (seen) *seen = m;
  return true;
}

// ---------------------------------------------------------------------------------------
// TMA
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled load: box at (x = inner coordinate in elements, y = row) into smem.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                            int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int32_t x, int32_t y,
                                            int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// 1-D bulk copy global -> shared (both 16-byte aligned, bytes a multiple of 16).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Hint the L2 to fetch [src, src + bytes) from HBM (no shared-memory destination, no
// completion to wait for).  src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)), "r"(bytes)
               : "memory");
}

// ---------------------------------------------------------------------------------------
// tcgen05: tensor memory and the 5th-generation tensor core
// ---------------------------------------------------------------------------------------
// One full warp allocates `ncols` (power of two, >= 32) TMEM columns; the base address is
// written to *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Instruction descriptor for kind::f16 with bf16 A/B, fp32 accumulate, both K-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(uint32_t M, uint32_t N) {
  return (1u << 4)            // D format: f32
         | (1u << 7)          // A format: bf16
         | (1u << 10)         // B format: bf16
         | (0u << 15)         // A K-major
         | (0u << 16)         // B K-major
         | ((N >> 3) << 17)   // N / 8
         | ((M >> 4) << 24);  // M / 16
}

// The same with A and B both fp16 (ab_f16 != 0) or both bf16: kind::f16 takes one type for
// both operands.
__host__ __device__ constexpr uint32_t idesc_f16kind_f32(uint32_t M, uint32_t N, int ab_f16) {
  return ab_f16 ? (idesc_bf16_f32(M, N) & ~((7u << 7) | (7u << 10))) : idesc_bf16_f32(M, N);
}

// Shared-memory matrix descriptor for a K-major operand stored with the 128-byte swizzle:
// rows of 128 bytes (64 bf16), groups of 8 rows 1024 bytes apart.  The tile base must be
// 1024-byte aligned; advancing along K inside the 128-byte row is done by adding the byte
// offset to the start address.
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3fffu);  // start address
  d |= (uint64_t)1u << 16;                      // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024u >> 4) << 32;            // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1u << 46;                      // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                      // layout: 128-byte swizzle
  return d;
}

// D[tmem] (+)= A[smem] * B[smem]^T
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on *bar when all previously issued tcgen05 operations of this thread finish.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Each thread of the warp reads 16 consecutive 32-bit columns of its own TMEM lane.  The
// load and its completion wait are one asm statement, so no use of the destination
// registers can be scheduled before the data has arrived.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// Two tmem_ld16 loads (any two column addresses of the thread's lane) under one completion
// wait.
__device__ __forceinline__ void tmem_ld16x2(uint32_t taddr0, uint32_t taddr1, uint32_t (&r)[16], uint32_t (&u)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%32];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%33];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]), "=r"(u[7]),
        "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]), "=r"(u[13]), "=r"(u[14]), "=r"(u[15])
      : "r"(taddr0), "r"(taddr1)
      : "memory");
}

// Each thread of the warp writes 16 consecutive 32-bit columns of its own TMEM lane.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// Named barrier among `nthreads` threads (multiple of 32) with id 1..15.
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also returns the OR of `pred` over all participating threads, so a
// group of warps can agree on leaving a loop together.
__device__ __forceinline__ bool named_bar_any(uint32_t id, uint32_t nthreads, bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((uint32_t)pred), "r"(id), "r"(nthreads)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "elect.sync _|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

}  // namespace lmoe
