// Thin inline-PTX wrappers for sm_100a: mbarriers, TMA tile loads, tcgen05
// (TMEM allocation, UMMA issue/commit, TMEM loads) and the shared-memory
// matrix descriptors the UMMA reads.  Written against the PTX ISA; the
// descriptor bit positions follow the public sm_100 UMMA descriptor layout
// (CUTLASS cute/arch/mma_sm100_desc.hpp documents the same fields).
//
// No multicast form of any load appears here: these kernels also run under
// the multi-GPU driver.
#pragma once

#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>

namespace gdn {

// Status codes written to the device status word (bitwise OR).
enum : unsigned int {
  kStatusOk = 0u,
  kStatusTmaTimeout = 1u,
  kStatusMmaTimeout = 2u,
  kStatusBadSeqlens = 4u,   // cu_seqlens not non-decreasing within [0, total_tokens]
  kStatusSelftestWait = 16u,   // the wait of the bounded-wait self-test ran out
};

// Upper bound on any spin on an mbarrier, in nanoseconds of %globaltimer.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
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

// try_wait with a suspend-time hint: a thread whose phase is not complete
// sleeps (up to the hint) instead of re-polling, leaving its sub-partition's
// issue slots to the warps that work.
#ifndef GDN_WAIT_HINT_NS
#define GDN_WAIT_HINT_NS 20000
#endif
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "n"(GDN_WAIT_HINT_NS)
      : "memory");
  return ok != 0;
}

// Bounded wait on the given phase parity.  Returns false when the limit ran
// out; the caller records an error status and leaves its loop.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (globaltimer_ns() - t0 > limit_ns) return false;
  }
}

// Plain arrival (release at CTA scope) by the calling thread.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Bounded wait that also gives up as soon as another thread of the CTA has
// raised `abort`, so that one timed-out wait ends every role's loop after at
// most one more limit.  Returns 1 when the phase completed, 0 when another
// thread raised `abort`, -1 when this thread's own limit ran out (it then
// raises `abort`).
__device__ __forceinline__ int mbar_wait_or_abort(uint64_t* bar, uint32_t parity,
                                                  volatile int* abort,
                                                  unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return 1;
  const unsigned long long t0 = globaltimer_ns();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity)) return 1;
    if (*abort) return 0;
    if (globaltimer_ns() - t0 > limit_ns) {
      *abort = 1;
      return -1;
    }
  }
}

// One lane of a converged warp (elect.sync); tcgen05.mma and commit are
// issued by that lane.
// Named barriers (ids 1-15; 0 is __syncthreads): `count` threads, whole warps.
// named_arrive signals without waiting; named_sync signals and waits.
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}
__device__ __forceinline__ void named_arrive(int id, int count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, e;\n\t}"
      : "=r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------- proxies
// Make generic-proxy shared-memory writes visible to the async proxy
// (UMMA operand reads, TMA writes).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- TMA
// 3-D tiled bulk tensor load global -> shared, completion counted in bytes on
// an mbarrier.  Coordinates are innermost first.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const void* tmap, uint64_t* bar,
                                            int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}

// ---------------------------------------------------------------- tcgen05
// TMEM allocation: executed by one full warp; the base address is written to
// shared memory.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, bf16 inputs, fp32 accumulate. Issued by one thread.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same UMMA issued by one elected lane of a converged warp: every lane
// executes the instruction sequence, only the elected one issues, and the warp
// never diverges (no reconvergence after the issue).
__device__ __forceinline__ void umma_bf16_elect(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p, e;\n\t.reg .b32 r;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit_elect(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .pred e;\n\t.reg .b32 r;\n\t"
      "elect.sync r|e, 0xffffffff;\n\t"
      "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Arrive on an mbarrier once every previously issued tcgen05 op of this thread completes.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 columns of 32-bit TMEM words: thread i of the warp receives
// lane (quadrant*32 + i), columns [col, col+32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&r)[32]) {
  uint32_t* u = reinterpret_cast<uint32_t*>(r);
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(u[0]), "=r"(u[1]), "=r"(u[2]), "=r"(u[3]), "=r"(u[4]), "=r"(u[5]), "=r"(u[6]),
        "=r"(u[7]), "=r"(u[8]), "=r"(u[9]), "=r"(u[10]), "=r"(u[11]), "=r"(u[12]),
        "=r"(u[13]), "=r"(u[14]), "=r"(u[15]), "=r"(u[16]), "=r"(u[17]), "=r"(u[18]),
        "=r"(u[19]), "=r"(u[20]), "=r"(u[21]), "=r"(u[22]), "=r"(u[23]), "=r"(u[24]),
        "=r"(u[25]), "=r"(u[26]), "=r"(u[27]), "=r"(u[28]), "=r"(u[29]), "=r"(u[30]),
        "=r"(u[31])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------- descriptors
// Shared-memory matrix descriptor, 128-byte swizzle.  Start address, leading
// byte offset (LBO) and stride byte offset (SBO) are encoded >> 4; bit 46 is
// the sm_100 descriptor version; bits 61-63 = 2 select SWIZZLE_128B.
//  * K-major operand: rows of 128 B (64 bf16 along K), 8-row groups SBO apart.
//  * MN-major operand: 128 B lines of 64 MN-contiguous elements, one line per
//    K index, 8-line groups SBO apart, 64-element MN blocks LBO apart.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// Descriptor of the same operand advanced by `byte_off` bytes (k-steps):
// adds to the 14-bit start-address field, which cannot carry for shared-memory
// addresses below 256 KiB.
__device__ __forceinline__ uint64_t sdesc_add(uint64_t desc, uint32_t byte_off) {
  return desc + static_cast<uint64_t>(byte_off >> 4);
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 D.
// a_mn / b_mn select MN-major operands.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, int a_mn, int b_mn) {
  return (1u << 4)                               // D format: f32
         | (1u << 7)                             // A format: bf16
         | (1u << 10)                            // B format: bf16
         | (static_cast<uint32_t>(a_mn) << 15)   // A major
         | (static_cast<uint32_t>(b_mn) << 16)   // B major
         | (static_cast<uint32_t>(N >> 3) << 17)  // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24); // M / 16
}

// Byte offset of (row, 16-byte chunk) inside a 128-byte-swizzled tile whose
// base is 1024-byte aligned.
__device__ __forceinline__ uint32_t sw128_off(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace gdn
