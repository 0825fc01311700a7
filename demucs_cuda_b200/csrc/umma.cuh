// sm_100a primitives: mbarriers, TMA tensor loads, tcgen05 (UMMA) MMA / TMEM.
//
// Conventions used by every tensor-core kernel in this library:
//  * operand tiles live in shared memory in the K-major, 128-byte-swizzled canonical
//    layout: rows of 64 fp16 (128 B), 8-row atoms of 1024 B stacked along M/N, 16-byte
//    chunk index XOR (row & 7); tile bases are 1024-byte aligned;
//  * one elected thread issues tcgen05.mma (cta_group::1, kind::f16, fp32 accumulate in
//    TMEM) and tcgen05.commit arrives on an mbarrier when the MMAs finish;
//  * every wait on an mbarrier is bounded (mbar_wait): after kWaitNs it records a bit in
//    g_dev_fault and gives up, so a protocol error ends the kernel instead of hanging the
//    GPU (the host reads the word with dcb_device_fault()).
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "common.cuh"

namespace dcb {

enum : uint32_t {
  kFaultFull = 1u,      // operand stage never filled
  kFaultEmpty = 2u,     // operand stage never released
  kFaultDone = 4u,      // accumulator never completed
  kFaultAttn = 8u,      // attention pipeline
};

static __device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

static __device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}
static __device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
static __device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
static __device__ __forceinline__ void mbar_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
static __device__ __forceinline__ bool mbar_try(uint64_t *bar, uint32_t parity) {
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
static __device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}
static __device__ __forceinline__ bool fault_pending() {
  return *(volatile uint32_t *)&g_dev_fault != 0;
}
// Bounded wait: false (and a fault bit) if the phase has not completed within
// g_wait_ns of wall-clock time, or at once if another CTA already recorded a fault, so a
// protocol error ends every CTA of the grid quickly instead of hanging the GPU.  The limit
// is 2 s (legitimate waits are microseconds); the host may shorten it (option
// "wait_limit_ms") so that a test can make a wait expire quickly.
// (g_wait_ns and the test hook g_test_withhold are defined in common.cuh.)
static __device__ __forceinline__ uint64_t wait_limit_ns() {
  return *(volatile uint64_t *)&g_wait_ns;
}
static __device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, uint32_t fault) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = global_ns(), lim = wait_limit_ns();
  for (uint32_t i = 1;; i++) {
    if (mbar_try(bar, parity)) return true;
    if ((i & 255u) == 0) {
      if (fault_pending()) return false;
      if (global_ns() - t0 > lim) {
        atomicOr(&g_dev_fault, fault);
        return false;
      }
    }
  }
}

// Warp-uniform outcome of a wait: tcgen05.ld / st (and the epilogues built on them) are
// .sync.aligned, so all 32 lanes must take the same path after a wait; a lane that gave up
// at the time limit while another saw the phase complete would otherwise leave the warp
// divergent in front of a TMEM access.  Every lane of the warp must call it.
static __device__ __forceinline__ bool warp_all(bool ok) { return __all_sync(0xffffffffu, ok); }

// Fault-path drain: wait (bounded by the same limit, but not cut short by the fault word)
// for a phase that this CTA's own copies complete, so that no copy is still landing in
// shared memory when the CTA exits.  Returns whether the phase completed.
static __device__ __forceinline__ bool mbar_drain(uint64_t *bar, uint32_t parity) {
  const uint64_t t0 = global_ns(), lim = wait_limit_ns();
  while (!mbar_try(bar, parity)) {
    if (global_ns() - t0 > lim) return false;
  }
  return true;
}

// generic-proxy smem writes -> visible to the async proxy (UMMA operand reads)
static __device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// TMA: tiled tensor loads into shared memory, completion counted on an mbarrier
static __device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map,
                                                   uint64_t *bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}
static __device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map,
                                                   uint64_t *bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"((uint64_t)map), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
static __device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}

// ---------------------------------------------------------------- tcgen05
static __device__ __forceinline__ void tmem_alloc(uint32_t *slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
static __device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
static __device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
static __device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
static __device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] . B[smem]^T, fp16 x fp16 -> fp32
static __device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` when every previously issued tcgen05.mma of this thread has completed
static __device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32-bit, 16 consecutive columns per thread
static __device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
// 32 lanes x 32-bit, 16 consecutive columns per thread, registers -> TMEM
static __device__ __forceinline__ void tmem_st16(uint32_t taddr, const float (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15]))
      : "memory");
}
// 32 lanes x 32-bit, 4 consecutive columns per thread (load and store)
static __device__ __forceinline__ void tmem_ld4(uint32_t taddr, float (&v)[4]) {
  uint32_t r0, r1, r2, r3;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(taddr)
               : "memory");
  v[0] = __uint_as_float(r0);
  v[1] = __uint_as_float(r1);
  v[2] = __uint_as_float(r2);
  v[3] = __uint_as_float(r3);
}
static __device__ __forceinline__ void tmem_st4(uint32_t taddr, const float (&v)[4]) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x4.b32 [%0], {%1,%2,%3,%4};" ::"r"(taddr),
               "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])),
               "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3]))
               : "memory");
}
// 32 lanes x 32-bit, one column per thread
static __device__ __forceinline__ float tmem_ld1(uint32_t taddr) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr)
               : "memory");
  return __uint_as_float(r);
}
static __device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}
static __device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major SWIZZLE_128B tile (sm100 format):
// start address >> 4 in bits 0-13, leading byte offset (unused for swizzled K-major,
// set to 1) in 16-29, stride byte offset 1024 B (>> 4 = 64) in 32-45, version 1 in
// bits 46-47, layout type SWIZZLE_128B (2) in bits 61-63.
static __device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3fffu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)64u << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)2u << 61;
  return d;
}

// Instruction descriptor, kind::f16: fp32 accumulator (bits 4-5 = 1), A and B fp16
// (formats 0), both K-major, N >> 3 in bits 17-22, M >> 4 in bits 24-28.
static __host__ __device__ constexpr uint32_t idesc_f16_f32(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// byte offset of the 16-byte chunk `c` (0..7) of row `r` inside a SW128 K-major tile
static __device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
}

static __device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b,
                                                    uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c),
               "r"(d)
               : "memory");
}

}  // namespace dcb
