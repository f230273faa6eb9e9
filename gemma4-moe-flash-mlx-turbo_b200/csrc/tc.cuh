// tcgen05 / TMA building blocks shared by the tensor-core kernels (prefill
// grouped GEMMs, the many-token router): TMA tile loads, bounded mbarrier
// waits, shared-memory and instruction descriptors, MMA issue and commit,
// TMEM loads; and the host-side tensor-map encoder.
#pragma once
#include <cuda.h>
#include <cudaTypedefs.h>
#include "common.cuh"
#include "internal.h"
#include "stage.cuh"

namespace fmoe {
namespace tc {

__device__ __forceinline__ void tma2d(void* dst, const CUtensorMap* m, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];\n" ::"r"(
          smem_u32(dst)),
      "l"(m), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void tma3d(void* dst, const CUtensorMap* m, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];\n" ::"r"(smem_u32(dst)),
      "l"(m), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ bool try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// Bounded wait; after a failure anywhere in the CTA every wait returns at once.
__device__ __forceinline__ bool pwait(uint64_t* bar, uint32_t parity, volatile int* failed, int* status, int site) {
  if (*failed) return false;
  for (int i = 0; i < kMaxWaitIters; ++i) {
    if (try_wait(bar, parity)) return true;
    if ((i & 1023) == 1023 && *failed) return false;
  }
  *failed = 1;
  if (status) atomicCAS(status, 0, site);
  return false;
}
// pwait for warps that wait long (a whole tile or item): after a short spin the
// poll backs off by `ns` nanoseconds, so the waiting warps leave the issue slots
// to the warps doing the work.  Bounded by the same poll count as pwait.
__device__ __forceinline__ bool pwait_sleep(uint64_t* bar, uint32_t parity, volatile int* failed, int* status, int site,
                                            unsigned ns) {
  if (*failed) return false;
  for (int i = 0; i < kMaxWaitIters; ++i) {
    if (try_wait(bar, parity)) return true;
    if (i >= 8) __nanosleep(ns);
    if ((i & 255) == 255 && *failed) return false;
  }
  *failed = 1;
  if (status) atomicCAS(status, 0, site);
  return false;
}
// Bounded wait that ignores the failure flag (draining copies / MMAs in flight).
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
  for (int i = 0; i < kMaxWaitIters && !try_wait(bar, parity); ++i) {
  }
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row atoms of
// 1024 bytes (SBO 1024, LBO unused = 1), descriptor version 1.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF) | (1ull << 16) | (64ull << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::f16: D f32, A / B bf16 K-major, M 128, N = n.
__device__ __forceinline__ uint32_t idesc_n(int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

// D (TMEM) += A (shared memory descriptor) . B (shared memory descriptor)^T
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory"); }
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

}  // namespace tc

// Host: encode a tiled tensor map through the driver entry point (resolved at
// run time, so the library does not link the driver library).  The OOB fill
// is zero; `what` names the tensor in the error text.
int encode(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
           const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle sw, const char* what);

}  // namespace fmoe
