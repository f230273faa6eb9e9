// Shared-memory staging helpers for the decode kernels.
//
// The decode kernels put every operand a CTA needs (weight tile, scales,
// biases, activation rows) in flight at CTA start with 16-byte cp.async
// copies, then compute from shared memory.  Each CTA therefore keeps its whole
// working set (tens of KB) outstanding against HBM, which is what a
// bandwidth-bound GEMV needs, and the compute phase never waits on L2.
#pragma once
#include "common.cuh"

namespace fmoe {

// Row stride in shared memory for rows of `row_bytes` (a multiple of 32) that
// lanes (g = lane/4, t = lane%4) read `access` bytes at a time:
//   8-byte reads: a half-warp covers rows g..g+3 (32 B each) -> stride = 8 or
//                 24 words mod 32 banks keeps them on distinct banks;
//   16-byte reads: a quarter-warp covers 2 rows (64 B each) -> 16 words mod 32.
__host__ __device__ inline int smem_stride(int row_bytes, int access) {
  const int w = row_bytes / 4;
  for (int p = 0; p < 32; p += 4) {
    const int m = (w + p) % 32;
    if (access == 8 ? (m == 8 || m == 24) : (m == 16)) return row_bytes + 4 * p;
  }
  return row_bytes;
}

__host__ __device__ inline size_t align16(size_t v) { return (v + 15) & ~size_t(15); }

// Programmatic dependent launch: wait for the preceding kernel in the stream
// (no-op when launched without the attribute), and allow the next one to be
// scheduled early.
__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void griddep_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory"); }

__device__ __forceinline__ uint4 lds_u4(const void* p) { return *static_cast<const uint4*>(p); }

// B fragments of group gi for token row n = g of a staged activation tile
// (rows `xs` bytes apart); rows >= nv contribute zeros.
__device__ __forceinline__ BFrag4 stage_bfrag4(const uint8_t* xsm, int XS, int nv, int gi, int g, int t) {
  uint4 lo = make_uint4(0, 0, 0, 0), hi = lo;
  if (g < nv) {
    const uint8_t* p = xsm + g * XS + gi * 128 + 32 * t;
    lo = lds_u4(p);
    hi = lds_u4(p + 16);
  }
  return make_bfrag4(lo, hi);
}

}  // namespace fmoe

namespace fmoe {

// ---------------------------------------------------------------------------
// TMA bulk copies (cp.async.bulk, no tensor map, no multicast) tracked by a
// shared-memory mbarrier.  One instruction moves a whole row or tile, so a CTA
// keeps tens of KB in flight without per-thread request slots.  Both
// addresses 16-byte aligned, size a multiple of 16.

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Makes the initialised barrier visible to the async (TMA) proxy.
__device__ __forceinline__ void mbar_fence_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
// Plain arrival (no transaction bytes), e.g. a consumer releasing a stage.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Prefetch [src, src + bytes) into L2 without touching shared memory.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;\n" ::"l"(src), "r"(bytes) : "memory");
}

// Bounded wait for phase `parity` of `bar`.  Every wait in this library gives
// up after kMaxWaitIters polls (each poll itself blocks for a short
// hardware-defined interval), records FMOE_ERR_TIMEOUT with a site code in
// *status and returns false, so a lost completion surfaces as an error status
// instead of a hung GPU.
constexpr int kMaxWaitIters = 1 << 22;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* status, int site) {
  const uint32_t a = smem_u32(bar);
  for (int i = 0; i < kMaxWaitIters; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  if (status) atomicCAS(status, 0, site);
  return false;
}

}  // namespace fmoe
