// Prefill MoE (many tokens): grouped GEMMs over token-sorted expert tiles on
// the 5th-generation tensor cores (tcgen05.mma, accumulators in TMEM), the
// batched form of Gemma4MoeBlock::forward's expert loop (src/model/moe.rs:
// 424-465: gate / up quantized_matmul, GELU-tanh gating, down, weighted
// combine).
//
//   route    router + top-k + per-expert pair lists (the decode router kernels)
//   gather   X_sorted[i] = x[token of pair i] (rows grouped by expert)
//   GEMM1    act = gelu(X_sorted . Wg_e^T) * (X_sorted . Wu_e^T)   per expert tile
//   GEMM2    Y_sorted = act . Wd_e^T                                 per expert tile
//   combine  y[t] = sum over the token's k slots of w * Y_sorted[row]  (slot order)
//
// GEMM kernel (persistent, one CTA per SM, 10 warps):
//   warp 0   producer: TMA tiles of A (128 sorted rows x 64 K, bf16, 128-byte
//            swizzle) and of the packed 4-bit weights (3-D tensor map over the
//            expert table), 1-D bulk copies of the step's scale / bias rows
//   warp 1   MMA issuer: 4 x tcgen05.mma (M 128, N 256, K 16) per K tile into
//            one of two TMEM accumulators; tcgen05.commit releases the stage
//   warps 2-5  dequantise the weight tile into the canonical K-major
//            128-byte-swizzled bf16 layout: w = bf16(fma(s, q, b)) per element
//   warps 6-9  epilogue: tcgen05.ld of the accumulator, GELU gating (GEMM1) or
//            plain bf16 store (GEMM2)
// Within every 8-element word of K the columns are stored in the order
// 0 4 1 5 2 6 3 7: a 4-bit word's nibbles j and j+4 then form one bf16 pair
// with a single AND/OR, so weights dequantise two at a time.  The gather
// writes X in that order, GEMM1's epilogue writes act in it; the dot products
// are unchanged.  Scale / bias rows of the expert table (88 bytes for 44
// groups) break TMA's 16-byte stride rule, so fmoe_moe_prefill_prepare keeps
// a transposed copy ([group][row]) from which one K tile's rows are contiguous.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <algorithm>
#include <mutex>
#include "internal.h"
#include "common.cuh"
#include "stage.cuh"

namespace fmoe {
namespace pf {

constexpr int BM = 128, BN = 256, BK = 64;
constexpr int NS = 3;
constexpr int A_BYTES = BM * BK * 2;   // 16 KB
constexpr int WB_BYTES = BN * BK * 2;  // 32 KB
constexpr int WQ_BYTES = BN * BK / 2;  // 8 KB
constexpr int SC_BYTES = 1024;         // scale | bias of 256 rows
constexpr int OFF_A = 0, OFF_WB = A_BYTES, OFF_WQ = OFF_WB + WB_BYTES, OFF_SC = OFF_WQ + WQ_BYTES;
constexpr int STAGE = OFF_SC + SC_BYTES;  // 57 KB, a multiple of 1024
constexpr int OFF_BAR = NS * STAGE;
constexpr int SMEM = OFF_BAR + 256 + 1024;  // + alignment slack for the 1024-byte swizzle atoms
constexpr int THREADS = 320;
constexpr int TMEM_COLS = 512;              // two 256-column fp32 accumulators
static_assert(STAGE % 1024 == 0, "stage alignment");

struct alignas(64) Maps {
  CUtensorMap a;   // A rows (bf16 [P][K], 128-byte swizzle, box 64 x 128)
  CUtensorMap w0;  // packed weights (u8 [E][rows][K/2], box 32 x 128 (GEMM1) / 256 (GEMM2) x 1)
  CUtensorMap w1;  // GEMM1: the up projection
};

struct Args {
  const int4* tiles;     // (expert, first sorted row, rows, 0)
  const int* ntiles;
  const bf16* prep;      // transposed scales / biases, expert stride eps elements
  int64_t eps;
  int64_t off_s0, off_b0, off_s1, off_b1;  // element offsets of this GEMM's arrays in an expert's block
  int H, I, E;
  bf16* out;             // GEMM1: act [P][I] (permuted words); GEMM2: Y [P][H]
  int* status;
};

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
  atomicCAS(status, 0, site);
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
// Instruction descriptor, kind::f16: D f32, A / B bf16 K-major, M 128, N 256.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) | ((uint32_t)(BM >> 4) << 24);

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, {%5, %6, %7, %8}, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(acc), "r"(0), "r"(0), "r"(0), "r"(0));
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

// Two bf16 from two floats, low half first.
__device__ __forceinline__ uint32_t bf2(float lo, float hi) { return pack_bf16x2(lo, hi); }

template <int MODE>  // 0: gate|up + GELU gating, 1: down
__global__ void __launch_bounds__(THREADS, 1) tc_gemm_kernel(const __grid_constant__ Maps maps, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
  uint64_t* deqd = full + NS;
  uint64_t* mmad = deqd + NS;
  uint64_t* accf = mmad + NS;
  uint64_t* acce = accf + 2;
  volatile int* failed = reinterpret_cast<volatile int*>(acce + 2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2) + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = MODE == 0 ? a.H : a.I;
  const int NJ = MODE == 0 ? (a.I + 127) / 128 : a.H / BN;
  const int NK = K / BK;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&deqd[s], 4);
      mbar_init(&mmad[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&accf[s], 1);
      mbar_init(&acce[s], 4);
    }
    *failed = 0;
    mbar_fence_init();
  }
  if (warp == 1) {  // the whole warp allocates the accumulators
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int nitems = __ldg(a.ntiles) * NJ;

  if (warp == 0) {
    // ---- producer
    if (lane == 0) {
      int q = 0;
      for (int it = blockIdx.x; it < nitems; it += gridDim.x) {
        const int4 tl = __ldg(a.tiles + it / NJ);
        const int j = it % NJ, e = tl.x, row0 = tl.y;
        const int rows_ok = MODE == 0 ? min(128, a.I - j * 128) : BN;
        const bf16* pe = a.prep + (int64_t)e * a.eps;
        for (int kt = 0; kt < NK; ++kt, ++q) {
          const int s = q % NS;
          if (q >= NS) pwait(&mmad[s], (uint32_t)((q / NS) - 1) & 1u, failed, a.status, 301);
          if (*failed) break;
          uint8_t* st = smem + s * STAGE;
          const int sc_bytes = MODE == 0 ? 4 * rows_ok * 2 : 2 * BN * 2;
          mbar_arrive_expect_tx(&full[s], (uint32_t)(A_BYTES + WQ_BYTES + sc_bytes));
          tma2d(st + OFF_A, &maps.a, kt * BK, row0, &full[s]);
          if (MODE == 0) {
            tma3d(st + OFF_WQ, &maps.w0, kt * 32, j * 128, e, &full[s]);
            tma3d(st + OFF_WQ + WQ_BYTES / 2, &maps.w1, kt * 32, j * 128, e, &full[s]);
            const int64_t r = (int64_t)kt * a.I + j * 128;
            bulk_g2s(st + OFF_SC, pe + a.off_s0 + r, rows_ok * 2, &full[s]);
            bulk_g2s(st + OFF_SC + 256, pe + a.off_b0 + r, rows_ok * 2, &full[s]);
            bulk_g2s(st + OFF_SC + 512, pe + a.off_s1 + r, rows_ok * 2, &full[s]);
            bulk_g2s(st + OFF_SC + 768, pe + a.off_b1 + r, rows_ok * 2, &full[s]);
          } else {
            tma3d(st + OFF_WQ, &maps.w0, kt * 32, j * BN, e, &full[s]);
            const int64_t r = (int64_t)kt * a.H + j * BN;
            bulk_g2s(st + OFF_SC, pe + a.off_s0 + r, BN * 2, &full[s]);
            bulk_g2s(st + OFF_SC + 512, pe + a.off_b0 + r, BN * 2, &full[s]);
          }
        }
        if (*failed) break;
      }
      // every copy issued lands before the CTA ends
      for (int k = q - NS < 0 ? 0 : q - NS; k < q; ++k) drain_wait(&full[k % NS], (uint32_t)(k / NS) & 1u);
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      int q = 0, n = 0;
      for (int it = blockIdx.x; it < nitems; it += gridDim.x, ++n) {
        const int ab = n & 1;
        if (n >= 2) pwait(&acce[ab], (uint32_t)((n / 2) - 1) & 1u, failed, a.status, 302);
        tc_fence_after();
        const uint32_t d = tmem + ab * BN;
        for (int kt = 0; kt < NK; ++kt, ++q) {
          const int s = q % NS;
          pwait(&deqd[s], (uint32_t)(q / NS) & 1u, failed, a.status, 303);
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * STAGE + OFF_A), sb = smem_u32(smem + s * STAGE + OFF_WB);
          if (!*failed) {
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) mma_bf16(d, sw128_desc(sa + 32 * k), sw128_desc(sb + 32 * k), (kt | k) != 0);
          }
          mma_commit(&mmad[s]);
        }
        mma_commit(&accf[ab]);
      }
      if (n > 0) drain_wait(&accf[(n - 1) & 1], (uint32_t)((n - 1) / 2) & 1u);  // the last MMAs are done
    }
  } else if (warp < 6) {
    // ---- dequantisers: rows dt and dt + 128 of every weight tile
    const int dt = threadIdx.x - 64;
    int q = 0;
    for (int it = blockIdx.x; it < nitems; it += gridDim.x) {
      const int j = it % NJ;
      for (int kt = 0; kt < NK; ++kt, ++q) {
        const int s = q % NS;
        pwait(&full[s], (uint32_t)(q / NS) & 1u, failed, a.status, 304);
        uint8_t* st = smem + s * STAGE;
        const bf16* sc = reinterpret_cast<const bf16*>(st + OFF_SC);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int rr = dt + 128 * h;
          bool ok;
          float sv, bv;
          if (MODE == 0) {
            ok = j * 128 + (rr & 127) < a.I;
            sv = ok ? bf2f(sc[h * 256 + (rr & 127)]) : 0.f;
            bv = ok ? bf2f(sc[h * 256 + 128 + (rr & 127)]) : 0.f;
          } else {
            ok = true;
            sv = bf2f(sc[rr]);
            bv = bf2f(sc[BN + rr]);
          }
          const uint4 w0 = *reinterpret_cast<const uint4*>(st + OFF_WQ + rr * 32);
          const uint4 w1 = *reinterpret_cast<const uint4*>(st + OFF_WQ + rr * 32 + 16);
          const uint32_t ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
          const __nv_bfloat162 s2 = __floats2bfloat162_rn(sv, sv), b2 = __floats2bfloat162_rn(bv, bv);
          const __nv_bfloat162 off = __floats2bfloat162_rn(128.f, 128.f);
          uint8_t* wrow = st + OFF_WB + rr * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            uint32_t o[4];
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
              // nibbles jj and jj+4 of the word -> bf16 (128 + q) pair -> q -> fma(q, s, b)
              const uint32_t v = and_or(ww[c] >> (4 * jj), 0x000F000Fu, 0x43004300u);
              __nv_bfloat162 qv = __hsub2(*reinterpret_cast<const __nv_bfloat162*>(&v), off);
              __nv_bfloat162 r = __hfma2(qv, s2, b2);
              o[jj] = ok ? *reinterpret_cast<uint32_t*>(&r) : 0u;
            }
            *reinterpret_cast<uint4*>(wrow + ((c ^ (rr & 7)) << 4)) = make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // generic writes -> tensor-core reads
        __syncwarp();
        if (lane == 0) mbar_arrive(&deqd[s]);
      }
    }
  } else {
    // ---- epilogue: TMEM lanes 32 * (warp % 4) ..
    const int qw = warp & 3, row = qw * 32 + lane;
    int n = 0;
    for (int it = blockIdx.x; it < nitems; it += gridDim.x, ++n) {
      const int4 tl = __ldg(a.tiles + it / NJ);
      const int j = it % NJ, row0 = tl.y, nrows = tl.z;
      const int ab = n & 1;
      pwait(&accf[ab], (uint32_t)(n / 2) & 1u, failed, a.status, 305);
      tc_fence_after();
      const uint32_t ta = tmem + ((uint32_t)(qw * 32) << 16) + ab * BN;
      const bool live = row < nrows && !*failed;
      if (MODE == 0) {
#pragma unroll 1
        for (int cc = 0; cc < 8; ++cc) {
          float g[16], u[16];
          tmem_ld16(ta + cc * 16, g);
          tmem_ld16(ta + 128 + cc * 16, u);
          tmem_ld_wait();
          const int col0 = j * 128 + cc * 16;
          if (live && col0 < a.I) {
            float act[16];
#pragma unroll
            for (int i = 0; i < 16; ++i) act[i] = gelu_tanh(round_bf(g[i])) * round_bf(u[i]);
            // store in the permuted word order: position 8w + 2jj + h holds element 8w + jj + 4h
            uint32_t o[8];
#pragma unroll
            for (int w = 0; w < 2; ++w)
#pragma unroll
              for (int jj = 0; jj < 4; ++jj) o[4 * w + jj] = bf2(act[8 * w + jj], act[8 * w + jj + 4]);
            uint4* dst = reinterpret_cast<uint4*>(a.out + (int64_t)(row0 + row) * a.I + col0);
            dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
            dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
          }
        }
      } else {
#pragma unroll 1
        for (int cc = 0; cc < BN / 16; ++cc) {
          float v[16];
          tmem_ld16(ta + cc * 16, v);
          tmem_ld_wait();
          if (live) {
            uint32_t o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = bf2(v[2 * i], v[2 * i + 1]);
            uint4* dst = reinterpret_cast<uint4*>(a.out + (int64_t)(row0 + row) * a.H + j * BN + cc * 16);
            dst[0] = make_uint4(o[0], o[1], o[2], o[3]);
            dst[1] = make_uint4(o[4], o[5], o[6], o[7]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acce[ab]);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(TMEM_COLS) : "memory");
}

// ---------------------------------------------------------------------------
// small kernels

// Transposed scale / bias copy of every expert: [gs | gb | us | ub] as
// [G1][I], then [ds | db] as [G2][H] (bf16), expert stride eps elements.
__global__ void prep_kernel(ExpertsDev ex, bf16* __restrict__ prep, int64_t eps) {
  const int e = blockIdx.y;
  const uint8_t* base = ex.base + (int64_t)e * ex.stride;
  const int G1 = ex.H / 64, G2 = ex.I / 64;
  bf16* pe = prep + (int64_t)e * eps;
  const int n1 = ex.I, n2 = ex.H;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < n1 + n2; r += gridDim.x * blockDim.x) {
    if (r < n1) {
      const int arr[4] = {1, 2, 4, 5};
      for (int t = 0; t < 4; ++t) {
        const bf16* src = reinterpret_cast<const bf16*>(base + ex.off[arr[t]]) + (int64_t)r * G1;
        for (int g = 0; g < G1; ++g) pe[(int64_t)t * G1 * n1 + (int64_t)g * n1 + r] = src[g];
      }
    } else {
      const int rr = r - n1;
      for (int t = 0; t < 2; ++t) {
        const bf16* src = reinterpret_cast<const bf16*>(base + ex.off[7 + t]) + (int64_t)rr * G2;
        for (int g = 0; g < G2; ++g) pe[4LL * G1 * n1 + (int64_t)t * G2 * n2 + (int64_t)g * n2 + rr] = src[g];
      }
    }
  }
}

// Tile list: per expert with n > 0 pairs, ceil(n / 128) tiles of sorted rows.
__global__ void tiles_kernel(const int32_t* __restrict__ start, int E, int4* __restrict__ tiles, int* __restrict__ ntiles) {
  if (threadIdx.x != 0) return;
  int n = 0;
  for (int e = 0; e < E; ++e) {
    const int r0 = start[e], r1 = start[e + 1];
    for (int r = r0; r < r1; r += BM) tiles[n++] = make_int4(e, r, min(BM, r1 - r), 0);
  }
  *ntiles = n;
}

// X_sorted[i] = x[pairs[i] / k] with each 8-column word in the order 0 4 1 5 2 6 3 7;
// inv[pairs[i]] = i.
__global__ void gather_kernel(const bf16* __restrict__ x, const int32_t* __restrict__ pairs, int P, int k, int H,
                              bf16* __restrict__ xs, int32_t* __restrict__ inv) {
  const int words = H / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)P * words;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / words), w = (int)(i % words);
    const int p = pairs[r];
    if (w == 0) inv[p] = r;
    const uint4 v = *reinterpret_cast<const uint4*>(x + (int64_t)(p / k) * H + 8 * w);
    // elements e0..e7 in (lo, hi) halves of v.x .. v.w -> e0 e4 e1 e5 e2 e6 e3 e7
    const uint32_t o0 = __byte_perm(v.x, v.z, 0x5410), o1 = __byte_perm(v.x, v.z, 0x7632);
    const uint32_t o2 = __byte_perm(v.y, v.w, 0x5410), o3 = __byte_perm(v.y, v.w, 0x7632);
    *reinterpret_cast<uint4*>(xs + (int64_t)r * H + 8 * w) = make_uint4(o0, o1, o2, o3);
  }
}

// y[t] = bf16(sum over slots of w[t, slot] * Y[inv[t * k + slot]]) in slot order.
__global__ void combine_kernel(const bf16* __restrict__ Y, const int32_t* __restrict__ inv,
                               const float* __restrict__ wts, int T, int k, int H, bf16* __restrict__ y) {
  const int words = H / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)T * words;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / words), w = (int)(i % words);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < k; ++s) {
      const float wv = wts[t * k + s];
      const uint4 v = *reinterpret_cast<const uint4*>(Y + (int64_t)inv[t * k + s] * H + 8 * w);
      const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] = fmaf(wv, bf16lo(vv[q]), acc[2 * q]);
        acc[2 * q + 1] = fmaf(wv, bf16hi(vv[q]), acc[2 * q + 1]);
      }
    }
    *reinterpret_cast<uint4*>(y + (int64_t)t * H + 8 * w) =
        make_uint4(bf2(acc[0], acc[1]), bf2(acc[2], acc[3]), bf2(acc[4], acc[5]), bf2(acc[6], acc[7]));
  }
}

}  // namespace pf

// ---------------------------------------------------------------------------
// host side

namespace {

int64_t prep_eps(const ExpertsDev& d) { return 4LL * (d.H / 64) * d.I + 2LL * (d.I / 64) * d.H; }

// The driver's tensor-map encoder, resolved through the runtime (the library
// does not link the driver library, so it loads on machines without one).
PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

int encode(CUtensorMap* m, CUtensorMapDataType dt, int rank, const void* base, const cuuint64_t* dims,
           const cuuint64_t* strides, const cuuint32_t* box, CUtensorMapSwizzle sw, const char* what) {
  cuuint32_t es[3] = {1, 1, 1};
  const auto enc = tmap_encoder();
  if (!enc) return set_error(FMOE_ERR_CUDA, "prefill: the driver's tensor-map encoder is unavailable");
  const CUresult r = enc(m, dt, rank, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FMOE_ERR_CUDA, "prefill: tensor map for %s failed (%d)", what, (int)r);
  return FMOE_OK;
}

int check_prefill(const ExpertsDev& d) {
  if (d.H % 256 || d.I % 64 || d.H > 8192 || d.E < 1)
    return set_error(FMOE_ERR_UNSUPPORTED, "prefill: hidden %d (multiple of 256), intermediate %d (multiple of 64)",
                     d.H, d.I);
  if (d.stride % 16 || !aligned(d.base, 16))
    return set_error(FMOE_ERR_ALIGN, "prefill: expert table must be 16-byte aligned with a 16-byte stride");
  for (int j = 0; j < 9; ++j)
    if (d.off[j] % 16) return set_error(FMOE_ERR_ALIGN, "prefill: expert tensor offsets must be 16-byte aligned");
  return FMOE_OK;
}

struct PfWs {
  WsHead h;
  RouterWs r;
  int32_t* ids;
  float* wts;
  RouteMeta m;
  int4* tiles;
  int* ntiles;
  int32_t* inv;
  bf16* xs;
  bf16* act;
  bf16* ys;
};

size_t carve_pf(Carver& c, int64_t T, const fmoe_router_t* r, const ExpertsDev& d, PfWs* w) {
  PfWs p;
  p.h = carve_head(c);
  carve_router(c, T, r, p.h, &p.r);
  const int64_t P = T * r->top_k;
  p.ids = c.take<int32_t>(P);
  p.wts = c.take<float>(P);
  p.m.start = c.take<int32_t>(d.E + 1);
  p.m.pairs = c.take<int32_t>(P);
  p.m.unique = c.take<int32_t>(d.E);
  p.m.num_unique = c.take<int32_t>(1);
  p.m.work_len = (int)std::min<int64_t>(P, d.E);
  p.m.work = c.take<int4>(p.m.work_len);
  p.tiles = c.take<int4>(P / pf::BM + d.E + 1);
  p.ntiles = c.take<int>(1);
  p.inv = c.take<int32_t>(P);
  p.xs = c.take<bf16>((size_t)P * d.H);
  p.act = c.take<bf16>((size_t)P * d.I);
  p.ys = c.take<bf16>((size_t)P * d.H);
  if (w) *w = p;
  return c.off;
}

}  // namespace

}  // namespace fmoe

using namespace fmoe;

extern "C" size_t fmoe_moe_prefill_prepare_bytes(const fmoe_experts_t* ex) {
  ExpertsDev d;
  if (to_experts(ex, &d) || check_prefill(d)) return 0;
  return (size_t)prep_eps(d) * d.E * 2;
}

extern "C" int fmoe_moe_prefill_prepare(const fmoe_experts_t* ex, void* prep, size_t bytes, void* stream) {
  ExpertsDev d;
  int rc;
  if ((rc = to_experts(ex, &d)) || (rc = check_prefill(d))) return rc;
  if (!prep || bytes < (size_t)prep_eps(d) * d.E * 2 || !aligned(prep, 16))
    return set_error(FMOE_ERR_WORKSPACE, "prefill_prepare: %zu bytes (16-byte aligned) required",
                     (size_t)prep_eps(d) * d.E * 2);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  {
    ProfScope prof_("prefill_prep_kernel", st);
    pf::prep_kernel<<<dim3((d.I + d.H + 255) / 256, d.E), 256, 0, st>>>(d, static_cast<bf16*>(prep), prep_eps(d));
  }
  return check_launch("prefill_prep_kernel");
}

extern "C" size_t fmoe_moe_prefill_workspace_bytes(int64_t T, const fmoe_router_t* r, const fmoe_experts_t* ex) {
  ExpertsDev d;
  if (T <= 0 || !r || to_experts(ex, &d) || check_prefill(d)) return 0;
  Carver c(nullptr);
  return carve_pf(c, T, r, d, nullptr) + 256;
}

extern "C" int fmoe_moe_prefill(const void* x, int64_t T, const fmoe_router_t* r, const fmoe_experts_t* ex,
                                const void* prep, void* y, int32_t* ids, float* weights, void* workspace,
                                size_t workspace_bytes, void* stream) {
  QW q;
  int rc;
  if ((rc = check_router(r, &q))) return rc;
  ExpertsDev d;
  if ((rc = to_experts(ex, &d)) || (rc = check_prefill(d))) return rc;
  if (!x || !y || !prep) return set_error(FMOE_ERR_INVALID, "prefill: null x / y / prepared scales");
  if (T <= 0) return FMOE_OK;
  if (q.in != d.H || q.out != d.E || d.first != 0)
    return set_error(FMOE_ERR_INVALID, "prefill: router [%d, %d] vs experts %d x hidden %d", q.out, q.in, d.E, d.H);
  if (!aligned(x, 16) || !aligned(y, 16)) return set_error(FMOE_ERR_ALIGN, "prefill: x / y not 16-byte aligned");
  const size_t need = fmoe_moe_prefill_workspace_bytes(T, r, ex);
  if (!workspace || workspace_bytes < need)
    return set_error(FMOE_ERR_WORKSPACE, "prefill: workspace %zu < %zu", workspace_bytes, need);
  const int k = r->top_k;
  const int64_t P = T * k;
  if (P > (1 << 30) / d.H) return set_error(FMOE_ERR_UNSUPPORTED, "prefill: T=%lld too large", (long long)T);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver c(workspace);
  PfWs w;
  carve_pf(c, T, r, d, &w);
  int32_t* ids_out = ids ? ids : w.ids;
  float* w_out = weights ? weights : w.wts;
  // route (builds the per-expert pair lists)
  if ((rc = run_router(static_cast<const bf16*>(x), T, r, q, w.r, ids_out, w_out, nullptr, &w.m, w.h.status, st)))
    return rc;
  {
    ProfScope prof_("prefill_tiles_kernel", st);
    pf::tiles_kernel<<<1, 32, 0, st>>>(w.m.start, d.E, w.tiles, w.ntiles);
  }
  if ((rc = check_launch("prefill_tiles_kernel"))) return rc;
  {
    ProfScope prof_("prefill_gather_kernel", st);
    pf::gather_kernel<<<2 * kNumSMs * 4, 256, 0, st>>>(static_cast<const bf16*>(x), w.m.pairs, (int)P, k, d.H, w.xs,
                                                        w.inv);
  }
  if ((rc = check_launch("prefill_gather_kernel"))) return rc;
  // tensor maps
  pf::Maps m1, m2;
  {
    const cuuint64_t dA[2] = {(cuuint64_t)d.H, (cuuint64_t)P}, sA[1] = {(cuuint64_t)d.H * 2};
    const cuuint32_t bA[2] = {64, 128};
    const cuuint64_t dW[3] = {(cuuint64_t)d.H / 2, (cuuint64_t)d.I, (cuuint64_t)d.E};
    const cuuint64_t sW[2] = {(cuuint64_t)d.H / 2, (cuuint64_t)d.stride};
    const cuuint32_t bW[3] = {32, 128, 1};
    if ((rc = encode(&m1.a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w.xs, dA, sA, bA, CU_TENSOR_MAP_SWIZZLE_128B, "x")) ||
        (rc = encode(&m1.w0, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, d.base + d.off[0], dW, sW, bW, CU_TENSOR_MAP_SWIZZLE_NONE,
                     "gate")) ||
        (rc = encode(&m1.w1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, d.base + d.off[3], dW, sW, bW, CU_TENSOR_MAP_SWIZZLE_NONE,
                     "up")))
      return rc;
    const cuuint64_t dA2[2] = {(cuuint64_t)d.I, (cuuint64_t)P}, sA2[1] = {(cuuint64_t)d.I * 2};
    const cuuint64_t dW2[3] = {(cuuint64_t)d.I / 2, (cuuint64_t)d.H, (cuuint64_t)d.E};
    const cuuint64_t sW2[2] = {(cuuint64_t)d.I / 2, (cuuint64_t)d.stride};
    const cuuint32_t bW2[3] = {32, (cuuint32_t)pf::BN, 1};
    if ((rc = encode(&m2.a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w.act, dA2, sA2, bA, CU_TENSOR_MAP_SWIZZLE_128B,
                     "act")) ||
        (rc = encode(&m2.w0, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, d.base + d.off[6], dW2, sW2, bW2,
                     CU_TENSOR_MAP_SWIZZLE_NONE, "down")))
      return rc;
    m2.w1 = m2.w0;
  }
  const int G1 = d.H / 64, G2 = d.I / 64;
  pf::Args a1{w.tiles, w.ntiles, static_cast<const bf16*>(prep), prep_eps(d), 0, (int64_t)G1 * d.I,
              2LL * G1 * d.I, 3LL * G1 * d.I, d.H, d.I, d.E, w.act, w.h.status};
  pf::Args a2 = a1;
  a2.off_s0 = 4LL * G1 * d.I;
  a2.off_b0 = 4LL * G1 * d.I + (int64_t)G2 * d.H;
  a2.out = w.ys;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(pf::tc_gemm_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, pf::SMEM);
    cudaFuncSetAttribute(pf::tc_gemm_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, pf::SMEM);
  });
  {
    ProfScope prof_("tc_gemm_kernel<gate_up>", st);
    pf::tc_gemm_kernel<0><<<kNumSMs, pf::THREADS, pf::SMEM, st>>>(m1, a1);
  }
  if ((rc = check_launch("tc_gemm_kernel<gate_up>"))) return rc;
  {
    ProfScope prof_("tc_gemm_kernel<down>", st);
    pf::tc_gemm_kernel<1><<<kNumSMs, pf::THREADS, pf::SMEM, st>>>(m2, a2);
  }
  if ((rc = check_launch("tc_gemm_kernel<down>"))) return rc;
  {
    ProfScope prof_("prefill_combine_kernel", st);
    pf::combine_kernel<<<2 * kNumSMs * 4, 256, 0, st>>>(w.ys, w.inv, w_out, (int)T, k, d.H, static_cast<bf16*>(y));
  }
  return check_launch("prefill_combine_kernel");
}
