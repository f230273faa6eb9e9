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
// GEMM kernel (persistent, one CTA per SM, 14 warps):
//   warp 0   producer: TMA tiles of A (128 sorted rows x 64 K, bf16, 128-byte
//            swizzle) and of the packed 4-bit weights (3-D tensor map over the
//            expert table), 1-D bulk copies of the step's scale / bias rows
//   warp 1   MMA issuer: per K tile, 2 x 4 tcgen05.mma (K 16) with the
//            dequantised weights as the M operand (two 128-row halves: gate
//            and up rows, or 256 down rows) and the tile's tokens as N (their
//            count rounded up to 16, so a lightly used expert wastes little);
//            one of two TMEM accumulators; tcgen05.commit releases the stage
//   warps 2-9  dequantise the weight tile into the canonical K-major
//            128-byte-swizzled bf16 layout in shared memory: w = bf16(fma(s, q, b))
//   warps 10-13  epilogue: tcgen05.ld of the accumulator (lane = weight row,
//            column = token), GELU gating (GEMM1) or plain bf16 store (GEMM2)
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
#include "tc.cuh"

namespace fmoe {
namespace pf {

using namespace tc;

constexpr int BM = 128;                // tokens per tile (the MMA's N, rounded up to 16)
constexpr int BN = 256, BK = 64;       // weight rows per item (two 128-row halves), K per tile
constexpr int NS = 3;                  // K-tile stages: token tile + dequantised weights (shared memory)
constexpr int NQ = 2;                  // packed-weight stages, KQ K tiles each
constexpr int KQ = 4;                  // K tiles per packed-weight stage (128 bytes of 4-bit codes per row)
constexpr int X_BYTES = BM * BK * 2;   // 16 KB
constexpr int WB_BYTES = BN * BK * 2;  // 32 KB
constexpr int WQ_BYTES = BN * BK * KQ / 2;  // 32 KB: 256 rows x 128 bytes, 128-byte swizzle
constexpr int SC_BYTES = 2 * BN * KQ * 2;   // 4 KB: scale and bias of 256 rows x KQ groups
constexpr int WQS = WQ_BYTES + SC_BYTES;    // one packed-weight stage (codes, then scales)
constexpr int OFF_X = 0, OFF_WB = X_BYTES;
constexpr int STAGE = OFF_WB + WB_BYTES;    // 48 KB, a multiple of 1024
constexpr int OFF_WQ = NS * STAGE;
constexpr int OFF_BAR = OFF_WQ + NQ * WQS;
constexpr int SMEM = OFF_BAR + 512 + 1024;  // + alignment slack for the 1024-byte swizzle atoms
constexpr int NDQ = 8;                      // dequantising warps (one weight row per thread)
constexpr int THREADS = (2 + NDQ + 4) * 32;
constexpr int TMEM_COLS = 512;              // accumulators [2 buffers][2 halves][BM tokens] fp32
static_assert(STAGE % 1024 == 0 && OFF_WQ % 1024 == 0 && WQS % 1024 == 0, "stage alignment");

struct alignas(64) Maps {
  CUtensorMap a;   // A rows (bf16 [P][K], 128-byte swizzle, box 64 x 128)
  CUtensorMap a_small[3];  // the same with boxes of 16, 32 and 64 rows (tiles of few tokens)
  CUtensorMap w0;  // packed weights (u8 [E][rows][K/2], 128-byte swizzle, box 128 x 128 (GEMM1) / 256 (GEMM2) x 1)
  CUtensorMap w1;  // GEMM1: the up projection
};

struct Args {
  const int4* tiles;     // (expert, first sorted row, rows, 0)
  const int* ntiles;
  const bf16* prep;      // scales / biases as [group / 4][row][4] per array, expert stride eps elements
  int64_t eps;
  int64_t off_s0, off_b0, off_s1, off_b1;  // element offsets of this GEMM's arrays in an expert's block
  int H, I, E;
  bf16* out;             // GEMM1: act [P][I] (permuted words); GEMM2: Y [P][H]
  int* status;
};

// Two bf16 from two floats, low half first.
__device__ __forceinline__ uint32_t bf2(float lo, float hi) { return pack_bf16x2(lo, hi); }

template <int MODE>  // 0: gate|up + GELU gating, 1: down
__global__ void __launch_bounds__(THREADS, 1) tc_gemm_kernel(const __grid_constant__ Maps maps, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* xfull = reinterpret_cast<uint64_t*>(smem + OFF_BAR);  // token tile landed
  uint64_t* deqd = xfull + NS;                                      // dequantised weights written
  uint64_t* mmad = deqd + NS;                                       // MMAs done with the stage
  uint64_t* wqf = mmad + NS;                                        // packed weights + scales landed
  uint64_t* wqe = wqf + NQ;                                         // dequantisers done with them
  uint64_t* accf = wqe + NQ;                                        // accumulator complete
  uint64_t* acce = accf + 2;                                        // accumulator read out
  volatile int* failed = reinterpret_cast<volatile int*>(acce + 2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2) + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int K = MODE == 0 ? a.H : a.I;
  const int NJ = MODE == 0 ? (a.I + 127) / 128 : a.H / BN;
  const int NK = K / BK;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&deqd[s], NDQ);
      mbar_init(&mmad[s], 1);
    }
    for (int s = 0; s < NQ; ++s) {
      mbar_init(&wqf[s], 1);
      mbar_init(&wqe[s], NDQ);
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
    // ---- producer: token tiles (one per K tile) and packed-weight stages (one per KQ K tiles)
    if (lane == 0) {
      int q = 0, qq = 0;
      for (int it = blockIdx.x; it < nitems; it += gridDim.x) {
        const int4 tl = __ldg(a.tiles + it / NJ);
        const int j = it % NJ, e = tl.x, row0 = tl.y;
        const int rows_ok = MODE == 0 ? min(128, a.I - j * 128) : BN;
        const bf16* pe = a.prep + (int64_t)e * a.eps;
        for (int kt = 0; kt < NK; ++kt, ++q) {
          if (kt % KQ == 0) {
            const int sq = qq % NQ;
            if (qq >= NQ) pwait(&wqe[sq], (uint32_t)((qq / NQ) - 1) & 1u, failed, a.status, 306);
            if (*failed) break;
            uint8_t* wq = smem + OFF_WQ + sq * WQS;
            uint8_t* sc = wq + WQ_BYTES;
            const int gb = kt / KQ;  // group block: KQ groups, one per K tile
            if (MODE == 0) {
              mbar_arrive_expect_tx(&wqf[sq], (uint32_t)(WQ_BYTES + 4 * rows_ok * KQ * 2));
              tma3d(wq, &maps.w0, kt * 32, j * 128, e, &wqf[sq]);
              tma3d(wq + WQ_BYTES / 2, &maps.w1, kt * 32, j * 128, e, &wqf[sq]);
              const int64_t r = ((int64_t)gb * a.I + j * 128) * KQ;
              bulk_g2s(sc, pe + a.off_s0 + r, rows_ok * KQ * 2, &wqf[sq]);
              bulk_g2s(sc + 1024, pe + a.off_b0 + r, rows_ok * KQ * 2, &wqf[sq]);
              bulk_g2s(sc + 2048, pe + a.off_s1 + r, rows_ok * KQ * 2, &wqf[sq]);
              bulk_g2s(sc + 3072, pe + a.off_b1 + r, rows_ok * KQ * 2, &wqf[sq]);
            } else {
              mbar_arrive_expect_tx(&wqf[sq], (uint32_t)(WQ_BYTES + 2 * BN * KQ * 2));
              tma3d(wq, &maps.w0, kt * 32, j * BN, e, &wqf[sq]);
              const int64_t r = ((int64_t)gb * a.H + j * BN) * KQ;
              bulk_g2s(sc, pe + a.off_s0 + r, BN * KQ * 2, &wqf[sq]);
              bulk_g2s(sc + 2048, pe + a.off_b0 + r, BN * KQ * 2, &wqf[sq]);
            }
            ++qq;
          }
          const int s = q % NS;
          if (q >= NS) pwait(&mmad[s], (uint32_t)((q / NS) - 1) & 1u, failed, a.status, 301);
          if (*failed) break;
          // only the tile's token rows (rounded up to a box of 16 / 32 / 64 / 128)
          const int ntok = tl.z, hb = ntok <= 16 ? 0 : ntok <= 32 ? 1 : ntok <= 64 ? 2 : 3;
          mbar_arrive_expect_tx(&xfull[s], (uint32_t)((16 << hb) * BK * 2));
          tma2d(smem + s * STAGE + OFF_X, hb < 3 ? &maps.a_small[hb] : &maps.a, kt * BK, row0, &xfull[s]);
        }
        if (*failed) break;
      }
      // every copy issued lands before the CTA ends
      for (int k = q - NS < 0 ? 0 : q - NS; k < q; ++k) drain_wait(&xfull[k % NS], (uint32_t)(k / NS) & 1u);
      for (int k = qq - NQ < 0 ? 0 : qq - NQ; k < qq; ++k) drain_wait(&wqf[k % NQ], (uint32_t)(k / NQ) & 1u);
    }
  } else if (warp == 1) {
    // ---- MMA issuer: weights as the M operand (two 128-row halves), the tile's tokens as N
    if (lane == 0) {
      int q = 0, n = 0;
      for (int it = blockIdx.x; it < nitems; it += gridDim.x, ++n) {
        const int ab = n & 1;
        const int ntok = __ldg(a.tiles + it / NJ).z;
        const uint32_t idesc = idesc_n((ntok + 15) & ~15);
        if (n >= 2) pwait(&acce[ab], (uint32_t)((n / 2) - 1) & 1u, failed, a.status, 302);
        tc_fence_after();
        for (int kt = 0; kt < NK; ++kt, ++q) {
          const int s = q % NS;
          pwait(&deqd[s], (uint32_t)(q / NS) & 1u, failed, a.status, 303);  // implies the token tile too
          tc_fence_after();
          const uint32_t sx = smem_u32(smem + s * STAGE + OFF_X), sw = smem_u32(smem + s * STAGE + OFF_WB);
          if (!*failed) {
#pragma unroll
            for (int h = 0; h < 2; ++h)
#pragma unroll
              for (int k = 0; k < BK / 16; ++k)
                mma_ss(tmem + ab * 2 * BM + h * BM, sw128_desc(sw + h * (128 * 128) + 32 * k),
                       sw128_desc(sx + 32 * k), idesc, (kt | k) != 0);
          }
          mma_commit(&mmad[s]);
        }
        mma_commit(&accf[ab]);
      }
      if (n > 0) drain_wait(&accf[(n - 1) & 1], (uint32_t)((n - 1) / 2) & 1u);  // the last MMAs are done
    }
  } else if (warp < 2 + NDQ) {
    // ---- dequantisers: thread = one row of the 256-row weight tile, written as 64 bf16 in
    // the canonical K-major 128-byte-swizzled layout (chunk c of row r at chunk c ^ (r % 8))
    const int rr = threadIdx.x - 64, h = rr >> 7;
    int q = 0, qq = 0;
    for (int it = blockIdx.x; it < nitems; it += gridDim.x) {
      const int j = it % NJ;
      for (int kt = 0; kt < NK; ++kt, ++q) {
        const int s = q % NS, sq = qq % NQ;
        if (kt % KQ == 0) pwait(&wqf[sq], (uint32_t)(qq / NQ) & 1u, failed, a.status, 307);
        pwait(&xfull[s], (uint32_t)(q / NS) & 1u, failed, a.status, 304);  // the stage is free again
        const uint8_t* wq = smem + OFF_WQ + sq * WQS;
        const bf16* sc = reinterpret_cast<const bf16*>(wq + WQ_BYTES);
        const int kq = kt % KQ, c0 = 2 * kq;  // this K tile's two 16-byte chunks of a 128-byte row
        bool ok;
        float sv, bv;
        if (MODE == 0) {
          ok = j * 128 + (rr & 127) < a.I;
          sv = ok ? bf2f(sc[h * 1024 + (rr & 127) * KQ + kq]) : 0.f;
          bv = ok ? bf2f(sc[h * 1024 + 512 + (rr & 127) * KQ + kq]) : 0.f;
        } else {
          ok = true;
          sv = bf2f(sc[rr * KQ + kq]);
          bv = bf2f(sc[BN * KQ + rr * KQ + kq]);
        }
        // 128-byte-swizzled rows: chunk c of row r sits at chunk c ^ (r % 8)
        const uint4 w0 = *reinterpret_cast<const uint4*>(wq + rr * 128 + ((c0 ^ (rr & 7)) << 4));
        const uint4 w1 = *reinterpret_cast<const uint4*>(wq + rr * 128 + (((c0 + 1) ^ (rr & 7)) << 4));
        const uint32_t ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
        const __nv_bfloat162 s2 = __floats2bfloat162_rn(sv, sv), b2 = __floats2bfloat162_rn(bv, bv);
        const __nv_bfloat162 off = __floats2bfloat162_rn(128.f, 128.f);
        uint8_t* wrow = smem + s * STAGE + OFF_WB + rr * 128;
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
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // generic writes -> tensor-core reads
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&deqd[s]);
          if (kt % KQ == KQ - 1 || kt == NK - 1) mbar_arrive(&wqe[sq]);
        }
        if (kt % KQ == KQ - 1 || kt == NK - 1) ++qq;
      }
    }
  } else {
    // ---- epilogue: TMEM lane = weight row (feature) 32 * (warp % 4) + lane, column = token
    const int qw = warp & 3, fr = qw * 32 + lane;
    int n = 0;
    for (int it = blockIdx.x; it < nitems; it += gridDim.x, ++n) {
      const int4 tl = __ldg(a.tiles + it / NJ);
      const int j = it % NJ, row0 = tl.y, nrows = tl.z, nc = (nrows + 15) / 16;
      const int ab = n & 1;
      pwait(&accf[ab], (uint32_t)(n / 2) & 1u, failed, a.status, 305);
      tc_fence_after();
      const uint32_t ta = tmem + ((uint32_t)(qw * 32) << 16) + ab * 2 * BM;
      const bool ok = !*failed;
      if (MODE == 0) {
        const int f = j * 128 + fr;  // intermediate index of this lane's gate / up rows
        // act is stored in the permuted word order: element 8w + jj + 4h at position 8w + 2jj + h
        const int pos = (f & ~7) | ((f & 3) << 1) | ((f >> 2) & 1);
#pragma unroll 1
        for (int cc = 0; cc < nc; ++cc) {
          float g[16], u[16];
          tmem_ld16(ta + cc * 16, g);
          tmem_ld16(ta + BM + cc * 16, u);
          tmem_ld_wait();
          if (ok && f < a.I) {
#pragma unroll
            for (int i = 0; i < 16; ++i) {
              const int tok = cc * 16 + i;
              if (tok < nrows)
                a.out[(int64_t)(row0 + tok) * a.I + pos] = __float2bfloat16_rn(gelu_tanh(round_bf(g[i])) * round_bf(u[i]));
            }
          }
        }
      } else {
#pragma unroll 1
        for (int hh = 0; hh < 2; ++hh) {
          const int f = j * BN + hh * 128 + fr;
#pragma unroll 1
          for (int cc = 0; cc < nc; ++cc) {
            float v[16];
            tmem_ld16(ta + hh * BM + cc * 16, v);
            tmem_ld_wait();
            if (ok) {
#pragma unroll
              for (int i = 0; i < 16; ++i) {
                const int tok = cc * 16 + i;
                if (tok < nrows) a.out[(int64_t)(row0 + tok) * a.H + f] = __float2bfloat16_rn(v[i]);
              }
            }
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

// Scale / bias copy of every expert laid out per K super-tile: for each array
// (gate s, gate b, up s, up b over [I] rows; down s, down b over [H] rows),
// [ceil(G / 4)][rows][4] bf16, groups past G zero.  One super-tile's 4 groups
// of a row block are then one contiguous run.
__device__ __forceinline__ int64_t prep_q1(const ExpertsDev& ex) { return (ex.H / 64 + 3) / 4; }
__device__ __forceinline__ int64_t prep_q2(const ExpertsDev& ex) { return (ex.I / 64 + 3) / 4; }
__global__ void prep_kernel(ExpertsDev ex, bf16* __restrict__ prep, int64_t eps) {
  const int e = blockIdx.y;
  const uint8_t* base = ex.base + (int64_t)e * ex.stride;
  const int G1 = ex.H / 64, G2 = ex.I / 64;
  const int64_t Q1 = prep_q1(ex), Q2 = prep_q2(ex);
  bf16* pe = prep + (int64_t)e * eps;
  const int n1 = ex.I, n2 = ex.H;
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < n1 + n2; r += gridDim.x * blockDim.x) {
    if (r < n1) {
      const int arr[4] = {1, 2, 4, 5};
      for (int t = 0; t < 4; ++t) {
        const bf16* src = reinterpret_cast<const bf16*>(base + ex.off[arr[t]]) + (int64_t)r * G1;
        bf16* dst = pe + (int64_t)t * Q1 * n1 * 4;
        for (int g = 0; g < (int)Q1 * 4; ++g)
          dst[((int64_t)(g / 4) * n1 + r) * 4 + g % 4] = g < G1 ? src[g] : __float2bfloat16_rn(0.f);
      }
    } else {
      const int rr = r - n1;
      for (int t = 0; t < 2; ++t) {
        const bf16* src = reinterpret_cast<const bf16*>(base + ex.off[7 + t]) + (int64_t)rr * G2;
        bf16* dst = pe + 4 * Q1 * n1 * 4 + (int64_t)t * Q2 * n2 * 4;
        for (int g = 0; g < (int)Q2 * 4; ++g)
          dst[((int64_t)(g / 4) * n2 + rr) * 4 + g % 4] = g < G2 ? src[g] : __float2bfloat16_rn(0.f);
      }
    }
  }
}

// Tile list: per expert with n > 0 pairs, ceil(n / 128) tiles of sorted rows
// (one warp: lane l takes experts l, l + 32, ...; a prefix over lanes).
__global__ void tiles_kernel(const int32_t* __restrict__ start, int E, int4* __restrict__ tiles, int* __restrict__ ntiles) {
  const int lane = threadIdx.x;
  int base = 0;
  for (int e0 = 0; e0 < E; e0 += 32) {
    const int e = e0 + lane;
    const int r0 = e < E ? start[e] : 0, r1 = e < E ? start[e + 1] : 0;
    const int n = (r1 - r0 + BM - 1) / BM;
    int incl = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    for (int t = 0; t < n; ++t) tiles[base + incl - n + t] = make_int4(e, r0 + t * BM, min(BM, r1 - r0 - t * BM), 0);
    base += __shfl_sync(0xffffffffu, incl, 31);
  }
  if (lane == 0) *ntiles = base;
}

// X_sorted[i] = x[pairs[i] / k] with each 8-column word in the order 0 4 1 5 2 6 3 7;
// inv[pairs[i]] = i, for the *nvalid pairs of local experts (inv is -1 elsewhere).
__global__ void gather_kernel(const bf16* __restrict__ x, const int32_t* __restrict__ pairs,
                              const int32_t* __restrict__ nvalid, int k, int H, bf16* __restrict__ xs,
                              int32_t* __restrict__ inv) {
  const int words = H / 8;
  const int P = *nvalid;
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

// y[t] = bf16(sum over local slots of w[t, slot] * Y[inv[t * k + slot]]) in slot order.
__global__ void combine_kernel(const bf16* __restrict__ Y, const int32_t* __restrict__ inv,
                               const float* __restrict__ wts, int T, int k, int H, bf16* __restrict__ y,
                               float* __restrict__ y32) {
  const int words = H / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)T * words;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / words), w = (int)(i % words);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < k; ++s) {
      const int j = inv[t * k + s];
      if (j < 0) continue;
      const float wv = wts[t * k + s];
      const uint4 v = *reinterpret_cast<const uint4*>(Y + (int64_t)j * H + 8 * w);
      const uint32_t vv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        acc[2 * q] = fmaf(wv, bf16lo(vv[q]), acc[2 * q]);
        acc[2 * q + 1] = fmaf(wv, bf16hi(vv[q]), acc[2 * q + 1]);
      }
    }
    if (y32) {
      float4* o = reinterpret_cast<float4*>(y32 + (int64_t)t * H + 8 * w);
      o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    } else {
      *reinterpret_cast<uint4*>(y + (int64_t)t * H + 8 * w) =
          make_uint4(bf2(acc[0], acc[1]), bf2(acc[2], acc[3]), bf2(acc[4], acc[5]), bf2(acc[6], acc[7]));
    }
  }
}

}  // namespace pf

// ---------------------------------------------------------------------------
// host side

namespace {

int64_t prep_q1h(const ExpertsDev& d) { return (d.H / 64 + 3) / 4; }
int64_t prep_q2h(const ExpertsDev& d) { return (d.I / 64 + 3) / 4; }
int64_t prep_eps(const ExpertsDev& d) { return 4 * (4 * prep_q1h(d) * d.I) + 2 * (4 * prep_q2h(d) * d.H); }

}  // namespace

// The driver's tensor-map encoder, resolved through the runtime (the library
// does not link the driver library, so it loads on machines without one).
static PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
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
  if (!enc) return set_error(FMOE_ERR_CUDA, "tensor map: the driver's encoder is unavailable");
  const CUresult r = enc(m, dt, rank, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         sw, CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return set_error(FMOE_ERR_CUDA, "tensor map for %s failed (%d)", what, (int)r);
  return FMOE_OK;
}

int check_prefill(const ExpertsDev& d) {
  if (d.slot_of) return set_error(FMOE_ERR_UNSUPPORTED, "prefill: expert tables with a slot map (decode kernels only)");
  if (d.H % 256 || d.I % 64 || d.H > 8192 || d.E < 1)
    return set_error(FMOE_ERR_UNSUPPORTED, "prefill: hidden %d (multiple of 256), intermediate %d (multiple of 64)",
                     d.H, d.I);
  if (d.stride % 16 || !aligned(d.base, 16))
    return set_error(FMOE_ERR_ALIGN, "prefill: expert table must be 16-byte aligned with a 16-byte stride");
  for (int j = 0; j < 9; ++j)
    if (d.off[j] % 16) return set_error(FMOE_ERR_ALIGN, "prefill: expert tensor offsets must be 16-byte aligned");
  return FMOE_OK;
}

size_t carve_pf_ex(Carver& c, int64_t T, int k, const ExpertsDev& d, PfExWs* w) {
  PfExWs p;
  const int64_t P = T * k;
  p.m.start = c.take<int32_t>(d.E + 1);
  p.m.pairs = c.take<int32_t>(P);
  p.m.unique = c.take<int32_t>(d.E);
  p.m.num_unique = c.take<int32_t>(1);
  p.m.work_len = (int)std::min<int64_t>(P, d.E);
  p.m.work = c.take<int4>(p.m.work_len);
  const int64_t rs = route_scratch_ints(P, d.E);
  p.m.scratch = rs ? c.take<int32_t>(rs) : nullptr;
  p.tiles = c.take<int4>(P / pf::BM + d.E + 1);
  p.ntiles = c.take<int>(1);
  p.inv = c.take<int32_t>(P);
  p.xs = c.take<bf16>((size_t)P * d.H);
  p.act = c.take<bf16>((size_t)P * d.I);
  p.ys = c.take<bf16>((size_t)P * d.H);
  if (w) *w = p;
  return c.off;
}

int run_prefill_experts(const bf16* x, int64_t T, int k, const int32_t* ids, const float* wts, const ExpertsDev& d,
                        const bf16* prep, bf16* y, const PfExWs& w, bool build_routes, int* status, cudaStream_t st,
                        float* y32) {
  int rc;
  const int64_t P = T * k;
  if (P > (1 << 30) / d.H) return set_error(FMOE_ERR_UNSUPPORTED, "prefill: T=%lld too large", (long long)T);
  if (build_routes && (rc = launch_route_build(ids, P, d, w.m, st))) return rc;
  {
    ProfScope prof_("prefill_tiles_kernel", st);
    pf::tiles_kernel<<<1, 32, 0, st>>>(w.m.start, d.E, w.tiles, w.ntiles);
  }
  if ((rc = check_launch("prefill_tiles_kernel"))) return rc;
  if (cudaMemsetAsync(w.inv, 0xFF, (size_t)P * sizeof(int32_t), st) != cudaSuccess)
    return set_error(FMOE_ERR_CUDA, "prefill: memset failed");
  {
    ProfScope prof_("prefill_gather_kernel", st);
    pf::gather_kernel<<<2 * kNumSMs * 4, 256, 0, st>>>(x, w.m.pairs, w.m.start + d.E, k, d.H, w.xs, w.inv);
  }
  if ((rc = check_launch("prefill_gather_kernel"))) return rc;
  // tensor maps
  pf::Maps m1, m2;
  {
    const cuuint64_t dA[2] = {(cuuint64_t)d.H, (cuuint64_t)P}, sA[1] = {(cuuint64_t)d.H * 2};
    const cuuint32_t bA[2] = {64, (cuuint32_t)pf::BM};
    const cuuint64_t dW[3] = {(cuuint64_t)d.H / 2, (cuuint64_t)d.I, (cuuint64_t)d.E};
    const cuuint64_t sW[2] = {(cuuint64_t)d.H / 2, (cuuint64_t)d.stride};
    const cuuint32_t bW[3] = {128, 128, 1};
    for (int h = 0; h < 3; ++h) {
      const cuuint32_t bS[2] = {64, (cuuint32_t)(16 << h)};
      if ((rc = encode(&m1.a_small[h], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w.xs, dA, sA, bS, CU_TENSOR_MAP_SWIZZLE_128B,
                       "x")))
        return rc;
    }
    if ((rc = encode(&m1.a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w.xs, dA, sA, bA, CU_TENSOR_MAP_SWIZZLE_128B, "x")) ||
        (rc = encode(&m1.w0, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, d.base + d.off[0], dW, sW, bW, CU_TENSOR_MAP_SWIZZLE_128B,
                     "gate")) ||
        (rc = encode(&m1.w1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, d.base + d.off[3], dW, sW, bW, CU_TENSOR_MAP_SWIZZLE_128B,
                     "up")))
      return rc;
    const cuuint64_t dA2[2] = {(cuuint64_t)d.I, (cuuint64_t)P}, sA2[1] = {(cuuint64_t)d.I * 2};
    const cuuint64_t dW2[3] = {(cuuint64_t)d.I / 2, (cuuint64_t)d.H, (cuuint64_t)d.E};
    const cuuint64_t sW2[2] = {(cuuint64_t)d.I / 2, (cuuint64_t)d.stride};
    const cuuint32_t bW2[3] = {128, (cuuint32_t)pf::BN, 1};
    for (int h = 0; h < 3; ++h) {
      const cuuint32_t bS[2] = {64, (cuuint32_t)(16 << h)};
      if ((rc = encode(&m2.a_small[h], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w.act, dA2, sA2, bS,
                       CU_TENSOR_MAP_SWIZZLE_128B, "act")))
        return rc;
    }
    if ((rc = encode(&m2.a, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w.act, dA2, sA2, bA, CU_TENSOR_MAP_SWIZZLE_128B,
                     "act")) ||
        (rc = encode(&m2.w0, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, d.base + d.off[6], dW2, sW2, bW2,
                     CU_TENSOR_MAP_SWIZZLE_128B, "down")))
      return rc;
    m2.w1 = m2.w0;
  }
  const int64_t A1 = 4 * prep_q1h(d) * d.I, A2 = 4 * prep_q2h(d) * d.H;  // elements per array
  pf::Args a1{w.tiles, w.ntiles, prep, prep_eps(d), 0, A1, 2 * A1, 3 * A1, d.H, d.I, d.E, w.act, status};
  pf::Args a2 = a1;
  a2.off_s0 = 4 * A1;
  a2.off_b0 = 4 * A1 + A2;
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
    pf::combine_kernel<<<2 * kNumSMs * 4, 256, 0, st>>>(w.ys, w.inv, wts, (int)T, k, d.H, y, y32);
  }
  return check_launch("prefill_combine_kernel");
}

namespace {

struct PfWs {
  WsHead h;
  RouterWs r;
  int32_t* ids;
  float* wts;
  PfExWs ex;
};

size_t carve_pf(Carver& c, int64_t T, const fmoe_router_t* r, const ExpertsDev& d, PfWs* w) {
  PfWs p;
  p.h = carve_head(c);
  carve_router(c, T, r, p.h, &p.r);
  const int64_t P = T * r->top_k;
  p.ids = c.take<int32_t>(P);
  p.wts = c.take<float>(P);
  carve_pf_ex(c, T, r->top_k, d, &p.ex);
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
  // route (builds the per-expert pair lists), then the expert stage
  if ((rc = run_router(static_cast<const bf16*>(x), T, r, q, w.r, ids_out, w_out, nullptr, &w.ex.m, w.h.status, st)))
    return rc;
  return run_prefill_experts(static_cast<const bf16*>(x), T, k, ids_out, w_out, d, static_cast<const bf16*>(prep),
                             static_cast<bf16*>(y), w.ex, false, w.h.status, st);
}

extern "C" size_t fmoe_moe_prefill_experts_workspace_bytes(int64_t T, int top_k, const fmoe_experts_t* ex) {
  ExpertsDev d;
  if (T <= 0 || top_k < 1 || top_k > 16 || to_experts(ex, &d) || check_prefill(d)) return 0;
  Carver c(nullptr);
  carve_head(c);
  return carve_pf_ex(c, T, top_k, d, nullptr) + 256;
}

extern "C" int fmoe_moe_prefill_experts(const void* x, int64_t T, int top_k, const int32_t* ids, const float* weights,
                                        const fmoe_experts_t* ex, const void* prep, void* y, void* workspace,
                                        size_t workspace_bytes, void* stream) {
  ExpertsDev d;
  int rc;
  if ((rc = to_experts(ex, &d)) || (rc = check_prefill(d))) return rc;
  if (!x || !ids || !weights || !y || !prep)
    return set_error(FMOE_ERR_INVALID, "prefill_experts: null x / ids / weights / y / prepared scales");
  if (top_k < 1 || top_k > 16) return set_error(FMOE_ERR_INVALID, "prefill_experts: top_k %d", top_k);
  if (T <= 0) return FMOE_OK;
  if (!aligned(x, 16) || !aligned(y, 16)) return set_error(FMOE_ERR_ALIGN, "prefill_experts: x / y not 16-byte aligned");
  const size_t need = fmoe_moe_prefill_experts_workspace_bytes(T, top_k, ex);
  if (!workspace || workspace_bytes < need)
    return set_error(FMOE_ERR_WORKSPACE, "prefill_experts: workspace %zu < %zu", workspace_bytes, need);
  Carver c(workspace);
  const WsHead h = carve_head(c);
  PfExWs w;
  carve_pf_ex(c, T, top_k, d, &w);
  return run_prefill_experts(static_cast<const bf16*>(x), T, top_k, ids, weights, d, static_cast<const bf16*>(prep),
                             static_cast<bf16*>(y), w, true, h.status, static_cast<cudaStream_t>(stream));
}
