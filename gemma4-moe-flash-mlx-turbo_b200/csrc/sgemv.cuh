// Streaming GEMV core for decode (T <= 8 tokens).  Every warp streams its own
// weight tiles from HBM into a private shared-memory ring with cp.async and
// multiplies them on the warp-level tensor cores (mma.sync m16n8k16, fp32
// accumulate) against input fragments the CTA prepared once in shared memory.
//
// A step = NG consecutive 64-wide groups of K of one 16-row tile (two tiles
// for a gate|up pair); the groups' MMA chains are independent (and each
// group's four MMAs run as two chains), so a warp keeps several in flight.  Each lane copies exactly the bytes it later feeds to the MMA — lane
// 4g + t holds 16 codes of rows g and g+8, columns 16t .. 16t+15 of the group
// in a lane-specific k order — so a warp instruction reads 8 rows x 64 bytes
// (as fast as contiguous streaming once every warp of the GPU has work: the
// work is split over warps by groups, see dlayer.cu) and a lane reads back
// only its own copies: no swizzle, no cross-lane barrier.  6-bit rows are the
// exception: a quad's 48-byte group row arrives as three 16-byte copies of
// lanes t = 0..2 and is read back after a __syncwarp (48-byte row slots put
// the 12-byte lane reads of 8 rows on 32 distinct banks).  The bytes in
// flight sit in shared memory, not registers; only one scale or bias word per
// tile and step waits in a register.
//
// Per-width operand recipes (the B fragments use the same k order):
//   4-bit  bf16 MMA, A = bf16(128 + q) from one LOP3 per code pair
//   6-bit  f16 MMA, A = f16(1024 + q) from the 96-bit lane stream
//   8-bit  f16 MMA, A = f16(1024 + q) from one PRMT per code pair
//   16-bit bf16 MMA, A = the bf16 weights themselves (no scale / bias)
// Affine fixup per group and row:  y += s * C + (b - off * s) * sum(x),
// C = sum (off + q) x, sum(x) over the same rounded x the MMA saw.
#pragma once
#include "common.cuh"
#include "qfrag.cuh"

namespace fmoe {
namespace sg {

__device__ __forceinline__ void cpa16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global.L2::128B [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cpa8(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global.L2::128B [%0], [%1], 8;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void wait_group() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint32_t s_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ uint32_t ldg_h(const bf16* p) {
  unsigned short r;
  asm volatile("ld.global.nc.u16 %0, [%1];\n" : "=h"(r) : "l"(p));
  return r;
}

// Stage layout of one width: LB bytes per lane and row half (6-bit: a 48-byte
// slot per row, shared by the quad), GB bytes of one group in a row.
template <int BITS>
struct Geo {
  static constexpr int GB = 64 * BITS / 8;
  static constexpr int LB = BITS == 4 ? 8 : BITS == 16 ? 32 : 16;
  static constexpr int HALF = BITS == 6 ? 8 * 48 : 32 * LB;  // bytes of one row half (8 rows)
  static constexpr float OFF = (BITS == 4 || BITS == 16) ? 128.0f : 1024.0f;
};
template <int BITS, int NT>
constexpr int stage_bytes() {
  return 2 * NT * Geo<BITS>::HALF;
}

// Issue this lane's copies of one step.  src[h] = row (g + 8h) of tile h/2 at
// the step's group, lane offset not yet applied.
template <int BITS, int NT>
__device__ __forceinline__ void issue_step(uint32_t st, const uint8_t* const (&src)[2 * NT], int lane, int t) {
  using Gm = Geo<BITS>;
#pragma unroll
  for (int h = 0; h < 2 * NT; ++h) {
    const uint32_t d = st + h * Gm::HALF;
    if constexpr (BITS == 4) {
      cpa8(d + lane * 8, src[h] + 8 * t);
    } else if constexpr (BITS == 8) {
      cpa16(d + lane * 16, src[h] + 16 * t);
    } else if constexpr (BITS == 16) {
      cpa16(d + lane * 32, src[h] + 32 * t);
      cpa16(d + lane * 32 + 16, src[h] + 32 * t + 16);
    } else {
      if (t < 3) cpa16(d + (lane >> 2) * 48 + 16 * t, src[h] + 16 * t);
    }
  }
}

// C[4] += (off + q) . x for one group of tile i of the stage.
template <int BITS>
__device__ __forceinline__ void mma_group(float (&c)[4], const uint8_t* st, int i, int lane, int t,
                                          const uint32_t (&b)[8]) {
  using Gm = Geo<BITS>;
  const uint8_t* lo = st + (2 * i) * Gm::HALF;
  const uint8_t* hi = lo + Gm::HALF;
  if constexpr (BITS == 4) {
    const uint2 l = *reinterpret_cast<const uint2*>(lo + lane * 8);
    const uint2 h = *reinterpret_cast<const uint2*>(hi + lane * 8);
    float c2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int s = 0; s < 4; s += 2) {
      mma16816(c, nib_pair(l.x, 4 * s), nib_pair(h.x, 4 * s), nib_pair(l.y, 4 * s), nib_pair(h.y, 4 * s), b[s],
               b[4 + s]);
      mma16816(c2, nib_pair(l.x, 4 * s + 4), nib_pair(h.x, 4 * s + 4), nib_pair(l.y, 4 * s + 4),
               nib_pair(h.y, 4 * s + 4), b[s + 1], b[5 + s]);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) c[e] += c2[e];
  } else if constexpr (BITS == 16) {
    const uint4 l0 = *reinterpret_cast<const uint4*>(lo + lane * 32), l1 = *reinterpret_cast<const uint4*>(lo + lane * 32 + 16);
    const uint4 h0 = *reinterpret_cast<const uint4*>(hi + lane * 32), h1 = *reinterpret_cast<const uint4*>(hi + lane * 32 + 16);
    const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
    const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    float c2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 4; j += 2) {
      mma16816(c, lw[j], hw[j], lw[j + 4], hw[j + 4], b[j], b[j + 4]);
      mma16816(c2, lw[j + 1], hw[j + 1], lw[j + 5], hw[j + 5], b[j + 1], b[j + 5]);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) c[e] += c2[e];
  } else {
    uint32_t a[4][4];
    if constexpr (BITS == 8)
      load_a_frags<8>(lo + lane * 16, hi + lane * 16, a);
    else
      load_a_frags<6>(lo + (lane >> 2) * 48 + 12 * t, hi + (lane >> 2) * 48 + 12 * t, a);
    float c2[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < 4; j += 2) {
      mma16816_f16(c, a[j][0], a[j][1], a[j][2], a[j][3], b[j], b[4 + j]);
      mma16816_f16(c2, a[j + 1][0], a[j + 1][1], a[j + 1][2], a[j + 1][3], b[j + 1], b[5 + j]);
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) c[e] += c2[e];
  }
}

// B fragment (8 words) of 16 input values in the lane's k order for BITS.
template <int BITS>
__device__ __forceinline__ void make_frag(const float (&v)[16], uint32_t (&b)[8]) {
  if constexpr (BITS == 4) {
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      b[s] = pack_bf16x2(v[s], v[s + 4]);
      b[4 + s] = pack_bf16x2(v[8 + s], v[12 + s]);
    }
  } else if constexpr (BITS == 16) {
#pragma unroll
    for (int j = 0; j < 8; ++j) b[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
  } else {
    make_b_frags<BITS>(v, b);
  }
}

// The value the MMA sees for input v (f16 operands round; bf16 ones keep bf16 inputs).
template <int BITS>
__device__ __forceinline__ float operand_round(float v) {
  if constexpr (BITS == 4 || BITS == 16) return round_bf(v);
  else return f16r(v);
}

// y += s*C + (b - off*s)*xs for rows g (lo) / g+8 (hi), columns 2t, 2t+1.
template <int BITS>
__device__ __forceinline__ void fixup(float (&y)[4], const float (&c)[4], float x0, float x1, uint32_t sl,
                                      uint32_t bl, uint32_t sh, uint32_t bh) {
  constexpr float off = Geo<BITS>::OFF;
  const float s_lo = __uint_as_float(sl << 16), s_hi = __uint_as_float(sh << 16);
  const float b_lo = fmaf(-off, s_lo, __uint_as_float(bl << 16)), b_hi = fmaf(-off, s_hi, __uint_as_float(bh << 16));
  y[0] = fmaf(s_lo, c[0], fmaf(b_lo, x0, y[0]));
  y[1] = fmaf(s_lo, c[1], fmaf(b_lo, x1, y[1]));
  y[2] = fmaf(s_hi, c[2], fmaf(b_hi, x0, y[2]));
  y[3] = fmaf(s_hi, c[3], fmaf(b_hi, x1, y[3]));
}

}  // namespace sg
}  // namespace fmoe
