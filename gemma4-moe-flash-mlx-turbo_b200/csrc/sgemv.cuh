// Streaming GEMV core for decode (T <= 8 tokens).  Every warp streams its own
// weight tiles from HBM into a private shared-memory ring with 16-byte
// cp.async copies (no producer warp, no mbarriers) and multiplies them on the
// warp-level tensor cores (mma.sync m16n8k16, fp32 accumulate) against input
// fragments the CTA prepared once in shared memory.
//
// A step = one 16-row tile (two for a gate|up pair) x up to NGM consecutive
// 64-wide groups of K.  The copy side reads each row's segment of the step as
// contiguous 16-byte chunks, 32 lanes covering whole 128-byte lines; the math
// side reads the same bytes back in the MMA fragment layout (lane = 4g + t
// holds 16 codes of rows g and g+8 per group), so rows are XOR-swizzled in
// 16-byte chunks to keep those reads free of bank conflicts.  The ring holds D
// steps: the bytes in flight sit in shared memory, not registers, so a CTA
// keeps tens of KB outstanding against HBM with few registers — leaving room
// on the SM for the next kernel of a programmatic-dependent chain to become
// resident and start its own stream before this one ends.
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
__device__ __forceinline__ void commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void wait_group() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
__device__ __forceinline__ uint32_t s_addr(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }
__device__ __forceinline__ uint32_t ldg_h(const bf16* p) {
  unsigned short r;
  asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];\n" : "=h"(r) : "l"(p));
  return r;
}

// Geometry of one width's stage: GB bytes per group and row, NGM groups per
// step, RB bytes per staged row (6-bit: padded to 52 words so the 12-byte lane
// reads of 8 rows hit 32 distinct banks), CPG chunks per group.
template <int BITS, int NGM>
struct Geo {
  static constexpr int GB = 64 * BITS / 8;
  static constexpr int CPG = GB / 16;
  static constexpr int RB = NGM * GB + (BITS == 6 ? 16 : 0);
  static constexpr float OFF = (BITS == 4 || BITS == 16) ? 128.0f : 1024.0f;
  static_assert(BITS != 4 || NGM % 4 == 0, "4-bit rows: whole 128-byte lines per step");
  static_assert(BITS != 8 || NGM % 2 == 0, "8-bit rows: whole 128-byte lines per step");
  static_assert(BITS != 6 || NGM == 4, "6-bit stage padding assumes 4 groups per step");
  static_assert(BITS != 16 || NGM == 1, "16-bit: one group (128 bytes) per step");
};

// Physical 16-byte chunk of logical chunk c in staged row r.
template <int BITS>
__device__ __forceinline__ int swz(int r, int c) {
  if constexpr (BITS == 8) return c ^ ((r & 1) << 2);
  else if constexpr (BITS == 4) return c ^ ((r & 3) << 1);
  else if constexpr (BITS == 16) return c ^ (r & 1);
  else return c;
}

// Byte offset (in the stage) of the lane's data for group gi of staged row r.
template <int BITS, int NGM>
__device__ __forceinline__ int lane_off(int r, int gi, int t) {
  using Gm = Geo<BITS, NGM>;
  if constexpr (BITS == 8) return r * Gm::RB + swz<8>(r, gi * 4 + t) * 16;
  else if constexpr (BITS == 4) return r * Gm::RB + swz<4>(r, gi * 2 + (t >> 1)) * 16 + (t & 1) * 8;
  else if constexpr (BITS == 6) return r * Gm::RB + gi * 48 + 12 * t;
  else return r * Gm::RB;  // 16-bit: two chunks, see mma_group
}

// C[4] += (off + q) . x for one group of a 16-row tile; lo / hi = stage
// offsets of rows g and g+8 (row index rl / rh for the 16-bit swizzle).
template <int BITS, int NGM>
__device__ __forceinline__ void mma_group(float (&c)[4], const uint8_t* st, int rl, int rh, int gi, int t,
                                          const uint32_t (&b)[8]) {
  if constexpr (BITS == 4) {
    const uint2 l = *reinterpret_cast<const uint2*>(st + lane_off<4, NGM>(rl, gi, t));
    const uint2 h = *reinterpret_cast<const uint2*>(st + lane_off<4, NGM>(rh, gi, t));
#pragma unroll
    for (int s = 0; s < 4; ++s)
      mma16816(c, nib_pair(l.x, 4 * s), nib_pair(h.x, 4 * s), nib_pair(l.y, 4 * s), nib_pair(h.y, 4 * s), b[s],
               b[4 + s]);
  } else if constexpr (BITS == 16) {
    constexpr int RB = Geo<16, NGM>::RB;
    const uint4 l0 = *reinterpret_cast<const uint4*>(st + rl * RB + swz<16>(rl, 2 * t) * 16);
    const uint4 l1 = *reinterpret_cast<const uint4*>(st + rl * RB + swz<16>(rl, 2 * t + 1) * 16);
    const uint4 h0 = *reinterpret_cast<const uint4*>(st + rh * RB + swz<16>(rh, 2 * t) * 16);
    const uint4 h1 = *reinterpret_cast<const uint4*>(st + rh * RB + swz<16>(rh, 2 * t + 1) * 16);
    const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
    const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) mma16816(c, lw[j], hw[j], lw[j + 4], hw[j + 4], b[j], b[j + 4]);
  } else {
    uint32_t a[4][4];
    load_a_frags<BITS>(st + lane_off<BITS, NGM>(rl, gi, t), st + lane_off<BITS, NGM>(rh, gi, t), a);
#pragma unroll
    for (int j = 0; j < 4; ++j) mma16816_f16(c, a[j][0], a[j][1], a[j][2], a[j][3], b[j], b[4 + j]);
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
  constexpr float off = Geo<BITS, BITS == 4 ? 4 : BITS == 6 ? 4 : BITS == 8 ? 2 : 1>::OFF;
  const float s_lo = __uint_as_float(sl << 16), s_hi = __uint_as_float(sh << 16);
  const float b_lo = fmaf(-off, s_lo, __uint_as_float(bl << 16)), b_hi = fmaf(-off, s_hi, __uint_as_float(bh << 16));
  y[0] = fmaf(s_lo, c[0], fmaf(b_lo, x0, y[0]));
  y[1] = fmaf(s_lo, c[1], fmaf(b_lo, x1, y[1]));
  y[2] = fmaf(s_hi, c[2], fmaf(b_hi, x0, y[2]));
  y[3] = fmaf(s_hi, c[3], fmaf(b_hi, x1, y[3]));
}

}  // namespace sg
}  // namespace fmoe
