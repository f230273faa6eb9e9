// Warp-level building blocks shared by the GEMV-shaped kernels: one warp
// computes a 16-row x 8-token tile of x . W^T over a set of 64-wide groups.
#pragma once
#include "common.cuh"

namespace fmoe {

// Lane t's 16 x values of group `gi` for token row `xrow` (nullptr -> zeros).
__device__ __forceinline__ void load_x16(const bf16* xrow, int gi, int t, uint4& lo, uint4& hi) {
  if (xrow) {
    const bf16* p = xrow + gi * 64 + 16 * t;
    lo = ldg_u4(p);
    hi = ldg_u4(p + 8);
  } else {
    lo = make_uint4(0, 0, 0, 0);
    hi = lo;
  }
}

// 8-bit codes: a word holds 4 codes (bytes).  Each byte is split into its low
// and high nibble so the same 128+q bf16 trick applies; the high-nibble k
// slots see 16*x, so sum_slots = sum q*x + 2176*sum x  (2176 = 128*17).
struct BFrag8 {
  uint32_t lo0[4], lo1[4];  // steps 0..3: (x[4s], x[4s+2]) and (x[4s+1], x[4s+3])
  uint32_t hi0[4], hi1[4];  // same pairs times 16
};
__device__ __forceinline__ BFrag8 make_bfrag8(uint4 lo, uint4 hi) {
  BFrag8 f;
  const uint32_t src[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
  const __nv_bfloat162 sixteen = __floats2bfloat162_rn(16.0f, 16.0f);
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    f.lo0[s] = prmt(src[2 * s], src[2 * s + 1], 0x5410u);
    f.lo1[s] = prmt(src[2 * s], src[2 * s + 1], 0x7632u);
    __nv_bfloat162 a = *reinterpret_cast<__nv_bfloat162*>(&f.lo0[s]);
    __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&f.lo1[s]);
    a = __hmul2(a, sixteen);
    b = __hmul2(b, sixteen);
    f.hi0[s] = *reinterpret_cast<uint32_t*>(&a);
    f.hi1[s] = *reinterpret_cast<uint32_t*>(&b);
  }
  return f;
}

// wlo / whi: the 4 words (16 codes) lane t holds for rows g and g+8.
__device__ __forceinline__ void mma_group_q8(float (&acc)[4], uint4 wlo, uint4 whi, const BFrag8& b) {
  const uint32_t l[4] = {wlo.x, wlo.y, wlo.z, wlo.w};
  const uint32_t h[4] = {whi.x, whi.y, whi.z, whi.w};
#pragma unroll
  for (int s = 0; s < 4; ++s)
    mma16816(acc, nib_pair(l[s], 0), nib_pair(h[s], 0), nib_pair(l[s], 8), nib_pair(h[s], 8), b.lo0[s], b.lo1[s]);
#pragma unroll
  for (int s = 0; s < 4; ++s)
    mma16816(acc, nib_pair(l[s], 4), nib_pair(h[s], 4), nib_pair(l[s], 12), nib_pair(h[s], 12), b.hi0[s], b.hi1[s]);
}
__device__ __forceinline__ void mma_group_ones8(float (&xs)[4], const BFrag8& b) {
  const uint32_t one = 0x3f803f80u;
#pragma unroll
  for (int s = 0; s < 4; ++s) mma16816(xs, one, one, one, one, b.lo0[s], b.lo1[s]);
}

// Apply one group's affine parameters: y += s*C + (b - off*s)*xs.
__device__ __forceinline__ void affine_fixup(float (&y)[4], const float (&c)[4], const float (&xs)[4], float s_lo,
                                             float b_lo, float s_hi, float b_hi, float off) {
  const float bl = fmaf(-off, s_lo, b_lo), bh = fmaf(-off, s_hi, b_hi);
  y[0] = fmaf(s_lo, c[0], fmaf(bl, xs[0], y[0]));
  y[1] = fmaf(s_lo, c[1], fmaf(bl, xs[1], y[1]));
  y[2] = fmaf(s_hi, c[2], fmaf(bh, xs[2], y[2]));
  y[3] = fmaf(s_hi, c[3], fmaf(bh, xs[3], y[3]));
}

// One warp: y[16 rows x 8 tokens] += W[row0.., groups] . x over the groups
// gi = gfirst, gfirst + gstep, ... < glast.  W rows are `wpr` words (or bf16
// pairs for BITS == 16) apart; spr = scales per row.  xrow: this lane's token
// (column g) or nullptr.
template <int BITS>
__device__ __forceinline__ void warp_tile_gemv(float (&y)[4], const void* w, const bf16* sc, const bf16* bi,
                                               int64_t r_lo, int64_t r_hi, int wpr, int spr, const bf16* xrow,
                                               int gfirst, int glast, int gstep, int t) {
  if constexpr (BITS == 16) {
    const bf16* W = static_cast<const bf16*>(w);
#pragma unroll 2
    for (int gi = gfirst; gi < glast; gi += gstep) {
      const bf16* plo = W + r_lo * (int64_t)wpr * 2 + gi * 64 + 16 * t;
      const bf16* phi = W + r_hi * (int64_t)wpr * 2 + gi * 64 + 16 * t;
      const uint4 w0 = ldg_stream_u4(plo), w1 = ldg_stream_u4(plo + 8);
      const uint4 w2 = ldg_stream_u4(phi), w3 = ldg_stream_u4(phi + 8);
      uint4 xl, xh;
      load_x16(xrow, gi, t, xl, xh);
      const BFrag4 b = make_bfrag4(xl, xh);
      const BFrag4 alo = make_bfrag4(w0, w1), ahi = make_bfrag4(w2, w3);
#pragma unroll
      for (int s = 0; s < 4; ++s) mma16816(y, alo.b0[s], ahi.b0[s], alo.b1[s], ahi.b1[s], b.b0[s], b.b1[s]);
    }
  } else if constexpr (BITS == 4) {
    const uint32_t* W = static_cast<const uint32_t*>(w);
#pragma unroll 2
    for (int gi = gfirst; gi < glast; gi += gstep) {
      const uint2 wl = ldg_stream_u2(W + r_lo * wpr + gi * 8 + 2 * t);
      const uint2 wh = ldg_stream_u2(W + r_hi * wpr + gi * 8 + 2 * t);
      const float sl = bfbits2f(ldg_u16(sc + r_lo * spr + gi)), bl = bfbits2f(ldg_u16(bi + r_lo * spr + gi));
      const float sh = bfbits2f(ldg_u16(sc + r_hi * spr + gi)), bh = bfbits2f(ldg_u16(bi + r_hi * spr + gi));
      uint4 xl, xh;
      load_x16(xrow, gi, t, xl, xh);
      const BFrag4 b = make_bfrag4(xl, xh);
      float c[4] = {0.f, 0.f, 0.f, 0.f}, xs[4] = {0.f, 0.f, 0.f, 0.f};
      mma_group_q4(c, wl, wh, b);
      mma_group_ones(xs, b);
      affine_fixup(y, c, xs, sl, bl, sh, bh, 128.0f);
    }
  } else {
    static_assert(BITS == 8, "unsupported width");
    const uint32_t* W = static_cast<const uint32_t*>(w);
#pragma unroll 2
    for (int gi = gfirst; gi < glast; gi += gstep) {
      const uint4 wl = ldg_stream_u4(W + r_lo * wpr + gi * 16 + 4 * t);
      const uint4 wh = ldg_stream_u4(W + r_hi * wpr + gi * 16 + 4 * t);
      const float sl = bfbits2f(ldg_u16(sc + r_lo * spr + gi)), bl = bfbits2f(ldg_u16(bi + r_lo * spr + gi));
      const float sh = bfbits2f(ldg_u16(sc + r_hi * spr + gi)), bh = bfbits2f(ldg_u16(bi + r_hi * spr + gi));
      uint4 xl, xh;
      load_x16(xrow, gi, t, xl, xh);
      const BFrag8 b = make_bfrag8(xl, xh);
      float c[4] = {0.f, 0.f, 0.f, 0.f}, xs[4] = {0.f, 0.f, 0.f, 0.f};
      mma_group_q8(c, wl, wh, b);
      mma_group_ones8(xs, b);
      affine_fixup(y, c, xs, sl, bl, sh, bh, 2176.0f);
    }
  }
}

}  // namespace fmoe
