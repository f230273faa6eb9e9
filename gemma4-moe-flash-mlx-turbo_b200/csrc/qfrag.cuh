// f16 "1024 + code" tensor-core operands for MLX-affine quantised weights
// (mma.sync m16n8k16, f16 in, fp32 accumulate).  The A operand is built in
// registers from packed codes (exact for codes < 1024); the B operand holds
// the input in the same k order.  Per 64-column group of a row:
//   y += s * C + (b - 1024 s) * sum(x),   C = sum (1024 + q) x.
#pragma once
#include "common.cuh"
#include "stage.cuh"

namespace fmoe {

// (a & m) | (b & ~m) in one instruction.
__device__ __forceinline__ uint32_t sel_bits(uint32_t a, uint32_t b, uint32_t m) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xE4;\n" : "=r"(r) : "r"(a), "r"(b), "r"(m));
  return r;
}

constexpr uint32_t kF16Magic = 0x64006400u;  // f16 1024.0 pairs; low mantissa bits take the code

// A fragments of one 64-column group for rows g (lo) and g+8 (hi), MMA j:
// a[j][0..3] = (row g, slots 2t..), (row g+8, slots 2t..), (row g, slots 2t+8..), (row g+8, slots 2t+8..).
template <int BITS>
__device__ __forceinline__ void load_a_frags(const uint8_t* rlo, const uint8_t* rhi, uint32_t (&a)[4][4]) {
  if constexpr (BITS == 8) {
    // lane's 16 codes = 4 words; word j -> k (4j, 4j+1) and (4j+2, 4j+3)
    const uint4 l = lds_u4(rlo), h = lds_u4(rhi);
    const uint32_t lw[4] = {l.x, l.y, l.z, l.w}, hw[4] = {h.x, h.y, h.z, h.w};
    const uint32_t K = 0x64646464u;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      a[j][0] = prmt(lw[j], K, 0x4140u);
      a[j][1] = prmt(hw[j], K, 0x4140u);
      a[j][2] = prmt(lw[j], K, 0x4342u);
      a[j][3] = prmt(hw[j], K, 0x4342u);
    }
  } else if constexpr (BITS == 4) {
    // lane's 16 codes = 2 words; nibbles (j, j+4) of word 0 and of word 1
    const uint2 l = lds_u2(rlo), h = lds_u2(rhi);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      a[j][0] = and_or(l.x >> (4 * j), 0x000F000Fu, kF16Magic);
      a[j][1] = and_or(h.x >> (4 * j), 0x000F000Fu, kF16Magic);
      a[j][2] = and_or(l.y >> (4 * j), 0x000F000Fu, kF16Magic);
      a[j][3] = and_or(h.y >> (4 * j), 0x000F000Fu, kF16Magic);
    }
  } else {
    static_assert(BITS == 6, "qgemv widths: 4, 6, 8");
    // lane's 16 codes v0..v15 = 96 bits = 3 words; v_i at stream bit 6i.
    // Codes whose bits sit exactly 16 apart share one select + shift:
    // pairs (v0,v8) (v1,v9) (v6,v14) (v7,v15) (v11,v3) (v12,v4), plus
    // (v2,v13) and (v5,v10) from shifted words.
    const uint32_t* pl = reinterpret_cast<const uint32_t*>(rlo);
    const uint32_t* ph = reinterpret_cast<const uint32_t*>(rhi);
    uint32_t r[2][8];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint32_t* p = h ? ph : pl;
      const uint32_t w0 = p[0], w1 = p[1], w2 = p[2];
      const uint32_t t01 = sel_bits(w0, w1, 0x0000FFFFu), t12 = sel_bits(w1, w2, 0x0000FFFFu);
      const uint32_t t20 = sel_bits(w2, w0, 0x0000FFFFu);
      const uint32_t M = 0x003F003Fu;
      r[h][0] = and_or(t01, M, kF16Magic);        // (v0, v8)
      r[h][1] = and_or(t01 >> 6, M, kF16Magic);   // (v1, v9)
      r[h][2] = and_or(t12 >> 4, M, kF16Magic);   // (v6, v14)
      r[h][3] = and_or(t12 >> 10, M, kF16Magic);  // (v7, v15)
      r[h][4] = and_or(t20 >> 2, M, kF16Magic);   // (v11, v3)
      r[h][5] = and_or(t20 >> 8, M, kF16Magic);   // (v12, v4)
      r[h][6] = and_or(sel_bits(w0 >> 12, w2 << 2, 0x0000FFFFu), M, kF16Magic);  // (v2, v13)
      r[h][7] = and_or(sel_bits(__funnelshift_r(w0, w1, 30), __funnelshift_r(w1, w2, 12), 0x0000FFFFu), M,
                       kF16Magic);  // (v5, v10)
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      a[j][0] = r[0][2 * j];
      a[j][1] = r[1][2 * j];
      a[j][2] = r[0][2 * j + 1];
      a[j][3] = r[1][2 * j + 1];
    }
  }
}

// The k pairing of load_a_frags, for the B fragments: MMA j takes
// b0 = (v[p0], v[p0']), b1 = (v[p1], v[p1']) of the lane's 16 inputs.
template <int BITS>
__device__ __forceinline__ void make_b_frags(const float (&v)[16], uint32_t (&b)[8]) {
  if constexpr (BITS == 6) {
    constexpr int lo[8] = {0, 1, 6, 7, 11, 12, 2, 5}, hi[8] = {8, 9, 14, 15, 3, 4, 13, 10};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      b[j] = pack_f16x2(v[lo[2 * j]], v[hi[2 * j]]);
      b[4 + j] = pack_f16x2(v[lo[2 * j + 1]], v[hi[2 * j + 1]]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if constexpr (BITS == 4) {
        b[j] = pack_f16x2(v[j], v[j + 4]);
        b[4 + j] = pack_f16x2(v[8 + j], v[12 + j]);
      } else {
        b[j] = pack_f16x2(v[4 * j], v[4 * j + 1]);
        b[4 + j] = pack_f16x2(v[4 * j + 2], v[4 * j + 3]);
      }
    }
  }
}

__device__ __forceinline__ float f16r(float v) { return __half2float(__float2half_rn(v)); }

}  // namespace fmoe
