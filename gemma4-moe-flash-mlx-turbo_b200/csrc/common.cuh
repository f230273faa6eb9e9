// Shared device helpers for libfmoe (sm_100a).
//
// Quantised weights follow MLX's affine layout: a row of `in` values is a
// little-endian bit stream of `bits`-wide codes packed into uint32 words, with
// one bf16 scale and one bf16 bias per `group` (64) consecutive values:
// w ~= scale * q + bias.
//
// Decode-time GEMVs run on the legacy warp-level tensor-core instruction
// (mma.sync m16n8k16, bf16 in, fp32 accumulate) because its A operand comes
// from registers: the 4-bit codes are turned into bf16 operands in registers
// (one LOP3 per code pair) and never touch shared memory.  Rows of the weight
// are the M dimension, tokens are N (8 per instruction), so one weight load
// serves up to 8 tokens.
//
// Fragment bookkeeping (PTX ISA, mma.m16n8k16 .bf16): lane = 4*g + t,
//   A: a0=(row g, k 2t..2t+1) a1=(row g+8, k 2t..) a2=(row g, k 2t+8..) a3=(row g+8, k 2t+8..)
//   B: b0=(k 2t..2t+1, col g)  b1=(k 2t+8..2t+9, col g)
//   C: c0=(row g, col 2t) c1=(row g, col 2t+1) c2=(row g+8, col 2t) c3=(row g+8, col 2t+1)
// A dot product does not depend on the order of its k terms, so the kernels
// assign physical columns to logical k slots in whatever order makes the
// weight side cheapest, and build the x (B) fragments with the same order.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace fmoe {

typedef __nv_bfloat16 bf16;

__device__ __forceinline__ float bf16lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
__device__ __forceinline__ float bf2f(bf16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float bfbits2f(uint16_t v) { return __uint_as_float(static_cast<uint32_t>(v) << 16); }

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// D = A * B + C, m16n8k16, bf16 operands, fp32 accumulators.
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Same shape with f16 operands (A and B both f16).
__device__ __forceinline__ void mma16816_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_f16x2(float lo, float hi) {
  __half2 v = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

// (a & b) | c in one instruction.
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
  uint32_t r;
  asm("lop3.b32 %0, %1, %2, %3, 0xEA;\n" : "=r"(r) : "r"(a), "r"(b), "r"(c));
  return r;
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;\n" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// Two 4-bit codes at bit offsets `sh` and `sh + 16` of `w` as the bf16 pair
// (128 + q_lo, 128 + q_hi): bf16 0x4300 is 128.0 with unit mantissa steps.
__device__ __forceinline__ uint32_t nib_pair(uint32_t w, int sh) {
  return and_or(w >> sh, 0x000f000fu, 0x43004300u);
}

// Read-only streaming loads that do not allocate in L1 (weights are read once).
__device__ __forceinline__ uint2 ldg_stream_u2(const void* p) {
  uint2 r;
  asm("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];\n" : "=r"(r.x), "=r"(r.y) : "l"(p));
  return r;
}
__device__ __forceinline__ uint4 ldg_stream_u4(const void* p) {
  uint4 r;
  asm("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];\n"
      : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
      : "l"(p));
  return r;
}
__device__ __forceinline__ uint16_t ldg_u16(const void* p) {
  unsigned short r;
  asm("ld.global.nc.u16 %0, [%1];\n" : "=h"(r) : "l"(p));
  return r;
}
__device__ __forceinline__ uint4 ldg_u4(const void* p) {
  uint4 r;
  asm("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];\n" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
// Coherent (non-.nc) 16-byte load, for buffers written earlier in the same
// kernel or by the previous kernel in a programmatic-dependent chain.
__device__ __forceinline__ uint4 ld_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];\n" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}

// Asynchronous 16-byte global -> shared copies (LDGSTS), bypassing L1.
__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory");
}
// Copy `bytes` (multiple of 16, both addresses 16-byte aligned) with the
// `nthr` threads of index `tid`.
__device__ __forceinline__ void cp_async_block(void* smem, const void* gmem, int bytes, int tid, int nthr) {
  uint8_t* d = static_cast<uint8_t*>(smem);
  const uint8_t* s = static_cast<const uint8_t*>(gmem);
  for (int o = tid * 16; o < bytes; o += nthr * 16) cp_async16(d + o, s + o);
}

__device__ __forceinline__ uint2 lds_u2(const void* p) { return *static_cast<const uint2*>(p); }
__device__ __forceinline__ float lds_bf(const bf16* p) { return __bfloat162float(*p); }

// B fragments for one 64-wide group of one token, 4-bit weight order.
// Lane t holds x[16t .. 16t+15] of the group as X[0..7] (bf16 pairs); the
// 4-bit A side puts codes (s, s+4) of a word in one register, so step s uses
//   b0 = (x[s], x[s+4]),  b1 = (x[8+s], x[12+s]).
struct BFrag4 {
  uint32_t b0[4], b1[4];
};
__device__ __forceinline__ BFrag4 make_bfrag4(uint4 lo, uint4 hi) {
  BFrag4 f;
  f.b0[0] = prmt(lo.x, lo.z, 0x5410u);
  f.b0[1] = prmt(lo.x, lo.z, 0x7632u);
  f.b0[2] = prmt(lo.y, lo.w, 0x5410u);
  f.b0[3] = prmt(lo.y, lo.w, 0x7632u);
  f.b1[0] = prmt(hi.x, hi.z, 0x5410u);
  f.b1[1] = prmt(hi.x, hi.z, 0x7632u);
  f.b1[2] = prmt(hi.y, hi.w, 0x5410u);
  f.b1[3] = prmt(hi.y, hi.w, 0x7632u);
  return f;
}

// acc[16 rows x 8 tokens] += (128 + q) . x over one 64-wide group of a 4-bit
// weight tile.  wlo / whi: words (2t, 2t+1) of the group for rows g and g+8.
__device__ __forceinline__ void mma_group_q4(float (&acc)[4], uint2 wlo, uint2 whi, const BFrag4& b) {
#pragma unroll
  for (int s = 0; s < 4; ++s)
    mma16816(acc, nib_pair(wlo.x, 4 * s), nib_pair(whi.x, 4 * s), nib_pair(wlo.y, 4 * s),
             nib_pair(whi.y, 4 * s), b.b0[s], b.b1[s]);
}

// Per-group sum of x for each of the 8 tokens, laid out like the C fragment,
// from one MMA chain against an all-ones A operand.
__device__ __forceinline__ void mma_group_ones(float (&xs)[4], const BFrag4& b) {
  const uint32_t one = 0x3f803f80u;
#pragma unroll
  for (int s = 0; s < 4; ++s) mma16816(xs, one, one, one, one, b.b0[s], b.b1[s]);
}

__device__ __forceinline__ float gelu_tanh(float g) {
  const float k0 = 0.7978845608028654f;
  return 0.5f * g * (1.0f + tanhf(k0 * (g + 0.044715f * g * g * g)));
}

__device__ __forceinline__ float round_bf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }

}  // namespace fmoe
