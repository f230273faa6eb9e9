// Warp-per-row KV-cache helpers shared by the cache kernels and the decode
// layer: TurboQuant constants (deterministic_signs(n, 42), src/cache.rs:29-43;
// N(0,1) Lloyd-Max tables, src/cache.rs:67-89), the in-register fast
// Walsh-Hadamard transform, MLX-affine quantisation of a row, and the
// TurboQuant round trip (src/cache.rs:94-129).  Lane l of a warp holds
// elements [l*P, (l+1)*P) of a D = 32*P row.
#pragma once
#include "common.cuh"

namespace fmoe {

// ---------------------------------------------------------------------------
// TurboQuant constants: deterministic_signs(n, 42) (src/cache.rs:29-43) and
// the N(0,1) Lloyd-Max tables (src/cache.rs:67-89).

// Sign i is bit i of the packed words (set: -1).  A lane reads the one word
// holding its P signs, so a warp touches at most 16 distinct words (a table
// of floats indexed by lane would serialise 32 ways in the constant cache).
struct SignBits {
  uint32_t w[16];
};
constexpr SignBits make_sign_bits() {
  SignBits t{};
  uint64_t st = 42;
  for (int i = 0; i < 512; ++i) {
    st = st * 6364136223846793005ull + 1442695040888963407ull;
    if ((st >> 63) & 1ull) t.w[i >> 5] |= 1u << (i & 31);
  }
  return t;
}
static __constant__ SignBits kRhtSignBits = make_sign_bits();

struct Codebook {
  float c[16];
  float b[15];
  int n;
};
static __constant__ Codebook kLloyd[3] = {
    {{-1.510f, -0.453f, 0.453f, 1.510f}, {-0.982f, 0.0f, 0.982f}, 4},
    {{-2.152f, -1.344f, -0.756f, -0.245f, 0.245f, 0.756f, 1.344f, 2.152f},
     {-1.748f, -1.050f, -0.501f, 0.0f, 0.501f, 1.050f, 1.748f},
     8},
    {{-2.733f, -2.069f, -1.618f, -1.256f, -0.942f, -0.657f, -0.388f, -0.128f, 0.128f, 0.388f, 0.657f, 0.942f, 1.256f,
      1.618f, 2.069f, 2.733f},
     {-2.401f, -1.844f, -1.437f, -1.099f, -0.800f, -0.522f, -0.258f, 0.0f, 0.258f, 0.522f, 0.800f, 1.099f, 1.437f,
      1.844f, 2.401f},
     16}};

// ---------------------------------------------------------------------------
// warp-per-row helpers

template <int P>
__device__ __forceinline__ void warp_fwht(float (&v)[P], int lane) {
#pragma unroll
  for (int h = 1; h < P; h <<= 1)
#pragma unroll
    for (int i = 0; i < P; i += 2 * h)
#pragma unroll
      for (int j = i; j < i + h; ++j) {
        const float a = v[j], b = v[j + h];
        v[j] = a + b;
        v[j + h] = a - b;
      }
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) {
    const bool upper = (lane & m) != 0;
#pragma unroll
    for (int j = 0; j < P; ++j) {
      const float o = __shfl_xor_sync(0xffffffffu, v[j], m);
      v[j] = upper ? __fsub_rn(o, v[j]) : __fadd_rn(v[j], o);
    }
  }
}

// MLX-affine quantisation of the warp's D values in groups of 64 (64/P lanes
// per group), the oracle's quantize_group arithmetic; codes stored as the
// little-endian bit stream (4-bit: P/8 words per lane, 8-bit: P/4 words).
template <int P, int BITS>
__device__ __forceinline__ void warp_quant_store(const float (&v)[P], int lane, uint32_t* wrow, bf16* srow,
                                                 bf16* brow) {
  constexpr int LG = 64 / P;
  float mn = v[0], mx = v[0];
#pragma unroll
  for (int i = 1; i < P; ++i) {
    mn = fminf(mn, v[i]);
    mx = fmaxf(mx, v[i]);
  }
#pragma unroll
  for (int o = 1; o < LG; o <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const float nmax = (float)((1u << BITS) - 1u);
  float scale = __fdiv_rn(__fsub_rn(mx, mn), nmax);
  if (!(scale >= 1e-7f)) scale = 1e-7f;
  const bf16 sb = __float2bfloat16_rn(scale), bb = __float2bfloat16_rn(mn);
  const float s = __bfloat162float(sb), b = __bfloat162float(bb);
  constexpr int VPW = 32 / BITS;
  uint32_t w[P / VPW];
#pragma unroll
  for (int i = 0; i < P / VPW; ++i) w[i] = 0;
#pragma unroll
  for (int i = 0; i < P; ++i) {
    float q = rintf(__fdiv_rn(__fsub_rn(v[i], b), s));
    q = fminf(fmaxf(q, 0.0f), nmax);
    w[i / VPW] |= (uint32_t)q << (BITS * (i % VPW));
  }
#pragma unroll
  for (int i = 0; i < P / VPW; ++i) wrow[lane * (P / VPW) + i] = w[i];
  if (lane % LG == 0) {
    srow[lane / LG] = sb;
    brow[lane / LG] = bb;
  }
}

// The same quantisation as warp_quant_store, the row replaced by what the
// cache will return for it: bf16(fma(s, q, b)) with the group's bf16 scale and
// bias (MLX dequantisation), in the same basis.
template <int P, int BITS>
__device__ __forceinline__ void warp_quant_round_trip(float (&v)[P], int lane) {
  constexpr int LG = 64 / P;
  float mn = v[0], mx = v[0];
#pragma unroll
  for (int i = 1; i < P; ++i) {
    mn = fminf(mn, v[i]);
    mx = fmaxf(mx, v[i]);
  }
#pragma unroll
  for (int o = 1; o < LG; o <<= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  const float nmax = (float)((1u << BITS) - 1u);
  float scale = __fdiv_rn(__fsub_rn(mx, mn), nmax);
  if (!(scale >= 1e-7f)) scale = 1e-7f;
  const float s = __bfloat162float(__float2bfloat16_rn(scale)), b = __bfloat162float(__float2bfloat16_rn(mn));
#pragma unroll
  for (int i = 0; i < P; ++i) {
    float q = rintf(__fdiv_rn(__fsub_rn(v[i], b), s));
    q = fminf(fmaxf(q, 0.0f), nmax);
    v[i] = __bfloat162float(__float2bfloat16_rn(fmaf(s, q, b)));
  }
}

// The round trip's constants for one lane: the codebook (uniform loads;
// boundaries past the last are +inf) and the lane's P sign bits.  They do not
// depend on the row, so callers can load them early (before a dependency wait).
struct TurboTab {
  float cc[16], bd[15];
  uint32_t sbits;
};
template <int P>
__device__ __forceinline__ TurboTab turbo_tab(int lane, int bits) {
  static_assert(P <= 16, "head_dim up to 512");
  const Codebook& cb = kLloyd[bits - 2];
  const int nc = cb.n;
  TurboTab t;
#pragma unroll
  for (int q = 0; q < 16; ++q) t.cc[q] = q < nc ? cb.c[q] : 0.f;
#pragma unroll
  for (int q = 0; q < 15; ++q) t.bd[q] = q < nc - 1 ? cb.b[q] : INFINITY;
  t.sbits = kRhtSignBits.w[(lane * P) >> 5] >> ((lane * P) & 31);
  return t;
}
// TurboQuant round trip of one row in registers, src/cache.rs:94-129.  With
// R = H diag(s), H the normalised Sylvester matrix:
//   y   = (v / (n + 1e-8)) R sqrt(D) = s (.) FWHT(v / (n + 1e-8))
//   out = n (c[idx] / sqrt(D)) R^T    = n / D * FWHT(s (.) c[idx])
// The centroid is picked by compare / select in registers (no divergent
// constant-memory indexing).
template <int P>
__device__ __forceinline__ void warp_turbo(float (&v)[P], int lane, const TurboTab& tb) {
  constexpr int D = 32 * P;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < P; ++i) ss = fmaf(v[i], v[i], ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float n = sqrtf(ss);
  const float den = n + 1e-8f;
#pragma unroll
  for (int i = 0; i < P; ++i) v[i] = v[i] / den;
  warp_fwht<P>(v, lane);
#pragma unroll
  for (int i = 0; i < P; ++i) {
    const float sg = ((tb.sbits >> i) & 1u) ? -1.0f : 1.0f;
    const float y = v[i] * sg;
    int idx = 0;
#pragma unroll
    for (int q = 0; q < 15; ++q) idx += (y >= tb.bd[q]) ? 1 : 0;
    float c = tb.cc[0];
#pragma unroll
    for (int q = 1; q < 16; ++q) c = idx == q ? tb.cc[q] : c;
    v[i] = c * sg;
  }
  warp_fwht<P>(v, lane);
  const float f = n / (float)D;
#pragma unroll
  for (int i = 0; i < P; ++i) v[i] *= f;
}
template <int P>
__device__ __forceinline__ void warp_turbo(float (&v)[P], int lane, int bits) {
  warp_turbo<P>(v, lane, turbo_tab<P>(lane, bits));
}

}  // namespace fmoe
