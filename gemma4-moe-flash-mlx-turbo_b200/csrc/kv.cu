// Quantised KV cache (append) and split-KV decode attention.
//
// Cache modes
//   FMOE_KV_BF16    K/V stored as bf16 rows: the reference's KVCache storage
//                   (src/cache.rs:266-310).  With turbo_bits 2/3/4 each appended
//                   row first passes through the TurboQuant quantise->dequantise
//                   round trip, as the reference's quantised cache does
//                   (src/cache.rs:290-308).
//   FMOE_KV_AFFINE  rows rotated by the normalised Walsh-Hadamard transform, then
//                   MLX-affine quantised: K 4-bit, V 8-bit, group 64 (the
//                   quantised-KV configuration of the benchmark; no reference
//                   counterpart).  Attention rotates the query by the same
//                   transform and rotates its output back (the normalised WHT
//                   is its own inverse), so callers see the original basis.
//
// Rows live in a ring of `capacity` slots per (batch, kv head): position p is
// slot p % capacity.  A capacity equal to the sliding window keeps exactly the
// last `window` positions (src/cache.rs:139-148, masks src/model/mod.rs:717-753)
// and decode attention attends every valid slot, in any order.
//
// One warp owns one D-vector (D = 256 or 512): lane l holds elements
// [l*P, (l+1)*P), P = D/32.  The WHT is the butterfly network of the oracle
// (stages h = 1, 2, 4, ...: (a, b) -> (a+b, a-b)), in-lane for h < P and over
// shfl_xor for h >= P, so the fp32 rotated values (hence the codes) are the
// oracle's bit for bit.
#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include "internal.h"
#include "common.cuh"
#include "stage.cuh"

namespace fmoe {

// ---------------------------------------------------------------------------
// TurboQuant constants: deterministic_signs(n, 42) (src/cache.rs:29-43) and
// the N(0,1) Lloyd-Max tables (src/cache.rs:67-89).

struct SignTable {
  float s[512];
};
constexpr SignTable make_sign_table() {
  SignTable t{};
  uint64_t st = 42;
  for (int i = 0; i < 512; ++i) {
    st = st * 6364136223846793005ull + 1442695040888963407ull;
    t.s[i] = ((st >> 63) & 1ull) ? -1.0f : 1.0f;
  }
  return t;
}
__constant__ SignTable kRhtSigns = make_sign_table();

struct Codebook {
  float c[16];
  float b[15];
  int n;
};
__constant__ Codebook kLloyd[3] = {
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

template <int P>
__device__ __forceinline__ void load_row_f32(const bf16* row, int lane, float (&v)[P]) {
  const uint4* p = reinterpret_cast<const uint4*>(row + lane * P);
#pragma unroll
  for (int i = 0; i < P / 8; ++i) {
    const uint4 w = p[i];
    v[8 * i + 0] = bf16lo(w.x);
    v[8 * i + 1] = bf16hi(w.x);
    v[8 * i + 2] = bf16lo(w.y);
    v[8 * i + 3] = bf16hi(w.y);
    v[8 * i + 4] = bf16lo(w.z);
    v[8 * i + 5] = bf16hi(w.z);
    v[8 * i + 6] = bf16lo(w.w);
    v[8 * i + 7] = bf16hi(w.w);
  }
}

template <int P>
__device__ __forceinline__ void store_row_bf16(bf16* row, int lane, const float (&v)[P]) {
  uint4* p = reinterpret_cast<uint4*>(row + lane * P);
#pragma unroll
  for (int i = 0; i < P / 8; ++i)
    p[i] = make_uint4(pack_bf16x2(v[8 * i], v[8 * i + 1]), pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                      pack_bf16x2(v[8 * i + 4], v[8 * i + 5]), pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
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

// TurboQuant round trip of one row in registers, src/cache.rs:94-129.  With
// R = H diag(s), H the normalised Sylvester matrix:
//   y   = (v / (n + 1e-8)) R sqrt(D) = s (.) FWHT(v / (n + 1e-8))
//   out = n (c[idx] / sqrt(D)) R^T    = n / D * FWHT(s (.) c[idx])
template <int P>
__device__ __forceinline__ void warp_turbo(float (&v)[P], int lane, int bits) {
  constexpr int D = 32 * P;
  const Codebook& cb = kLloyd[bits - 2];
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
    const float sg = kRhtSigns.s[lane * P + i];
    const float y = v[i] * sg;
    int idx = 0;
    for (int q = 0; q < cb.n - 1; ++q) idx += (y >= cb.b[q]) ? 1 : 0;
    v[i] = cb.c[idx] * sg;
  }
  warp_fwht<P>(v, lane);
  const float f = n / (float)D;
#pragma unroll
  for (int i = 0; i < P; ++i) v[i] *= f;
}

// ---------------------------------------------------------------------------
// append: one warp per new (batch, kv head, token) row, K and V together

template <int P>
__global__ void __launch_bounds__(256) kv_append_kernel(KvDev c, const bf16* __restrict__ kin,
                                                        const bf16* __restrict__ vin, int64_t Tn, int64_t pos,
                                                        const int64_t* __restrict__ pos_dev, int turbo_bits,
                                                        float inv_sqrt_d) {
  constexpr int D = 32 * P, G = D / 64;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);  // (b, h, t)
  if (row >= (int64_t)c.B * c.Hkv * Tn) return;
  const int64_t t = row % Tn;
  if (t < Tn - c.cap) return;  // its slot is overwritten by a later token of the same call
  const int64_t bh = row / Tn;
  const int64_t p0 = pos_dev ? *pos_dev : pos;
  const int64_t dst = bh * c.cap + (p0 + t) % c.cap;
  float kv[P], vv[P];
  load_row_f32<P>(kin + row * D, lane, kv);
  load_row_f32<P>(vin + row * D, lane, vv);
  if (c.mode == FMOE_KV_BF16) {
    if (turbo_bits) {
      warp_turbo<P>(kv, lane, turbo_bits);
      warp_turbo<P>(vv, lane, turbo_bits);
    }
    store_row_bf16<P>(reinterpret_cast<bf16*>(c.k) + dst * D, lane, kv);
    store_row_bf16<P>(reinterpret_cast<bf16*>(c.v) + dst * D, lane, vv);
    return;
  }
  warp_fwht<P>(kv, lane);
  warp_fwht<P>(vv, lane);
#pragma unroll
  for (int i = 0; i < P; ++i) {
    kv[i] *= inv_sqrt_d;
    vv[i] *= inv_sqrt_d;
  }
  warp_quant_store<P, 4>(kv, lane, reinterpret_cast<uint32_t*>(c.k) + dst * (D / 8), c.ks + dst * G, c.kb + dst * G);
  warp_quant_store<P, 8>(vv, lane, reinterpret_cast<uint32_t*>(c.v) + dst * (D / 4), c.vs + dst * G, c.vb + dst * G);
}

template <int P>
__global__ void __launch_bounds__(256) turbo_round_trip_kernel(const bf16* __restrict__ x, int64_t rows, int bits,
                                                               bf16* __restrict__ out) {
  constexpr int D = 32 * P;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  float v[P];
  load_row_f32<P>(x + row * D, lane, v);
  warp_turbo<P>(v, lane, bits);
  store_row_bf16<P>(out + row * D, lane, v);
}

// ---------------------------------------------------------------------------
// Split-KV decode attention.  CTA = (split, kv head, batch); its GQ = Hq/Hkv
// query heads are the N columns of the score MMAs.  A split covers S
// consecutive slots, processed in chunks of CH positions through an NST-stage
// ring of TMA bulk copies (K and V rows with their scales / biases), so the
// next chunk streams in while this one is computed:
//   scores  mma.sync, K rows as A (16 positions x 64-wide group) straight from
//           the 4-bit codes ((128+q) bf16 built in registers), query as B.
//           The rotated query is fp32; it is split into bf16 hi + lo parts
//           (two MMAs) so the scores keep ~16 mantissa bits.  Affine fixup
//           per group: s * C + (b - 128 s) * sum(q).
//   softmax running max / sum per head across chunks (online rescaling).
//   P.V     CUDA cores: a thread owns 4 columns, V dequantised in fp32
//           (fmaf(scale, q, bias), the oracle's dequantisation).
// A split's (m, l, o) goes to the workspace; the last CTA of a (batch, kv
// head) to finish merges the splits (log-sum-exp), normalises, applies the
// inverse rotation and writes the output, so one launch does the whole op.

template <int P, int MODE>
struct AtCfg {
  static constexpr int D = 32 * P, G = D / 64;
  static constexpr int KRB = MODE == FMOE_KV_BF16 ? 2 * D : D / 2;  // K bytes per position
  static constexpr int VRB = MODE == FMOE_KV_BF16 ? 2 * D : D;      // V bytes per position
  static constexpr int SB = MODE == FMOE_KV_BF16 ? 0 : 2 * G;       // bytes of one scale / bias row
  static constexpr int CH = MODE == FMOE_KV_BF16 ? (P == 8 ? 64 : 32) : (P == 8 ? 128 : 64);
  static constexpr int NST = 2;
  static constexpr int KS = CH * KRB, KB = KS + CH * SB, VC = KB + CH * SB, VS = VC + CH * VRB, VB = VS + CH * SB;
  static constexpr int STAGE = VB + CH * SB;  // 53,248 (affine) / 65,536 (bf16) bytes
  static constexpr int TPC = CH / 16;         // 16-position tiles per chunk
  static constexpr int WPT = 8 / TPC;         // warps per tile (they split the groups)
  static constexpr int GPW = G / WPT;         // groups per warp
  static constexpr int U = D / 4;             // P.V: 4-column units per row
  static constexpr int NPH = 256 / U;         // P.V: position phases
  static_assert(STAGE % 128 == 0 && CH % 32 == 0 && G % WPT == 0 && 256 % U == 0, "attention tiling");
};

constexpr int kMaxSplits = 1024;

template <int P, int MODE, int GQ>
struct AtSmem {
  using C = AtCfg<P, MODE>;
  static constexpr int D = C::D;
  static constexpr int BAR = C::NST * C::STAGE;                              // mbarriers
  static constexpr int QH = BAR + 64;                                        // bf16 [GQ][D] query (hi part)
  static constexpr int QL = QH + GQ * D * 2;                                 // bf16 [GQ][D] lo part (affine)
  static constexpr int QS = QL + (MODE == FMOE_KV_AFFINE ? GQ * D * 2 : 0);  // f32 [GQ][G] group sums
  static constexpr int SC = QS + 16 * ((GQ * C::G * 4 + 15) / 16);           // f32 [WPT][GQ][CH] scores
  static constexpr int PR = SC + C::WPT * GQ * C::CH * 4;                    // f32 [GQ][CH] probabilities
  static constexpr int ST = PR + GQ * C::CH * 4;                             // f32 m[8] l[8] f[8], int flags[8]
  static constexpr int BYTES = ST + 32 * 4;
  // aliases of the stage area once every chunk is consumed
  static constexpr int RED = 0;                 // f32 [NPH][GQ][D] P.V phase partials
  static constexpr int WTS = 0;                 // f32 [GQ][kMaxSplits] merge weights
  static constexpr int RED2 = 8 * kMaxSplits * 4;  // f32 [GQ][D] merged rows
  static_assert(C::NPH * GQ * D * 4 <= BAR && RED2 + GQ * D * 4 <= BAR, "attention smem aliases");
};

__device__ __forceinline__ void mma_group_q4_hl(float (&acc)[4], uint2 wlo, uint2 whi, const BFrag4& bh,
                                                const BFrag4& bl) {
#pragma unroll
  for (int s = 0; s < 4; ++s) {
    const uint32_t a0 = nib_pair(wlo.x, 4 * s), a1 = nib_pair(whi.x, 4 * s);
    const uint32_t a2 = nib_pair(wlo.y, 4 * s), a3 = nib_pair(whi.y, 4 * s);
    mma16816(acc, a0, a1, a2, a3, bh.b0[s], bh.b1[s]);
    mma16816(acc, a0, a1, a2, a3, bl.b0[s], bl.b1[s]);
  }
}

// Output row of one head: v / l, rotated back in affine mode.
template <int P, int MODE>
__device__ __forceinline__ void finish_row(float (&v)[P], float l, float inv_sqrt_d, int lane, bf16* orow) {
  const float il = l > 0.f ? 1.0f / l : 0.f;
#pragma unroll
  for (int i = 0; i < P; ++i) v[i] *= il;
  if (MODE == FMOE_KV_AFFINE) {
    warp_fwht<P>(v, lane);
#pragma unroll
    for (int i = 0; i < P; ++i) v[i] *= inv_sqrt_d;
  }
  store_row_bf16<P>(orow, lane, v);
}

template <int P, int MODE, int GQ>
__global__ void __launch_bounds__(256, GQ >= 8 ? 1 : 2)
    attn_decode_kernel(const KvDev c, const bf16* __restrict__ q, int Hq, int S, int nsplit, int64_t nvalid,
                       const int64_t* __restrict__ nvalid_dev, float scale, float inv_sqrt_d,
                       float2* __restrict__ part_ml, float* __restrict__ part_o, unsigned* __restrict__ ctr,
                       bf16* __restrict__ out, int* __restrict__ status) {
  using C = AtCfg<P, MODE>;
  using Sm = AtSmem<P, MODE, GQ>;
  constexpr int D = C::D, G = C::G, CH = C::CH, NST = C::NST;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Sm::BAR);
  bf16* qh = reinterpret_cast<bf16*>(smem + Sm::QH);
  bf16* ql = reinterpret_cast<bf16*>(smem + Sm::QL);
  float* qsum = reinterpret_cast<float*>(smem + Sm::QS);
  float* sc = reinterpret_cast<float*>(smem + Sm::SC);
  float* pr = reinterpret_cast<float*>(smem + Sm::PR);
  float* st_m = reinterpret_cast<float*>(smem + Sm::ST);
  float* st_l = st_m + 8;
  float* st_f = st_m + 16;
  int* flags = reinterpret_cast<int*>(st_m + 24);  // [0] a wait gave up, [1] last arriver

  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int64_t bh = (int64_t)b * c.Hkv + hk;
  int64_t nv = nvalid;
  if (nvalid_dev) nv = min(max(*nvalid_dev, (int64_t)0), c.cap);
  const int64_t p_begin = (int64_t)split * S;
  const int nS = (int)max((int64_t)0, min((int64_t)S, nv - p_begin));
  const int nch = (nS + CH - 1) / CH;

  const int64_t row0 = bh * c.cap + p_begin;  // first slot of this split
  const uint8_t* kc_g = reinterpret_cast<const uint8_t*>(c.k) + row0 * C::KRB;
  const uint8_t* vc_g = reinterpret_cast<const uint8_t*>(c.v) + row0 * C::VRB;
  const uint8_t* ks_g = reinterpret_cast<const uint8_t*>(c.ks) + row0 * C::SB;
  const uint8_t* kb_g = reinterpret_cast<const uint8_t*>(c.kb) + row0 * C::SB;
  const uint8_t* vs_g = reinterpret_cast<const uint8_t*>(c.vs) + row0 * C::SB;
  const uint8_t* vb_g = reinterpret_cast<const uint8_t*>(c.vb) + row0 * C::SB;

  // Chunk ch -> stage ch % NST.  Rows are copied in even counts (16-byte
  // multiples for the 8-byte scale rows); the capacity is a multiple of 16,
  // so the extra row exists.
  auto issue = [&](int chn) {
    const int s = chn % NST;
    const int rows = (min(CH, nS - chn * CH) + 1) & ~1;
    const int64_t r0 = (int64_t)chn * CH;
    uint8_t* sb = smem + s * C::STAGE;
    if (MODE == FMOE_KV_BF16) {
      mbar_arrive_expect_tx(&bar[s], (uint32_t)rows * (C::KRB + C::VRB));
      bulk_g2s(sb, kc_g + r0 * C::KRB, rows * C::KRB, &bar[s]);
      bulk_g2s(sb + C::VC, vc_g + r0 * C::VRB, rows * C::VRB, &bar[s]);
    } else {
      mbar_arrive_expect_tx(&bar[s], (uint32_t)rows * (C::KRB + C::VRB + 4 * C::SB));
      bulk_g2s(sb, kc_g + r0 * C::KRB, rows * C::KRB, &bar[s]);
      bulk_g2s(sb + C::KS, ks_g + r0 * C::SB, rows * C::SB, &bar[s]);
      bulk_g2s(sb + C::KB, kb_g + r0 * C::SB, rows * C::SB, &bar[s]);
      bulk_g2s(sb + C::VC, vc_g + r0 * C::VRB, rows * C::VRB, &bar[s]);
      bulk_g2s(sb + C::VS, vs_g + r0 * C::SB, rows * C::SB, &bar[s]);
      bulk_g2s(sb + C::VB, vb_g + r0 * C::SB, rows * C::SB, &bar[s]);
    }
  };

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < NST; ++s) mbar_init(&bar[s], 1);
    mbar_fence_init();
  }
  if (tid < 8) {
    st_m[tid] = -INFINITY;
    st_l[tid] = 0.f;
    st_f[tid] = 0.f;
    flags[tid] = 0;
  }
  __syncthreads();
  int issued = 0;  // meaningful in thread 0 only
  if (tid == 0)
    for (; issued < min(NST, nch); ++issued) issue(issued);

  // query rows of the CTA's heads, while the first chunks stream in
  if (warp < GQ) {
    float v[P];
    load_row_f32<P>(q + ((int64_t)b * Hq + hk * GQ + warp) * D, lane, v);
    if (MODE == FMOE_KV_AFFINE) {
      warp_fwht<P>(v, lane);
      float hi[P], lo[P], s = 0.f;
#pragma unroll
      for (int i = 0; i < P; ++i) {
        v[i] *= inv_sqrt_d;
        hi[i] = round_bf(v[i]);
        lo[i] = round_bf(v[i] - hi[i]);
        s += hi[i] + lo[i];
      }
      store_row_bf16<P>(qh + warp * D, lane, hi);
      store_row_bf16<P>(ql + warp * D, lane, lo);
#pragma unroll
      for (int o = 1; o < 64 / P; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (lane % (64 / P) == 0) qsum[warp * G + lane / (64 / P)] = s;
    } else {
      store_row_bf16<P>(qh + warp * D, lane, v);
    }
  }
  __syncthreads();

  float o[GQ][4];
#pragma unroll
  for (int h = 0; h < GQ; ++h)
#pragma unroll
    for (int j = 0; j < 4; ++j) o[h][j] = 0.f;

  int ch = 0;
  for (; ch < nch; ++ch) {
    const int stg = ch % NST;
    const int nrow = min(CH, nS - ch * CH);
    const uint8_t* sb = smem + stg * C::STAGE;
    if (!mbar_wait(&bar[stg], (uint32_t)(ch / NST) & 1u, status, 51)) atomicOr(&flags[0], 1);

    // ---- scores (unscaled) -> sc[wp][h][i]
    {
      const int tile = warp % C::TPC, wp = warp / C::TPC, r0 = tile * 16;
      if (r0 < nrow) {
        const int rl = min(r0 + g, nrow - 1), rh = min(r0 + g + 8, nrow - 1);
        float y[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int gg = 0; gg < C::GPW; ++gg) {
          const int gi = wp * C::GPW + gg;
          BFrag4 bq = make_bfrag4(make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0));
          if (g < GQ) {
            const uint8_t* pq = reinterpret_cast<const uint8_t*>(qh) + g * D * 2 + gi * 128 + 32 * t;
            bq = make_bfrag4(lds_u4(pq), lds_u4(pq + 16));
          }
          if (MODE == FMOE_KV_BF16) {
            const uint8_t* kl = sb + rl * C::KRB + gi * 128 + 32 * t;
            const uint8_t* kh = sb + rh * C::KRB + gi * 128 + 32 * t;
            const BFrag4 alo = make_bfrag4(lds_u4(kl), lds_u4(kl + 16));
            const BFrag4 ahi = make_bfrag4(lds_u4(kh), lds_u4(kh + 16));
#pragma unroll
            for (int s4 = 0; s4 < 4; ++s4)
              mma16816(y, alo.b0[s4], ahi.b0[s4], alo.b1[s4], ahi.b1[s4], bq.b0[s4], bq.b1[s4]);
          } else {
            BFrag4 bl = make_bfrag4(make_uint4(0, 0, 0, 0), make_uint4(0, 0, 0, 0));
            if (g < GQ) {
              const uint8_t* pq = reinterpret_cast<const uint8_t*>(ql) + g * D * 2 + gi * 128 + 32 * t;
              bl = make_bfrag4(lds_u4(pq), lds_u4(pq + 16));
            }
            const uint2 wl = lds_u2(sb + rl * C::KRB + gi * 32 + 8 * t);
            const uint2 wh = lds_u2(sb + rh * C::KRB + gi * 32 + 8 * t);
            float cc[4] = {0.f, 0.f, 0.f, 0.f};
            mma_group_q4_hl(cc, wl, wh, bq, bl);
            const bf16* ksc = reinterpret_cast<const bf16*>(sb + C::KS);
            const bf16* kbi = reinterpret_cast<const bf16*>(sb + C::KB);
            const float sl = bf2f(ksc[rl * G + gi]), bl_ = bf2f(kbi[rl * G + gi]);
            const float sh = bf2f(ksc[rh * G + gi]), bh_ = bf2f(kbi[rh * G + gi]);
            const float q0 = 2 * t < GQ ? qsum[(2 * t) * G + gi] : 0.f;
            const float q1 = 2 * t + 1 < GQ ? qsum[(2 * t + 1) * G + gi] : 0.f;
            y[0] += fmaf(sl, cc[0], fmaf(-128.f, sl, bl_) * q0);
            y[1] += fmaf(sl, cc[1], fmaf(-128.f, sl, bl_) * q1);
            y[2] += fmaf(sh, cc[2], fmaf(-128.f, sh, bh_) * q0);
            y[3] += fmaf(sh, cc[3], fmaf(-128.f, sh, bh_) * q1);
          }
        }
        // C fragment: rows = positions (g, g+8), columns = heads (2t, 2t+1)
        float* scw = sc + wp * GQ * CH;
        if (2 * t < GQ) {
          if (r0 + g < nrow) scw[(2 * t) * CH + r0 + g] = y[0];
          if (r0 + g + 8 < nrow) scw[(2 * t) * CH + r0 + g + 8] = y[2];
        }
        if (2 * t + 1 < GQ) {
          if (r0 + g < nrow) scw[(2 * t + 1) * CH + r0 + g] = y[1];
          if (r0 + g + 8 < nrow) scw[(2 * t + 1) * CH + r0 + g + 8] = y[3];
        }
      }
    }
    __syncthreads();
    if (flags[0]) break;  // a copy never landed: every thread leaves the loop here

    // ---- online softmax per head (warp h)
    for (int h = warp; h < GQ; h += 8) {
      float sv[CH / 32];
      float cm = -INFINITY;
#pragma unroll
      for (int j = 0; j < CH / 32; ++j) {
        const int i = lane + 32 * j;
        float s = -INFINITY;
        if (i < nrow) {
          s = 0.f;
#pragma unroll
          for (int w = 0; w < C::WPT; ++w) s += sc[(w * GQ + h) * CH + i];
          s *= scale;
        }
        sv[j] = s;
        cm = fmaxf(cm, s);
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, off));
      const float m_old = st_m[h];
      const float m_new = fmaxf(m_old, cm);
      const float f = expf(m_old - m_new);
      float ls = 0.f;
#pragma unroll
      for (int j = 0; j < CH / 32; ++j) {
        const int i = lane + 32 * j;
        const float p = i < nrow ? expf(sv[j] - m_new) : 0.f;
        pr[h * CH + i] = p;
        ls += p;
      }
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ls += __shfl_xor_sync(0xffffffffu, ls, off);
      __syncwarp();
      if (lane == 0) {
        st_l[h] = fmaf(st_l[h], f, ls);
        st_m[h] = m_new;
        st_f[h] = f;
      }
    }
    __syncthreads();

    // ---- P.V
    {
      const int unit = tid % C::U, ph = tid / C::U;
#pragma unroll
      for (int h = 0; h < GQ; ++h) {
        const float f = st_f[h];
#pragma unroll
        for (int j = 0; j < 4; ++j) o[h][j] *= f;
      }
      for (int i = ph; i < nrow; i += C::NPH) {
        float v4[4];
        if (MODE == FMOE_KV_BF16) {
          const uint2 w = lds_u2(sb + C::VC + i * C::VRB + unit * 8);
          v4[0] = bf16lo(w.x);
          v4[1] = bf16hi(w.x);
          v4[2] = bf16lo(w.y);
          v4[3] = bf16hi(w.y);
        } else {
          const uint32_t w = *reinterpret_cast<const uint32_t*>(sb + C::VC + i * C::VRB + unit * 4);
          const int gi = unit >> 4;
          const float sv = bf2f(reinterpret_cast<const bf16*>(sb + C::VS)[i * G + gi]);
          const float bv = bf2f(reinterpret_cast<const bf16*>(sb + C::VB)[i * G + gi]);
          // byte j placed in the low mantissa bits of 2^23: the subtraction
          // leaves the code exactly
#pragma unroll
          for (int j = 0; j < 4; ++j)
            v4[j] = fmaf(sv, __uint_as_float(prmt(w, 0x4B000000u, 0x7650u | j)) - 8388608.0f, bv);
        }
#pragma unroll
        for (int h = 0; h < GQ; ++h) {
          const float p = pr[h * CH + i];
#pragma unroll
          for (int j = 0; j < 4; ++j) o[h][j] = fmaf(p, v4[j], o[h][j]);
        }
      }
    }
    __syncthreads();
    if (tid == 0 && issued < nch) issue(issued++);
  }
  // Chunks still in flight (only after a wait gave up) must land before the
  // stage area is reused.
  if (tid == 0)
    for (int k = ch; k < issued; ++k) mbar_wait(&bar[k % NST], (uint32_t)(k / NST) & 1u, status, 52);
  const bool failed = flags[0] != 0;
  __syncthreads();

  // ---- reduce the P.V phases, then finish or publish the split
  float* red = reinterpret_cast<float*>(smem + Sm::RED);
  {
    const int unit = tid % C::U, ph = tid / C::U;
#pragma unroll
    for (int h = 0; h < GQ; ++h)
      *reinterpret_cast<float4*>(red + (ph * GQ + h) * D + unit * 4) = make_float4(o[h][0], o[h][1], o[h][2], o[h][3]);
  }
  __syncthreads();
  if (warp < GQ) {
    const int h = warp;
    float v[P];
#pragma unroll
    for (int i = 0; i < P; ++i) {
      float s = 0.f;
#pragma unroll
      for (int ph = 0; ph < C::NPH; ++ph) s += red[(ph * GQ + h) * D + lane * P + i];
      v[i] = s;
    }
    const float m = st_m[h], l = failed ? 0.f : st_l[h];
    const int64_t row = (int64_t)b * Hq + hk * GQ + h;
    if (nsplit == 1) {
      finish_row<P, MODE>(v, l, inv_sqrt_d, lane, out + row * D);
    } else {
      float4* po = reinterpret_cast<float4*>(part_o + (row * nsplit + split) * D + lane * P);
#pragma unroll
      for (int i = 0; i < P / 4; ++i) __stcg(po + i, make_float4(v[4 * i], v[4 * i + 1], v[4 * i + 2], v[4 * i + 3]));
      if (lane == 0) __stcg(part_ml + row * nsplit + split, make_float2(m, l));
    }
  }
  if (nsplit == 1) return;

  // ---- the last CTA of this (batch, kv head) merges the splits
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const unsigned prev = atomicAdd(&ctr[bh], 1u);
    flags[1] = prev == (unsigned)(nsplit - 1);
    if (flags[1]) ctr[bh] = 0u;  // every split has arrived: ready for the next call
  }
  __syncthreads();
  if (!flags[1]) return;
  __threadfence();
  float* wts = reinterpret_cast<float*>(smem + Sm::WTS);
  float* red2 = reinterpret_cast<float*>(smem + Sm::RED2);
  if (warp < GQ) {
    const int64_t row = (int64_t)b * Hq + hk * GQ + warp;
    float M = -INFINITY;
    for (int s = lane; s < nsplit; s += 32) {
      const float2 ml = __ldcg(part_ml + row * nsplit + s);
      if (ml.y > 0.f) M = fmaxf(M, ml.x);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) M = fmaxf(M, __shfl_xor_sync(0xffffffffu, M, off));
    float L = 0.f;
    for (int s = lane; s < nsplit; s += 32) {
      const float2 ml = __ldcg(part_ml + row * nsplit + s);
      const float w = ml.y > 0.f ? expf(ml.x - M) : 0.f;
      wts[warp * kMaxSplits + s] = w;
      L = fmaf(w, ml.y, L);
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) L += __shfl_xor_sync(0xffffffffu, L, off);
    if (lane == 0) st_l[warp] = L;
  }
  __syncthreads();
  for (int pi = tid; pi < GQ * (D / 4); pi += 256) {
    const int h = pi / (D / 4), d4 = pi % (D / 4);
    const int64_t row = (int64_t)b * Hq + hk * GQ + h;
    const float4* src = reinterpret_cast<const float4*>(part_o + row * nsplit * D) + d4;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 4
    for (int s = 0; s < nsplit; ++s) {
      const float w = wts[h * kMaxSplits + s];
      const float4 x = __ldcg(src + (int64_t)s * (D / 4));
      if (w != 0.f) {
        a.x = fmaf(w, x.x, a.x);
        a.y = fmaf(w, x.y, a.y);
        a.z = fmaf(w, x.z, a.z);
        a.w = fmaf(w, x.w, a.w);
      }
    }
    *reinterpret_cast<float4*>(red2 + h * D + d4 * 4) = a;
  }
  __syncthreads();
  if (warp < GQ) {
    float v[P];
#pragma unroll
    for (int i = 0; i < P; ++i) v[i] = red2[warp * D + lane * P + i];
    finish_row<P, MODE>(v, st_l[warp], inv_sqrt_d, lane, out + ((int64_t)b * Hq + hk * GQ + warp) * D);
  }
}

// ---------------------------------------------------------------------------
// host side

static int chunk_positions(int mode, int D) {
  return mode == FMOE_KV_BF16 ? (D == 256 ? AtCfg<8, FMOE_KV_BF16>::CH : AtCfg<16, FMOE_KV_BF16>::CH)
                              : (D == 256 ? AtCfg<8, FMOE_KV_AFFINE>::CH : AtCfg<16, FMOE_KV_AFFINE>::CH);
}

// CTAs the split planner aims for: two resident per SM (each keeps one chunk
// in flight while it computes the other).  The environment variable
// FMOE_ATTN_TARGET_CTAS overrides it (read once; a tuning knob).
static int attn_target_ctas() {
  static const int v = [] {
    const char* e = std::getenv("FMOE_ATTN_TARGET_CTAS");
    const int x = e ? std::atoi(e) : 0;
    return x > 0 ? x : 2 * kNumSMs;
  }();
  return v;
}

AttnPlan attn_plan(const KvDev& c, int64_t n) {
  const int CH = chunk_positions(c.mode, c.D);
  const int64_t chunks = n > 0 ? (n + CH - 1) / CH : 1;
  const int64_t heads = (int64_t)c.B * c.Hkv;
  int64_t ns = (attn_target_ctas() + heads - 1) / heads;
  ns = std::max<int64_t>(1, std::min<int64_t>({ns, chunks, (int64_t)kMaxSplits}));
  const int64_t per = (chunks + ns - 1) / ns;
  AttnPlan p;
  p.S = (int)std::min<int64_t>(per * CH, 1 << 30);
  p.nsplit = (int)((chunks + per - 1) / per);
  return p;
}

struct AttnWs {
  int* status;
  unsigned* ctr;
  float2* ml;
  float* po;
  size_t bytes;
};
static AttnWs carve_attn_ws(void* ws, const KvDev& c, int Hq, int nsplit) {
  uint8_t* base = static_cast<uint8_t*>(ws);
  const size_t rows = (size_t)c.B * Hq;
  AttnWs w;
  size_t off = 256;  // status word
  w.status = reinterpret_cast<int*>(base);
  w.ctr = reinterpret_cast<unsigned*>(base + off);
  off = align_up(off + sizeof(unsigned) * c.B * c.Hkv, 256);
  w.ml = reinterpret_cast<float2*>(base + off);
  off = align_up(off + sizeof(float2) * rows * nsplit, 256);
  w.po = reinterpret_cast<float*>(base + off);
  w.bytes = off + sizeof(float) * rows * nsplit * c.D;
  return w;
}

// Upper bound of attn_plan(c, n).nsplit over every n <= capacity (the split
// count before rounding S up to whole chunks; rounding only lowers it).
static int attn_max_splits(const KvDev& c) {
  const int CH = chunk_positions(c.mode, c.D);
  const int64_t chunks = (c.cap + CH - 1) / CH;
  const int64_t heads = (int64_t)c.B * c.Hkv;
  const int64_t ns = (attn_target_ctas() + heads - 1) / heads;
  return (int)std::max<int64_t>(1, std::min<int64_t>({ns, chunks, (int64_t)kMaxSplits}));
}

size_t attn_workspace_bytes(const KvDev& c, int Hq) {
  return carve_attn_ws(nullptr, c, Hq, attn_max_splits(c)).bytes;
}

int launch_kv_append(const KvDev& c, const bf16* k, const bf16* v, int64_t Tn, int64_t pos, const int64_t* pos_dev,
                     int turbo_bits, cudaStream_t st) {
  const int64_t rows = (int64_t)c.B * c.Hkv * Tn;
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  const float inv = 1.0f / std::sqrt((float)c.D);
  if (c.D == 256) {
    ProfScope prof_("kv_append_kernel", st);
    kv_append_kernel<8><<<blocks, 256, 0, st>>>(c, k, v, Tn, pos, pos_dev, turbo_bits, inv);
  } else {
    ProfScope prof_("kv_append_kernel", st);
    kv_append_kernel<16><<<blocks, 256, 0, st>>>(c, k, v, Tn, pos, pos_dev, turbo_bits, inv);
  }
  return check_launch("kv_append_kernel");
}

int launch_turbo_round_trip(const bf16* x, int64_t rows, int D, int bits, bf16* out, cudaStream_t st) {
  const unsigned blocks = (unsigned)((rows + 7) / 8);
  if (D == 256) {
    ProfScope prof_("turbo_round_trip_kernel", st);
    turbo_round_trip_kernel<8><<<blocks, 256, 0, st>>>(x, rows, bits, out);
  } else {
    ProfScope prof_("turbo_round_trip_kernel", st);
    turbo_round_trip_kernel<16><<<blocks, 256, 0, st>>>(x, rows, bits, out);
  }
  return check_launch("turbo_round_trip_kernel");
}

template <int P, int MODE, int GQ>
static int launch_attn_t(const KvDev& c, const bf16* q, int Hq, const AttnPlan& p, int64_t nvalid,
                         const int64_t* nvalid_dev, float scale, const AttnWs& w, bf16* out, cudaStream_t st) {
  constexpr int bytes = AtSmem<P, MODE, GQ>::BYTES;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [] {
    attr_err =
        cudaFuncSetAttribute(attn_decode_kernel<P, MODE, GQ>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  });
  if (attr_err != cudaSuccess)
    return set_error(FMOE_ERR_CUDA, "attn_decode: shared memory attribute: %s", cudaGetErrorString(attr_err));
  const float inv = 1.0f / std::sqrt((float)(32 * P));
  dim3 grid(p.nsplit, c.Hkv, c.B);
  ProfScope prof_("attn_decode_kernel", st);
  attn_decode_kernel<P, MODE, GQ><<<grid, 256, bytes, st>>>(c, q, Hq, p.S, p.nsplit, nvalid, nvalid_dev, scale, inv,
                                                            w.ml, w.po, w.ctr, out, w.status);
  return check_launch("attn_decode_kernel");
}

template <int P, int MODE>
static int launch_attn_m(const KvDev& c, int GQ, const bf16* q, int Hq, const AttnPlan& p, int64_t nvalid,
                         const int64_t* nvalid_dev, float scale, const AttnWs& w, bf16* out, cudaStream_t st) {
  switch (GQ) {
    case 1: return launch_attn_t<P, MODE, 1>(c, q, Hq, p, nvalid, nvalid_dev, scale, w, out, st);
    case 2: return launch_attn_t<P, MODE, 2>(c, q, Hq, p, nvalid, nvalid_dev, scale, w, out, st);
    case 4: return launch_attn_t<P, MODE, 4>(c, q, Hq, p, nvalid, nvalid_dev, scale, w, out, st);
    case 8: return launch_attn_t<P, MODE, 8>(c, q, Hq, p, nvalid, nvalid_dev, scale, w, out, st);
  }
  return set_error(FMOE_ERR_UNSUPPORTED, "attn_decode: %d query heads per kv head (kernels: 1, 2, 4, 8)", GQ);
}

int launch_attn_decode(const KvDev& c, const bf16* q, int Hq, int64_t nvalid, const int64_t* nvalid_dev, float scale,
                       void* ws, bf16* out, cudaStream_t st) {
  const AttnPlan p = attn_plan(c, nvalid_dev ? c.cap : nvalid);
  const AttnWs w = carve_attn_ws(ws, c, Hq, p.nsplit);
  const int GQ = Hq / c.Hkv;
  if (c.D == 256)
    return c.mode == FMOE_KV_BF16 ? launch_attn_m<8, FMOE_KV_BF16>(c, GQ, q, Hq, p, nvalid, nvalid_dev, scale, w, out, st)
                                  : launch_attn_m<8, FMOE_KV_AFFINE>(c, GQ, q, Hq, p, nvalid, nvalid_dev, scale, w, out,
                                                                     st);
  return c.mode == FMOE_KV_BF16 ? launch_attn_m<16, FMOE_KV_BF16>(c, GQ, q, Hq, p, nvalid, nvalid_dev, scale, w, out, st)
                                : launch_attn_m<16, FMOE_KV_AFFINE>(c, GQ, q, Hq, p, nvalid, nvalid_dev, scale, w, out,
                                                                    st);
}

}  // namespace fmoe

// ---------------------------------------------------------------------------
// extern "C" entry points

using namespace fmoe;

namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Byte offsets of a cache's arrays inside one buffer: bf16 mode k, v;
// affine mode k codes, k scales, k biases, v codes, v scales, v biases.
struct KvLayout {
  size_t off[6];
  int n;
  size_t bytes;
};
int kv_layout(int mode, int B, int Hkv, int D, int64_t cap, KvLayout* L) {
  if (mode != FMOE_KV_BF16 && mode != FMOE_KV_AFFINE) return set_error(FMOE_ERR_INVALID, "kv: mode %d", mode);
  if (D != 256 && D != 512) return set_error(FMOE_ERR_UNSUPPORTED, "kv: head_dim %d (kernels: 256, 512)", D);
  if (B <= 0 || Hkv <= 0 || cap <= 0 || cap % 16)
    return set_error(FMOE_ERR_INVALID, "kv: batch %d kv_heads %d capacity %lld (capacity: a positive multiple of 16)",
                     B, Hkv, (long long)cap);
  const size_t rows = (size_t)B * Hkv * cap;
  size_t sizes[6];
  if (mode == FMOE_KV_BF16) {
    L->n = 2;
    sizes[0] = sizes[1] = rows * D * 2;
  } else {
    L->n = 6;
    sizes[0] = rows * D / 2;
    sizes[3] = rows * D;
    sizes[1] = sizes[2] = sizes[4] = sizes[5] = rows * (D / 64) * 2;
  }
  size_t off = 0;
  for (int i = 0; i < L->n; ++i) {
    L->off[i] = off;
    off = align_up(off + sizes[i], 256);
  }
  L->bytes = off;
  return FMOE_OK;
}

int to_kv(const fmoe_kv_cache_t* c, KvDev* d) {
  if (!c) return set_error(FMOE_ERR_INVALID, "kv: null cache");
  KvLayout L;
  int rc = kv_layout(c->mode, c->batch, c->kv_heads, c->head_dim, c->capacity, &L);
  if (rc) return rc;
  if (c->mode == FMOE_KV_AFFINE && (c->k_bits != 4 || c->v_bits != 8 || c->group_size != 64))
    return set_error(FMOE_ERR_UNSUPPORTED, "kv: affine mode k_bits %d v_bits %d group %d (kernels: 4, 8, 64)",
                     c->k_bits, c->v_bits, c->group_size);
  if (!c->k || !c->v || !aligned16(c->k) || !aligned16(c->v))
    return set_error(FMOE_ERR_ALIGN, "kv: k/v null or not 16-byte aligned");
  if (c->mode == FMOE_KV_AFFINE &&
      (!c->k_scales || !c->k_biases || !c->v_scales || !c->v_biases || !aligned16(c->k_scales) ||
       !aligned16(c->k_biases) || !aligned16(c->v_scales) || !aligned16(c->v_biases)))
    return set_error(FMOE_ERR_ALIGN, "kv: scales/biases null or not 16-byte aligned");
  d->mode = c->mode;
  d->B = c->batch;
  d->Hkv = c->kv_heads;
  d->D = c->head_dim;
  d->cap = c->capacity;
  d->k = c->k;
  d->v = c->v;
  d->ks = static_cast<bf16*>(c->k_scales);
  d->kb = static_cast<bf16*>(c->k_biases);
  d->vs = static_cast<bf16*>(c->v_scales);
  d->vb = static_cast<bf16*>(c->v_biases);
  return FMOE_OK;
}

}  // namespace

extern "C" {

size_t fmoe_kv_cache_bytes(int mode, int batch, int kv_heads, int head_dim, int64_t capacity) {
  KvLayout L;
  return kv_layout(mode, batch, kv_heads, head_dim, capacity, &L) == FMOE_OK ? L.bytes : 0;
}

int fmoe_kv_cache_init(fmoe_kv_cache_t* c, int mode, int batch, int kv_heads, int head_dim, int64_t capacity,
                       void* buffer, size_t buffer_bytes) {
  if (!c) return set_error(FMOE_ERR_INVALID, "kv_cache_init: null cache");
  KvLayout L;
  int rc = kv_layout(mode, batch, kv_heads, head_dim, capacity, &L);
  if (rc) return rc;
  if (!buffer || buffer_bytes < L.bytes)
    return set_error(FMOE_ERR_WORKSPACE, "kv_cache_init: buffer of %zu bytes, %zu needed", buffer_bytes, L.bytes);
  if (!aligned16(buffer)) return set_error(FMOE_ERR_ALIGN, "kv_cache_init: buffer not 16-byte aligned");
  uint8_t* p = static_cast<uint8_t*>(buffer);
  std::memset(c, 0, sizeof(*c));
  c->mode = mode;
  c->batch = batch;
  c->kv_heads = kv_heads;
  c->head_dim = head_dim;
  c->capacity = capacity;
  if (mode == FMOE_KV_BF16) {
    c->k_bits = c->v_bits = 16;
    c->group_size = 0;
    c->k = p + L.off[0];
    c->v = p + L.off[1];
  } else {
    c->k_bits = 4;
    c->v_bits = 8;
    c->group_size = 64;
    c->k = p + L.off[0];
    c->k_scales = p + L.off[1];
    c->k_biases = p + L.off[2];
    c->v = p + L.off[3];
    c->v_scales = p + L.off[4];
    c->v_biases = p + L.off[5];
  }
  return FMOE_OK;
}

int fmoe_kv_append(const fmoe_kv_cache_t* cache, const void* k, const void* v, int64_t T_new, int64_t pos,
                   const int64_t* pos_dev, int turbo_bits, void* stream) {
  KvDev c;
  int rc = to_kv(cache, &c);
  if (rc) return rc;
  if (T_new < 0 || pos < 0) return set_error(FMOE_ERR_INVALID, "kv_append: T_new %lld pos %lld", (long long)T_new,
                                             (long long)pos);
  if (T_new == 0) return FMOE_OK;
  if (!k || !v || !aligned16(k) || !aligned16(v)) return set_error(FMOE_ERR_ALIGN, "kv_append: k/v null or misaligned");
  if (turbo_bits != 0 && (c.mode != FMOE_KV_BF16 || turbo_bits < 2 || turbo_bits > 4))
    return set_error(FMOE_ERR_INVALID, "kv_append: turbo_bits %d (0, or 2..4 with the bf16 mode)", turbo_bits);
  return launch_kv_append(c, static_cast<const bf16*>(k), static_cast<const bf16*>(v), T_new, pos, pos_dev,
                          turbo_bits, static_cast<cudaStream_t>(stream));
}

size_t fmoe_attn_decode_workspace_bytes(const fmoe_kv_cache_t* cache, int q_heads) {
  KvDev c;
  if (to_kv(cache, &c) != FMOE_OK || q_heads <= 0) return 0;
  return attn_workspace_bytes(c, q_heads);
}

int fmoe_attn_decode(const fmoe_kv_cache_t* cache, const void* q, int q_heads, int64_t n_valid,
                     const int64_t* n_valid_dev, float scale, void* out, void* workspace, size_t workspace_bytes,
                     void* stream) {
  KvDev c;
  int rc = to_kv(cache, &c);
  if (rc) return rc;
  if (q_heads <= 0 || q_heads % c.Hkv || q_heads / c.Hkv > 8)
    return set_error(FMOE_ERR_UNSUPPORTED, "attn_decode: %d query heads over %d kv heads (1..8 per kv head)", q_heads,
                     c.Hkv);
  const int gq = q_heads / c.Hkv;
  if (gq != 1 && gq != 2 && gq != 4 && gq != 8)
    return set_error(FMOE_ERR_UNSUPPORTED, "attn_decode: %d query heads per kv head (kernels: 1, 2, 4, 8)", gq);
  if (!q || !out || !aligned16(q) || !aligned16(out))
    return set_error(FMOE_ERR_ALIGN, "attn_decode: q/out null or not 16-byte aligned");
  if (n_valid < 0) return set_error(FMOE_ERR_INVALID, "attn_decode: n_valid %lld", (long long)n_valid);
  const size_t need = attn_workspace_bytes(c, q_heads);
  if (!workspace || workspace_bytes < need || !aligned16(workspace))
    return set_error(FMOE_ERR_WORKSPACE, "attn_decode: workspace of %zu bytes, %zu needed (16-byte aligned)",
                     workspace_bytes, need);
  return launch_attn_decode(c, static_cast<const bf16*>(q), q_heads, std::min<int64_t>(n_valid, c.cap), n_valid_dev,
                            scale, workspace, static_cast<bf16*>(out), static_cast<cudaStream_t>(stream));
}

int fmoe_turbo_round_trip(const void* x, int64_t rows, int head_dim, int bits, void* out, void* stream) {
  if (head_dim != 256 && head_dim != 512)
    return set_error(FMOE_ERR_UNSUPPORTED, "turbo_round_trip: head_dim %d (kernels: 256, 512)", head_dim);
  if (bits < 2 || bits > 4) return set_error(FMOE_ERR_INVALID, "turbo_round_trip: bits %d (2..4)", bits);
  if (rows < 0) return set_error(FMOE_ERR_INVALID, "turbo_round_trip: rows %lld", (long long)rows);
  if (rows == 0) return FMOE_OK;
  if (!x || !out || !aligned16(x) || !aligned16(out))
    return set_error(FMOE_ERR_ALIGN, "turbo_round_trip: x/out null or not 16-byte aligned");
  return launch_turbo_round_trip(static_cast<const bf16*>(x), rows, head_dim, bits, static_cast<bf16*>(out),
                                 static_cast<cudaStream_t>(stream));
}

}  // extern "C"
