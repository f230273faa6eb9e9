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
#include "rowops.cuh"
#include "kvrow.cuh"

namespace fmoe {

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
// Decode-step attention input: the q / k / v projections (fp32, one row per
// sequence) -> per-head RMSNorm -> RoPE -> query rows for attention and the
// new K / V rows appended to the cache, one warp per (sequence, head) row; a
// kv head's K and V rows take separate warps (the TurboQuant round trip of each
// is a chain of dependent shuffles, so the two run side by side).
// Follows Gemma4Attention::forward, src/model/gemma4_attention.rs:46-84:
//   q = rope(q_norm(q_proj x));  k = rope(k_norm(k_proj x));
//   v = v_norm(v_proj x), or v_norm(k_proj x) before k_norm when K == V;
// every tensor rounded to bf16 as the reference's bf16 arrays are.  RoPE is
// MLX fast::rope, non-traditional: the first rope_dims dims rotate in pairs
// (i, i + rope_dims/2) by angle pos * inv_freq[i].

// v[i] = sum over the `parts` fp32 slices (part_stride apart, added in slice
// order) of src[i], i < P (src 16-byte aligned); every slice of a batch in
// flight together.
template <int P>
__device__ __forceinline__ void sum_slices(const float* src, int parts, int64_t part_stride, float (&v)[P]) {
#pragma unroll
  for (int i = 0; i < P; ++i) v[i] = 0.f;
  constexpr int NB = P <= 8 ? 8 : 4;  // slices per batch
  for (int p0 = 0; p0 < parts; p0 += NB) {
    float4 w[NB][P / 4];  // the lane's P contiguous floats as 16-byte loads (coalesced)
#pragma unroll
    for (int u = 0; u < NB; ++u)
#pragma unroll
      for (int i = 0; i < P / 4; ++i)
        w[u][i] = p0 + u < parts ? __ldcg(reinterpret_cast<const float4*>(src + (p0 + u) * part_stride) + i)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int u = 0; u < NB; ++u)
      if (p0 + u < parts)
#pragma unroll
        for (int i = 0; i < P / 4; ++i) {
          v[4 * i] += w[u][i].x;
          v[4 * i + 1] += w[u][i].y;
          v[4 * i + 2] += w[u][i].z;
          v[4 * i + 3] += w[u][i].w;
        }
  }
}

template <int P>
__global__ void __launch_bounds__(256) qkv_post_kernel(KvDev c, const float* __restrict__ qkv, int ld, int parts,
                                                       int64_t part_stride, int Hq,
                                                       int k_eq_v, const bf16* __restrict__ q_norm,
                                                       const bf16* __restrict__ k_norm, float eps, int rope_dims,
                                                       float log2_theta, int64_t pos,
                                                       const int64_t* __restrict__ pos_dev, bf16* __restrict__ q_out,
                                                       int turbo_bits, float inv_sqrt_d) {
  constexpr int D = 32 * P, G = D / 64;
  const int lane = threadIdx.x & 31;
  const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int Hkv = c.Hkv, T = c.B;  // one token per sequence
  const bool is_q = row < T * Hq;
  // rows past the queries: (sequence, kv head) pairs, K then V on separate warps
  const bool is_v = !is_q && ((row - T * Hq) & 1);
  // Before the dependency wait, what does not depend on the projections: the
  // norm weights and the RoPE cos / sin of this step's position.  The device
  // position is written at least two kernels earlier in the stream (before
  // the preceding kernel's own wait), so it is final here.
  const int64_t p0 = pos_dev ? *pos_dev : pos;
  float nwv[P], cs[P], sn[P];
  const bf16* nwp = is_q ? q_norm : (is_v ? nullptr : k_norm);
  uint4 nraw[P / 8];  // the norm weights' bits, in flight across the wait
#pragma unroll
  for (int i = 0; i < P / 8; ++i) nraw[i] = nwp ? reinterpret_cast<const uint4*>(nwp + lane * P)[i] : make_uint4(0, 0, 0, 0);
  rope_angles<P>(rope_dims, log2_theta, (float)p0, lane, cs, sn);
  TurboTab ttab;  // the round trip's constants, loaded before the wait
  if (turbo_bits && !is_q && c.mode == FMOE_KV_BF16) ttab = turbo_tab<P>(lane, turbo_bits);
  griddep_wait();  // the projections come from the preceding kernel
  griddep_launch_dependents();
#pragma unroll
  for (int i = 0; i < P / 8; ++i) {
    const uint32_t w4[4] = {nraw[i].x, nraw[i].y, nraw[i].z, nraw[i].w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      nwv[8 * i + 2 * e] = nwp ? bf16lo(w4[e]) : 1.f;
      nwv[8 * i + 2 * e + 1] = nwp ? bf16hi(w4[e]) : 1.f;
    }
  }
  if (row >= T * (Hq + 2 * Hkv)) return;
  float v[P];
  if (is_q) {
    const int t = row / Hq, h = row % Hq;
    sum_slices<P>(qkv + (int64_t)t * ld + h * D + lane * P, parts, part_stride, v);
#pragma unroll
    for (int i = 0; i < P; ++i) v[i] = round_bf(v[i]);
    warp_rms_norm_w<P>(v, nwv, q_norm != nullptr, eps, lane);
    warp_rope_cs<P>(v, rope_dims, cs, sn, lane);
    store_row_bf16<P>(q_out + ((int64_t)t * Hq + h) * D, lane, v);
    return;
  }
  const int r = (row - T * Hq) >> 1, t = r / Hkv, hk = r % Hkv;
  const float* ks = qkv + (int64_t)t * ld + (Hq + hk) * D + lane * P;
  // V: the value projection, or the raw key projection when K == V (before k_norm)
  const float* src = !is_v ? ks : k_eq_v ? ks : qkv + (int64_t)t * ld + (Hq + Hkv + hk) * D + lane * P;
  float x[P];
  sum_slices<P>(src, parts, part_stride, x);
#pragma unroll
  for (int i = 0; i < P; ++i) x[i] = round_bf(x[i]);
  if (is_v) {
    warp_rms_norm<P>(x, nullptr, eps, lane);  // v_norm: no learned scale
  } else {
    warp_rms_norm_w<P>(x, nwv, k_norm != nullptr, eps, lane);
    warp_rope_cs<P>(x, rope_dims, cs, sn, lane);
  }
  const int64_t dst = ((int64_t)t * Hkv + hk) * c.cap + p0 % c.cap;
  if (c.mode == FMOE_KV_BF16) {
    if (turbo_bits) warp_turbo<P>(x, lane, ttab);
    store_row_bf16<P>(reinterpret_cast<bf16*>(is_v ? c.v : c.k) + dst * D, lane, x);
    return;
  }
  warp_fwht<P>(x, lane);
#pragma unroll
  for (int i = 0; i < P; ++i) x[i] *= inv_sqrt_d;
  if (is_v)
    warp_quant_store<P, 8>(x, lane, reinterpret_cast<uint32_t*>(c.v) + dst * (D / 4), c.vs + dst * G, c.vb + dst * G);
  else
    warp_quant_store<P, 4>(x, lane, reinterpret_cast<uint32_t*>(c.k) + dst * (D / 8), c.ks + dst * G, c.kb + dst * G);
}

// ---------------------------------------------------------------------------
// Split-KV decode attention.  CTA = (split, kv head, batch); its GQ = Hq/Hkv
// query heads are the N columns of the MMAs.  A split covers S consecutive
// slots, processed in chunks of CH positions through a two-stage ring of TMA
// bulk copies (K and V rows with their scales / biases): the next chunk
// streams in while this one is computed.  Per chunk:
//   scores  mma.sync, K rows as A (16 positions x 64-wide group).  Affine
//           cache: A = (128 + q) bf16 built in registers from the 4-bit codes;
//           the rotated query is fp32, split into bf16 hi + lo parts (two
//           MMAs, ~16 mantissa bits kept), B fragments prepared once per CTA;
//           per-group fixup s * C + (b - 128 s) * sum(q).  bf16 cache: A = K.
//   softmax running max / sum per head across chunks (online rescaling); the
//           tile maxima are exchanged through shared memory, probabilities
//           stay with the warp that scored them.
//   P.V     affine: tensor cores (f16): A = V codes as (1024 + q), two
//           positions per register; B = p * v_scale; a second MMA with
//           A = -1024 removes the offset; the bias half of V is summed in fp32.
//           bf16: CUDA cores, a thread owns 4 columns of one position phase.
// A split's (m, l, o) goes to the workspace; the last CTA of a (batch, kv
// head) to finish merges the splits (log-sum-exp), normalises, applies the
// inverse rotation and writes the output, so one launch does the whole op.

template <int P, int MODE>
struct AtCfg {
  static constexpr int D = 32 * P, G = D / 64;
  static constexpr int KRB = MODE == FMOE_KV_BF16 ? 2 * D : D / 2;  // K bytes per position
  static constexpr int VRB = MODE == FMOE_KV_BF16 ? 2 * D : D;      // V bytes per position
  static constexpr int SB = MODE == FMOE_KV_BF16 ? 0 : 2 * G;       // bytes of one scale / bias row
  // bf16 cache at head_dim 256: 32-position chunks (two 32 KB stages) leave room
  // on the SM for the next kernel of a decode chain
  static constexpr int CH = MODE == FMOE_KV_BF16 ? 32 : (P == 8 ? 128 : 64);
  static constexpr int NST = 2;
  static constexpr int KS = CH * KRB, KB = KS + CH * SB, VC = KB + CH * SB, VS = VC + CH * VRB, VB = VS + CH * SB;
  static constexpr int STAGE = VB + CH * SB;  // 53,248 (affine) / 32,768 or 65,536 (bf16) bytes
  static constexpr int TPC = CH / 16;         // 16-position tiles per chunk
  static constexpr int WPT = 8 / TPC;         // warps per tile (they split the groups)
  static constexpr int GPW = G / WPT;         // groups per warp
  // bf16 P.V on CUDA cores: a thread owns 4 columns of one position phase
  static constexpr int U = D / 4;
  static constexpr int NPH = 256 / U;
  // affine P.V on tensor cores: a warp owns one 64-column group and KTW of
  // the chunk's KT 16-position k-tiles
  static constexpr int KT = CH / 16;
  static constexpr int WPG = 8 / G;
  static constexpr int KTW = KT / WPG;
  static constexpr int RSL = MODE == FMOE_KV_BF16 ? NPH : WPG;  // partial rows reduced at the end
  static_assert(STAGE % 128 == 0 && CH % 32 == 0 && G % WPT == 0 && 256 % U == 0 && KT % WPG == 0,
                "attention tiling");
};

constexpr int kMaxSplits = 1024;
constexpr int kRed2Off = 8 * kMaxSplits * 4;  // merged rows, after the merge weights

// Global sources of one split (first slot p_begin of (batch, kv head) bh).
struct SplitSrc {
  const uint8_t *kc, *ks, *kb, *vc, *vs, *vb;
};
template <class C>
__device__ __forceinline__ SplitSrc split_src(const KvDev& c, int64_t row0) {
  SplitSrc s;
  s.kc = reinterpret_cast<const uint8_t*>(c.k) + row0 * C::KRB;
  s.vc = reinterpret_cast<const uint8_t*>(c.v) + row0 * C::VRB;
  s.ks = reinterpret_cast<const uint8_t*>(c.ks) + row0 * C::SB;
  s.kb = reinterpret_cast<const uint8_t*>(c.kb) + row0 * C::SB;
  s.vs = reinterpret_cast<const uint8_t*>(c.vs) + row0 * C::SB;
  s.vb = reinterpret_cast<const uint8_t*>(c.vb) + row0 * C::SB;
  return s;
}

// Chunk chn of the split -> stage chn % NST.  Rows are copied in even counts
// (16-byte multiples for the 8-byte scale rows); the capacity is a multiple of
// 16, so the extra row exists.
template <class C, int MODE>
__device__ __forceinline__ void issue_chunk(uint8_t* smem, uint64_t* bar, const SplitSrc& src, int chn, int nS) {
  const int s = chn % C::NST;
  const int rows = (min(C::CH, nS - chn * C::CH) + 1) & ~1;
  const int64_t r0 = (int64_t)chn * C::CH;
  uint8_t* sb = smem + s * C::STAGE;
  if (MODE == FMOE_KV_BF16) {
    mbar_arrive_expect_tx(&bar[s], (uint32_t)rows * (C::KRB + C::VRB));
    bulk_g2s(sb, src.kc + r0 * C::KRB, rows * C::KRB, &bar[s]);
    bulk_g2s(sb + C::VC, src.vc + r0 * C::VRB, rows * C::VRB, &bar[s]);
  } else {
    mbar_arrive_expect_tx(&bar[s], (uint32_t)rows * (C::KRB + C::VRB + 4 * C::SB));
    bulk_g2s(sb, src.kc + r0 * C::KRB, rows * C::KRB, &bar[s]);
    bulk_g2s(sb + C::KS, src.ks + r0 * C::SB, rows * C::SB, &bar[s]);
    bulk_g2s(sb + C::KB, src.kb + r0 * C::SB, rows * C::SB, &bar[s]);
    bulk_g2s(sb + C::VC, src.vc + r0 * C::VRB, rows * C::VRB, &bar[s]);
    bulk_g2s(sb + C::VS, src.vs + r0 * C::SB, rows * C::SB, &bar[s]);
    bulk_g2s(sb + C::VB, src.vb + r0 * C::SB, rows * C::SB, &bar[s]);
  }
}

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

// End of a split, called by every thread of the CTA.  red holds RSL partial
// rows per head ([RSL][GQ][D] f32, at the start of the stage area), st_m /
// st_l the split's running max / sum per head.  One split: finish the rows.
// Several: publish (m, l, o) and let the last CTA of the (batch, kv head)
// merge them.
template <int P, int MODE, int GQ, int RSL>
__device__ __forceinline__ void attn_epilogue(uint8_t* smem, const float* st_m, float* st_l, int* flags, bool failed,
                                              int Hq, int b, int hk, int64_t bh, int split, int nsplit,
                                              float inv_sqrt_d, float2* part_ml, float* part_o, unsigned* ctr,
                                              bf16* out) {
  constexpr int D = 32 * P;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const float* red = reinterpret_cast<const float*>(smem);
  if (warp < GQ) {
    const int h = warp;
    float v[P];
#pragma unroll
    for (int i = 0; i < P; ++i) {
      float s = 0.f;
#pragma unroll
      for (int r = 0; r < RSL; ++r) s += red[(r * GQ + h) * D + lane * P + i];
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
  float* wts = reinterpret_cast<float*>(smem);
  float* red2 = reinterpret_cast<float*>(smem + kRed2Off);
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
  for (int pi = tid; pi < GQ * (D / 4); pi += blockDim.x) {
    const int h = pi / (D / 4), d4 = pi % (D / 4);
    const int64_t row = (int64_t)b * Hq + hk * GQ + h;
    const float4* src = reinterpret_cast<const float4*>(part_o + row * nsplit * D) + d4;
    float4 a = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int s0 = 0; s0 < nsplit; s0 += 8) {  // 8 loads in flight, summed in split order
      float4 x[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        x[j] = s0 + j < nsplit ? __ldcg(src + (int64_t)(s0 + j) * (D / 4)) : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float w = s0 + j < nsplit ? wts[h * kMaxSplits + s0 + j] : 0.f;
        if (w != 0.f) {
          a.x = fmaf(w, x[j].x, a.x);
          a.y = fmaf(w, x[j].y, a.y);
          a.z = fmaf(w, x[j].z, a.z);
          a.w = fmaf(w, x[j].w, a.w);
        }
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

// ---- affine (WHT-rotated 4-bit K / 8-bit V) cache

template <int P, int GQ>
struct AffSmem {
  using C = AtCfg<P, FMOE_KV_AFFINE>;
  static constexpr int D = C::D, G = C::G;
  static constexpr int BAR = C::NST * C::STAGE;                    // mbarriers
  static constexpr int QF = BAR + 64;                              // uint4 [G][hi, lo][4*GQ lanes][2] B fragments
  static constexpr int QR = QF + G * 2 * 4 * GQ * 32;              // bf16 [hi, lo][GQ][D] rotated query rows
  static constexpr int QS = QR + 2 * GQ * D * 2;                   // f32 [GQ][G] group sums of hi + lo
  static constexpr int SC = QS + 16 * ((GQ * G * 4 + 15) / 16);    // f32 [GQ][CH] second-half partial scores
  static constexpr int TM = SC + (C::WPT > 1 ? GQ * C::CH * 4 : 0);  // f32 [TPC][8] tile maxima / sums
  static constexpr int PR = TM + C::TPC * 8 * 4;                   // f32 [GQ][CH] probabilities
  static constexpr int ST = PR + GQ * C::CH * 4;                   // f32 m[8] l[8] pad[8], int flags[8]
  static constexpr int BYTES = ST + 32 * 4;
  static_assert(C::RSL * GQ * D * 4 <= BAR && kRed2Off + GQ * D * 4 <= BAR, "attention smem aliases");
};

template <int P, int GQ>
__global__ void __launch_bounds__(256, GQ >= 8 ? 1 : 2)
    attn_affine_kernel(const KvDev c, const bf16* __restrict__ q, int Hq, int S, int nsplit, int64_t nvalid,
                       const int64_t* __restrict__ nvalid_dev, float scale, float inv_sqrt_d,
                       float2* __restrict__ part_ml, float* __restrict__ part_o, unsigned* __restrict__ ctr,
                       bf16* __restrict__ out, int* __restrict__ status, int64_t newest,
                     const int64_t* __restrict__ newest_dev) {
  using C = AtCfg<P, FMOE_KV_AFFINE>;
  using Sm = AffSmem<P, GQ>;
  // Launched as a programmatic dependent, q and the newest cache rows come
  // from the preceding kernel: every chunk but the one holding the row
  // appended at position `newest` (slot newest % cap; -1: none) is copied
  // before the dependency wait.  The position and slot count are written at
  // least two kernels earlier in the stream, so they are final here.
  constexpr int D = C::D, G = C::G, CH = C::CH, NST = C::NST, TPC = C::TPC, WPT = C::WPT, GPW = C::GPW;
  static_assert(GPW == 4, "a scale row of a warp's groups is one 8-byte load");
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Sm::BAR);
  uint4* qf = reinterpret_cast<uint4*>(smem + Sm::QF);
  bf16* qrow = reinterpret_cast<bf16*>(smem + Sm::QR);
  float* qsum = reinterpret_cast<float*>(smem + Sm::QS);
  float* scp = reinterpret_cast<float*>(smem + Sm::SC);
  float* tmax = reinterpret_cast<float*>(smem + Sm::TM);
  float* pr = reinterpret_cast<float*>(smem + Sm::PR);
  float* st_m = reinterpret_cast<float*>(smem + Sm::ST);
  float* st_l = st_m + 8;
  int* flags = reinterpret_cast<int*>(st_m + 24);  // [0] a wait gave up, [1] last arriver

  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int64_t bh = (int64_t)b * c.Hkv + hk;
  int64_t nv = nvalid;
  if (nvalid_dev) nv = min(max(*nvalid_dev, (int64_t)0), c.cap);
  const int64_t p_begin = (int64_t)split * S;
  const int nS = (int)max((int64_t)0, min((int64_t)S, nv - p_begin));
  const int nch = (nS + CH - 1) / CH;
  const SplitSrc src = split_src<C>(c, bh * c.cap + p_begin);

  if (tid == 0) {
#pragma unroll
    for (int s = 0; s < NST; ++s) mbar_init(&bar[s], 1);
    mbar_fence_init();
  }
  if (tid < 8) {
    st_m[tid] = -INFINITY;
    st_l[tid] = 0.f;
    flags[tid] = 0;
  }
  __syncthreads();
  int64_t pn = newest;
  if (newest_dev) pn = *newest_dev;
  const int64_t slot_new = pn >= 0 ? pn % c.cap : -1;
  const int chn_new = slot_new >= p_begin && slot_new < p_begin + nS ? (int)((slot_new - p_begin) / CH) : -1;
  int issued = 0;  // meaningful in thread 0 only
  if (tid == 0)
    for (; issued < min(NST, nch); ++issued)
      if (issued != chn_new) issue_chunk<C, FMOE_KV_AFFINE>(smem, bar, src, issued, nS);
  griddep_wait();
  griddep_launch_dependents();
  if (tid == 0 && chn_new >= 0 && chn_new < min(NST, nch)) issue_chunk<C, FMOE_KV_AFFINE>(smem, bar, src, chn_new, nS);

  // rotated query rows (hi / lo bf16 parts) and their group sums
  if (warp < GQ) {
    float v[P];
    load_row_f32<P>(q + ((int64_t)b * Hq + hk * GQ + warp) * D, lane, v);
    warp_fwht<P>(v, lane);
    float hi[P], lo[P], s = 0.f;
#pragma unroll
    for (int i = 0; i < P; ++i) {
      v[i] *= inv_sqrt_d;
      hi[i] = round_bf(v[i]);
      lo[i] = round_bf(v[i] - hi[i]);
      s += hi[i] + lo[i];
    }
    store_row_bf16<P>(qrow + warp * D, lane, hi);
    store_row_bf16<P>(qrow + (GQ + warp) * D, lane, lo);
#pragma unroll
    for (int o = 1; o < 64 / P; o <<= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane % (64 / P) == 0) qsum[warp * G + lane / (64 / P)] = s;
  }
  __syncthreads();
  // B fragments of the query, one warp per group; lanes g >= GQ use zeros
  if (warp < G && lane < 4 * GQ) {
#pragma unroll
    for (int hl = 0; hl < 2; ++hl) {
      const uint8_t* p = reinterpret_cast<const uint8_t*>(qrow + (hl * GQ + g) * D) + warp * 128 + 32 * t;
      const BFrag4 f = make_bfrag4(lds_u4(p), lds_u4(p + 16));
      uint4* dst = qf + ((warp * 2 + hl) * 4 * GQ + lane) * 2;
      dst[0] = make_uint4(f.b0[0], f.b0[1], f.b0[2], f.b0[3]);
      dst[1] = make_uint4(f.b1[0], f.b1[1], f.b1[2], f.b1[3]);
    }
  }
  __syncthreads();
  float qs0[G], qs1[G];  // group sums of heads 2t, 2t+1 (the C fragment's columns)
#pragma unroll
  for (int gi = 0; gi < G; ++gi) {
    qs0[gi] = 2 * t < GQ ? qsum[(2 * t) * G + gi] : 0.f;
    qs1[gi] = 2 * t + 1 < GQ ? qsum[(2 * t + 1) * G + gi] : 0.f;
  }

  const int tile = warp % TPC, wp = warp / TPC, r0 = tile * 16;
  const int pv_grp = warp % G, pv_slot = warp / G;
  float m_run0 = -INFINITY, m_run1 = -INFINITY;  // heads 2t, 2t+1 (same in every thread)
  float l_run0 = 0.f, l_run1 = 0.f;              // this lane's rows of its tile
  float acc[4][4], cor[4], bacc0 = 0.f, bacc1 = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    cor[i] = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;
  }

  int ch = 0;
  for (; ch < nch; ++ch) {
    const int stg = ch % NST;
    const int nrow = min(CH, nS - ch * CH);
    const uint8_t* sb = smem + stg * C::STAGE;
    if (!mbar_wait(&bar[stg], (uint32_t)(ch / NST) & 1u, status, 51)) atomicOr(&flags[0], 1);

    // ---- scores of tile `tile` over the warp's groups (fp32, unscaled)
    const bool live = r0 < nrow;
    float y[4] = {0.f, 0.f, 0.f, 0.f};
    if (live) {
      const int rl = min(r0 + g, nrow - 1), rh = min(r0 + g + 8, nrow - 1);
      const uint2 ksl = lds_u2(sb + C::KS + (rl * G + wp * GPW) * 2), kbl = lds_u2(sb + C::KB + (rl * G + wp * GPW) * 2);
      const uint2 ksh = lds_u2(sb + C::KS + (rh * G + wp * GPW) * 2), kbh = lds_u2(sb + C::KB + (rh * G + wp * GPW) * 2);
      const float sl[4] = {bf16lo(ksl.x), bf16hi(ksl.x), bf16lo(ksl.y), bf16hi(ksl.y)};
      const float bl[4] = {bf16lo(kbl.x), bf16hi(kbl.x), bf16lo(kbl.y), bf16hi(kbl.y)};
      const float sh[4] = {bf16lo(ksh.x), bf16hi(ksh.x), bf16lo(ksh.y), bf16hi(ksh.y)};
      const float bh_[4] = {bf16lo(kbh.x), bf16hi(kbh.x), bf16lo(kbh.y), bf16hi(kbh.y)};
#pragma unroll
      for (int gg = 0; gg < GPW; ++gg) {
        const int gi = wp * GPW + gg;
        BFrag4 fh, fl;
        if (g < GQ) {
          const uint4* src4 = qf + ((gi * 2) * 4 * GQ + lane) * 2;
          const uint4 h0 = src4[0], h1 = src4[1];
          const uint4 l0 = src4[8 * GQ], l1 = src4[8 * GQ + 1];
          fh = BFrag4{{h0.x, h0.y, h0.z, h0.w}, {h1.x, h1.y, h1.z, h1.w}};
          fl = BFrag4{{l0.x, l0.y, l0.z, l0.w}, {l1.x, l1.y, l1.z, l1.w}};
        } else {
          fh = BFrag4{{0u, 0u, 0u, 0u}, {0u, 0u, 0u, 0u}};
          fl = fh;
        }
        const uint2 wl = lds_u2(sb + rl * C::KRB + gi * 32 + 8 * t);
        const uint2 wh = lds_u2(sb + rh * C::KRB + gi * 32 + 8 * t);
        float cc[4] = {0.f, 0.f, 0.f, 0.f};
        mma_group_q4_hl(cc, wl, wh, fh, fl);
        // static register indexes (wp is 0 or 1)
        const float q0 = wp ? qs0[(GPW + gg) % G] : qs0[gg], q1 = wp ? qs1[(GPW + gg) % G] : qs1[gg];
        const float ol = fmaf(-128.f, sl[gg], bl[gg]), oh = fmaf(-128.f, sh[gg], bh_[gg]);
        y[0] += fmaf(sl[gg], cc[0], ol * q0);
        y[1] += fmaf(sl[gg], cc[1], ol * q1);
        y[2] += fmaf(sh[gg], cc[2], oh * q0);
        y[3] += fmaf(sh[gg], cc[3], oh * q1);
      }
    }
    if constexpr (WPT > 1) {  // the second half of the groups adds through shared memory
      if (wp == 1 && live) {
        if (2 * t < GQ) {
          scp[(2 * t) * CH + r0 + g] = y[0];
          scp[(2 * t) * CH + r0 + g + 8] = y[2];
        }
        if (2 * t + 1 < GQ) {
          scp[(2 * t + 1) * CH + r0 + g] = y[1];
          scp[(2 * t + 1) * CH + r0 + g + 8] = y[3];
        }
      }
      __syncthreads();
      if (wp == 0 && live) {
        if (2 * t < GQ) {
          y[0] += scp[(2 * t) * CH + r0 + g];
          y[2] += scp[(2 * t) * CH + r0 + g + 8];
        }
        if (2 * t + 1 < GQ) {
          y[1] += scp[(2 * t + 1) * CH + r0 + g];
          y[3] += scp[(2 * t + 1) * CH + r0 + g + 8];
        }
      }
    }
    // C fragment: y[0] (row g, head 2t), y[1] (g, 2t+1), y[2] (g+8, 2t), y[3] (g+8, 2t+1)
    const bool v0 = r0 + g < nrow, v1 = r0 + g + 8 < nrow;
    const float s00 = y[0] * scale, s01 = y[1] * scale, s10 = y[2] * scale, s11 = y[3] * scale;
    if (wp == 0) {
      float mx0 = fmaxf(v0 ? s00 : -INFINITY, v1 ? s10 : -INFINITY);
      float mx1 = fmaxf(v0 ? s01 : -INFINITY, v1 ? s11 : -INFINITY);
#pragma unroll
      for (int off = 4; off < 32; off <<= 1) {
        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
      }
      if (g == 0) {
        tmax[tile * 8 + 2 * t] = mx0;
        tmax[tile * 8 + 2 * t + 1] = mx1;
      }
    }
    __syncthreads();
    if (flags[0]) break;  // a copy never landed: every thread leaves the loop here

    // ---- running max (identical in every thread), probabilities of the tile
    float cm0 = -INFINITY, cm1 = -INFINITY;
#pragma unroll
    for (int w = 0; w < TPC; ++w) {
      cm0 = fmaxf(cm0, tmax[w * 8 + 2 * t]);
      cm1 = fmaxf(cm1, tmax[w * 8 + 2 * t + 1]);
    }
    const float mn0 = fmaxf(m_run0, cm0), mn1 = fmaxf(m_run1, cm1);
    const float f0 = expf(m_run0 - mn0), f1 = expf(m_run1 - mn1);
    m_run0 = mn0;
    m_run1 = mn1;
    if (wp == 0) {
      float p00 = 0.f, p01 = 0.f, p10 = 0.f, p11 = 0.f;
      if (live) {
        p00 = v0 ? expf(s00 - mn0) : 0.f;
        p01 = v0 ? expf(s01 - mn1) : 0.f;
        p10 = v1 ? expf(s10 - mn0) : 0.f;
        p11 = v1 ? expf(s11 - mn1) : 0.f;
        if (2 * t < GQ) {
          pr[(2 * t) * CH + r0 + g] = p00;
          pr[(2 * t) * CH + r0 + g + 8] = p10;
        }
        if (2 * t + 1 < GQ) {
          pr[(2 * t + 1) * CH + r0 + g] = p01;
          pr[(2 * t + 1) * CH + r0 + g + 8] = p11;
        }
      }
      l_run0 = fmaf(l_run0, f0, p00 + p10);
      l_run1 = fmaf(l_run1, f1, p01 + p11);
    }
    __syncthreads();

    // ---- P.V: o^T[d, h] += V^T[d, pos] (p s)[pos, h] (see the header comment);
    // m-tile i of the group: rows g / g+8 are columns grp*64 + 8g + 2i / +1
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc[i][0] *= f0;
      acc[i][1] *= f1;
      acc[i][2] *= f0;
      acc[i][3] *= f1;
    }
    cor[0] *= f0;
    cor[1] *= f1;
    cor[2] *= f0;
    cor[3] *= f1;
    bacc0 *= f0;
    bacc1 *= f1;
    {
      const bf16* vsc = reinterpret_cast<const bf16*>(sb + C::VS);
      const bf16* vbi = reinterpret_cast<const bf16*>(sb + C::VB);
      const uint8_t* vcol = sb + C::VC + pv_grp * 64 + 8 * g;
      float bs = 0.f;  // sum of p * v_bias over this lane's positions, head g
#pragma unroll
      for (int kk = 0; kk < C::KTW; ++kk) {
        const int pk = (pv_slot * C::KTW + kk) * 16;
        if (pk < nrow) {
          const int p0 = pk + 2 * t, p2 = p0 + 8;
          uint32_t b0 = 0u, b1 = 0u;
          if (g < GQ) {
            const float2 pa = *reinterpret_cast<const float2*>(pr + g * CH + p0);
            const float2 pc = *reinterpret_cast<const float2*>(pr + g * CH + p2);
            const bool q0 = p0 < nrow, q1 = p0 + 1 < nrow, q2 = p2 < nrow, q3 = p2 + 1 < nrow;
            const float w0 = q0 ? pa.x * bf2f(vsc[p0 * G + pv_grp]) : 0.f;
            const float w1 = q1 ? pa.y * bf2f(vsc[(p0 + 1) * G + pv_grp]) : 0.f;
            const float w2 = q2 ? pc.x * bf2f(vsc[p2 * G + pv_grp]) : 0.f;
            const float w3 = q3 ? pc.y * bf2f(vsc[(p2 + 1) * G + pv_grp]) : 0.f;
            if (q0) bs = fmaf(pa.x, bf2f(vbi[p0 * G + pv_grp]), bs);
            if (q1) bs = fmaf(pa.y, bf2f(vbi[(p0 + 1) * G + pv_grp]), bs);
            if (q2) bs = fmaf(pc.x, bf2f(vbi[p2 * G + pv_grp]), bs);
            if (q3) bs = fmaf(pc.y, bf2f(vbi[(p2 + 1) * G + pv_grp]), bs);
            b0 = pack_f16x2(w0, w1);
            b1 = pack_f16x2(w2, w3);
          }
          const uint2 wa = lds_u2(vcol + p0 * C::VRB), wb = lds_u2(vcol + (p0 + 1) * C::VRB);
          const uint2 wc = lds_u2(vcol + p2 * C::VRB), wd = lds_u2(vcol + (p2 + 1) * C::VRB);
          // bytes j of two position rows side by side, then f16 (1024 + q) pairs
          const uint32_t ab0 = prmt(wa.x, wb.x, 0x5140u), ab1 = prmt(wa.x, wb.x, 0x7362u);
          const uint32_t ab2 = prmt(wa.y, wb.y, 0x5140u), ab3 = prmt(wa.y, wb.y, 0x7362u);
          const uint32_t cd0 = prmt(wc.x, wd.x, 0x5140u), cd1 = prmt(wc.x, wd.x, 0x7362u);
          const uint32_t cd2 = prmt(wc.y, wd.y, 0x5140u), cd3 = prmt(wc.y, wd.y, 0x7362u);
          const uint32_t K = 0x64646464u;
          mma16816_f16(acc[0], prmt(ab0, K, 0x4140u), prmt(ab0, K, 0x4342u), prmt(cd0, K, 0x4140u),
                       prmt(cd0, K, 0x4342u), b0, b1);
          mma16816_f16(acc[1], prmt(ab1, K, 0x4140u), prmt(ab1, K, 0x4342u), prmt(cd1, K, 0x4140u),
                       prmt(cd1, K, 0x4342u), b0, b1);
          mma16816_f16(acc[2], prmt(ab2, K, 0x4140u), prmt(ab2, K, 0x4342u), prmt(cd2, K, 0x4140u),
                       prmt(cd2, K, 0x4342u), b0, b1);
          mma16816_f16(acc[3], prmt(ab3, K, 0x4140u), prmt(ab3, K, 0x4342u), prmt(cd3, K, 0x4140u),
                       prmt(cd3, K, 0x4342u), b0, b1);
          const uint32_t m1024 = 0xE400E400u;  // f16 -1024 pairs
          mma16816_f16(cor, m1024, m1024, m1024, m1024, b0, b1);
        }
      }
      // head g's bias sum -> the lanes holding heads 2t / 2t+1
      bs += __shfl_xor_sync(0xffffffffu, bs, 1);
      bs += __shfl_xor_sync(0xffffffffu, bs, 2);
      bacc0 += __shfl_sync(0xffffffffu, bs, 8 * t);
      bacc1 += __shfl_sync(0xffffffffu, bs, 8 * t + 4);
    }
    __syncthreads();
    if (tid == 0 && issued < nch) issue_chunk<C, FMOE_KV_AFFINE>(smem, bar, src, issued++, nS);
  }
  // Chunks still in flight (only after a wait gave up) must land before the
  // stage area is reused.
  if (tid == 0)
    for (int k = ch; k < issued; ++k) mbar_wait(&bar[k % NST], (uint32_t)(k / NST) & 1u, status, 52);
  const bool failed = flags[0] != 0;
  // split sums: this lane's tile rows -> tile -> split
  if (wp == 0) {
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      l_run0 += __shfl_xor_sync(0xffffffffu, l_run0, off);
      l_run1 += __shfl_xor_sync(0xffffffffu, l_run1, off);
    }
  }
  __syncthreads();  // every thread is past its last read of tmax
  if (wp == 0 && g == 0) {
    tmax[tile * 8 + 2 * t] = l_run0;
    tmax[tile * 8 + 2 * t + 1] = l_run1;
  }
  if (warp == 0 && g == 0) {
    if (2 * t < GQ) st_m[2 * t] = m_run0;
    if (2 * t + 1 < GQ) st_m[2 * t + 1] = m_run1;
  }
  float* red = reinterpret_cast<float*>(smem);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = pv_grp * 64 + 8 * g + 2 * i;
    if (2 * t < GQ) {
      float* r = red + (pv_slot * GQ + 2 * t) * D + d;
      r[0] = acc[i][0] + cor[0] + bacc0;
      r[1] = acc[i][2] + cor[2] + bacc0;
    }
    if (2 * t + 1 < GQ) {
      float* r = red + (pv_slot * GQ + 2 * t + 1) * D + d;
      r[0] = acc[i][1] + cor[1] + bacc1;
      r[1] = acc[i][3] + cor[3] + bacc1;
    }
  }
  __syncthreads();
  if (tid < GQ) {
    float l = 0.f;
#pragma unroll
    for (int w = 0; w < TPC; ++w) l += tmax[w * 8 + tid];
    st_l[tid] = l;
  }
  __syncthreads();
  attn_epilogue<P, FMOE_KV_AFFINE, GQ, C::RSL>(smem, st_m, st_l, flags, failed, Hq, b, hk, bh, split, nsplit,
                                               inv_sqrt_d, part_ml, part_o, ctr, out);
}

// ---- bf16 cache (the reference's storage)

template <int P, int GQ>
struct Bf16Smem {
  using C = AtCfg<P, FMOE_KV_BF16>;
  static constexpr int D = C::D;
  static constexpr int BAR = C::NST * C::STAGE;
  static constexpr int QH = BAR + 64;                 // bf16 [GQ][D] query rows
  static constexpr int SC = QH + GQ * D * 2;          // f32 [WPT][GQ][CH] partial scores
  static constexpr int PR = SC + C::WPT * GQ * C::CH * 4;  // f32 [GQ][CH] probabilities
  static constexpr int ST = PR + GQ * C::CH * 4;      // f32 m[8] l[8] f[8], int flags[8]
  static constexpr int BYTES = ST + 32 * 4;
  static_assert(C::RSL * GQ * D * 4 <= BAR && kRed2Off + GQ * D * 4 <= BAR, "attention smem aliases");
};

template <int P, int GQ>
__global__ void __launch_bounds__(256, GQ >= 8 ? 1 : 2)
    attn_bf16_kernel(const KvDev c, const bf16* __restrict__ q, int Hq, int S, int nsplit, int64_t nvalid,
                     const int64_t* __restrict__ nvalid_dev, float scale, float inv_sqrt_d,
                     float2* __restrict__ part_ml, float* __restrict__ part_o, unsigned* __restrict__ ctr,
                     bf16* __restrict__ out, int* __restrict__ status, int64_t newest,
                     const int64_t* __restrict__ newest_dev) {
  using C = AtCfg<P, FMOE_KV_BF16>;
  using Sm = Bf16Smem<P, GQ>;
  // Launched as a programmatic dependent, q and the newest cache rows come
  // from the preceding kernel: every chunk but the one holding the row
  // appended at position `newest` (slot newest % cap; -1: none) is copied
  // before the dependency wait.  The position and slot count are written at
  // least two kernels earlier in the stream, so they are final here.
  constexpr int D = C::D, CH = C::CH, NST = C::NST;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + Sm::BAR);
  bf16* qh = reinterpret_cast<bf16*>(smem + Sm::QH);
  float* sc = reinterpret_cast<float*>(smem + Sm::SC);
  float* pr = reinterpret_cast<float*>(smem + Sm::PR);
  float* st_m = reinterpret_cast<float*>(smem + Sm::ST);
  float* st_l = st_m + 8;
  float* st_f = st_m + 16;
  int* flags = reinterpret_cast<int*>(st_m + 24);

  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int64_t bh = (int64_t)b * c.Hkv + hk;
  int64_t nv = nvalid;
  if (nvalid_dev) nv = min(max(*nvalid_dev, (int64_t)0), c.cap);
  const int64_t p_begin = (int64_t)split * S;
  const int nS = (int)max((int64_t)0, min((int64_t)S, nv - p_begin));
  const int nch = (nS + CH - 1) / CH;
  const SplitSrc src = split_src<C>(c, bh * c.cap + p_begin);

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
  int64_t pn = newest;
  if (newest_dev) pn = *newest_dev;
  const int64_t slot_new = pn >= 0 ? pn % c.cap : -1;
  const int chn_new = slot_new >= p_begin && slot_new < p_begin + nS ? (int)((slot_new - p_begin) / CH) : -1;
  int issued = 0;  // meaningful in thread 0 only
  if (tid == 0)
    for (; issued < min(NST, nch); ++issued)
      if (issued != chn_new) issue_chunk<C, FMOE_KV_BF16>(smem, bar, src, issued, nS);
  griddep_wait();
  griddep_launch_dependents();
  if (tid == 0 && chn_new >= 0 && chn_new < min(NST, nch)) issue_chunk<C, FMOE_KV_BF16>(smem, bar, src, chn_new, nS);
  if (warp < GQ) {
    float v[P];
    load_row_f32<P>(q + ((int64_t)b * Hq + hk * GQ + warp) * D, lane, v);
    store_row_bf16<P>(qh + warp * D, lane, v);
  }
  __syncthreads();

  float o[GQ][4];  // column 4*unit + j of head h, this thread's position phase
#pragma unroll
  for (int h = 0; h < GQ; ++h)
#pragma unroll
    for (int j = 0; j < 4; ++j) o[h][j] = 0.f;

  int ch = 0;
  for (; ch < nch; ++ch) {
    const int stg = ch % NST;
    const int nrow = min(CH, nS - ch * CH);
    const uint8_t* sb = smem + stg * C::STAGE;
    if (!mbar_wait(&bar[stg], (uint32_t)(ch / NST) & 1u, status, 53)) atomicOr(&flags[0], 1);
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
          const uint8_t* kl = sb + rl * C::KRB + gi * 128 + 32 * t;
          const uint8_t* kh = sb + rh * C::KRB + gi * 128 + 32 * t;
          const BFrag4 alo = make_bfrag4(lds_u4(kl), lds_u4(kl + 16));
          const BFrag4 ahi = make_bfrag4(lds_u4(kh), lds_u4(kh + 16));
#pragma unroll
          for (int s4 = 0; s4 < 4; ++s4)
            mma16816(y, alo.b0[s4], ahi.b0[s4], alo.b1[s4], ahi.b1[s4], bq.b0[s4], bq.b1[s4]);
        }
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
    if (flags[0]) break;
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
    {
      const int unit = tid % C::U, ph = tid / C::U;
#pragma unroll
      for (int h = 0; h < GQ; ++h) {
        const float f = st_f[h];
#pragma unroll
        for (int j = 0; j < 4; ++j) o[h][j] *= f;
      }
      for (int i = ph; i < nrow; i += C::NPH) {
        const uint2 w = lds_u2(sb + C::VC + i * C::VRB + unit * 8);
        const float v4[4] = {bf16lo(w.x), bf16hi(w.x), bf16lo(w.y), bf16hi(w.y)};
#pragma unroll
        for (int h = 0; h < GQ; ++h) {
          const float p = pr[h * CH + i];
#pragma unroll
          for (int j = 0; j < 4; ++j) o[h][j] = fmaf(p, v4[j], o[h][j]);
        }
      }
    }
    __syncthreads();
    if (tid == 0 && issued < nch) issue_chunk<C, FMOE_KV_BF16>(smem, bar, src, issued++, nS);
  }
  if (tid == 0)
    for (int k = ch; k < issued; ++k) mbar_wait(&bar[k % NST], (uint32_t)(k / NST) & 1u, status, 54);
  const bool failed = flags[0] != 0;
  __syncthreads();
  float* red = reinterpret_cast<float*>(smem);
  {
    const int unit = tid % C::U, ph = tid / C::U;
#pragma unroll
    for (int h = 0; h < GQ; ++h)
      *reinterpret_cast<float4*>(red + (ph * GQ + h) * D + unit * 4) = make_float4(o[h][0], o[h][1], o[h][2], o[h][3]);
  }
  __syncthreads();
  attn_epilogue<P, FMOE_KV_BF16, GQ, C::RSL>(smem, st_m, st_l, flags, failed, Hq, b, hk, bh, split, nsplit,
                                             inv_sqrt_d, part_ml, part_o, ctr, out);
}

// ---------------------------------------------------------------------------
// host side

static int chunk_positions(int mode, int D) {
  return mode == FMOE_KV_BF16 ? (D == 256 ? AtCfg<8, FMOE_KV_BF16>::CH : AtCfg<16, FMOE_KV_BF16>::CH)
                              : (D == 256 ? AtCfg<8, FMOE_KV_AFFINE>::CH : AtCfg<16, FMOE_KV_AFFINE>::CH);
}

// Split planner.  Two CTAs are resident per SM; a launch of about one wave
// (2 x 148 CTAs) has the lowest fixed cost (prologue, merge), four waves
// balance the SMs better once every split still streams >= 8 chunks.  The
// environment variable FMOE_ATTN_TARGET_CTAS, when set, replaces the choice
// with one fixed CTA target (read once; a tuning knob).
static int attn_target_override() {
  static const int v = [] {
    const char* e = std::getenv("FMOE_ATTN_TARGET_CTAS");
    const int x = e ? std::atoi(e) : 0;
    return x > 0 ? x : 0;
  }();
  return v;
}

static int64_t attn_split_candidate(int64_t chunks, int64_t heads) {
  const int64_t one = (2 * kNumSMs + heads - 1) / heads, four = (8 * kNumSMs + heads - 1) / heads;
  if (attn_target_override()) return (attn_target_override() + heads - 1) / heads;
  return chunks >= 8 * four ? four : one;
}

// The last-arriving split of a (batch, kv head) merges nsplit partial rows
// of GQ x D floats; past kMergeFloats per head that serial merge outweighs what
// more splits save (full-attention layers: GQ 8 x D 512), so the split count
// is capped there.
constexpr int64_t kMergeFloats = 65536;
static int64_t merge_cap(const KvDev& c, int Hq) {
  const int64_t gqd = (int64_t)(Hq / c.Hkv) * c.D;
  return std::max<int64_t>(1, kMergeFloats / std::max<int64_t>(gqd, 1));
}

AttnPlan attn_plan(const KvDev& c, int64_t n, int Hq) {
  const int CH = chunk_positions(c.mode, c.D);
  const int64_t chunks = n > 0 ? (n + CH - 1) / CH : 1;
  const int64_t heads = (int64_t)c.B * c.Hkv;
  const int64_t ns = std::max<int64_t>(1, std::min<int64_t>({attn_split_candidate(chunks, heads), chunks,
                                                              merge_cap(c, Hq), (int64_t)kMaxSplits}));
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

// Upper bound of attn_plan(c, n).nsplit over every n <= capacity: the larger
// candidate, before rounding S up to whole chunks (rounding only lowers it).
static int attn_max_splits(const KvDev& c, int Hq) {
  const int CH = chunk_positions(c.mode, c.D);
  const int64_t chunks = (c.cap + CH - 1) / CH;
  const int64_t heads = (int64_t)c.B * c.Hkv;
  const int64_t ns = std::max(attn_split_candidate(0, heads), attn_split_candidate(INT64_MAX / 2, heads));
  return (int)std::max<int64_t>(1, std::min<int64_t>({ns, chunks, merge_cap(c, Hq), (int64_t)kMaxSplits}));
}

size_t attn_workspace_bytes(const KvDev& c, int Hq) {
  return carve_attn_ws(nullptr, c, Hq, attn_max_splits(c, Hq)).bytes;
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

int launch_qkv_post(const KvDev& c, const float* qkv, int ld, int parts, int64_t part_stride, int Hq, int k_eq_v,
                    const bf16* q_norm,
                    const bf16* k_norm, float eps, int rope_dims, float rope_theta, int64_t pos,
                    const int64_t* pos_dev, bf16* q_out, int turbo_bits, bool pdl, cudaStream_t st) {
  const float l2t = (float)std::log2((double)rope_theta);
  const int rows = c.B * (Hq + 2 * c.Hkv);  // query rows, then K and V rows on separate warps
  const float inv = 1.0f / std::sqrt((float)c.D);
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3((rows + 7) / 8);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  ProfScope prof_("qkv_post_kernel", st);
  if (c.D == 256)
    cudaLaunchKernelEx(&cfg, qkv_post_kernel<8>, c, qkv, ld, parts, part_stride, Hq, k_eq_v, q_norm, k_norm, eps,
                       rope_dims, l2t, pos, pos_dev, q_out, turbo_bits, inv);
  else
    cudaLaunchKernelEx(&cfg, qkv_post_kernel<16>, c, qkv, ld, parts, part_stride, Hq, k_eq_v, q_norm, k_norm, eps,
                       rope_dims, l2t, pos, pos_dev, q_out, turbo_bits, inv);
  return check_launch("qkv_post_kernel");
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
                         const int64_t* nvalid_dev, float scale, const AttnWs& w, bf16* out, cudaStream_t st,
                         bool pdl, int64_t newest, const int64_t* newest_dev) {
  constexpr bool aff = MODE == FMOE_KV_AFFINE;
  constexpr int bytes = aff ? AffSmem<P, GQ>::BYTES : Bf16Smem<P, GQ>::BYTES;
  auto kern = aff ? attn_affine_kernel<P, GQ> : attn_bf16_kernel<P, GQ>;
  static std::once_flag once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(once, [kern] {
    attr_err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  });
  if (attr_err != cudaSuccess)
    return set_error(FMOE_ERR_CUDA, "attn_decode: shared memory attribute: %s", cudaGetErrorString(attr_err));
  const float inv = 1.0f / std::sqrt((float)(32 * P));
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(p.nsplit, c.Hkv, c.B);
  cfg.blockDim = dim3(256);
  cfg.dynamicSmemBytes = bytes;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  ProfScope prof_(aff ? "attn_affine_kernel" : "attn_bf16_kernel", st);
  cudaLaunchKernelEx(&cfg, kern, c, q, Hq, p.S, p.nsplit, nvalid, nvalid_dev, scale, inv, w.ml, w.po, w.ctr, out,
                     w.status, newest, newest_dev);
  return check_launch("attn_decode kernel");
}

template <int P, int MODE>
static int launch_attn_m(const KvDev& c, int GQ, const bf16* q, int Hq, const AttnPlan& p, int64_t nvalid,
                         const int64_t* nvalid_dev, float scale, const AttnWs& w, bf16* out, cudaStream_t st,
                         bool pdl, int64_t newest, const int64_t* newest_dev) {
  switch (GQ) {
    case 1: return launch_attn_t<P, MODE, 1>(c, q, Hq, p, nvalid, nvalid_dev, scale, w, out, st, pdl, newest,
                                                  newest_dev);
    case 2: return launch_attn_t<P, MODE, 2>(c, q, Hq, p, nvalid, nvalid_dev, scale, w, out, st, pdl, newest,
                                                  newest_dev);
    case 4: return launch_attn_t<P, MODE, 4>(c, q, Hq, p, nvalid, nvalid_dev, scale, w, out, st, pdl, newest,
                                                  newest_dev);
    case 8: return launch_attn_t<P, MODE, 8>(c, q, Hq, p, nvalid, nvalid_dev, scale, w, out, st, pdl, newest,
                                                  newest_dev);
  }
  return set_error(FMOE_ERR_UNSUPPORTED, "attn_decode: %d query heads per kv head (kernels: 1, 2, 4, 8)", GQ);
}

int launch_attn_decode(const KvDev& c, const bf16* q, int Hq, int64_t nvalid, const int64_t* nvalid_dev, float scale,
                       void* ws, bf16* out, cudaStream_t st, bool pdl, int64_t newest, const int64_t* newest_dev) {
  const AttnPlan p = attn_plan(c, nvalid_dev ? c.cap : nvalid, Hq);
  const AttnWs w = carve_attn_ws(ws, c, Hq, p.nsplit);
  const int GQ = Hq / c.Hkv;
  if (c.D == 256)
    return c.mode == FMOE_KV_BF16
               ? launch_attn_m<8, FMOE_KV_BF16>(c, GQ, q, Hq, p, nvalid, nvalid_dev, scale, w, out, st, pdl, newest,
                                                newest_dev)
               : launch_attn_m<8, FMOE_KV_AFFINE>(c, GQ, q, Hq, p, nvalid, nvalid_dev, scale, w, out, st, pdl, newest,
                                                  newest_dev);
  return c.mode == FMOE_KV_BF16
             ? launch_attn_m<16, FMOE_KV_BF16>(c, GQ, q, Hq, p, nvalid, nvalid_dev, scale, w, out, st, pdl, newest,
                                               newest_dev)
             : launch_attn_m<16, FMOE_KV_AFFINE>(c, GQ, q, Hq, p, nvalid, nvalid_dev, scale, w, out, st, pdl, newest,
                                                 newest_dev);
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
  if (c->turbo_bits != 0 && (c->mode != FMOE_KV_BF16 || c->turbo_bits < 2 || c->turbo_bits > 4))
    return set_error(FMOE_ERR_INVALID, "kv: turbo_bits %d (0, or 2..4 with the bf16 mode)", c->turbo_bits);
  if (c->mode == FMOE_KV_AFFINE &&
      (!c->k_scales || !c->k_biases || !c->v_scales || !c->v_biases || !aligned16(c->k_scales) ||
       !aligned16(c->k_biases) || !aligned16(c->v_scales) || !aligned16(c->v_biases)))
    return set_error(FMOE_ERR_ALIGN, "kv: scales/biases null or not 16-byte aligned");
  d->mode = c->mode;
  d->B = c->batch;
  d->Hkv = c->kv_heads;
  d->D = c->head_dim;
  d->cap = c->capacity;
  d->turbo = c->turbo_bits;
  d->k = c->k;
  d->v = c->v;
  d->ks = static_cast<bf16*>(c->k_scales);
  d->kb = static_cast<bf16*>(c->k_biases);
  d->vs = static_cast<bf16*>(c->v_scales);
  d->vb = static_cast<bf16*>(c->v_biases);
  return FMOE_OK;
}

}  // namespace

namespace fmoe {
int kv_to_dev(const fmoe_kv_cache_t* c, KvDev* d) { return to_kv(c, d); }
}  // namespace fmoe

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
