// Prefill of one decoder layer: T prompt tokens of one sequence at positions
// pos0 .. pos0+T-1, DecoderLayer::forward_gemma4 (src/model/mod.rs:67-119)
// with l > 1:
//   xn   = input_norm(x)                                    pf_norm_rows_kernel
//   q|k|v = xn . W^T                                        qgemm (one launch)
//   q = rope(q_norm(q)); k = rope(k_norm(k)); v = v_norm(v) pf_qkv_post_kernel
//        (TurboQuant round trip of the new k / v rows when the cache has it)
//   att = SDPA(q, cached K/V + new K/V, causal / sliding mask)  pf_attn_kernel
//   the new rows -> the cache ring                           kv_append_kernel
//   h = x + post_attn_norm(att . Wo^T)                       qgemm, pf_ff_in_kernel
//   d = down(gelu(gate(h1)) * up(h1)), moe = MoE(h2)         qgemm (gated), qgemm,
//                                                            fmoe_moe_prefill
//   x = (h + post_ff_norm(pff1(d) + pff2(moe))) * scalar     pf_ff_out_kernel
// Attention follows the reference's prefill: the cache's update_and_fetch
// returns the stored rows plus the new ones (src/cache.rs:266-310), and the
// mask admits key position j for the query at position p when j <= p and, on
// sliding layers, p - j < window (src/model/mod.rs:682-753).  Here the stored
// rows stay in the ring (slot p % capacity) and the new rows in a staging
// buffer until attention is done; only then are they appended, so a prompt
// longer than the window does not overwrite rows that its first queries need.
#include <cmath>
#include <cstring>
#include "internal.h"
#include "common.cuh"
#include "stage.cuh"
#include "rowops.cuh"
#include "kvrow.cuh"

namespace fmoe {

int launch_kv_append(const KvDev& c, const bf16* k, const bf16* v, int64_t Tn, int64_t pos, const int64_t* pos_dev,
                     int turbo_bits, cudaStream_t st);

namespace pfl {

// Row kernels: one CTA per token row of H values, each thread holding up to
// kRowVec 8-value vectors of every tensor in registers (one pass over memory;
// H a multiple of 8, at most kRowMaxH).
constexpr int kRowThreads = 384, kRowVec = 2, kRowMaxH = 8 * kRowThreads * kRowVec;

__device__ __forceinline__ float blk_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red is reused across calls
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < kRowThreads / 32; ++w) s += red[w];
  return s;
}
__device__ __forceinline__ void ld8(const bf16* p, float (&v)[8]) {
  const uint4 w = *reinterpret_cast<const uint4*>(p);
  v[0] = bf16lo(w.x);
  v[1] = bf16hi(w.x);
  v[2] = bf16lo(w.y);
  v[3] = bf16hi(w.y);
  v[4] = bf16lo(w.z);
  v[5] = bf16hi(w.z);
  v[6] = bf16lo(w.w);
  v[7] = bf16hi(w.w);
}
__device__ __forceinline__ void st8(bf16* p, const float (&v)[8]) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                            pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
}
__device__ __forceinline__ float sumsq8(const float (&v)[8], float acc) {
#pragma unroll
  for (int i = 0; i < 8; ++i) acc = fmaf(v[i], v[i], acc);
  return acc;
}

// y = bf16(rms_norm(x) * w), one CTA per row (fast::rms_norm, src/model/norm.rs:11-29)
__global__ void __launch_bounds__(kRowThreads) pf_norm_rows_kernel(const bf16* __restrict__ x, int H,
                                                                   const bf16* __restrict__ w, float eps,
                                                                   bf16* __restrict__ y) {
  __shared__ float red[kRowThreads / 32];
  const int64_t base = (int64_t)blockIdx.x * H;
  float xv[kRowVec][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kRowVec; ++k) {
    const int c = threadIdx.x + k * kRowThreads;
    if (8 * c < H) {
      ld8(x + base + 8 * c, xv[k]);
      ss = sumsq8(xv[k], ss);
    }
  }
  const float r = rsqrtf(blk_sum(ss, red) / (float)H + eps);
#pragma unroll
  for (int k = 0; k < kRowVec; ++k) {
    const int c = threadIdx.x + k * kRowThreads;
    if (8 * c < H) {
      float wv[8], o[8];
      ld8(w + 8 * c, wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = xv[k][i] * r * wv[i];
      st8(y + base + 8 * c, o);
    }
  }
}

// h = bf16(x + bf16(rms_norm(o) * w_pa)) -> x (in place); h1 / h2 = the two
// pre-feed-forward norms of h.  The same steps as the decode ff_in kernel.
__global__ void __launch_bounds__(kRowThreads) pf_ff_in_kernel(bf16* __restrict__ x, const bf16* __restrict__ o, int H,
                                                               const bf16* __restrict__ w_pa,
                                                               const bf16* __restrict__ w_pf,
                                                               const bf16* __restrict__ w_pf2, float eps,
                                                               bf16* __restrict__ h1, bf16* __restrict__ h2) {
  __shared__ float red[kRowThreads / 32];
  const int64_t base = (int64_t)blockIdx.x * H;
  float ov[kRowVec][8], hv[kRowVec][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kRowVec; ++k) {
    const int c = threadIdx.x + k * kRowThreads;
    if (8 * c < H) {
      ld8(o + base + 8 * c, ov[k]);
      ld8(x + base + 8 * c, hv[k]);
      ss = sumsq8(ov[k], ss);
    }
  }
  const float r1 = rsqrtf(blk_sum(ss, red) / (float)H + eps);
  ss = 0.f;
#pragma unroll
  for (int k = 0; k < kRowVec; ++k) {
    const int c = threadIdx.x + k * kRowThreads;
    if (8 * c < H) {
      float wv[8];
      ld8(w_pa + 8 * c, wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) hv[k][i] = round_bf(hv[k][i] + round_bf(ov[k][i] * r1 * wv[i]));
      st8(x + base + 8 * c, hv[k]);
      ss = sumsq8(hv[k], ss);
    }
  }
  const float r2 = rsqrtf(blk_sum(ss, red) / (float)H + eps);
#pragma unroll
  for (int k = 0; k < kRowVec; ++k) {
    const int c = threadIdx.x + k * kRowThreads;
    if (8 * c < H) {
      float w1[8], w2[8], a1[8], a2[8];
      ld8(w_pf + 8 * c, w1);
      ld8(w_pf2 + 8 * c, w2);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        a1[i] = hv[k][i] * r2 * w1[i];
        a2[i] = hv[k][i] * r2 * w2[i];
      }
      st8(h1 + base + 8 * c, a1);
      st8(h2 + base + 8 * c, a2);
    }
  }
}

// x = bf16(bf16(h + bf16(rms_norm(s) * w)) * scalar), s = bf16(pff1(d) + pff2(moe)),
// h = x on entry.  The same steps as the decode ff_out kernel.
// h: the residual stream h of each row (x itself in the prefill, which then
// updates x in place; the batched decode layer's separate h rows).
__global__ void __launch_bounds__(kRowThreads) pf_ff_out_kernel(bf16* x, const bf16* h, const bf16* __restrict__ d,
                                                                const bf16* __restrict__ moe, int H,
                                                                const bf16* __restrict__ w1,
                                                                const bf16* __restrict__ w2,
                                                                const bf16* __restrict__ w, float eps, float scalar) {
  __shared__ float red[kRowThreads / 32];
  const int64_t base = (int64_t)blockIdx.x * H;
  float dv[kRowVec][8], mv[kRowVec][8];
  float sd = 0.f, sm = 0.f;
#pragma unroll
  for (int k = 0; k < kRowVec; ++k) {
    const int c = threadIdx.x + k * kRowThreads;
    if (8 * c < H) {
      ld8(d + base + 8 * c, dv[k]);
      ld8(moe + base + 8 * c, mv[k]);
      sd = sumsq8(dv[k], sd);
      sm = sumsq8(mv[k], sm);
    }
  }
  const float rd = rsqrtf(blk_sum(sd, red) / (float)H + eps);
  const float rm = rsqrtf(blk_sum(sm, red) / (float)H + eps);
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kRowVec; ++k) {
    const int c = threadIdx.x + k * kRowThreads;
    if (8 * c < H) {
      float a[8], b[8];
      ld8(w1 + 8 * c, a);
      ld8(w2 + 8 * c, b);
#pragma unroll
      for (int i = 0; i < 8; ++i) dv[k][i] = round_bf(round_bf(dv[k][i] * rd * a[i]) + round_bf(mv[k][i] * rm * b[i]));
      ss = sumsq8(dv[k], ss);
    }
  }
  const float rs = rsqrtf(blk_sum(ss, red) / (float)H + eps);
  const float sc = round_bf(scalar);
#pragma unroll
  for (int k = 0; k < kRowVec; ++k) {
    const int c = threadIdx.x + k * kRowThreads;
    if (8 * c < H) {
      float hv[8], wv[8];
      ld8(h + base + 8 * c, hv);
      ld8(w + 8 * c, wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) hv[i] = round_bf(hv[i] + round_bf(dv[k][i] * rs * wv[i])) * sc;
      st8(x + base + 8 * c, hv);
    }
  }
}

// One CTA per token, one warp per (token, head) row of the projections:
// queries normed and rotated in place ([T][Hq][D]); keys / values normed (and
// rotated), through the TurboQuant round trip when `turbo`, into the staging
// rows [Hkv][T][D].  Gemma4Attention::forward, src/model/gemma4_attention.rs:
// 46-84.  The token's RoPE cos / sin (rope_dims / 2 angles, the decode path's
// formula) are computed once into shared memory and shared by its heads.
constexpr int kPostWarps = 8;
template <int P>
__global__ void __launch_bounds__(32 * kPostWarps) pf_qkv_post_kernel(
    bf16* __restrict__ q, const bf16* __restrict__ k, const bf16* __restrict__ v, int T, int Hq, int Hkv,
    const bf16* __restrict__ qn, const bf16* __restrict__ kn, float eps, int rope_dims, float log2_theta,
    int64_t pos0, int turbo, bf16* __restrict__ ks, bf16* __restrict__ vs) {
  constexpr int D = 32 * P;
  __shared__ float tc[D / 2], tsn[D / 2];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int t = blockIdx.x;
  const float pos = (float)(pos0 + t);
  const int half = rope_dims / 2;
  for (int j = threadIdx.x; j < half; j += blockDim.x)
    sincosf(pos * exp2f(-(float)(2 * j) / (float)rope_dims * log2_theta), &tsn[j], &tc[j]);
  __syncthreads();
  float cs[P], sn[P];
#pragma unroll
  for (int i = 0; i < P; ++i) {
    const int e = lane * P + i;
    const int j = e < half ? e : e - half;
    cs[i] = e < rope_dims ? tc[j] : 1.f;
    sn[i] = e < rope_dims ? tsn[j] : 0.f;
  }
  for (int hh = warp; hh < Hq + Hkv; hh += kPostWarps) {
    if (hh < Hq) {
      float x[P];
      bf16* r = q + ((int64_t)t * Hq + hh) * D;
      load_row_f32<P>(r, lane, x);
      warp_rms_norm<P>(x, qn, eps, lane);
      warp_rope_cs<P>(x, rope_dims, cs, sn, lane);
      store_row_bf16<P>(r, lane, x);
      continue;
    }
    const int g = hh - Hq;
    float kv[P], vv[P];
    load_row_f32<P>(k + ((int64_t)t * Hkv + g) * D, lane, kv);
    if (v)
      load_row_f32<P>(v + ((int64_t)t * Hkv + g) * D, lane, vv);
    else {  // K == V: the raw key projection, before its norm
#pragma unroll
      for (int i = 0; i < P; ++i) vv[i] = kv[i];
    }
    warp_rms_norm<P>(kv, kn, eps, lane);
    warp_rope_cs<P>(kv, rope_dims, cs, sn, lane);
    warp_rms_norm<P>(vv, nullptr, eps, lane);
    if (turbo) {
      warp_turbo<P>(kv, lane, turbo);
      warp_turbo<P>(vv, lane, turbo);
    }
    store_row_bf16<P>(ks + ((int64_t)g * T + t) * D, lane, kv);
    store_row_bf16<P>(vs + ((int64_t)g * T + t) * D, lane, vv);
  }
}

// The affine (rotated K4 / V8) cache's prefill: queries rotated in place by the
// normalised WHT (the basis the cache keeps K and V in); the new K / V rows
// rotated and taken through the cache's quantise -> dequantise round trip into
// kr / vr [Hkv][T][D], which attention reads for them (the rows it will read
// back from the cache for every later token).  One warp per row; the rotation
// and quantisation are kv_append_kernel's, step for step.
template <int P>
__global__ void __launch_bounds__(256) pf_affine_prep_kernel(bf16* __restrict__ q, const bf16* __restrict__ ks,
                                                             const bf16* __restrict__ vs, int T, int Hq, int Hkv,
                                                             float inv_sqrt_d, bf16* __restrict__ kr,
                                                             bf16* __restrict__ vr) {
  constexpr int D = 32 * P;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  const int64_t nq = (int64_t)T * Hq, nkv = (int64_t)Hkv * T;
  if (row >= nq + 2 * nkv) return;
  float x[P];
  if (row < nq) {
    load_row_f32<P>(q + row * D, lane, x);
    warp_fwht<P>(x, lane);
#pragma unroll
    for (int i = 0; i < P; ++i) x[i] *= inv_sqrt_d;
    store_row_bf16<P>(q + row * D, lane, x);
    return;
  }
  const bool is_v = row - nq >= nkv;
  const int64_t r = is_v ? row - nq - nkv : row - nq;
  load_row_f32<P>((is_v ? vs : ks) + r * D, lane, x);
  warp_fwht<P>(x, lane);
#pragma unroll
  for (int i = 0; i < P; ++i) x[i] *= inv_sqrt_d;
  if (is_v)
    warp_quant_round_trip<P, 8>(x, lane);
  else
    warp_quant_round_trip<P, 4>(x, lane);
  store_row_bf16<P>((is_v ? vr : kr) + r * D, lane, x);
}

// Rows back from the rotated basis (the normalised WHT is its own inverse).
template <int P>
__global__ void __launch_bounds__(256) pf_rotate_rows_kernel(bf16* __restrict__ x, int64_t rows, float inv_sqrt_d) {
  constexpr int D = 32 * P;
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + (threadIdx.x >> 5);
  if (row >= rows) return;
  float v[P];
  load_row_f32<P>(x + row * D, lane, v);
  warp_fwht<P>(v, lane);
#pragma unroll
  for (int i = 0; i < P; ++i) v[i] *= inv_sqrt_d;
  store_row_bf16<P>(x + row * D, lane, v);
}

// ---------------------------------------------------------------------------
// Prefill attention: one CTA per (tile of 64 query rows, kv head).  A row is a
// (token, query head of the kv head's group) pair, token-major, so a tile holds
// 64 / R tokens (R = Hq / Hkv).  Key tiles of 32 positions stream through two
// cp.async stages; position j comes from the ring (j < pos0) or the staging
// rows (j >= pos0).  Warp (rb, dp): 16 rows, output dims [256 dp, 256 dp + 256);
// S = Q K^T over all D (both warps of a row block when D = 512), online
// softmax in fp32 (log2 domain), O += P V with P rounded to bf16, all on
// mma.sync m16n8k16.  Shared-memory rows are D bf16 with 16-byte chunk c of
// row r at chunk c ^ (r % 8), so every ldmatrix is conflict-free.

constexpr int KT = 32;  // keys per tile
constexpr int QR = 64;  // query rows per CTA

template <int D>
struct PaCfg {
  static constexpr int DP = D / 256;
  static constexpr int THREADS = 128 * DP;
  static constexpr int ROWB = D * 2;
  static constexpr int Q_BYTES = QR * ROWB;
  static constexpr int KV_BYTES = KT * ROWB;
  static constexpr int STAGE = 2 * KV_BYTES;
  static constexpr int SMEM = Q_BYTES + 2 * STAGE;
};

struct PaArgs {
  const bf16* q;    // [T][Hq][D]
  const bf16* kr;   // ring rows [Hkv][cap][D] of the sequence
  const bf16* vr;
  const bf16* ks;   // staged new rows [Hkv][T][D]
  const bf16* vs;
  bf16* out;        // [T][Hq * D]
  int T, Hq, R, QT, win;
  int64_t pos0, cap;
  float sl;         // attention scale * log2(e)
  // affine (WHT-rotated K4 / V8) ring instead of kr / vr: codes, scales, biases
  const uint32_t* kq;
  const bf16 *kss, *kbb;
  const uint32_t* vq;
  const bf16 *vss, *vbb;
};

// Chunk c (values 8c .. 8c+7) of an affine ring row dequantised to bf16, as the
// cache returns it: bf16(fma(s, q, b)) with the group's scale and bias.
template <int D>
__device__ __forceinline__ uint4 affine_chunk(const uint32_t* codes, int bits, const bf16* sc, const bf16* bi,
                                              int64_t row, int c) {
  const int g = c >> 3;  // 64 values per group = 8 chunks
  const float s = bf2f(sc[row * (D / 64) + g]), b = bf2f(bi[row * (D / 64) + g]);
  float v[8];
  if (bits == 4) {
    const uint32_t w = codes[row * (D / 8) + c];
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = round_bf(fmaf(s, (float)((w >> (4 * i)) & 15u), b));
  } else {
    const uint32_t w0 = codes[row * (D / 4) + 2 * c], w1 = codes[row * (D / 4) + 2 * c + 1];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[i] = round_bf(fmaf(s, (float)((w0 >> (8 * i)) & 255u), b));
      v[4 + i] = round_bf(fmaf(s, (float)((w1 >> (8 * i)) & 255u), b));
    }
  }
  return make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                    pack_bf16x2(v[6], v[7]));
}

__device__ __forceinline__ void cp16(void* dst, const void* src, int n) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(smem_u32(dst)), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void ldsm4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}
__device__ __forceinline__ void ldsm4t(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(smem_u32(p)));
}

template <int D, bool AFF>  // AFF: the ring is the rotated affine cache, dequantised as it is read
__global__ void __launch_bounds__(PaCfg<D>::THREADS, D == 256 ? 2 : 1) pf_attn_kernel(const PaArgs a) {
  using C = PaCfg<D>;
  constexpr int CH = D / 8;  // 16-byte chunks per row
  extern __shared__ __align__(128) uint8_t sm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int tt = gridDim.x - 1 - blockIdx.x;  // the longest tiles first
  const int g = blockIdx.y;
  const int t0 = tt * a.QT;
  const int tlast = min(t0 + a.QT, a.T) - 1;
  const int64_t plo = a.pos0 + t0, phi = a.pos0 + tlast;
  const int64_t kb0 = a.win ? max((int64_t)0, plo - a.win + 1) : (int64_t)0;
  const int nkt = (int)((phi - kb0 + KT) / KT);

  for (int i = tid; i < QR * CH; i += C::THREADS) {
    const int r = i / CH, c = i % CH;
    const int t = t0 + r / a.R;
    uint8_t* dst = sm + r * C::ROWB + ((c ^ (r & 7)) << 4);
    if (t < a.T)
      cp16(dst, a.q + ((int64_t)t * a.Hq + g * a.R + r % a.R) * D + c * 8, 16);
    else
      cp16(dst, a.q, 0);  // zero fill
  }
  auto load_kv = [&](int i, int st) {
    uint8_t* kd = sm + C::Q_BYTES + st * C::STAGE;
    uint8_t* vd = kd + C::KV_BYTES;
    for (int j = tid; j < KT * CH; j += C::THREADS) {
      const int r = j / CH, c = j % CH;
      const int64_t kp = kb0 + (int64_t)i * KT + r;
      const bf16 *ksrc = a.q, *vsrc = a.q;
      int n = 0;
      if (kp <= phi) {
        n = 16;
        if (kp < a.pos0) {
          const int64_t row = (int64_t)g * a.cap + kp % a.cap;
          if (AFF) {  // plain loads, dequantised into the tile
            const int off = r * C::ROWB + ((c ^ (r & 7)) << 4);
            *reinterpret_cast<uint4*>(kd + off) = affine_chunk<D>(a.kq, 4, a.kss, a.kbb, row, c);
            *reinterpret_cast<uint4*>(vd + off) = affine_chunk<D>(a.vq, 8, a.vss, a.vbb, row, c);
            continue;
          }
          ksrc = a.kr + row * D + c * 8;
          vsrc = a.vr + row * D + c * 8;
        } else {
          const int64_t row = (int64_t)g * a.T + (kp - a.pos0);
          ksrc = a.ks + row * D + c * 8;
          vsrc = a.vs + row * D + c * 8;
        }
      }
      const int off = r * C::ROWB + ((c ^ (r & 7)) << 4);
      cp16(kd + off, ksrc, n);
      cp16(vd + off, vsrc, n);
    }
  };
  load_kv(0, 0);
  cp_async_commit();

  const int rb = warp & 3, dp = warp >> 2;
  const int r0 = rb * 16 + (lane >> 2), r1 = r0 + 8;
  const bool ok0 = t0 + r0 / a.R < a.T, ok1 = t0 + r1 / a.R < a.T;
  const int64_t p0 = a.pos0 + t0 + r0 / a.R, p1 = a.pos0 + t0 + r1 / a.R;
  float o[32][4];
#pragma unroll
  for (int j = 0; j < 32; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const int qrow = rb * 16 + (lane & 15);
  const uint8_t* qbase = sm + qrow * C::ROWB;

  for (int i = 0; i < nkt; ++i) {
    if (i + 1 < nkt) {
      load_kv(i + 1, (i + 1) & 1);
      cp_async_commit();
      asm volatile("cp.async.wait_group 1;\n" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;\n" ::: "memory");
    }
    __syncthreads();
    const uint8_t* kd = sm + C::Q_BYTES + (i & 1) * C::STAGE;
    const uint8_t* vd = kd + C::KV_BYTES;
    float s[4][4];
#pragma unroll
    for (int n = 0; n < 4; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll 4
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a0, a1, a2, a3;
      ldsm4(qbase + (((2 * kk + (lane >> 4)) ^ (qrow & 7)) << 4), a0, a1, a2, a3);
#pragma unroll
      for (int np = 0; np < 2; ++np) {
        const int krow = np * 16 + ((lane >> 4) << 3) + (lane & 7);
        const int kc = 2 * kk + ((lane >> 3) & 1);
        uint32_t b0, b1, b2, b3;
        ldsm4(kd + krow * C::ROWB + ((kc ^ (krow & 7)) << 4), b0, b1, b2, b3);
        mma16816(s[2 * np], a0, a1, a2, a3, b0, b1);
        mma16816(s[2 * np + 1], a0, a1, a2, a3, b2, b3);
      }
    }
    // mask, scale, online softmax
    const int64_t kbase = kb0 + (int64_t)i * KT;
    float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int64_t kp = kbase + n * 8 + 2 * (lane & 3) + e;
        const bool v0 = ok0 && kp <= p0 && (!a.win || p0 - kp < a.win);
        const bool v1 = ok1 && kp <= p1 && (!a.win || p1 - kp < a.win);
        s[n][e] = v0 ? s[n][e] * a.sl : -INFINITY;
        s[n][2 + e] = v1 ? s[n][2 + e] * a.sl : -INFINITY;
        mx0 = fmaxf(mx0, s[n][e]);
        mx1 = fmaxf(mx1, s[n][2 + e]);
      }
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
    mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
    mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
    const float mn0 = fmaxf(m0, mx0), mn1 = fmaxf(m1, mx1);
    const float c0 = mn0 == -INFINITY ? 0.f : mn0, c1 = mn1 == -INFINITY ? 0.f : mn1;
    const float al0 = exp2f(m0 - c0), al1 = exp2f(m1 - c1);
    m0 = mn0;
    m1 = mn1;
    float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
    for (int n = 0; n < 4; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        s[n][e] = exp2f(s[n][e] - c0);
        s[n][2 + e] = exp2f(s[n][2 + e] - c1);
        ps0 += s[n][e];
        ps1 += s[n][2 + e];
      }
    l0 = l0 * al0 + ps0;
    l1 = l1 * al1 + ps1;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      o[j][0] *= al0;
      o[j][1] *= al0;
      o[j][2] *= al1;
      o[j][3] *= al1;
    }
    uint32_t pa[2][4];
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      pa[kk][0] = pack_bf16x2(s[2 * kk][0], s[2 * kk][1]);
      pa[kk][1] = pack_bf16x2(s[2 * kk][2], s[2 * kk][3]);
      pa[kk][2] = pack_bf16x2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pa[kk][3] = pack_bf16x2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
    }
#pragma unroll
    for (int kk = 0; kk < 2; ++kk) {
      const int vrow = 16 * kk + ((lane >> 3) & 1) * 8 + (lane & 7);
      const uint8_t* vb = vd + vrow * C::ROWB;
#pragma unroll
      for (int np = 0; np < 16; ++np) {
        const int vc = dp * 32 + np * 2 + (lane >> 4);
        uint32_t b0, b1, b2, b3;
        ldsm4t(vb + ((vc ^ (vrow & 7)) << 4), b0, b1, b2, b3);
        mma16816(o[2 * np], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b0, b1);
        mma16816(o[2 * np + 1], pa[kk][0], pa[kk][1], pa[kk][2], pa[kk][3], b2, b3);
      }
    }
    __syncthreads();  // the stage is refilled two tiles later
  }
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float i0 = l0 > 0.f ? 1.f / l0 : 0.f, i1 = l1 > 0.f ? 1.f / l1 : 0.f;
  const int col = dp * 256 + 2 * (lane & 3);
  if (ok0) {
    bf16* orow = a.out + ((int64_t)(t0 + r0 / a.R) * a.Hq + g * a.R + r0 % a.R) * D + col;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      *reinterpret_cast<uint32_t*>(orow + j * 8) = pack_bf16x2(o[j][0] * i0, o[j][1] * i0);
  }
  if (ok1) {
    bf16* orow = a.out + ((int64_t)(t0 + r1 / a.R) * a.Hq + g * a.R + r1 % a.R) * D + col;
#pragma unroll
    for (int j = 0; j < 32; ++j)
      *reinterpret_cast<uint32_t*>(orow + j * 8) = pack_bf16x2(o[j][2] * i1, o[j][3] * i1);
  }
}

}  // namespace pfl

// Attention of T new tokens (one sequence) at positions pos0.. over the ring's
// rows of earlier positions and the staged new rows.
// Output norms, residual and layer scalar of `rows` rows (the decode layer's
// batched feed-forward half): x = (h + post_ff(pff1(d) + pff2(moe))) * scalar.
int launch_ff_out_rows(bf16* x, const bf16* h, const bf16* d, const bf16* moe, int64_t rows, int H, const bf16* w1,
                       const bf16* w2, const bf16* w, float eps, float scalar, cudaStream_t st) {
  if (H % 8 || H > pfl::kRowThreads * pfl::kRowVec * 8)
    return set_error(FMOE_ERR_UNSUPPORTED, "ff_out_rows: hidden %d", H);
  ProfScope prof_("pf_ff_out_kernel", st);
  pfl::pf_ff_out_kernel<<<(unsigned)rows, pfl::kRowThreads, 0, st>>>(x, h, d, moe, H, w1, w2, w, eps, scalar);
  return check_launch("pf_ff_out_kernel");
}

int launch_attn_prefill(const KvDev& c, const bf16* q, int Hq, int64_t T, int64_t pos0, int window,
                        const bf16* ks, const bf16* vs, bf16* out, float scale, cudaStream_t st, bool affine_ok) {
  using namespace pfl;
  if (T <= 0) return FMOE_OK;
  if (c.mode != FMOE_KV_BF16 && !(affine_ok && c.mode == FMOE_KV_AFFINE))
    return set_error(FMOE_ERR_UNSUPPORTED, "attn_prefill: bf16-storage caches only");
  const bool aff = c.mode == FMOE_KV_AFFINE;
  if (c.B != 1) return set_error(FMOE_ERR_INVALID, "attn_prefill: one sequence per call (batch %d)", c.B);
  if (c.D != 256 && c.D != 512) return set_error(FMOE_ERR_UNSUPPORTED, "attn_prefill: head_dim %d", c.D);
  const int R = Hq / c.Hkv;
  if (Hq % c.Hkv || R < 1 || R > QR || (R & (R - 1)))
    return set_error(FMOE_ERR_UNSUPPORTED, "attn_prefill: %d query heads over %d kv heads", Hq, c.Hkv);
  if (window < 0) return set_error(FMOE_ERR_INVALID, "attn_prefill: window %d", window);
  // every stored position the queries need must still be in the ring
  if (window ? (c.cap < window) : (pos0 + T > c.cap))
    return set_error(FMOE_ERR_INVALID, "attn_prefill: capacity %lld too small (window %d, positions to %lld)",
                     (long long)c.cap, window, (long long)(pos0 + T));
  if (T > (1 << 24) || pos0 < 0) return set_error(FMOE_ERR_INVALID, "attn_prefill: T %lld, pos0 %lld", (long long)T,
                                                  (long long)pos0);
  if (!aligned(q, 16) || !aligned(ks, 16) || !aligned(vs, 16) || !aligned(out, 16))
    return set_error(FMOE_ERR_ALIGN, "attn_prefill: buffers must be 16-byte aligned");
  PaArgs a;
  a.q = q;
  a.kr = static_cast<const bf16*>(c.k);
  a.vr = static_cast<const bf16*>(c.v);
  a.ks = ks;
  a.vs = vs;
  a.out = out;
  a.T = (int)T;
  a.Hq = Hq;
  a.R = R;
  a.QT = QR / R;
  a.win = window;
  a.pos0 = pos0;
  a.cap = c.cap;
  a.sl = scale * 1.4426950408889634f;
  a.kq = aff ? static_cast<const uint32_t*>(c.k) : nullptr;
  a.vq = aff ? static_cast<const uint32_t*>(c.v) : nullptr;
  a.kss = c.ks;
  a.kbb = c.kb;
  a.vss = c.vs;
  a.vbb = c.vb;
  if (aff) a.kr = a.vr = nullptr;
  const dim3 grid((unsigned)((T + a.QT - 1) / a.QT), (unsigned)c.Hkv);
  if (c.D == 256) {
    auto k = aff ? pf_attn_kernel<256, true> : pf_attn_kernel<256, false>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, PaCfg<256>::SMEM);
    ProfScope prof_(aff ? "pf_attn_kernel<256, affine>" : "pf_attn_kernel<256>", st);
    k<<<grid, PaCfg<256>::THREADS, PaCfg<256>::SMEM, st>>>(a);
  } else {
    auto k = aff ? pf_attn_kernel<512, true> : pf_attn_kernel<512, false>;
    cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, PaCfg<512>::SMEM);
    ProfScope prof_(aff ? "pf_attn_kernel<512, affine>" : "pf_attn_kernel<512>", st);
    k<<<grid, PaCfg<512>::THREADS, PaCfg<512>::SMEM, st>>>(a);
  }
  return check_launch("pf_attn_kernel");
}

namespace {

struct PfLayerWs {
  bf16 *xn, *q, *k, *v, *ks, *vs, *kr, *vr, *att, *h1, *h2, *act, *d, *moe;
  void* moe_ws;
  size_t moe_bytes;
};

// The MoE prefill's workspace comes first, so its status word is the layer's.
// n_ranks > 0: the routed experts are this rank's slice, run by the
// expert-parallel MoE (exact exchange, cap = T).
size_t carve_pf_layer(Carver& c, const fmoe_decoder_layer_t* L, int64_t T, PfLayerWs* w, int n_ranks = 0) {
  PfLayerWs p{};
  const size_t mb = n_ranks > 0 ? fmoe_ep_moe_workspace_bytes(n_ranks, T, &L->router, &L->experts)
                                : fmoe_moe_prefill_workspace_bytes(T, &L->router, &L->experts);
  if (!mb) return 0;
  p.moe_ws = c.take<uint8_t>(mb);
  p.moe_bytes = mb;
  const int64_t H = L->q_proj.in_features, Q = (int64_t)L->num_heads * L->head_dim,
                KV = (int64_t)L->num_kv_heads * L->head_dim, I = L->mlp_gate.out_features;
  p.xn = c.take<bf16>(T * H);
  p.q = c.take<bf16>(T * Q);
  p.k = c.take<bf16>(T * KV);
  p.v = L->k_eq_v ? nullptr : c.take<bf16>(T * KV);
  p.ks = c.take<bf16>(T * KV);
  p.vs = c.take<bf16>(T * KV);
  p.kr = c.take<bf16>(T * KV);  // affine caches: the new rows as the cache returns them (rotated basis)
  p.vr = c.take<bf16>(T * KV);
  p.att = c.take<bf16>(T * Q);
  p.h1 = c.take<bf16>(T * H);
  p.h2 = c.take<bf16>(T * H);
  p.act = c.take<bf16>(T * I);
  p.d = c.take<bf16>(T * H);
  p.moe = c.take<bf16>(T * H);
  if (w) *w = p;
  return c.off;
}

int launch_pf_qkv_post(bf16* q, const bf16* k, const bf16* v, int64_t T, int Hq, int Hkv, int D, const bf16* qn,
                       const bf16* kn, float eps, int rope_dims, float theta, int64_t pos0, int turbo, bf16* ks,
                       bf16* vs, cudaStream_t st) {
  const unsigned blocks = (unsigned)T;
  const float l2t = std::log2(theta);
  ProfScope prof_("pf_qkv_post_kernel", st);
  if (D == 256)
    pfl::pf_qkv_post_kernel<8><<<blocks, 32 * pfl::kPostWarps, 0, st>>>(q, k, v, (int)T, Hq, Hkv, qn, kn, eps,
                                                                        rope_dims, l2t, pos0, turbo, ks, vs);
  else
    pfl::pf_qkv_post_kernel<16><<<blocks, 32 * pfl::kPostWarps, 0, st>>>(q, k, v, (int)T, Hq, Hkv, qn, kn, eps,
                                                                         rope_dims, l2t, pos0, turbo, ks, vs);
  return check_launch("pf_qkv_post_kernel");
}

}  // namespace

}  // namespace fmoe

using namespace fmoe;

extern "C" int fmoe_attn_prefill(const fmoe_kv_cache_t* cache, const void* q, int q_heads, int64_t T, int64_t pos0,
                                 int window, const void* k_new, const void* v_new, void* out, float scale,
                                 void* stream) {
  KvDev c;
  int rc;
  if (!cache) return set_error(FMOE_ERR_INVALID, "attn_prefill: null cache");
  if ((rc = kv_to_dev(cache, &c))) return rc;
  if (!q || !k_new || !v_new || !out) return set_error(FMOE_ERR_INVALID, "attn_prefill: null q / k / v / out");
  return launch_attn_prefill(c, static_cast<const bf16*>(q), q_heads, T, pos0, window,
                             static_cast<const bf16*>(k_new), static_cast<const bf16*>(v_new), static_cast<bf16*>(out),
                             scale, static_cast<cudaStream_t>(stream));
}

extern "C" size_t fmoe_mlp_workspace_bytes(int64_t T, const fmoe_qweight_t* gate) {
  if (T <= 0 || !gate || gate->out_features <= 0) return 0;
  return align_up(sizeof(bf16) * (size_t)T * gate->out_features, 256) + 512;
}

extern "C" int fmoe_mlp_forward(const void* x, int64_t T, const fmoe_qweight_t* gate, const fmoe_qweight_t* up,
                                const fmoe_qweight_t* down, void* y, void* workspace, size_t workspace_bytes,
                                void* stream) {
  QW g, u, d;
  int rc;
  if ((rc = to_qw(gate, &g)) || (rc = to_qw(up, &u)) || (rc = to_qw(down, &d))) return rc;
  if (!x || !y) return set_error(FMOE_ERR_INVALID, "mlp: null x / y");
  if (T <= 0) return FMOE_OK;
  if (g.out != u.out || g.in != u.in || d.in != g.out || d.out != g.in)
    return set_error(FMOE_ERR_INVALID, "mlp: gate [%d, %d], up [%d, %d], down [%d, %d]", g.out, g.in, u.out, u.in,
                     d.out, d.in);
  if (!qgemm_supported(g, gate->group_size, g.in) || !qgemm_supported(u, up->group_size, u.in) ||
      !qgemm_supported(d, down->group_size, d.in) || g.bits != u.bits)
    return set_error(FMOE_ERR_UNSUPPORTED, "mlp: 4 / 8-bit group-64 weights with 16-byte aligned codes only");
  const size_t need = fmoe_mlp_workspace_bytes(T, gate);
  if (!workspace || workspace_bytes < need)
    return set_error(FMOE_ERR_WORKSPACE, "mlp: workspace %zu < %zu", workspace_bytes, need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver c(workspace);
  int* status = c.take<int>(64);
  bf16* act = c.take<bf16>((size_t)T * g.out);
  const QmOut gu[2] = {{&g, act, g.out}, {&u, act, g.out}};
  if ((rc = launch_qgemm(static_cast<const bf16*>(x), T, g.in, gu, 2, true, status, st))) return rc;
  const QmOut dn{&d, static_cast<bf16*>(y), d.out};
  return launch_qgemm(act, T, d.in, &dn, 1, false, status, st);
}

namespace {

size_t pf_layer_bytes(const fmoe_decoder_layer_t* L, int64_t T, int n_ranks) {
  if (!L || T <= 0) return 0;
  Carver c(nullptr);
  const size_t n = carve_pf_layer(c, L, T, nullptr, n_ranks);
  return n ? n + 256 : 0;
}

int layer_prefill(const fmoe_decoder_layer_t* L, const fmoe_kv_cache_t* cache, fmoe_ep_comm_t* comm, void* x,
                  int64_t T, int64_t pos0, int window, const void* expert_prep, void* workspace,
                  size_t workspace_bytes, void* stream) {
  if (!L || !cache || !x) return set_error(FMOE_ERR_INVALID, "layer_prefill: null layer / cache / x");
  if (T <= 0) return FMOE_OK;
  if (!expert_prep) return set_error(FMOE_ERR_INVALID, "layer_prefill: null prepared expert scales");
  KvDev c;
  int rc;
  if ((rc = kv_to_dev(cache, &c))) return rc;
  const int Hq = L->num_heads, Hkv = L->num_kv_heads, D = L->head_dim;
  if (c.Hkv != Hkv || c.D != D)
    return set_error(FMOE_ERR_INVALID, "layer_prefill: cache heads %d x %d vs layer %d x %d", c.Hkv, c.D, Hkv, D);
  QW q, k, v, o, g, u, dn;
  if ((rc = to_qw(&L->q_proj, &q)) || (rc = to_qw(&L->k_proj, &k)) || (!L->k_eq_v && (rc = to_qw(&L->v_proj, &v))) ||
      (rc = to_qw(&L->o_proj, &o)) || (rc = to_qw(&L->mlp_gate, &g)) || (rc = to_qw(&L->mlp_up, &u)) ||
      (rc = to_qw(&L->mlp_down, &dn)))
    return rc;
  const int H = q.in;
  if (q.out != Hq * D || k.out != Hkv * D || (!L->k_eq_v && v.out != Hkv * D) || o.in != Hq * D || o.out != H ||
      g.in != H || dn.out != H)
    return set_error(FMOE_ERR_INVALID, "layer_prefill: projection shapes do not match the heads");
  if (H % 8 || !aligned(x, 16)) return set_error(FMOE_ERR_ALIGN, "layer_prefill: x must be 16-byte aligned, H %% 8 == 0");
  if (H > pfl::kRowMaxH) return set_error(FMOE_ERR_UNSUPPORTED, "layer_prefill: hidden %d > %d", H, pfl::kRowMaxH);
  if (L->rope_dims < 0 || L->rope_dims > D || L->rope_dims % 2)
    return set_error(FMOE_ERR_INVALID, "layer_prefill: rope_dims %d for head_dim %d", L->rope_dims, D);
  const int n_ranks = ep_comm_ranks(comm);
  const size_t need = pf_layer_bytes(L, T, n_ranks);
  if (!need) return set_error(FMOE_ERR_UNSUPPORTED, "layer_prefill: the routed experts have no prefill path");
  if (!workspace || workspace_bytes < need)
    return set_error(FMOE_ERR_WORKSPACE, "layer_prefill: workspace %zu < %zu", workspace_bytes, need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver cv(workspace);
  PfLayerWs w;
  carve_pf_layer(cv, L, T, &w, n_ranks);
  int* status = static_cast<int*>(workspace);  // the MoE workspace's header
  bf16* xb = static_cast<bf16*>(x);
  const unsigned rows = (unsigned)T;
  // attention block
  {
    ProfScope prof_("pf_norm_rows_kernel", st);
    pfl::pf_norm_rows_kernel<<<rows, pfl::kRowThreads, 0, st>>>(xb, H, static_cast<const bf16*>(L->input_norm),
                                                                  L->eps, w.xn);
  }
  if ((rc = check_launch("pf_norm_rows_kernel"))) return rc;
  {
    const QmOut qkv[3] = {{&q, w.q, q.out}, {&k, w.k, k.out}, {&v, w.v, Hkv * D}};
    if ((rc = launch_qgemm(w.xn, T, H, qkv, L->k_eq_v ? 2 : 3, false, status, st))) return rc;
  }
  if ((rc = launch_pf_qkv_post(w.q, w.k, L->k_eq_v ? nullptr : w.v, T, Hq, Hkv, D,
                               static_cast<const bf16*>(L->q_norm), static_cast<const bf16*>(L->k_norm), L->eps,
                               L->rope_dims, L->rope_theta, pos0, c.mode == FMOE_KV_BF16 ? c.turbo : 0, w.ks, w.vs,
                               st)))
    return rc;
  const bool aff = c.mode == FMOE_KV_AFFINE;
  const float inv = 1.0f / std::sqrt((float)D);
  if (aff) {  // attention in the cache's rotated basis
    const int64_t rows = T * Hq + 2 * (int64_t)Hkv * T;
    const unsigned blocks = (unsigned)((rows + 7) / 8);
    ProfScope prof_("pf_affine_prep_kernel", st);
    if (D == 256)
      pfl::pf_affine_prep_kernel<8><<<blocks, 256, 0, st>>>(w.q, w.ks, w.vs, (int)T, Hq, Hkv, inv, w.kr, w.vr);
    else
      pfl::pf_affine_prep_kernel<16><<<blocks, 256, 0, st>>>(w.q, w.ks, w.vs, (int)T, Hq, Hkv, inv, w.kr, w.vr);
    if ((rc = check_launch("pf_affine_prep_kernel"))) return rc;
  }
  if ((rc = launch_attn_prefill(c, w.q, Hq, T, pos0, window, aff ? w.kr : w.ks, aff ? w.vr : w.vs, w.att,
                                L->attn_scale, st, true)))
    return rc;
  if (aff) {  // the output back to the original basis
    const int64_t rows = T * Hq;
    const unsigned blocks = (unsigned)((rows + 7) / 8);
    ProfScope prof_("pf_rotate_rows_kernel", st);
    if (D == 256)
      pfl::pf_rotate_rows_kernel<8><<<blocks, 256, 0, st>>>(w.att, rows, inv);
    else
      pfl::pf_rotate_rows_kernel<16><<<blocks, 256, 0, st>>>(w.att, rows, inv);
    if ((rc = check_launch("pf_rotate_rows_kernel"))) return rc;
  }
  // the staged rows: already round-tripped (TurboQuant) and appended as they
  // are, or (affine) rotated and quantised by the append itself
  if ((rc = launch_kv_append(c, w.ks, w.vs, T, pos0, nullptr, 0, st))) return rc;
  {
    const QmOut oo{&o, w.xn, H};
    if ((rc = launch_qgemm(w.att, T, Hq * D, &oo, 1, false, status, st))) return rc;
  }
  {
    ProfScope prof_("pf_ff_in_kernel", st);
    pfl::pf_ff_in_kernel<<<rows, pfl::kRowThreads, 0, st>>>(
        xb, w.xn, H, static_cast<const bf16*>(L->post_attn_norm), static_cast<const bf16*>(L->pre_ff_norm),
        static_cast<const bf16*>(L->pre_ff_norm_2), L->eps, w.h1, w.h2);
  }
  if ((rc = check_launch("pf_ff_in_kernel"))) return rc;
  // dense GeLU MLP and routed experts
  {
    const QmOut gu[2] = {{&g, w.act, g.out}, {&u, w.act, g.out}};
    if ((rc = launch_qgemm(w.h1, T, H, gu, 2, true, status, st))) return rc;
    const QmOut dd{&dn, w.d, H};
    if ((rc = launch_qgemm(w.act, T, g.out, &dd, 1, false, status, st))) return rc;
  }
  if (comm) {  // this rank's expert slice; every rank passes the same T (cap)
    if ((rc = fmoe_ep_moe_forward(comm, w.h2, T, T, &L->router, &L->experts, expert_prep, w.moe, nullptr, nullptr,
                                  FMOE_EP_EXACT, w.moe_ws, w.moe_bytes, st)))
      return rc;
  } else if ((rc = fmoe_moe_prefill(w.h2, T, &L->router, &L->experts, expert_prep, w.moe, nullptr, nullptr, w.moe_ws,
                                    w.moe_bytes, st))) {
    return rc;
  }
  {
    ProfScope prof_("pf_ff_out_kernel", st);
    pfl::pf_ff_out_kernel<<<rows, pfl::kRowThreads, 0, st>>>(
        xb, xb, w.d, w.moe, H, static_cast<const bf16*>(L->post_ff_norm_1), static_cast<const bf16*>(L->post_ff_norm_2),
        static_cast<const bf16*>(L->post_ff_norm), L->eps, L->layer_scalar);
  }
  return check_launch("pf_ff_out_kernel");
}

}  // namespace

extern "C" size_t fmoe_decoder_layer_prefill_workspace_bytes(const fmoe_decoder_layer_t* L, int64_t T) {
  return pf_layer_bytes(L, T, 0);
}

extern "C" int fmoe_decoder_layer_prefill(const fmoe_decoder_layer_t* L, const fmoe_kv_cache_t* cache, void* x,
                                          int64_t T, int64_t pos0, int window, const void* expert_prep,
                                          void* workspace, size_t workspace_bytes, void* stream) {
  return layer_prefill(L, cache, nullptr, x, T, pos0, window, expert_prep, workspace, workspace_bytes, stream);
}

extern "C" size_t fmoe_decoder_layer_prefill_ep_workspace_bytes(const fmoe_decoder_layer_t* L, int64_t T,
                                                                 int n_ranks) {
  if (n_ranks < 1) return 0;
  return pf_layer_bytes(L, T, n_ranks);
}

extern "C" int fmoe_decoder_layer_prefill_ep(const fmoe_decoder_layer_t* L, const fmoe_kv_cache_t* cache,
                                             fmoe_ep_comm_t* comm, void* x, int64_t T, int64_t pos0, int window,
                                             const void* expert_prep, void* workspace, size_t workspace_bytes,
                                             void* stream) {
  if (!comm) return set_error(FMOE_ERR_INVALID, "layer_prefill_ep: null communicator");
  return layer_prefill(L, cache, comm, x, T, pos0, window, expert_prep, workspace, workspace_bytes, stream);
}
