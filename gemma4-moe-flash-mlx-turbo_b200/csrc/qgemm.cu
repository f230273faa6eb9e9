// Dense quantised linear layers over many tokens (prefill) on the 5th-generation
// tensor cores: y[T][N] = x[T][K] . dequant(W)[N][K]^T for MLX-affine 4- or
// 8-bit weights with groups of 64, the many-token form of
// QuantizedLinear::forward (src/model/mlp.rs:15-25) and of GeLUMLP's gate / up /
// down (src/model/mlp.rs:28-41).
//
// Persistent kernel.  An item is 128 (plain form, two CTAs per SM, 10 warps)
// or 256 (gated form, one CTA per SM, 14 warps) weight rows x one tile of up to
// 128 tokens; items run weight-tile-major, so the CTAs that run at the same
// time share a weight tile in L2, and x stays in L2.
//   warp 0      producer: TMA of the token tile (bf16 [tokens][64], 128-byte
//               swizzle, one per K tile; a ring of 4 (gated) or 2 (plain)) and
//               of the packed codes (boxes of 128 rows x 128 bytes = 2 (8-bit)
//               or 4 (4-bit) K tiles, 128-byte swizzle; 3 or 2 stages ahead of
//               the dequantisers)
//   warp 1      MMA issuer: per K tile 4 tcgen05.mma (K 16) per half with the
//               dequantised weights as the M = 128 operand and
//               the tokens as N (rounded up to 16), into one of two TMEM
//               accumulators
//   next 4 / 8  dequantise one weight row each: w = bf16(s * q + b), s * q + b
//               in fp32, written in the canonical K-major 128-byte-swizzled
//               layout (a ring of 2 K tiles, each released by the MMA's commit);
//               the row's scale and bias are loaded from global memory one
//               packed stage ahead
//   last 4      epilogue: tcgen05.ld (TMEM lane = weight row, column = token),
//               bf16 stores, or (gated mode) gelu(gate) * up from the two
//               halves, the first projection of the GeLU MLP
// The plain mode takes up to three weights that share x (q, k and v), each a
// run of items with its own output.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <mutex>
#include "tc.cuh"

namespace fmoe {
namespace qm {

using namespace tc;

constexpr int BK = 64;                 // K per tile = one quantisation group
constexpr int X_BYTES = 128 * BK * 2;  // 16 KB: up to 128 tokens x 64 bf16

// Tile configuration by the number of 128-row halves (M = 128 MMAs) per item.
// NH = 2: 256 weight rows per item, one CTA per SM (the gated MLP form needs
// the gate and up halves together).  NH = 1: 128 rows per item and about
// 97 KB of shared memory and 256 TMEM columns, so two CTAs share an SM and one
// covers the other's dependency latency.
template <int NH>
struct Cfg {
  static constexpr int BN = 128 * NH;            // weight rows per item
  static constexpr int NX = NH == 2 ? 4 : 2;     // token-tile ring (TMA lookahead of the MMA)
  static constexpr int NW = 2;                   // dequantised-weight ring
  static constexpr int NQ = NH == 2 ? 3 : 2;     // packed-code stages (lookahead of the dequantisers)
  static constexpr int WB_BYTES = BN * BK * 2;   // BN rows x 64 bf16
  static constexpr int WQ_BYTES = BN * 128;      // BN rows x 128 bytes of codes
  static constexpr int OFF_X = 0;
  static constexpr int OFF_WB = OFF_X + NX * X_BYTES;
  static constexpr int OFF_WQ = OFF_WB + NW * WB_BYTES;
  static constexpr int OFF_BAR = OFF_WQ + NQ * WQ_BYTES;
  static constexpr int SMEM = OFF_BAR + 256 + 1024;  // + slack to align the base to 1024 bytes
  static constexpr int NDQ = 4 * NH;                 // dequantising warps: one thread per weight row
  static constexpr int THREADS = (2 + NDQ + 4) * 32;
  static constexpr int ACC = 128 * NH;               // TMEM columns of one accumulator ([halves][128 tokens])
  static constexpr int TMEM_COLS = 2 * ACC;          // two accumulators
  static constexpr int MINB = NH == 2 ? 1 : 2;       // CTAs per SM
  static_assert(OFF_WB % 1024 == 0 && OFF_WQ % 1024 == 0 && OFF_BAR % 1024 == 0, "ring alignment");
  static_assert(SMEM <= 227 * 1024 && MINB * (SMEM + 1024) <= 228 * 1024, "shared memory");
};

struct Seg {
  const bf16* s;  // scales [N][G]
  const bf16* b;  // biases [N][G]
  bf16* out;      // row t of the output at out + t * ld
  int N, ld;
  int item0;      // first item of the segment
};
struct alignas(64) Maps {
  CUtensorMap x[2];  // token tiles: boxes of 128 and 64 rows
  CUtensorMap w[kQmMaxSeg];
};
struct Args {
  Seg seg[kQmMaxSeg];
  int nseg, K, G, T, tb, nt, nitems;
  int* status;
};

struct Item {
  int sg, j, t0, ntok;
};
// Item `it` -> (segment, weight tile, first token, tokens).  The gated mode has
// one segment pair: gate (seg 0) and up (seg 1) rows j*128 .. j*128+127.
template <int MODE>
__device__ __forceinline__ Item item_at(const Args& a, int it) {
  int sg = 0;
  if (MODE == 0) {
#pragma unroll
    for (int s = 1; s < kQmMaxSeg; ++s)
      if (s < a.nseg && it >= a.seg[s].item0) sg = s;
  }
  const int loc = it - a.seg[sg].item0;
  Item r;
  r.sg = sg;
  r.j = loc / a.nt;
  r.t0 = (loc % a.nt) * a.tb;
  r.ntok = min(a.tb, a.T - r.t0);
  return r;
}

// 16-bit load issued where it stands (volatile: the compiler may not sink it to
// its first use, a packed stage later)
__device__ __forceinline__ uint16_t ldg_u16_now(const void* p) {
  unsigned short r;
  asm volatile("ld.global.nc.u16 %0, [%1];\n" : "=h"(r) : "l"(p));
  return r;
}

// code byte i of w as a float: 0x4B000000 | q is 2^23 + q
__device__ __forceinline__ float u8f(uint32_t w, int i) {
  return __uint_as_float(prmt(w, 0x4B000000u, 0x7540u | (uint32_t)i)) - 8388608.f;
}
__device__ __forceinline__ float u4f(uint32_t w, int i) {
  return __uint_as_float(((w >> (4 * i)) & 0xFu) | 0x4B000000u) - 8388608.f;
}

template <int BITS, int MODE, int NH>  // MODE 0: plain bf16 output; 1: gelu(gate) * up
__global__ void __launch_bounds__(Cfg<NH>::THREADS, Cfg<NH>::MINB)
    qgemm_kernel(const __grid_constant__ Maps maps, const Args a) {
  using C = Cfg<NH>;
  static_assert(MODE == 0 || NH == 2, "the gated form takes gate and up halves together");
  constexpr int BN = C::BN, NX = C::NX, NW = C::NW, NQ = C::NQ, NDQ = C::NDQ;
  constexpr int WB_BYTES = C::WB_BYTES, WQ_BYTES = C::WQ_BYTES;
  constexpr int OFF_X = C::OFF_X, OFF_WB = C::OFF_WB, OFF_WQ = C::OFF_WQ, OFF_BAR = C::OFF_BAR;
  constexpr int TMEM_COLS = C::TMEM_COLS, ACC = C::ACC;
  constexpr int KQ = 128 / (8 * BITS);  // K tiles per packed stage
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  uint64_t* xfull = reinterpret_cast<uint64_t*>(smem + OFF_BAR);  // token tile landed
  uint64_t* xfree = xfull + NX;                                     // MMAs done with the token tile
  uint64_t* deqd = xfree + NX;                                      // dequantised weights written
  uint64_t* wfree = deqd + NW;                                      // MMAs done with those weights
  uint64_t* wqf = wfree + NW;                                       // packed codes landed
  uint64_t* wqe = wqf + NQ;                                         // dequantisers done with them
  uint64_t* accf = wqe + NQ;                                        // accumulator complete
  uint64_t* acce = accf + 2;                                        // accumulator read out
  volatile int* failed = reinterpret_cast<volatile int*>(acce + 2);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acce + 2) + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int NK = a.K / BK;
  const int NKQ = (NK + KQ - 1) / KQ;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NX; ++s) {
      mbar_init(&xfull[s], 1);
      mbar_init(&xfree[s], 1);
    }
    for (int s = 0; s < NW; ++s) {
      mbar_init(&deqd[s], NDQ);
      mbar_init(&wfree[s], 1);
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
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ---- producer
    if (lane == 0) {
      int q = 0, qq = 0;
      const CUtensorMap* xm = &maps.x[a.tb == 128 ? 0 : 1];
      for (int it = blockIdx.x; it < a.nitems; it += gridDim.x) {
        const Item t = item_at<MODE>(a, it);
        for (int kt = 0; kt < NK; ++kt, ++q) {
          if (kt % KQ == 0) {
            const int sq = qq % NQ;
            if (qq >= NQ) pwait_sleep(&wqe[sq], (uint32_t)((qq / NQ) - 1) & 1u, failed, a.status, 401, 64);
            if (*failed) break;
            uint8_t* wq = smem + OFF_WQ + sq * WQ_BYTES;
            const int xb = (kt / KQ) * 128;  // byte column of the boxes
            mbar_arrive_expect_tx(&wqf[sq], (uint32_t)WQ_BYTES);
            if (MODE == 0) {
              tma2d(wq, &maps.w[t.sg], xb, t.j * BN, &wqf[sq]);
              if (NH == 2) tma2d(wq + WQ_BYTES / 2, &maps.w[t.sg], xb, t.j * BN + 128, &wqf[sq]);
            } else {
              tma2d(wq, &maps.w[0], xb, t.j * 128, &wqf[sq]);
              tma2d(wq + WQ_BYTES / 2, &maps.w[1], xb, t.j * 128, &wqf[sq]);
            }
            ++qq;
          }
          const int s = q % NX;
          if (q >= NX) pwait_sleep(&xfree[s], (uint32_t)((q / NX) - 1) & 1u, failed, a.status, 402, 64);
          if (*failed) break;
          mbar_arrive_expect_tx(&xfull[s], (uint32_t)(a.tb * BK * 2));
          tma2d(smem + OFF_X + s * X_BYTES, xm, kt * BK, t.t0, &xfull[s]);
        }
        if (*failed) break;
      }
      // every copy issued lands before the CTA ends
      for (int k = q - NX < 0 ? 0 : q - NX; k < q; ++k) drain_wait(&xfull[k % NX], (uint32_t)(k / NX) & 1u);
      for (int k = qq - NQ < 0 ? 0 : qq - NQ; k < qq; ++k) drain_wait(&wqf[k % NQ], (uint32_t)(k / NQ) & 1u);
    }
  } else if (warp == 1) {
    // ---- MMA issuer
    if (lane == 0) {
      int q = 0, n = 0;
      for (int it = blockIdx.x; it < a.nitems; it += gridDim.x, ++n) {
        const int ab = n & 1;
        const Item t = item_at<MODE>(a, it);
        const uint32_t idesc = idesc_n((t.ntok + 15) & ~15);
        if (n >= 2) pwait(&acce[ab], (uint32_t)((n / 2) - 1) & 1u, failed, a.status, 403);
        tc_fence_after();
        for (int kt = 0; kt < NK; ++kt, ++q) {
          const int s = q % NX, w = q % NW;
          pwait(&xfull[s], (uint32_t)(q / NX) & 1u, failed, a.status, 404);
          pwait(&deqd[w], (uint32_t)(q / NW) & 1u, failed, a.status, 405);
          tc_fence_after();
          const uint32_t sx = smem_u32(smem + OFF_X + s * X_BYTES), sw = smem_u32(smem + OFF_WB + w * WB_BYTES);
          if (!*failed) {
#pragma unroll
            for (int h = 0; h < NH; ++h)
#pragma unroll
              for (int k = 0; k < BK / 16; ++k)
                mma_ss(tmem + ab * ACC + h * 128, sw128_desc(sw + h * (128 * 128) + 32 * k), sw128_desc(sx + 32 * k),
                       idesc, (kt | k) != 0);
          }
          mma_commit(&xfree[s]);
          mma_commit(&wfree[w]);
        }
        mma_commit(&accf[ab]);
      }
      if (n > 0) drain_wait(&accf[(n - 1) & 1], (uint32_t)((n - 1) / 2) & 1u);
    }
  } else if (warp < 2 + NDQ) {
    // ---- dequantisers: thread rr = row rr of the item's 256 rows (half rr / 128)
    const int rr = threadIdx.x - 64, h = rr >> 7;
    // raw bf16 scale / bias of the packed stage (item it, group block kg), KQ groups
    auto load_sb = [&](int it, int kg, uint32_t (&sb)[KQ]) {
#pragma unroll
      for (int i = 0; i < KQ; ++i) sb[i] = 0u;
      if (it >= a.nitems) return;
      const Item t = item_at<MODE>(a, it);
      const Seg& sg = a.seg[MODE == 0 ? t.sg : h];
      const int row = MODE == 0 ? t.j * BN + rr : t.j * 128 + (rr & 127);
      if (row >= sg.N) return;
      const bf16* sp = sg.s + (int64_t)row * a.G;
      const bf16* bp = sg.b + (int64_t)row * a.G;
#pragma unroll
      for (int i = 0; i < KQ; ++i) {
        const int kt = kg * KQ + i;
        if (kt < NK) sb[i] = (uint32_t)ldg_u16_now(sp + kt) | ((uint32_t)ldg_u16_now(bp + kt) << 16);
      }
    };
    uint32_t cur[KQ], nxt[KQ];
    load_sb(blockIdx.x, 0, nxt);
    int q = 0, qq = 0;
    for (int it = blockIdx.x; it < a.nitems; it += gridDim.x) {
      for (int kt = 0; kt < NK; ++kt, ++q) {
        const int s = q % NW, sq = qq % NQ, kq = kt % KQ;
        if (kq == 0) {
#pragma unroll
          for (int i = 0; i < KQ; ++i) cur[i] = nxt[i];
          const int kg = kt / KQ + 1;
          if (kg < NKQ)
            load_sb(it, kg, nxt);
          else
            load_sb(it + gridDim.x, 0, nxt);
          pwait(&wqf[sq], (uint32_t)(qq / NQ) & 1u, failed, a.status, 406);
        }
        // the MMAs of the slot's previous use are done with its weights
        if (q >= NW) pwait(&wfree[s], (uint32_t)((q / NW) - 1) & 1u, failed, a.status, 407);
        uint32_t sbv = 0u;
#pragma unroll
        for (int i = 0; i < KQ; ++i)
          if (i == kq) sbv = cur[i];
        const float sv = __uint_as_float(sbv << 16), bv = __uint_as_float(sbv & 0xFFFF0000u);
        const uint8_t* wrow_q = smem + OFF_WQ + sq * WQ_BYTES + rr * 128;
        uint8_t* wrow = smem + OFF_WB + s * WB_BYTES + rr * 128;
        if (BITS == 8) {
          // K tile kq = 16-byte chunks 4kq .. 4kq+3 of the 128-byte row (swizzled by row % 8)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const uint4 w = *reinterpret_cast<const uint4*>(wrow_q + (((4 * kq + c) ^ (rr & 7)) << 4));
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int hc = 0; hc < 2; ++hc) {  // output chunk 2c + hc = words 2hc, 2hc+1
              const uint32_t w0 = ww[2 * hc], w1 = ww[2 * hc + 1];
              const uint4 o = make_uint4(pack_bf16x2(fmaf(u8f(w0, 0), sv, bv), fmaf(u8f(w0, 1), sv, bv)),
                                         pack_bf16x2(fmaf(u8f(w0, 2), sv, bv), fmaf(u8f(w0, 3), sv, bv)),
                                         pack_bf16x2(fmaf(u8f(w1, 0), sv, bv), fmaf(u8f(w1, 1), sv, bv)),
                                         pack_bf16x2(fmaf(u8f(w1, 2), sv, bv), fmaf(u8f(w1, 3), sv, bv)));
              *reinterpret_cast<uint4*>(wrow + (((2 * c + hc) ^ (rr & 7)) << 4)) = o;
            }
          }
        } else {
          // K tile kq = 16-byte chunks 2kq, 2kq+1; one word = 8 codes = one output chunk
#pragma unroll
          for (int c = 0; c < 2; ++c) {
            const uint4 w = *reinterpret_cast<const uint4*>(wrow_q + (((2 * kq + c) ^ (rr & 7)) << 4));
            const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int wi = 0; wi < 4; ++wi) {
              const uint32_t v = ww[wi];
              const uint4 o = make_uint4(pack_bf16x2(fmaf(u4f(v, 0), sv, bv), fmaf(u4f(v, 1), sv, bv)),
                                         pack_bf16x2(fmaf(u4f(v, 2), sv, bv), fmaf(u4f(v, 3), sv, bv)),
                                         pack_bf16x2(fmaf(u4f(v, 4), sv, bv), fmaf(u4f(v, 5), sv, bv)),
                                         pack_bf16x2(fmaf(u4f(v, 6), sv, bv), fmaf(u4f(v, 7), sv, bv)));
              *reinterpret_cast<uint4*>(wrow + (((4 * c + wi) ^ (rr & 7)) << 4)) = o;
            }
          }
        }
        asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");  // generic writes -> tensor-core reads
        __syncwarp();
        const bool last = kq == KQ - 1 || kt == NK - 1;
        if (lane == 0) {
          mbar_arrive(&deqd[s]);
          if (last) mbar_arrive(&wqe[sq]);
        }
        if (last) ++qq;
      }
    }
  } else {
    // ---- epilogue: TMEM lane = weight row 32 * (warp % 4) + lane, column = token
    const int qw = warp & 3;
    int n = 0;
    for (int it = blockIdx.x; it < a.nitems; it += gridDim.x, ++n) {
      const Item t = item_at<MODE>(a, it);
      const int ab = n & 1, nc = (t.ntok + 15) / 16;
      pwait_sleep(&accf[ab], (uint32_t)(n / 2) & 1u, failed, a.status, 408, 256);
      tc_fence_after();
      const uint32_t ta = tmem + ((uint32_t)(qw * 32) << 16) + ab * ACC;
      const bool ok = !*failed;
      if (MODE == 0) {
        const Seg& sg = a.seg[t.sg];
#pragma unroll 1
        for (int hh = 0; hh < NH; ++hh) {
          const int row = t.j * BN + hh * 128 + qw * 32 + lane;
          bf16* o = sg.out + (int64_t)t.t0 * sg.ld + row;
#pragma unroll 1
          for (int cc = 0; cc < nc; ++cc) {
            float v[16];
            tmem_ld16(ta + hh * 128 + cc * 16, v);
            tmem_ld_wait();
            if (ok && row < sg.N) {
#pragma unroll
              for (int i = 0; i < 16; ++i)
                if (cc * 16 + i < t.ntok) o[(int64_t)(cc * 16 + i) * sg.ld] = __float2bfloat16_rn(v[i]);
            }
          }
        }
      } else {
        const Seg& sg = a.seg[0];
        const int f = t.j * 128 + qw * 32 + lane;
        bf16* o = sg.out + (int64_t)t.t0 * sg.ld + f;
#pragma unroll 1
        for (int cc = 0; cc < nc; ++cc) {
          float g[16], u[16];
          tmem_ld16(ta + cc * 16, g);
          tmem_ld16(ta + 128 + cc * 16, u);
          tmem_ld_wait();
          if (ok && f < sg.N) {
#pragma unroll
            for (int i = 0; i < 16; ++i)
              if (cc * 16 + i < t.ntok)
                o[(int64_t)(cc * 16 + i) * sg.ld] = __float2bfloat16_rn(gelu_tanh(round_bf(g[i])) * round_bf(u[i]));
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

}  // namespace qm

bool qgemm_supported(const QW& w, int group, int K) {
  return (w.bits == 4 || w.bits == 8) && group == 64 && w.in == K && K % 64 == 0 && K >= 64 && w.out >= 1 &&
         aligned(w.w, 16) && w.s && w.b;
}

int launch_qgemm(const bf16* x, int64_t T, int K, const QmOut* o, int nseg, bool gated, int* status,
                 cudaStream_t st) {
  using namespace qm;
  if (T <= 0) return FMOE_OK;
  if (nseg < 1 || nseg > kQmMaxSeg || (gated && nseg != 2))
    return set_error(FMOE_ERR_INVALID, "qgemm: %d weights", nseg);
  if (!aligned(x, 16)) return set_error(FMOE_ERR_ALIGN, "qgemm: x not 16-byte aligned");
  if (T > (1 << 30) / K) return set_error(FMOE_ERR_UNSUPPORTED, "qgemm: T=%lld too large", (long long)T);
  const int bits = o[0].w->bits;
  for (int s = 0; s < nseg; ++s) {
    if (!qgemm_supported(*o[s].w, 64, K) || o[s].w->bits != bits)
      return set_error(FMOE_ERR_UNSUPPORTED, "qgemm: weight %d (bits %d, in %d) is not a 4/8-bit group-64 weight of K %d",
                       s, o[s].w->bits, o[s].w->in, K);
    if (!o[s].out) return set_error(FMOE_ERR_INVALID, "qgemm: null output");
  }
  if (gated && o[0].w->out != o[1].w->out) return set_error(FMOE_ERR_INVALID, "qgemm: gate / up rows differ");
  Args a = {};
  a.nseg = nseg;
  a.K = K;
  a.G = K / 64;
  a.T = (int)T;
  a.status = status;
  // plain form: 128-row items, two CTAs per SM; gated form: gate + up halves, one
  const int BN = gated ? Cfg<2>::BN : Cfg<1>::BN;
  const int slots = gated ? kNumSMs : 2 * kNumSMs;
  // tiles of 64 tokens when 128-token tiles would leave CTA slots idle
  int nj = 0;
  for (int s = 0; s < nseg; ++s) nj += gated ? 0 : (o[s].w->out + BN - 1) / BN;
  if (gated) nj = (o[0].w->out + 127) / 128;
  a.tb = (T > 64 && (int64_t)nj * ((T + 127) / 128) < slots) ? 64 : 128;
  if (T <= 64) a.tb = 64;
  a.nt = (int)((T + a.tb - 1) / a.tb);
  int item = 0;
  for (int s = 0; s < nseg; ++s) {
    a.seg[s] = Seg{o[s].w->s, o[s].w->b, o[s].out, o[s].w->out, o[s].ld, item};
    if (!gated) item += ((o[s].w->out + BN - 1) / BN) * a.nt;
  }
  a.nitems = gated ? nj * a.nt : item;
  Maps m;
  int rc;
  {
    const cuuint64_t dX[2] = {(cuuint64_t)K, (cuuint64_t)T}, sX[1] = {(cuuint64_t)K * 2};
    const cuuint32_t b128[2] = {64, 128}, b64[2] = {64, 64};
    if ((rc = encode(&m.x[0], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, dX, sX, b128, CU_TENSOR_MAP_SWIZZLE_128B, "x")) ||
        (rc = encode(&m.x[1], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, dX, sX, b64, CU_TENSOR_MAP_SWIZZLE_128B, "x")))
      return rc;
    const cuuint64_t rowb = (cuuint64_t)K * bits / 8;
    for (int s = 0; s < nseg; ++s) {
      const cuuint64_t dW[2] = {rowb, (cuuint64_t)o[s].w->out}, sW[1] = {rowb};
      const cuuint32_t bW[2] = {128, 128};
      if ((rc = encode(&m.w[s], CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, o[s].w->w, dW, sW, bW, CU_TENSOR_MAP_SWIZZLE_128B,
                       "weight codes")))
        return rc;
    }
    for (int s = nseg; s < kQmMaxSeg; ++s) m.w[s] = m.w[0];
  }
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(qgemm_kernel<4, 0, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<1>::SMEM);
    cudaFuncSetAttribute(qgemm_kernel<4, 1, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<2>::SMEM);
    cudaFuncSetAttribute(qgemm_kernel<8, 0, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<1>::SMEM);
    cudaFuncSetAttribute(qgemm_kernel<8, 1, 2>, cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg<2>::SMEM);
  });
  const int grid = a.nitems < slots ? a.nitems : slots;
  const char* name = bits == 8 ? (gated ? "qgemm_kernel<8, gated>" : "qgemm_kernel<8>")
                               : (gated ? "qgemm_kernel<4, gated>" : "qgemm_kernel<4>");
  {
    ProfScope prof_(name, st);
    if (bits == 8) {
      if (gated)
        qgemm_kernel<8, 1, 2><<<grid, Cfg<2>::THREADS, Cfg<2>::SMEM, st>>>(m, a);
      else
        qgemm_kernel<8, 0, 1><<<grid, Cfg<1>::THREADS, Cfg<1>::SMEM, st>>>(m, a);
    } else {
      if (gated)
        qgemm_kernel<4, 1, 2><<<grid, Cfg<2>::THREADS, Cfg<2>::SMEM, st>>>(m, a);
      else
        qgemm_kernel<4, 0, 1><<<grid, Cfg<1>::THREADS, Cfg<1>::SMEM, st>>>(m, a);
    }
  }
  return check_launch(name);
}

}  // namespace fmoe
