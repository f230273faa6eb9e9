// Decode step of a Gemma-4 layer (T <= 8 sequences, one token each, every
// expert resident on this GPU) as six launches chained by programmatic
// dependent launch, DecoderLayer::forward_gemma4 (src/model/mod.rs:67-119):
//
//   1 qkv   q|k|v = input_norm(x) . [Wq Wk Wv]^T            per head: q/k/v norms, RoPE,
//           KV append (bf16 / TurboQuant / affine)          (gemma4_attention.rs:46-84)
//   2 attention over the cache (kv.cu, split-KV with in-kernel merge)
//   3 o     o = attn . Wo^T                                 last CTA: residual and the
//           feed-forward input norms (h, h1, h2, router input)
//   4 ffn1  router logits (bf16 / 4-bit) + dense gate|up    per gate|up pair: GELU gating;
//           last CTA: top-k routing, sorted unique experts  (moe.rs:325-380)
//   5 ffn2  dense down + routed experts' gate|up            per expert pair: GELU gating
//   6 ffn3  routed experts' down                            per 16-row tile: weighted combine
//           in ascending expert order (moe.rs:443-453); last CTA: output norms, residual,
//           layer scalar -> x
// and the tied lm_head with softcap and greedy argmax (mod.rs:336-362).
//
// Every GEMV streams through the per-warp cp.async rings of sgemv.cuh.  Work
// is dealt stream-K style: a family's S = units x groups-per-unit groups go to
// its warps in equal contiguous ranges, so a unit (a 16-row tile over all of K,
// or a gate|up tile pair) may be shared by consecutive warps.  Each writes its
// partial sums as a "piece"; the warp that brings the unit's piece count
// (a device counter) to its total sums the pieces in warp order and finishes
// the unit.  Finished units feed group epilogues (a head, a tile across
// experts) through a second counter, and launch epilogues through a grid
// counter whose last CTA runs the row-wide work.  Sums run in a fixed order,
// so results are deterministic; every counter is reset by its consumer, so
// the workspace is ready for the next call or CUDA-graph replay.
//
// A launch's weights never depend on its predecessor, so each warp issues its
// first ring steps before griddepcontrol.wait (the routed experts' gate|up
// weights are the exception: their ids come from the previous launch).
#include <algorithm>
#include <cmath>
#include <mutex>
#include <utility>
#include <vector>

#include "internal.h"
#include "common.cuh"
#include "stage.cuh"
#include "rowops.cuh"
#include "kvrow.cuh"
#include "sgemv.cuh"

namespace fmoe {
namespace dl {

constexpr int NW = 12;  // warps per CTA
constexpr int NTHR = NW * 32;
constexpr int kMaxT = 8;
constexpr int kMaxHidden = 4096;      // hidden rows staged in shared memory by the row epilogues (<= 16 B each in the rings)
constexpr int kMaxSlotsPerCta = 3;    // expert inputs one ffn3 CTA may need
constexpr int kMaxUnique = 64;        // unique experts of one call (T * k <= 64)
constexpr int kRingSlot = 6144;       // bytes of one warp's ring
constexpr int kRingBytes = NW * kRingSlot;
constexpr int kMaxPend = 8;           // groups one warp may complete in one launch
static_assert(16 * kMaxHidden <= kRingBytes, "row epilogues stage 16 bytes per hidden element in the rings");

// ---------------------------------------------------------------------------
// Work families

enum { SRC_MAT = 0, SRC_EXPERT = 1 };

struct Fam {
  int bits, nt;        // code width; row tiles per unit (2: gate tile + up tile)
  int K, G;            // inputs and 64-wide groups
  int us;              // ring steps per unit (G / groups per step)
  int w0, nw;          // global warps [w0, w0 + nw)
  int tiles;           // units per matrix (per expert slot for SRC_EXPERT)
  int64_t rowbytes;
  int src;
  // SRC_MAT: segments stacked by rows, seg_tile0 in units; nt == 2: seg 0 gate, seg 1 up
  int nseg;
  int seg_tile0[5];
  const uint8_t* w[4];
  const bf16* s[4];
  const bf16* b[4];
  int mat;              // SRC_EXPERT: tensor index of the codes (0: gate|up, 6: down)
  float* piece;         // [units][maxp][nt][T][16]
  int maxp;
  unsigned* uctr;       // per-unit piece counters
  float* fin;           // finished units [units][nt][T][16] (families whose results are read later)
  unsigned* gctr;       // group counters
  int frag_off, xsum_off;  // shared-memory offsets of the input fragments
};

// Work split of a family over its nw warps, counted in ring steps (us per
// unit).  U > nw units: every warp takes whole units (never split).  U <= nw:
// unit u is cut into k or k + 1 contiguous slices (the first `extra` units
// k + 1), one per warp, so a unit has a fixed, known number of pieces; warps
// past U * us slices (when nw / U > us) stay idle.
struct Split {
  int U, nw, us, k, extra;
};
__host__ __device__ inline Split make_split(int U, int nw, int us) {
  Split p{U, nw, us, 0, 0};
  if (U > 0 && U <= nw) {
    p.k = nw / U;
    if (p.k >= us) {
      p.k = us;
    } else {
      p.extra = nw % U;
    }
  }
  return p;
}
__host__ __device__ inline void split_range(const Split& p, int lw, int* lo, int* hi) {
  *lo = *hi = 0;
  if (lw < 0 || lw >= p.nw || p.U <= 0) return;
  if (p.k == 0) {
    *lo = (int)((int64_t)p.U * lw / p.nw) * p.us;
    *hi = (int)((int64_t)p.U * (lw + 1) / p.nw) * p.us;
    return;
  }
  const int big = p.extra * (p.k + 1);
  int u, q, ku;
  if (lw < big) {
    u = lw / (p.k + 1);
    q = lw - u * (p.k + 1);
    ku = p.k + 1;
  } else {
    const int l2 = lw - big;
    u = p.extra + l2 / p.k;
    q = l2 - (u - p.extra) * p.k;
    ku = p.k;
    if (u >= p.U) return;  // idle
  }
  *lo = u * p.us + p.us * q / ku;
  *hi = u * p.us + p.us * (q + 1) / ku;
}
__device__ __forceinline__ int2 srange(const Split& p, int lw) {
  int lo, hi;
  split_range(p, lw, &lo, &hi);
  return make_int2(lo, hi);
}
// Pieces of unit u and the family-local warp holding its first slice.
__host__ __device__ inline int split_pieces(const Split& p, int u) {
  return p.k == 0 ? 1 : (u < p.extra ? p.k + 1 : p.k);
}
__host__ __device__ inline int split_first(const Split& p, int u) {
  return p.k == 0 ? 0 : (u < p.extra ? u * (p.k + 1) : p.extra * (p.k + 1) + (u - p.extra) * p.k);
}
// Largest piece count of any unit for U in [U_min, ...).
__host__ __device__ inline int split_maxp(int U_min, int nw, int us) {
  const Split p = make_split(U_min, nw, us);
  return p.k == 0 ? 1 : p.k + 1;
}

template <int NT>
struct Acc {
  float v[NT][4];
};
struct FragPtr {
  const uint4* frag;
  const float* xsum;
};

template <int NT>
struct UnitPtr {
  const uint8_t* w[NT];
  const bf16* s[NT];
  const bf16* b[NT];
};

template <int NT>
__device__ __forceinline__ UnitPtr<NT> mat_unit(const Fam& f, int u) {
  UnitPtr<NT> p;
  if (NT == 2) {
    const int64_t r0 = (int64_t)u * 16;
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      p.w[i] = f.w[i] + r0 * f.rowbytes;
      p.s[i] = f.s[i] + r0 * f.G;
      p.b[i] = f.b[i] + r0 * f.G;
    }
  } else {
    int sg = 0;
#pragma unroll
    for (int i = 1; i < 4; ++i)
      if (i < f.nseg && u >= f.seg_tile0[i]) sg = i;
    const int64_t r0 = (int64_t)(u - f.seg_tile0[sg]) * 16;
    p.w[0] = f.w[sg] + r0 * f.rowbytes;
    p.s[0] = f.s[sg] + r0 * f.G;
    p.b[0] = f.b[sg] + r0 * f.G;
  }
  return p;
}

template <int NT>
__device__ __forceinline__ UnitPtr<NT> expert_unit(const Fam& f, const ExpertsDev& ex, const int32_t* uniq, int u) {
  UnitPtr<NT> p;
  const int slot = u / f.tiles, j = u - slot * f.tiles;
  const uint8_t* eb = expert_base(ex, uniq[slot]);
  const int64_t r0 = (int64_t)j * 16;
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    const int m = f.mat + 3 * i;
    p.w[i] = eb + ex.off[m] + r0 * f.rowbytes;
    p.s[i] = reinterpret_cast<const bf16*>(eb + ex.off[m + 1]) + r0 * f.G;
    p.b[i] = reinterpret_cast<const bf16*>(eb + ex.off[m + 2]) + r0 * f.G;
  }
  return p;
}

// ---------------------------------------------------------------------------
// Per-warp streaming engine over one contiguous group range of a family.

template <int BITS, int NT, int NG, int D>
struct Engine {
  using Gm = sg::Geo<BITS>;
  static constexpr int GS = sg::stage_bytes<BITS, NT>();  // one group's copies
  static constexpr int SB = NG * GS;                      // stage bytes
  static_assert(D * SB <= kRingSlot, "ring slot");
  uint32_t ring;
  const uint8_t* ringp;
  int lane, g, t, G, us;
  int64_t rowbytes;
  int s0, s1;
  int ipos, iu, ig;               // issue cursor (ig: step within the unit)
  const uint8_t* rp[2 * NT];      // rows g / g+8 of the issue unit's tiles (group 0)
  const bf16* sp[NT];             // this lane's scale or bias word of the issue unit (group 0)
  uint32_t sreg[D][NT][NG];

  __device__ __forceinline__ void init(uint8_t* r, int ln, const Fam& f, int a, int b_) {
    ringp = r;
    ring = sg::s_addr(r);
    lane = ln;
    g = ln >> 2;
    t = ln & 3;
    G = f.G;
    us = f.us;
    rowbytes = f.rowbytes;
    s0 = a;
    s1 = b_;
  }
  __device__ __forceinline__ void set_unit(const UnitPtr<NT>& p) {
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      rp[2 * i] = p.w[i] + (int64_t)g * rowbytes;
      rp[2 * i + 1] = rp[2 * i] + 8 * rowbytes;
      // quad-cooperative scales: lane t holds s / b (t & 1) of row g + 8 (t >> 1)
      sp[i] = ((t & 1) ? p.b[i] : p.s[i]) + (g + 8 * (t >> 1)) * G;
    }
  }

  template <class Addr>
  __device__ __forceinline__ void issue(int j, Addr& addr) {
#pragma unroll
    for (int k = 0; k < NG; ++k) {
      const int gi = ig * NG + k;
      const uint8_t* src[2 * NT];
#pragma unroll
      for (int h = 0; h < 2 * NT; ++h) src[h] = rp[h] + gi * Gm::GB;
      sg::issue_step<BITS, NT>(ring + j * SB + k * GS, src, lane, t);
      if constexpr (BITS != 16) {
#pragma unroll
        for (int i = 0; i < NT; ++i) sreg[j][i][k] = sg::ldg_h(sp[i] + gi);
      }
    }
    ++ipos;
    if (++ig == us) {
      ig = 0;
      ++iu;
      if (ipos < s1) set_unit(addr(iu));
    }
  }

  template <class Addr>
  __device__ __forceinline__ void prime(Addr& addr) {
    ipos = s0;
    iu = s0 / us;
    ig = s0 - iu * us;
    if (ipos < s1) set_unit(addr(iu));
#pragma unroll
    for (int j = 0; j < D; ++j) {
      if (ipos < s1) issue(j, addr);
      sg::commit();
    }
  }

  // fr(u) -> FragPtr: the input fragments of unit u; done(u, Acc, piece_begin, piece_end).
  template <class Addr, class Frag, class Done>
  __device__ __forceinline__ void run(Addr& addr, Frag& fr, Done& done, int T) {
    int cpos = s0, cu = s0 / us;
    int cs = s0 - cu * us;
    int pst = s0;
    Acc<NT> y;
#pragma unroll
    for (int i = 0; i < NT; ++i) y.v[i][0] = y.v[i][1] = y.v[i][2] = y.v[i][3] = 0.f;
    FragPtr fp = {nullptr, nullptr};
    if (s0 < s1) fp = fr(cu);
    const int qb = lane & ~3;
    const bool live_col = g < T;
    const int gcol = live_col ? g : 0;
    while (cpos < s1) {
#pragma unroll
      for (int j = 0; j < D; ++j) {
        if (cpos < s1) {
          sg::wait_group<D - 1>();
          if constexpr (BITS == 6) __syncwarp();  // the quad's shared row slots
          const uint8_t* st = ringp + j * SB;
          float cc[NG][NT][4];
          float2 xv[NG];
          // all of the step's MMA chains first (independent), then the fixups
#pragma unroll
          for (int k = 0; k < NG; ++k) {
            const int gg = cs * NG + k;
            const uint4* p = fp.frag + ((gg * T + gcol) * 4 + t) * 2;
            const uint4 f0 = p[0], f1 = p[1];
            const uint32_t b[8] = {live_col ? f0.x : 0u, live_col ? f0.y : 0u, live_col ? f0.z : 0u,
                                   live_col ? f0.w : 0u, live_col ? f1.x : 0u, live_col ? f1.y : 0u,
                                   live_col ? f1.z : 0u, live_col ? f1.w : 0u};
            xv[k] = *reinterpret_cast<const float2*>(fp.xsum + gg * 8 + 2 * t);
#pragma unroll
            for (int i = 0; i < NT; ++i) {
              cc[k][i][0] = cc[k][i][1] = cc[k][i][2] = cc[k][i][3] = 0.f;
              sg::mma_group<BITS>(cc[k][i], st + k * GS, i, lane, t, b);
            }
          }
#pragma unroll
          for (int k = 0; k < NG; ++k)
#pragma unroll
            for (int i = 0; i < NT; ++i) {
              if constexpr (BITS == 16) {
                y.v[i][0] += cc[k][i][0], y.v[i][1] += cc[k][i][1], y.v[i][2] += cc[k][i][2], y.v[i][3] += cc[k][i][3];
              } else {
                const uint32_t v = sreg[j][i][k];
                const uint32_t sl = __shfl_sync(0xffffffffu, v, qb), bl = __shfl_sync(0xffffffffu, v, qb | 1);
                const uint32_t sh = __shfl_sync(0xffffffffu, v, qb | 2), bh = __shfl_sync(0xffffffffu, v, qb | 3);
                sg::fixup<BITS>(y.v[i], cc[k][i], xv[k].x, xv[k].y, sl, bl, sh, bh);
              }
            }
          ++cpos;
          if (++cs == us || cpos == s1) {
            done(cu, y, pst, cpos);
#pragma unroll
            for (int i = 0; i < NT; ++i) y.v[i][0] = y.v[i][1] = y.v[i][2] = y.v[i][3] = 0.f;
            pst = cpos;
          }
          if (cs == us) {
            cs = 0;
            ++cu;
            if (cpos < s1) fp = fr(cu);
          }
          if constexpr (BITS == 6) __syncwarp();  // the slots are read before they are refilled
          if (ipos < s1) issue(j, addr);
        }
        sg::commit();
      }
    }
    sg::wait_group<0>();
  }
};

// ---------------------------------------------------------------------------
// Pieces, unit completion, counters

// Count this warp's published writes toward counter `c`: lane 0 adds with
// acquire-release semantics after a __syncwarp (which orders the other lanes'
// writes before it), so the warp that brings the count to `target` sees every
// earlier warp's writes; it resets the counter and owns the next step.
__device__ __forceinline__ unsigned atom_add_acqrel(unsigned* c, unsigned v) {
  unsigned prev;
  asm volatile("atom.acq_rel.gpu.global.add.u32 %0, [%1], %2;\n" : "=r"(prev) : "l"(c), "r"(v) : "memory");
  return prev;
}
__device__ __forceinline__ bool arrive(unsigned* c, int target, int lane) {
  __syncwarp();
  unsigned last = 0;
  if (lane == 0) {
    last = atom_add_acqrel(c, 1u) == (unsigned)target - 1u;
    if (last) *c = 0u;
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  __syncwarp();
  return last != 0;
}

// CTA-level: true in the last CTA of the grid to get here (counter reset).
__device__ __forceinline__ bool grid_last(unsigned* ctr, int* flag) {
  __syncthreads();
  if (threadIdx.x == 0) {
    asm volatile("fence.acq_rel.gpu;\n" ::: "memory");
    *flag = atom_add_acqrel(ctr, 1u) == gridDim.x - 1;
    if (*flag) *ctr = 0u;
  }
  __syncthreads();
  return *flag != 0;
}

// The lane's fragment values (rows g / g+8, tokens 2t / 2t+1) stored to a
// [NT][T][16] block.
template <int NT>
__device__ __forceinline__ void store_block(float* base, int T, const Acc<NT>& y, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    float* pi = base + i * T * 16;
    if (2 * t < T) {
      pi[(2 * t) * 16 + g] = y.v[i][0];
      pi[(2 * t) * 16 + g + 8] = y.v[i][2];
    }
    if (2 * t + 1 < T) {
      pi[(2 * t + 1) * 16 + g] = y.v[i][1];
      pi[(2 * t + 1) * 16 + g + 8] = y.v[i][3];
    }
  }
}
// Sum of np blocks (stride `stride` floats) in the lane's fragment layout; all
// loads issued before the sums.
template <int NT>
__device__ __forceinline__ void sum_blocks(const float* base, int64_t stride, int np, int T, Acc<NT>& y, int lane) {
  const int g = lane >> 2, t = lane & 3;
  const int t0 = min(2 * t, T - 1), t1 = min(2 * t + 1, T - 1);
#pragma unroll
  for (int i = 0; i < NT; ++i) y.v[i][0] = y.v[i][1] = y.v[i][2] = y.v[i][3] = 0.f;
  for (int p0 = 0; p0 < np; p0 += 4) {
    float v[4][NT][4];
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        const float* pb = base + (p0 + q) * stride + i * T * 16;
        const bool ok = p0 + q < np;
        v[q][i][0] = ok ? __ldcg(pb + t0 * 16 + g) : 0.f;
        v[q][i][1] = ok ? __ldcg(pb + t1 * 16 + g) : 0.f;
        v[q][i][2] = ok ? __ldcg(pb + t0 * 16 + g + 8) : 0.f;
        v[q][i][3] = ok ? __ldcg(pb + t1 * 16 + g + 8) : 0.f;
      }
#pragma unroll
    for (int q = 0; q < 4; ++q)
#pragma unroll
      for (int i = 0; i < NT; ++i)
#pragma unroll
        for (int e = 0; e < 4; ++e) y.v[i][e] += v[q][i][e];
  }
}

// A warp's piece of unit u is done but the warp did not cover the whole unit:
// publish the piece; ok = 1 (with the unit's full sums in y) for the warp whose
// piece completed the unit.  Out of line: the ring's unrolled steps keep only
// a call.
template <int NT>
struct Fin {
  Acc<NT> y;
  int ok;
};
template <int NT>
__device__ __noinline__ Fin<NT> finish_piece(const Fam& f, const Split sp, int T, int lw, int u, Acc<NT> y,
                                             int lane, int slot) {
  const int64_t stride = (int64_t)NT * T * 16;
  float* base = f.piece + (int64_t)slot * f.maxp * stride;
  store_block<NT>(base + (lw - split_first(sp, u)) * stride, T, y, lane);
  const int np = split_pieces(sp, u);
  Fin<NT> r;
  r.ok = arrive(f.uctr + slot, np, lane) ? 1 : 0;
  if (r.ok) sum_blocks<NT>(base, stride, np, T, r.y, lane);
  return r;
}
// True when unit u's sums are complete in y (the whole unit was this warp's,
// or this warp's piece completed it).
#define DL_UNIT_DONE(NT, f, S, T, lw, u, y, pst, pe, lane, slot)                           \
  ((pst) == (u) * (f).us && (pe) == ((u) + 1) * (f).us                                         \
       ? true                                                                                 \
       : [&] {                                                                                \
           const Fin<NT> r_ = finish_piece<NT>((f), (S), (T), (lw), (u), (y), (lane), (slot));  \
           if (r_.ok) (y) = r_.y;                                                            \
           return r_.ok != 0;                                                                \
         }())

// ---------------------------------------------------------------------------
// Input fragments (prologue)

// Per-token 1 / rms of x rows (warp per token), into rms[tk]; every load of
// the row is issued before the first use.
__device__ __forceinline__ void row_rms(const bf16* x, int64_t ldx, int K, int T, float eps, float* rms) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int NL = (kMaxHidden + 255) / 256;
  for (int tk = warp; tk < T; tk += NW) {
    const bf16* xr = x + tk * ldx;
    uint4 w[NL];
#pragma unroll
    for (int q = 0; q < NL; ++q) {
      const int i = lane * 8 + q * 256;
      w[q] = i < K ? __ldcg(reinterpret_cast<const uint4*>(xr + i)) : make_uint4(0, 0, 0, 0);
    }
    float ss = 0.f;
#pragma unroll
    for (int q = 0; q < NL; ++q) {
      const uint32_t ww[4] = {w[q].x, w[q].y, w[q].z, w[q].w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float lo = bf16lo(ww[e]), hi = bf16hi(ww[e]);
        ss = fmaf(lo, lo, fmaf(hi, hi, ss));
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (lane == 0) rms[tk] = rsqrtf(ss / (float)K + eps);
  }
}

// frag [G][T][4][2 uint4] and xsum [G][8] of x rows (bf16, ldx apart) for BITS;
// rms != nullptr: x -> bf16(x * rms[tk] * nw) first (nw may be null).
template <int BITS>
__device__ void build_frags(uint8_t* smem, int frag_off, int xsum_off, int G, int T, const bf16* x, int64_t ldx,
                            const float* rms, const bf16* nw) {
  uint4* frag = reinterpret_cast<uint4*>(smem + frag_off);
  float* xsum = reinterpret_cast<float*>(smem + xsum_off);
  const int items = G * T * 4;
  for (int i0 = 0; i0 < items; i0 += NTHR) {
    const int it = i0 + threadIdx.x;
    const bool live = it < items;
    const int tq = it & 3, tk = live ? (it >> 2) % T : 0, gl = live ? (it >> 2) / T : 0;
    float v[16];
    if (live) {
      const int c0 = gl * 64 + 16 * tq;
      const bf16* xr = x + tk * ldx + c0;
      const uint4 a = __ldcg(reinterpret_cast<const uint4*>(xr)), bq = __ldcg(reinterpret_cast<const uint4*>(xr + 8));
      const uint32_t ww[8] = {a.x, a.y, a.z, a.w, bq.x, bq.y, bq.z, bq.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[2 * e] = bf16lo(ww[e]);
        v[2 * e + 1] = bf16hi(ww[e]);
      }
      if (rms) {
        const float r = rms[tk];
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = round_bf(nw ? v[e] * r * bf2f(nw[c0 + e]) : v[e] * r);
      }
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) v[e] = 0.f;
    }
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      v[e] = sg::operand_round<BITS>(v[e]);
      s += v[e];
    }
    uint32_t b[8];
    sg::make_frag<BITS>(v, b);
    if (live) {
      uint4* dst = frag + ((gl * T + tk) * 4 + tq) * 2;
      dst[0] = make_uint4(b[0], b[1], b[2], b[3]);
      dst[1] = make_uint4(b[4], b[5], b[6], b[7]);
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (live && tq == 0) xsum[gl * 8 + tk] = s;
  }
  for (int i = threadIdx.x; i < G * 8; i += NTHR)
    if ((i & 7) >= T) xsum[i] = 0.f;
}

__host__ __device__ inline int frag_bytes(int G, int T) { return G * T * 128; }

// ---------------------------------------------------------------------------
// CTA-wide helpers for the row epilogues

__device__ __forceinline__ float cta_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) s += red[w];
  return s;
}

// Finished value of row r, token tk, of a plain (nt = 1) family.
__device__ __forceinline__ float fin_at(const Fam& f, int T, int tk, int r) {
  return __ldcg(f.fin + (int64_t)(r >> 4) * T * 16 + tk * 16 + (r & 15));
}

// Rows [0, H) of token tk of a finished plain family into dst (shared memory),
// loads issued in batches before use.
__device__ __forceinline__ void fin_row(const Fam& f, int T, int tk, int H, float* dst) {
  for (int i0 = 0; i0 < H; i0 += 4 * NTHR) {
    float v[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int i = i0 + q * NTHR + threadIdx.x;
      v[q] = i < H ? fin_at(f, T, tk, i) : 0.f;
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const int i = i0 + q * NTHR + threadIdx.x;
      if (i < H) dst[i] = v[q];
    }
  }
}

// ---------------------------------------------------------------------------
// 1. q | k | v projections with the per-head epilogue

struct QkvArgs {
  Fam f;
  const bf16* x;
  const bf16* in_norm;
  float eps;
  int T, H;
  KvDev kv;
  int Hq, Hkv, D, k_eq_v;
  const bf16* q_norm;
  const bf16* k_norm;
  int rope_dims;
  float l2theta;
  int64_t pos;
  const int64_t* pos_dev;
  int turbo;
  float inv_sqrt_d;
  bf16* q_out;
};

// Head groups: q heads [0, Hq), then kv heads (their k tiles and v tiles).
__device__ __forceinline__ int qkv_group_of(const QkvArgs& a, int u) {
  const int h = u / (a.D / 16);
  return h < a.Hq + a.Hkv ? h : h - a.Hkv;
}
__device__ __forceinline__ int qkv_group_units(const QkvArgs& a, int grp) {
  return (grp < a.Hq || a.k_eq_v) ? a.D / 16 : a.D / 8;
}

// A finished q|k|v tile: store it and count it toward its head group; the
// group when this tile completed it, else -1.
__device__ __noinline__ int qkv_unit_finished(const QkvArgs& a, int u, const Acc<1> y, int lane) {
  store_block<1>(a.f.fin + (int64_t)u * a.T * 16, a.T, y, lane);
  const int grp = qkv_group_of(a, u);
  return arrive(a.f.gctr + grp, qkv_group_units(a, grp), lane) ? grp : -1;
}

// Warp epilogue of one head group (P = D / 32 values per lane).
template <int P>
__device__ __noinline__ void qkv_epilogue(const QkvArgs& a, int grp, int lane) {
  constexpr int D = 32 * P, G = D / 64;
  const int tpd = D / 16;
  const int64_t p0 = a.pos_dev ? __ldcg(a.pos_dev) : a.pos;
  const float fpos = (float)p0;
  const int e0 = lane * P;
  auto load = [&](int head_tile0, int tk, float (&v)[P]) {
    const float* src = a.f.fin + (int64_t)(head_tile0 + e0 / 16) * a.T * 16 + tk * 16 + e0 % 16;
#pragma unroll
    for (int e = 0; e < P; e += 4) {
      const float4 q = __ldcg(reinterpret_cast<const float4*>(src + e));
      v[e] = round_bf(q.x), v[e + 1] = round_bf(q.y), v[e + 2] = round_bf(q.z), v[e + 3] = round_bf(q.w);
    }
  };
  for (int tk = 0; tk < a.T; ++tk) {
    if (grp < a.Hq) {
      float v[P];
      load(grp * tpd, tk, v);
      warp_rms_norm<P>(v, a.q_norm, a.eps, lane);
      warp_rope<P>(v, a.rope_dims, a.l2theta, fpos, lane);
      store_row_bf16<P>(a.q_out + ((int64_t)tk * a.Hq + grp) * D, lane, v);
      continue;
    }
    const int hk = grp - a.Hq;
    float kv[P], vv[P];
    load((a.Hq + hk) * tpd, tk, kv);
    if (a.k_eq_v) {
#pragma unroll
      for (int i = 0; i < P; ++i) vv[i] = kv[i];
    } else {
      load((a.Hq + a.Hkv + hk) * tpd, tk, vv);
    }
    warp_rms_norm<P>(vv, nullptr, a.eps, lane);  // v_norm: no learned scale
    warp_rms_norm<P>(kv, a.k_norm, a.eps, lane);
    warp_rope<P>(kv, a.rope_dims, a.l2theta, fpos, lane);
    const KvDev& c = a.kv;
    const int64_t dst = ((int64_t)tk * a.Hkv + hk) * c.cap + p0 % c.cap;
    if (c.mode == FMOE_KV_BF16) {
      if (a.turbo) {
        warp_turbo<P>(kv, lane, a.turbo);
        warp_turbo<P>(vv, lane, a.turbo);
      }
      store_row_bf16<P>(reinterpret_cast<bf16*>(c.k) + dst * D, lane, kv);
      store_row_bf16<P>(reinterpret_cast<bf16*>(c.v) + dst * D, lane, vv);
    } else {
      warp_fwht<P>(kv, lane);
      warp_fwht<P>(vv, lane);
#pragma unroll
      for (int i = 0; i < P; ++i) {
        kv[i] *= a.inv_sqrt_d;
        vv[i] *= a.inv_sqrt_d;
      }
      warp_quant_store<P, 4>(kv, lane, reinterpret_cast<uint32_t*>(c.k) + dst * (D / 8), c.ks + dst * G,
                             c.kb + dst * G);
      warp_quant_store<P, 8>(vv, lane, reinterpret_cast<uint32_t*>(c.v) + dst * (D / 4), c.vs + dst * G,
                             c.vb + dst * G);
    }
  }
}

template <int BITS, int D_>
__global__ void __launch_bounds__(NTHR, 1) qkv_kernel(const __grid_constant__ QkvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float rms[kMaxT];
  __shared__ int pend[NW][kMaxPend];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * NW + warp;
  const Fam& f = a.f;
  const Split S = make_split(f.tiles, f.nw, f.us);
  const int lw = gw - f.w0;
  Engine<BITS, 1, 2, D_> en;
  const int2 rg = srange(S, lw);
  en.init(smem + warp * kRingSlot, lane, f, rg.x, rg.y);
  auto addr = [&](int u) { return mat_unit<1>(f, u); };
  en.prime(addr);
  griddep_wait();
  griddep_launch_dependents();
  row_rms(a.x, a.H, a.H, a.T, a.eps, rms);
  __syncthreads();
  build_frags<BITS>(smem, f.frag_off, f.xsum_off, f.G, a.T, a.x, a.H, rms, a.in_norm);
  __syncthreads();
  auto fr = [&](int) {
    return FragPtr{reinterpret_cast<const uint4*>(smem + f.frag_off), reinterpret_cast<const float*>(smem + f.xsum_off)};
  };
  int npend = 0;
  auto done = [&](int u, Acc<1> y, int pst, int pe) {
    if (!DL_UNIT_DONE(1, f, S, a.T, lw, u, y, pst, pe, lane, u)) return;
    const int grp = qkv_unit_finished(a, u, y, lane);
    if (grp >= 0) {
      if (lane == 0 && npend < kMaxPend) pend[warp][npend] = grp;
      ++npend;
    }
  };
  en.run(addr, fr, done, a.T);
  __syncwarp();
  // head epilogues after the stream (no out-of-line call inside the ring)
  for (int i = 0; i < npend && i < kMaxPend; ++i) {
    if (a.D == 256) qkv_epilogue<8>(a, pend[warp][i], lane);
    else qkv_epilogue<16>(a, pend[warp][i], lane);
  }
}

// ---------------------------------------------------------------------------
// 3. o projection; the last CTA applies the feed-forward input norms

struct OArgs {
  Fam f;
  const bf16* attn;  // [T][QD]
  int T, H, QD;
  const bf16* x;     // residual input of the layer
  const bf16* w_post_attn;
  const bf16* w_pre_ff;
  const bf16* w_pre_ff2;
  const bf16* rscale;
  float eps, root;
  bf16 *h, *h1, *h2, *xs;
  unsigned* grid_ctr;
};

// h = bf16(x + bf16(rms(bf16(o)) * w_post_attn)); h1 / h2 = bf16(rms(h) * w);
// xs = bf16(bf16(bf16(rms(h2)) * bf16(root)) * router_scale)   (mod.rs:84-104, moe.rs:325-329)
// Every input of a token is first loaded into shared memory (`rows`: the
// CTA's rings, idle by now) in one batch of independent loads, then the
// norms run from there: one memory round trip per token, not one per pass.
__device__ __noinline__ void ff_in_rows(const OArgs& a, float* red, uint8_t* rows) {
  const int H = a.H;
  float* ro = reinterpret_cast<float*>(rows);  // o, then h2
  float* rh = ro + H;                          // x, then h
  bf16* wv = reinterpret_cast<bf16*>(rh + H);  // [4][H]: post_attn, pre_ff, pre_ff_2, router_scale
  const bf16* srcw[4] = {a.w_post_attn, a.w_pre_ff, a.w_pre_ff2, a.rscale};
  for (int tk = 0; tk < a.T; ++tk) {
#pragma unroll
    for (int k = 0; k < (kMaxHidden + NTHR - 1) / NTHR; ++k) {
      const int i = threadIdx.x + k * NTHR;
      if (i < H) {
        const float o = fin_at(a.f, a.T, tk, i);
        const float x = __bfloat162float(__ldcg(a.x + (int64_t)tk * H + i));
        bf16 w4[4];
        if (tk == 0) {
#pragma unroll
          for (int q = 0; q < 4; ++q) w4[q] = srcw[q] ? srcw[q][i] : __float2bfloat16_rn(1.0f);
        }
        ro[i] = o;
        rh[i] = x;
        if (tk == 0) {
#pragma unroll
          for (int q = 0; q < 4; ++q) wv[q * H + i] = w4[q];
        }
      }
    }
    __syncthreads();
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += NTHR) {
      const float o = round_bf(ro[i]);
      ro[i] = o;
      ss = fmaf(o, o, ss);
    }
    const float r1 = rsqrtf(cta_sum(ss, red) / (float)H + a.eps);
    ss = 0.f;
    for (int i = threadIdx.x; i < H; i += NTHR) {
      const float h = round_bf(rh[i] + round_bf(ro[i] * r1 * bf2f(wv[i])));
      rh[i] = h;
      ss = fmaf(h, h, ss);
    }
    const float r2 = rsqrtf(cta_sum(ss, red) / (float)H + a.eps);
    ss = 0.f;
    for (int i = threadIdx.x; i < H; i += NTHR) {
      const float h = rh[i];
      const int64_t o = (int64_t)tk * H + i;
      a.h[o] = __float2bfloat16_rn(h);
      a.h1[o] = __float2bfloat16_rn(h * r2 * bf2f(wv[H + i]));
      const float h2 = round_bf(h * r2 * bf2f(wv[2 * H + i]));
      a.h2[o] = __float2bfloat16_rn(h2);
      ro[i] = h2;
      ss = fmaf(h2, h2, ss);
    }
    const float r3 = rsqrtf(cta_sum(ss, red) / (float)H + a.eps);
    const float rb = round_bf(a.root);
    for (int i = threadIdx.x; i < H; i += NTHR) {
      float v = round_bf(round_bf(ro[i] * r3) * rb);
      if (a.rscale) v = round_bf(v * bf2f(wv[3 * H + i]));
      a.xs[(int64_t)tk * H + i] = __float2bfloat16_rn(v);
    }
    __syncthreads();  // rows reused by the next token
  }
}

template <int BITS, int D_>
__global__ void __launch_bounds__(NTHR, 1) o_kernel(const __grid_constant__ OArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float red[NW];
  __shared__ int flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * NW + warp;
  const Fam& f = a.f;
  const Split S = make_split(f.tiles, f.nw, f.us);
  const int lw = gw - f.w0;
  Engine<BITS, 1, 2, D_> en;
  const int2 rg = srange(S, lw);
  en.init(smem + warp * kRingSlot, lane, f, rg.x, rg.y);
  auto addr = [&](int u) { return mat_unit<1>(f, u); };
  en.prime(addr);
  griddep_wait();
  griddep_launch_dependents();
  build_frags<BITS>(smem, f.frag_off, f.xsum_off, f.G, a.T, a.attn, a.QD, nullptr, nullptr);
  __syncthreads();
  auto fr = [&](int) {
    return FragPtr{reinterpret_cast<const uint4*>(smem + f.frag_off), reinterpret_cast<const float*>(smem + f.xsum_off)};
  };
  auto done = [&](int u, Acc<1> y, int pst, int pe) {
    if (DL_UNIT_DONE(1, f, S, a.T, lw, u, y, pst, pe, lane, u)) store_block<1>(f.fin + (int64_t)u * a.T * 16, a.T, y, lane);
  };
  en.run(addr, fr, done, a.T);
  if (grid_last(a.grid_ctr, &flag)) ff_in_rows(a, red, smem);
}

// ---------------------------------------------------------------------------
// GELU gating of a finished gate|up tile pair: act[tk][16 u + r], the lane's
// rows g / g+8 and tokens 2t / 2t+1 (moe.rs:437, mlp.rs:37).
__device__ __noinline__ void glu_store(const Acc<2> y, int T, int u, bf16* act, int64_t ld, int lane) {
  const int g = lane >> 2, t = lane & 3;
#pragma unroll
  for (int h = 0; h < 2; ++h)
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const int tk = 2 * t + c;
      if (tk < T) {
        const float gv = round_bf(y.v[0][2 * h + c]), uv = round_bf(y.v[1][2 * h + c]);
        act[tk * ld + 16 * u + g + 8 * h] = __float2bfloat16_rn(gelu_tanh(gv) * uv);
      }
    }
}

// ---------------------------------------------------------------------------
// 4. router logits + dense gate|up; last CTA: routing

struct Ffn1Args {
  Fam fr;             // router (bits 16 or 4), input xs
  Fam fg;             // dense gate|up pairs (4-bit), input h1
  const bf16* xs;
  const bf16* h1;
  int T, H, E, k, Id;
  const float* logit_bias;
  const bf16* pes;
  bf16* act_d;        // [T][Id]
  int32_t* ids;       // [T][k] descending logit
  float* wts;
  int32_t* uniq;      // [kMaxUnique] ascending
  int32_t* nuniq;
  int32_t* slot;      // [T][k] index of ids[t][j] in uniq
  unsigned* grid_ctr;
};

// Routing: logits rounded to bf16 (the router's output dtype in the
// reference), top-k by value with ties to the lower id, weights = softmax
// over the selected logits times per_expert_scale; then the sorted unique
// experts and each pair's slot among them.
__device__ __noinline__ void route_rows(const Ffn1Args& a, int* used) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int E = a.E, k = a.k;
  for (int tk = warp; tk < a.T; tk += NW) {
    float lv[8];  // E <= 256
    int li[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int e = lane + 32 * q;
      li[q] = e;
      lv[q] = e < E ? fin_at(a.fr, a.T, tk, e) : 0.f;
    }
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int e = lane + 32 * q;
      if (e < E) {
        float v = lv[q];
        if (a.logit_bias) v += a.logit_bias[e];
        lv[q] = round_bf(v);
      } else {
        lv[q] = -INFINITY;
        li[q] = 0x7fffffff;
      }
    }
    float sel[8];
    int sid[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (j >= k) break;
      float bv = -INFINITY;
      int bi = 0x7fffffff;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (li[q] != 0x7fffffff && (lv[q] > bv || (lv[q] == bv && li[q] < bi))) {
          bv = lv[q];
          bi = li[q];
        }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (ov > bv || (ov == bv && oi < bi)) {
          bv = ov;
          bi = oi;
        }
      }
      sel[j] = bv;
      sid[j] = bi;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (li[q] == bi) li[q] = 0x7fffffff;  // taken
    }
    if (lane == 0) {
      const float mx = sel[0];
      float den = 0.f;
      for (int j = 0; j < k; ++j) den += expf(sel[j] - mx);
      for (int j = 0; j < k; ++j) {
        float w = expf(sel[j] - mx) / den;
        if (a.pes) w *= bf2f(a.pes[sid[j]]);
        a.ids[tk * k + j] = sid[j];
        a.wts[tk * k + j] = w;
      }
    }
  }
  __threadfence_block();
  for (int e = threadIdx.x; e < E; e += NTHR) used[e] = 0;
  __syncthreads();
  for (int i = threadIdx.x; i < a.T * k; i += NTHR) used[a.ids[i]] = 1;
  __syncthreads();
  if (warp == 0) {
    int base = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const bool u = e < E && used[e];
      const unsigned m = __ballot_sync(0xffffffffu, u);
      if (u) {
        const int pos = base + __popc(m & ((1u << lane) - 1u));
        a.uniq[pos] = e;
        used[e] = pos + 1;  // slot + 1
      }
      base += __popc(m);
    }
    if (lane == 0) *a.nuniq = base;
  }
  __syncthreads();
  for (int i = threadIdx.x; i < a.T * k; i += NTHR) a.slot[i] = used[a.ids[i]] - 1;
}

__global__ void __launch_bounds__(NTHR, 1) ffn1_kernel(const __grid_constant__ Ffn1Args a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int flag;
  __shared__ int used[256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * NW + warp;
  const bool is_r = gw < a.fr.w0 + a.fr.nw;
  const Fam& f = is_r ? a.fr : a.fg;
  const Split S = make_split(f.tiles, f.nw, f.us);
  const int lw = gw - f.w0;
  const int2 rg = srange(S, lw);
  const int lo = rg.x, hi = rg.y;
  uint8_t* ring = smem + warp * kRingSlot;
  auto fr_ = [&](int) {
    return FragPtr{reinterpret_cast<const uint4*>(smem + f.frag_off), reinterpret_cast<const float*>(smem + f.xsum_off)};
  };
  auto prologue = [&]() {
    griddep_wait();
    griddep_launch_dependents();
    if (a.fr.bits == 16)
      build_frags<16>(smem, a.fr.frag_off, a.fr.xsum_off, a.fr.G, a.T, a.xs, a.H, nullptr, nullptr);
    else
      build_frags<4>(smem, a.fr.frag_off, a.fr.xsum_off, a.fr.G, a.T, a.xs, a.H, nullptr, nullptr);
    build_frags<4>(smem, a.fg.frag_off, a.fg.xsum_off, a.fg.G, a.T, a.h1, a.H, nullptr, nullptr);
    __syncthreads();
  };
  if (is_r) {
    auto addr = [&](int u) { return mat_unit<1>(f, u); };
    auto done = [&](int u, Acc<1> y, int pst, int pe) {
      if (DL_UNIT_DONE(1, f, S, a.T, lw, u, y, pst, pe, lane, u)) store_block<1>(f.fin + (int64_t)u * a.T * 16, a.T, y, lane);
    };
    if (a.fr.bits == 16) {
      Engine<16, 1, 1, 3> en;
      en.init(ring, lane, f, lo, hi);
      en.prime(addr);
      prologue();
      en.run(addr, fr_, done, a.T);
    } else {
      Engine<4, 1, 2, 6> en;
      en.init(ring, lane, f, lo, hi);
      en.prime(addr);
      prologue();
      en.run(addr, fr_, done, a.T);
    }
  } else {
    auto addr = [&](int u) { return mat_unit<2>(f, u); };
    auto done = [&](int u, Acc<2> y, int pst, int pe) {
      if (DL_UNIT_DONE(2, f, S, a.T, lw, u, y, pst, pe, lane, u)) glu_store(y, a.T, u, a.act_d, a.Id, lane);
    };
    Engine<4, 2, 2, 3> en;
    en.init(ring, lane, f, lo, hi);
    en.prime(addr);
    prologue();
    en.run(addr, fr_, done, a.T);
  }
  if (grid_last(a.grid_ctr, &flag)) route_rows(a, used);
}

// ---------------------------------------------------------------------------
// 5. dense down + routed experts' gate|up

struct Ffn2Args {
  Fam fd;             // dense down (4-bit), input act_d
  Fam fx;             // experts gate|up pairs (4-bit), input h2
  ExpertsDev ex;
  const bf16* act_d;  // [T][Id]
  const bf16* h2;     // [T][H]
  int T, H, Id, Ie;
  const int32_t* uniq;
  const int32_t* nuniq;
  bf16* act_e;        // [slot][T][Ie]
};

__global__ void __launch_bounds__(NTHR, 1) ffn2_kernel(const __grid_constant__ Ffn2Args a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int32_t uq[kMaxUnique];
  __shared__ int nu_s;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * NW + warp;
  const bool is_d = gw < a.fd.w0 + a.fd.nw;
  uint8_t* ring = smem + warp * kRingSlot;
  auto prologue = [&]() {
    griddep_wait();
    griddep_launch_dependents();
    if (threadIdx.x == 0) nu_s = min(__ldcg(a.nuniq), kMaxUnique);
    if (threadIdx.x < kMaxUnique) uq[threadIdx.x] = __ldcg(a.uniq + threadIdx.x);
    build_frags<4>(smem, a.fd.frag_off, a.fd.xsum_off, a.fd.G, a.T, a.act_d, a.Id, nullptr, nullptr);
    build_frags<4>(smem, a.fx.frag_off, a.fx.xsum_off, a.fx.G, a.T, a.h2, a.H, nullptr, nullptr);
    __syncthreads();
  };
  if (is_d) {
    const Fam& f = a.fd;
    const Split S = make_split(f.tiles, f.nw, f.us);
    const int lw = gw - f.w0;
    auto addr = [&](int u) { return mat_unit<1>(f, u); };
    auto fr_ = [&](int) {
      return FragPtr{reinterpret_cast<const uint4*>(smem + f.frag_off),
                     reinterpret_cast<const float*>(smem + f.xsum_off)};
    };
    auto done = [&](int u, Acc<1> y, int pst, int pe) {
      if (DL_UNIT_DONE(1, f, S, a.T, lw, u, y, pst, pe, lane, u)) store_block<1>(f.fin + (int64_t)u * a.T * 16, a.T, y, lane);
    };
    Engine<4, 1, 1, 8> en;
    const int2 rg = srange(S, lw);
    en.init(ring, lane, f, rg.x, rg.y);
    en.prime(addr);
    prologue();
    en.run(addr, fr_, done, a.T);
  } else {
    prologue();
    const Fam& f = a.fx;
    const Split S = make_split(nu_s * f.tiles, f.nw, f.us);
    const int lw = gw - f.w0;
    auto addr = [&](int u) { return expert_unit<2>(f, a.ex, uq, u); };
    auto fr_ = [&](int) {
      return FragPtr{reinterpret_cast<const uint4*>(smem + f.frag_off),
                     reinterpret_cast<const float*>(smem + f.xsum_off)};
    };
    auto done = [&](int u, Acc<2> y, int pst, int pe) {
      if (!DL_UNIT_DONE(2, f, S, a.T, lw, u, y, pst, pe, lane, u)) return;
      const int slot = u / f.tiles, j = u - slot * f.tiles;
      glu_store(y, a.T, j, a.act_e + (int64_t)slot * a.T * a.Ie, a.Ie, lane);
    };
    Engine<4, 2, 2, 3> en;
    const int2 rg = srange(S, lw);
    en.init(ring, lane, f, rg.x, rg.y);
    en.prime(addr);
    en.run(addr, fr_, done, a.T);
  }
}

// ---------------------------------------------------------------------------
// 6. routed experts' down + combine; last CTA: output norms -> x

struct Ffn3Args {
  Fam fy;             // experts down (4-bit), input act_e per slot
  Fam fd;             // dense down of ffn2 (finished units)
  ExpertsDev ex;
  const bf16* act_e;  // [slot][T][Ie]
  int T, H, Ie, k;
  const int32_t* uniq;
  const int32_t* nuniq;
  const int32_t* ids;
  const float* wts;
  const int32_t* slot;
  bf16* moe;          // [T][H]
  const bf16* h;      // residual (ff_in)
  const bf16* w1;     // post_ff_norm_1 (dense)
  const bf16* w2;     // post_ff_norm_2 (moe)
  const bf16* w;      // post_ff_norm
  float eps, scalar;
  bf16* x_out;
  unsigned* grid_ctr;
};

// A finished expert-down unit (slot, tile j): store it and count it toward
// tile j; j when every slot's tile j is now finished, else -1.
__device__ __noinline__ int down_unit_finished(const Fam& f, int T, int nu, int u, const Acc<1> y, int lane) {
  store_block<1>(f.fin + (int64_t)u * T * 16, T, y, lane);
  const int j = u % f.tiles;
  return arrive(f.gctr + j, nu, lane) ? j : -1;
}

// Tile-group epilogue: moe[tk][rows of tile j] = bf16(sum over tk's slots in
// ascending expert id of w * down_e), fp32 (moe.rs:443-453).
__device__ __noinline__ void combine_tile(const Ffn3Args& a, int j, int lane) {
  const Fam& f = a.fy;
  for (int i = lane; i < a.T * 16; i += 32) {
    const int tk = i >> 4, r = i & 15;
    float d[8], wv[8];
    int e[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      if (q < a.k) {
        const int s = a.slot[tk * a.k + q];
        e[q] = a.ids[tk * a.k + q];
        wv[q] = a.wts[tk * a.k + q];
        d[q] = __ldcg(f.fin + ((int64_t)s * f.tiles + j) * a.T * 16 + tk * 16 + r);
      } else {
        e[q] = 0x7fffffff;
      }
    }
    // ascending expert id (ids are distinct within a token)
    float acc = 0.f;
    int last = -1;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      int best = 0x7fffffff, bq = 0;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (e[q] > last && e[q] < best) {
          best = e[q];
          bq = q;
        }
      if (best == 0x7fffffff) break;
      last = best;
      float dv = 0.f, ww = 0.f;
#pragma unroll
      for (int q = 0; q < 8; ++q)
        if (q == bq) {
          dv = d[q];
          ww = wv[q];
        }
      acc += ww * dv;
    }
    a.moe[(int64_t)tk * a.H + 16 * j + r] = __float2bfloat16_rn(acc);
  }
}

// x = bf16(bf16(h + bf16(rms(s) * w_post_ff)) * scalar),
// s = bf16(bf16(rms(bf16(d)) * w1) + bf16(rms(moe) * w2))   (mod.rs:105-118)
// Inputs staged in shared memory in one batch, as in ff_in_rows.
__device__ __noinline__ void ff_out_rows(const Ffn3Args& a, float* red, uint8_t* rows) {
  const int H = a.H;
  float* rd = reinterpret_cast<float*>(rows);  // d, then s
  float* rm = rd + H;                          // moe
  bf16* rh = reinterpret_cast<bf16*>(rm + H);  // h
  bf16* wv = rh + H;                           // [3][H]: post_ff_norm_1, post_ff_norm_2, post_ff_norm
  const bf16* srcw[3] = {a.w1, a.w2, a.w};
  const float sc = round_bf(a.scalar);
  for (int tk = 0; tk < a.T; ++tk) {
#pragma unroll
    for (int k = 0; k < (kMaxHidden + NTHR - 1) / NTHR; ++k) {
      const int i = threadIdx.x + k * NTHR;
      if (i < H) {
        const float d = fin_at(a.fd, a.T, tk, i);
        const float m = __bfloat162float(__ldcg(a.moe + (int64_t)tk * H + i));
        const bf16 h = __ldcg(a.h + (int64_t)tk * H + i);
        bf16 w3[3];
        if (tk == 0) {
#pragma unroll
          for (int q = 0; q < 3; ++q) w3[q] = srcw[q][i];
        }
        rd[i] = d;
        rm[i] = m;
        rh[i] = h;
        if (tk == 0) {
#pragma unroll
          for (int q = 0; q < 3; ++q) wv[q * H + i] = w3[q];
        }
      }
    }
    __syncthreads();
    float sd = 0.f, sm = 0.f;
    for (int i = threadIdx.x; i < H; i += NTHR) {
      const float d = round_bf(rd[i]), m = rm[i];
      rd[i] = d;
      sd = fmaf(d, d, sd);
      sm = fmaf(m, m, sm);
    }
    const float rdn = rsqrtf(cta_sum(sd, red) / (float)H + a.eps);
    const float rmn = rsqrtf(cta_sum(sm, red) / (float)H + a.eps);
    float ss = 0.f;
    for (int i = threadIdx.x; i < H; i += NTHR) {
      const float v = round_bf(round_bf(rd[i] * rdn * bf2f(wv[i])) + round_bf(rm[i] * rmn * bf2f(wv[H + i])));
      rd[i] = v;
      ss = fmaf(v, v, ss);
    }
    const float rs = rsqrtf(cta_sum(ss, red) / (float)H + a.eps);
    for (int i = threadIdx.x; i < H; i += NTHR) {
      const float o = round_bf(bf2f(rh[i]) + round_bf(rd[i] * rs * bf2f(wv[2 * H + i])));
      a.x_out[(int64_t)tk * H + i] = __float2bfloat16_rn(o * sc);
    }
    __syncthreads();
  }
}

__global__ void __launch_bounds__(NTHR, 1) ffn3_kernel(const __grid_constant__ Ffn3Args a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int32_t uq[kMaxUnique];
  __shared__ int nu_s;
  __shared__ float red[NW];
  __shared__ int flag;
  __shared__ int pend[NW][kMaxPend];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int gw = blockIdx.x * NW + warp;
  const Fam& f = a.fy;
  // The routing was written by ffn1, two launches back.  This grid starts only
  // after every ffn2 CTA passed its own dependency wait (which ends ffn1), so
  // the routing can be read — and this launch's expert weights streamed —
  // before waiting for ffn2 (L2 reads: no stale L1 lines).
  if (threadIdx.x == 0) nu_s = min(__ldcg(a.nuniq), kMaxUnique);
  if (threadIdx.x < kMaxUnique) uq[threadIdx.x] = __ldcg(a.uniq + threadIdx.x);
  __syncthreads();
  const int nu = nu_s;
  const Split S = make_split(nu * f.tiles, f.nw, f.us);
  const int lw = gw - f.w0;
  const int2 rg = srange(S, lw);
  const int lo = rg.x, hi = rg.y;
  // expert slots this CTA's warps touch: their inputs' fragments
  int cl = 0x7fffffff, ch = 0;
  for (int w = 0; w < NW; ++w) {
    const int2 r = srange(S, blockIdx.x * NW + w - f.w0);
    if (r.y > r.x) {
      cl = min(cl, r.x);
      ch = max(ch, r.y);
    }
  }
  if (ch == 0) cl = 0;
  const int per = f.tiles * f.us;
  const int s_first = cl / per, s_last = ch > cl ? (ch - 1) / per : s_first;
  auto addr = [&](int u) { return expert_unit<1>(f, a.ex, uq, u); };
  Engine<4, 1, 1, 8> en;
  en.init(smem + warp * kRingSlot, lane, f, lo, hi);
  en.prime(addr);
  griddep_wait();  // the activations come from ffn2
  griddep_launch_dependents();
  const int fb = frag_bytes(f.G, a.T), xb = f.G * 8 * 4;
  for (int s = s_first; s <= s_last && s < nu && s - s_first < kMaxSlotsPerCta; ++s)
    build_frags<4>(smem, f.frag_off + (s - s_first) * fb, f.xsum_off + (s - s_first) * xb, f.G, a.T,
                   a.act_e + (int64_t)s * a.T * a.Ie, a.Ie, nullptr, nullptr);
  __syncthreads();
  auto fr_ = [&](int u) {
    const int s = min(max(u / f.tiles - s_first, 0), kMaxSlotsPerCta - 1);
    return FragPtr{reinterpret_cast<const uint4*>(smem + f.frag_off + s * fb),
                   reinterpret_cast<const float*>(smem + f.xsum_off + s * xb)};
  };
  int npend = 0;
  auto done = [&](int u, Acc<1> y, int pst, int pe) {
    if (!DL_UNIT_DONE(1, f, S, a.T, lw, u, y, pst, pe, lane, u)) return;
    const int j = down_unit_finished(f, a.T, nu, u, y, lane);
    if (j >= 0) {
      if (lane == 0 && npend < kMaxPend) pend[warp][npend] = j;
      ++npend;
    }
  };
  en.run(addr, fr_, done, a.T);
  __syncwarp();
  for (int i = 0; i < npend && i < kMaxPend; ++i) combine_tile(a, pend[warp][i], lane);
  if (grid_last(a.grid_ctr, &flag)) ff_out_rows(a, red, smem);
}

// ---------------------------------------------------------------------------
// lm_head: final norm, tied embedding, softcap, greedy argmax

struct LmArgs {
  Fam f;
  const bf16* x;
  const bf16* norm;
  float eps, cap;
  int T, H;
  int64_t V;
  float* logits;      // [T][V]
  float2* cand;       // [gridDim][T]
  int32_t* next_ids;
  int64_t* pos;
  unsigned* grid_ctr;
};

__device__ __forceinline__ float softcap_bf(float v, float cap) {
  v = round_bf(v);
  if (cap > 0.f) v = round_bf(round_bf(tanhf(round_bf(v / cap))) * cap);
  return v;
}
__device__ __forceinline__ void best_merge(float& bv, int& bi, float ov, int oi) {
  if (ov > bv || (ov == bv && oi < bi)) {
    bv = ov;
    bi = oi;
  }
}
// Running greedy candidates of a lane: tokens 2t and 2t+1.
struct Best {
  float v0, v1;
  int i0, i1;
};
// Softcap and store a finished lm_head tile; fold it into the lane's best.
__device__ __noinline__ Best lm_unit_finished(const LmArgs& a, int u, const Acc<1> y, Best b, int lane) {
  const int g = lane >> 2, t = lane & 3;
  const int r0 = 16 * u + g;
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int tk = 2 * t + c;
    if (tk < a.T) {
      const float v0 = softcap_bf(y.v[0][c], a.cap), v1 = softcap_bf(y.v[0][2 + c], a.cap);
      a.logits[tk * a.V + r0] = v0;
      a.logits[tk * a.V + r0 + 8] = v1;
      float& bv = c ? b.v1 : b.v0;
      int& bi = c ? b.i1 : b.i0;
      best_merge(bv, bi, v0, r0);
      best_merge(bv, bi, v1, r0 + 8);
    }
  }
  return b;
}

template <int BITS, int D_>
__global__ void __launch_bounds__(NTHR, 1) lm_kernel(const __grid_constant__ LmArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float rms[kMaxT];
  __shared__ float wbv[NW][kMaxT];
  __shared__ int wbi[NW][kMaxT];
  __shared__ int flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int gw = blockIdx.x * NW + warp;
  const Fam& f = a.f;
  const Split S = make_split(f.tiles, f.nw, f.us);
    const int lw = gw - f.w0;
  Engine<BITS, 1, 2, D_> en;
  const int2 rg = srange(S, lw);
  en.init(smem + warp * kRingSlot, lane, f, rg.x, rg.y);
  auto addr = [&](int u) { return mat_unit<1>(f, u); };
  en.prime(addr);
  griddep_wait();
  griddep_launch_dependents();
  row_rms(a.x, a.H, a.H, a.T, a.eps, rms);
  __syncthreads();
  build_frags<BITS>(smem, f.frag_off, f.xsum_off, f.G, a.T, a.x, a.H, rms, a.norm);
  __syncthreads();
  Best best = {-INFINITY, -INFINITY, 0x7fffffff, 0x7fffffff};
  auto fr_ = [&](int) {
    return FragPtr{reinterpret_cast<const uint4*>(smem + f.frag_off), reinterpret_cast<const float*>(smem + f.xsum_off)};
  };
  // Ranges are at least one unit long (planned so): a unit is split over at
  // most two warps, its pieces and counter keyed by its first warp.
  auto done = [&](int u, Acc<1> y, int pst, int pe) {
    if (!DL_UNIT_DONE(1, f, S, a.T, lw, u, y, pst, pe, lane, u)) return;
    best = lm_unit_finished(a, u, y, best, lane);
  };
  en.run(addr, fr_, done, a.T);
  float bv[2] = {best.v0, best.v1};
  int bi[2] = {best.i0, best.i1};
#pragma unroll
  for (int c = 0; c < 2; ++c)
#pragma unroll
    for (int o = 4; o < 32; o <<= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv[c], o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi[c], o);
      best_merge(bv[c], bi[c], ov, oi);
    }
  if (g == 0) {
#pragma unroll
    for (int c = 0; c < 2; ++c)
      if (2 * t + c < a.T) {
        wbv[warp][2 * t + c] = bv[c];
        wbi[warp][2 * t + c] = bi[c];
      }
  }
  __syncthreads();
  if (threadIdx.x < a.T) {
    float b = -INFINITY;
    int i = 0x7fffffff;
    for (int w = 0; w < NW; ++w) best_merge(b, i, wbv[w][threadIdx.x], wbi[w][threadIdx.x]);
    a.cand[blockIdx.x * a.T + threadIdx.x] = make_float2(b, __int_as_float(i));
  }
  if (grid_last(a.grid_ctr, &flag)) {
    if (threadIdx.x < a.T) {
      float b = -INFINITY;
      int i = 0x7fffffff;
      for (int c = 0; c < (int)gridDim.x; ++c) {
        const float2 cv = __ldcg(a.cand + c * a.T + threadIdx.x);
        best_merge(b, i, cv.x, __float_as_int(cv.y));
      }
      a.next_ids[threadIdx.x] = i == 0x7fffffff ? 0 : i;
    }
    if (threadIdx.x == 0 && a.pos) {
      a.pos[0] += 1;
      a.pos[1] += 1;
    }
  }
}

}  // namespace dl
}  // namespace fmoe

// ===========================================================================
// Host side: plan, workspace, launches

namespace fmoe {
namespace dl {

constexpr int kGrid = kNumSMs;      // one CTA per SM
constexpr int kWarps = kGrid * NW;  // warps of a launch

static bool fits32(long S, long nw) { return S > 0 && (S + 1) * nw + S < (1l << 32); }

static Fam mat_fam(int bits, int K, const QW* segs, int nseg, int w0, int nw, int ng) {
  Fam f = {};
  f.bits = bits;
  f.nt = 1;
  f.K = K;
  f.G = K / 64;
  f.us = f.G / ng;
  f.w0 = w0;
  f.nw = nw;
  f.src = SRC_MAT;
  f.rowbytes = (int64_t)K * bits / 8;
  f.nseg = nseg;
  int t0 = 0;
  for (int i = 0; i < nseg; ++i) {
    f.seg_tile0[i] = t0;
    f.w[i] = static_cast<const uint8_t*>(segs[i].w);
    f.s[i] = segs[i].s;
    f.b[i] = segs[i].b;
    t0 += segs[i].out / 16;
  }
  f.seg_tile0[nseg] = t0;
  f.tiles = t0;
  return f;
}
static Fam glu_fam(const QW& gate, const QW& up, int w0, int nw, int ng) {
  const QW s[2] = {gate, up};
  Fam f = mat_fam(gate.bits, gate.in, s, 2, w0, nw, ng);
  f.nt = 2;
  f.tiles = gate.out / 16;
  return f;
}
static Fam expert_fam(int mat, int nt, int K, int rows, int w0, int nw, int ng) {
  Fam f = {};
  f.bits = 4;
  f.nt = nt;
  f.K = K;
  f.G = K / 64;
  f.us = f.G / ng;
  f.w0 = w0;
  f.nw = nw;
  f.src = SRC_EXPERT;
  f.rowbytes = K / 2;
  f.mat = mat;
  f.tiles = rows / 16;
  return f;
}

// Warps of a two-family launch, by bytes (each family >= 1 warp, <= 1 per group).
static void split_warps(double b0, double b1, long S0, long S1, int* n0, int* n1) {
  int a = (int)std::lround(kWarps * b0 / (b0 + b1));
  a = std::max(1, std::min(a, kWarps - 1));
  a = (int)std::min<long>(a, S0);
  int b = kWarps - a;
  if (b > S1) {
    b = (int)S1;
    a = (int)std::min<long>(kWarps - b, S0);
  }
  *n0 = a;
  *n1 = b;
}

// Raise a kernel's dynamic shared-memory limit once per (kernel, device): the
// opt-in block limit minus the kernel's static shared memory.
template <class F>
static int smem_attr(F kern, const char* name) {
  static std::mutex mu;
  static std::vector<std::pair<const void*, int>> done;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return set_error(FMOE_ERR_CUDA, "%s: no device", name);
  const void* key = reinterpret_cast<const void*>(kern);
  std::lock_guard<std::mutex> lk(mu);
  for (const auto& d : done)
    if (d.first == key && d.second == dev) return FMOE_OK;
  cudaFuncAttributes fa;
  int optin = 0;
  cudaError_t e = cudaFuncGetAttributes(&fa, kern);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, optin - (int)fa.sharedSizeBytes);
  if (e != cudaSuccess) return set_error(FMOE_ERR_CUDA, "%s: shared memory attribute: %s", name, cudaGetErrorString(e));
  done.emplace_back(key, dev);
  return FMOE_OK;
}

template <class F, class A>
static int launch(F kern, const A& args, size_t smem, cudaStream_t st, const char* name, unsigned grid = kGrid) {
  int rc = smem_attr(kern, name);
  if (rc) return rc;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(NTHR);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  ProfScope prof_(name, st);
  cudaLaunchKernelEx(&cfg, kern, args);
  return check_launch(name);
}

// Ring depth per code width (two groups per step): <BITS, steps in flight>.
#define DL_DISPATCH(bits, KERNEL, ...)                                                 \
  ((bits) == 8 ? launch(KERNEL<8, 3>, __VA_ARGS__)                                     \
               : (bits) == 6 ? launch(KERNEL<6, 4>, __VA_ARGS__) : launch(KERNEL<4, 6>, __VA_ARGS__))

}  // namespace dl

using namespace dl;

int dl_plan(const fmoe_decoder_layer_t* L, const KvDev& kv, int64_t T, DlPlan* p) {
  DlPlan d = {};
  if (T < 1 || T > kMaxT) return FMOE_ERR_UNSUPPORTED;
  QW q, k, v, o, gq, uq, dq, rq;
  ExpertsDev ex;
  if (to_qw(&L->q_proj, &q) || to_qw(&L->k_proj, &k) || to_qw(&L->o_proj, &o) || to_qw(&L->mlp_gate, &gq) ||
      to_qw(&L->mlp_up, &uq) || to_qw(&L->mlp_down, &dq) || check_router(&L->router, &rq) ||
      to_experts(&L->experts, &ex))
    return FMOE_ERR_INVALID;
  if (!L->k_eq_v && to_qw(&L->v_proj, &v)) return FMOE_ERR_INVALID;
  const int H = q.in;
  auto width_ok = [](const QW& w, int group, int b0, int b1) {
    return (w.bits == b0 || w.bits == b1) && (w.bits == 16 || group == 64) && w.in % 64 == 0 && w.out % 16 == 0 &&
           aligned(w.w, 16) && (w.bits == 16 || (w.s && w.b));
  };
  const int wb = q.bits == 6 ? 6 : 8;
  if (!width_ok(q, L->q_proj.group_size, wb, 4) || !width_ok(k, L->k_proj.group_size, q.bits, q.bits) ||
      (!L->k_eq_v && !width_ok(v, L->v_proj.group_size, q.bits, q.bits)) ||
      !width_ok(o, L->o_proj.group_size, o.bits == 6 ? 6 : 8, 4) || !width_ok(gq, L->mlp_gate.group_size, 4, 4) ||
      !width_ok(uq, L->mlp_up.group_size, 4, 4) || !width_ok(dq, L->mlp_down.group_size, 4, 4) ||
      !width_ok(rq, L->router.proj.group_size, 4, 16))
    return FMOE_ERR_UNSUPPORTED;
  if (ex.first != 0 || ex.E != rq.out || ex.H != H || ex.I % 64 || H % 64 || H > kMaxHidden || rq.out > 256 ||
      rq.out % 16 || L->router.top_k < 1 || L->router.top_k > 8 || T * L->router.top_k > kMaxUnique ||
      uq.out != gq.out || dq.in != gq.out || dq.out != H)
    return FMOE_ERR_UNSUPPORTED;
  for (int i = 0; i < 9; ++i)
    if (ex.off[i] % 16) return FMOE_ERR_UNSUPPORTED;
  if (ex.stride % 16 || !aligned(ex.base, 16)) return FMOE_ERR_UNSUPPORTED;
  const int D = L->head_dim;
  if ((D != 256 && D != 512) || kv.D != D || kv.B != T) return FMOE_ERR_UNSUPPORTED;
  const int Hq = L->num_heads, Hkv = L->num_kv_heads;
  if (Hq + Hkv > 64) return FMOE_ERR_UNSUPPORTED;
  d.T = (int)T;
  d.H = H;
  d.D = D;
  d.Hq = Hq;
  d.Hkv = Hkv;
  d.QD = Hq * D;
  d.Id = gq.out;
  d.Ie = ex.I;
  d.E = rq.out;
  d.k = L->router.top_k;
  d.Umax = std::min(d.E, d.T * d.k);
  d.qbits = q.bits;
  d.obits = o.bits;
  d.rbits = rq.bits;
  d.qkv_tiles = (Hq + (L->k_eq_v ? 1 : 2) * Hkv) * D / 16;
  const long Gh = H / 64, Gq = d.QD / 64, Gi = d.Id / 64, Ge = d.Ie / 64;
  // groups per ring step of each family (see the kernels' Engine instances)
  if (Gh % 2 || Gq % 2) return FMOE_ERR_UNSUPPORTED;
  const long Uh = Gh / 2, Uq = Gq / 2, Ur = d.rbits == 16 ? Gh : Gh / 2, Ui = Gi, Ue = Ge;
  const long S_qkv = (long)d.qkv_tiles * Uh, S_o = (long)(H / 16) * Uq;
  const long S_r = (long)(d.E / 16) * Ur, S_g = (long)(d.Id / 16) * Uh, S_d = (long)(H / 16) * Ui;
  const long S_x = (long)d.k * (d.Ie / 16) * Uh, S_y = (long)d.k * (H / 16) * Ue;  // fewest slots: k
  const double b_r = (double)d.E * H * (d.rbits == 16 ? 2.0 : 0.5625);
  const double b_g = 2.0 * d.Id * H * 0.5625, b_d = (double)H * d.Id * 0.5625;
  const double b_x = (double)d.Umax * 2.0 * d.Ie * H * 0.5625;
  split_warps(b_r, b_g, S_r, S_g, &d.nw_r, &d.nw_g);
  split_warps(b_d, b_x, S_d, S_x, &d.nw_d, &d.nw_x);
  if (S_qkv < kWarps || S_o < kWarps || S_y < kWarps) return FMOE_ERR_UNSUPPORTED;
  const long S_xmax = (long)d.Umax * (d.Ie / 16) * Uh, S_ymax = (long)d.Umax * (H / 16) * Ue;
  if (!fits32(S_qkv, kWarps) || !fits32(S_o, kWarps) || !fits32(S_xmax, d.nw_x) || !fits32(S_ymax, kWarps) ||
      !fits32(S_r, d.nw_r) || !fits32(S_g, d.nw_g) || !fits32(S_d, d.nw_d))
    return FMOE_ERR_UNSUPPORTED;
  d.mp_qkv = split_maxp(d.qkv_tiles, kWarps, (int)Uh);
  d.mp_o = split_maxp(H / 16, kWarps, (int)Uq);
  d.mp_r = split_maxp(d.E / 16, d.nw_r, (int)Ur);
  d.mp_g = split_maxp(d.Id / 16, d.nw_g, (int)Uh);
  d.mp_d = split_maxp(H / 16, d.nw_d, (int)Ui);
  d.mp_x = split_maxp(d.k * (d.Ie / 16), d.nw_x, (int)Uh);  // fewest slots: k
  d.mp_y = split_maxp(d.k * (H / 16), kWarps, (int)Ue);
  if (std::min({d.mp_qkv, d.mp_o, d.mp_r, d.mp_g, d.mp_d, d.mp_x, d.mp_y}) < 0) return FMOE_ERR_UNSUPPORTED;
  const size_t fT = 128 * (size_t)T;
  d.sm_qkv = kRingBytes + Gh * fT + Gh * 32;
  d.sm_o = kRingBytes + Gq * fT + Gq * 32;
  d.sm_1 = kRingBytes + 2 * (Gh * fT + Gh * 32);
  d.sm_2 = kRingBytes + Gi * fT + Gi * 32 + Gh * fT + Gh * 32;
  d.sm_3 = kRingBytes + kMaxSlotsPerCta * (Ge * fT + Ge * 32);
  if (std::max({d.sm_qkv, d.sm_o, d.sm_1, d.sm_2, d.sm_3}) > 200 * 1024) return FMOE_ERR_UNSUPPORTED;
  *p = d;
  return FMOE_OK;
}

size_t dl_carve(Carver& c, const DlPlan& p, DlWs* w) {
  DlWs d = {};
  const size_t T = p.T, blk = 16 * T;
  const size_t u_qkv = p.qkv_tiles, u_o = p.H / 16, u_r = p.E / 16, u_g = p.Id / 16, u_d = p.H / 16;
  const size_t u_x = (size_t)p.Umax * (p.Ie / 16), u_y = (size_t)p.Umax * (p.H / 16);
  d.uc_qkv = c.take<unsigned>(u_qkv);
  d.uc_o = c.take<unsigned>(u_o);
  d.uc_r = c.take<unsigned>(u_r);
  d.uc_g = c.take<unsigned>(u_g);
  d.uc_d = c.take<unsigned>(u_d);
  d.uc_x = c.take<unsigned>(u_x);
  d.uc_y = c.take<unsigned>(u_y);
  d.gc_qkv = c.take<unsigned>(64);
  d.gc_y = c.take<unsigned>(p.H / 16);
  d.grid = c.take<unsigned>(4);
  d.p_qkv = c.take<float>(u_qkv * p.mp_qkv * blk);
  d.p_o = c.take<float>(u_o * p.mp_o * blk);
  d.p_r = c.take<float>(u_r * p.mp_r * blk);
  d.p_g = c.take<float>(u_g * p.mp_g * 2 * blk);
  d.p_d = c.take<float>(u_d * p.mp_d * blk);
  d.p_x = c.take<float>(u_x * p.mp_x * 2 * blk);
  d.p_y = c.take<float>(u_y * p.mp_y * blk);
  d.f_qkv = c.take<float>(u_qkv * blk);
  d.f_o = c.take<float>(u_o * blk);
  d.f_r = c.take<float>(u_r * blk);
  d.f_d = c.take<float>(u_d * blk);
  d.f_y = c.take<float>(u_y * blk);
  d.act_d = c.take<bf16>(T * p.Id);
  d.act_e = c.take<bf16>((size_t)p.Umax * T * p.Ie);
  d.ids = c.take<int32_t>(T * p.k);
  d.slot = c.take<int32_t>(T * p.k);
  d.wts = c.take<float>(T * p.k);
  d.uniq = c.take<int32_t>(kMaxUnique);
  d.nuniq = c.take<int32_t>(1);
  if (w) *w = d;
  return c.off;
}

int dl_layer_forward(const fmoe_decoder_layer_t* L, const KvDev& kv, const DlPlan& p, const DlWs& w, bf16* x,
                     int64_t pos, const int64_t* pos_dev, const DlBufs& b, cudaStream_t st) {
  QW q, k, v = {}, o, gq, uq, dq, rq;
  ExpertsDev ex;
  to_qw(&L->q_proj, &q);
  to_qw(&L->k_proj, &k);
  to_qw(&L->o_proj, &o);
  to_qw(&L->mlp_gate, &gq);
  to_qw(&L->mlp_up, &uq);
  to_qw(&L->mlp_down, &dq);
  check_router(&L->router, &rq);
  to_experts(&L->experts, &ex);
  if (!L->k_eq_v) to_qw(&L->v_proj, &v);
  const int T = p.T, H = p.H;
  const int fT = 128 * T;
  int rc;
  // 1 q | k | v
  {
    QkvArgs a = {};
    const QW segs[3] = {q, k, v};
    a.f = mat_fam(p.qbits, H, segs, L->k_eq_v ? 2 : 3, 0, kWarps, 2);
    a.f.piece = w.p_qkv;
    a.f.maxp = p.mp_qkv;
    a.f.uctr = w.uc_qkv;
    a.f.fin = w.f_qkv;
    a.f.gctr = w.gc_qkv;
    a.f.frag_off = kRingBytes;
    a.f.xsum_off = kRingBytes + a.f.G * fT;
    a.x = x;
    a.in_norm = static_cast<const bf16*>(L->input_norm);
    a.eps = L->eps;
    a.T = T;
    a.H = H;
    a.kv = kv;
    a.Hq = p.Hq;
    a.Hkv = p.Hkv;
    a.D = p.D;
    a.k_eq_v = L->k_eq_v;
    a.q_norm = static_cast<const bf16*>(L->q_norm);
    a.k_norm = static_cast<const bf16*>(L->k_norm);
    a.rope_dims = L->rope_dims;
    a.l2theta = (float)std::log2((double)L->rope_theta);
    a.pos = pos;
    a.pos_dev = pos_dev;
    a.turbo = kv.turbo;
    a.inv_sqrt_d = 1.0f / std::sqrt((float)p.D);
    a.q_out = b.q;
    if ((rc = DL_DISPATCH(p.qbits, qkv_kernel, a, p.sm_qkv, st, "dl_qkv_kernel"))) return rc;
  }
  // 2 attention
  {
    const int64_t nvalid = pos + 1 < kv.cap ? pos + 1 : kv.cap;
    if ((rc = launch_attn_decode(kv, b.q, p.Hq, nvalid, pos_dev ? pos_dev + 1 : nullptr, L->attn_scale, b.attn_ws,
                                 b.attn, st, true, pos, pos_dev)))
      return rc;
  }
  // 3 o + feed-forward input norms
  {
    OArgs a = {};
    a.f = mat_fam(p.obits, p.QD, &o, 1, 0, kWarps, 2);
    a.f.piece = w.p_o;
    a.f.maxp = p.mp_o;
    a.f.uctr = w.uc_o;
    a.f.fin = w.f_o;
    a.f.frag_off = kRingBytes;
    a.f.xsum_off = kRingBytes + a.f.G * fT;
    a.attn = b.attn;
    a.T = T;
    a.H = H;
    a.QD = p.QD;
    a.x = x;
    a.w_post_attn = static_cast<const bf16*>(L->post_attn_norm);
    a.w_pre_ff = static_cast<const bf16*>(L->pre_ff_norm);
    a.w_pre_ff2 = static_cast<const bf16*>(L->pre_ff_norm_2);
    a.rscale = static_cast<const bf16*>(L->router.router_scale);
    a.eps = L->eps;
    a.root = L->router.root_size;
    a.h = b.h;
    a.h1 = b.h1;
    a.h2 = b.h2;
    a.xs = b.xs;
    a.grid_ctr = w.grid + 0;
    if ((rc = DL_DISPATCH(p.obits, o_kernel, a, p.sm_o, st, "dl_o_kernel"))) return rc;
  }
  // 4 router + dense gate|up
  {
    Ffn1Args a = {};
    a.fr = mat_fam(p.rbits, H, &rq, 1, 0, p.nw_r, p.rbits == 16 ? 1 : 2);
    a.fr.piece = w.p_r;
    a.fr.maxp = p.mp_r;
    a.fr.uctr = w.uc_r;
    a.fr.fin = w.f_r;
    a.fr.frag_off = kRingBytes;
    a.fr.xsum_off = kRingBytes + a.fr.G * fT;
    a.fg = glu_fam(gq, uq, p.nw_r, p.nw_g, 2);
    a.fg.piece = w.p_g;
    a.fg.maxp = p.mp_g;
    a.fg.uctr = w.uc_g;
    a.fg.frag_off = a.fr.xsum_off + a.fr.G * 32;
    a.fg.xsum_off = a.fg.frag_off + a.fg.G * fT;
    a.xs = b.xs;
    a.h1 = b.h1;
    a.T = T;
    a.H = H;
    a.E = p.E;
    a.k = p.k;
    a.Id = p.Id;
    a.logit_bias = L->router.logit_bias;
    a.pes = static_cast<const bf16*>(L->router.per_expert_scale);
    a.act_d = w.act_d;
    a.ids = w.ids;
    a.wts = w.wts;
    a.uniq = w.uniq;
    a.nuniq = w.nuniq;
    a.slot = w.slot;
    a.grid_ctr = w.grid + 1;
    if ((rc = launch(ffn1_kernel, a, p.sm_1, st, "dl_ffn1_kernel"))) return rc;
  }
  // 5 dense down + experts' gate|up
  Fam fd;
  {
    Ffn2Args a = {};
    a.fd = mat_fam(4, p.Id, &dq, 1, 0, p.nw_d, 1);
    a.fd.piece = w.p_d;
    a.fd.maxp = p.mp_d;
    a.fd.uctr = w.uc_d;
    a.fd.fin = w.f_d;
    a.fd.frag_off = kRingBytes;
    a.fd.xsum_off = kRingBytes + a.fd.G * fT;
    a.fx = expert_fam(0, 2, H, p.Ie, p.nw_d, p.nw_x, 2);
    a.fx.piece = w.p_x;
    a.fx.maxp = p.mp_x;
    a.fx.uctr = w.uc_x;
    a.fx.frag_off = a.fd.xsum_off + a.fd.G * 32;
    a.fx.xsum_off = a.fx.frag_off + a.fx.G * fT;
    a.ex = ex;
    a.act_d = w.act_d;
    a.h2 = b.h2;
    a.T = T;
    a.H = H;
    a.Id = p.Id;
    a.Ie = p.Ie;
    a.uniq = w.uniq;
    a.nuniq = w.nuniq;
    a.act_e = w.act_e;
    fd = a.fd;
    if ((rc = launch(ffn2_kernel, a, p.sm_2, st, "dl_ffn2_kernel"))) return rc;
  }
  // 6 experts' down + combine + output norms
  {
    Ffn3Args a = {};
    a.fy = expert_fam(6, 1, p.Ie, H, 0, kWarps, 1);
    a.fy.piece = w.p_y;
    a.fy.maxp = p.mp_y;
    a.fy.uctr = w.uc_y;
    a.fy.fin = w.f_y;
    a.fy.gctr = w.gc_y;
    a.fy.frag_off = kRingBytes;
    a.fy.xsum_off = kRingBytes + kMaxSlotsPerCta * a.fy.G * fT;
    a.fd = fd;
    a.ex = ex;
    a.act_e = w.act_e;
    a.T = T;
    a.H = H;
    a.Ie = p.Ie;
    a.k = p.k;
    a.uniq = w.uniq;
    a.nuniq = w.nuniq;
    a.ids = w.ids;
    a.wts = w.wts;
    a.slot = w.slot;
    a.moe = b.moe;
    a.h = b.h;
    a.w1 = static_cast<const bf16*>(L->post_ff_norm_1);
    a.w2 = static_cast<const bf16*>(L->post_ff_norm_2);
    a.w = static_cast<const bf16*>(L->post_ff_norm);
    a.eps = L->eps;
    a.scalar = L->layer_scalar;
    a.x_out = x;
    a.grid_ctr = w.grid + 2;
    if ((rc = launch(ffn3_kernel, a, p.sm_3, st, "dl_ffn3_kernel"))) return rc;
  }
  return FMOE_OK;
}

// ---------------------------------------------------------------------------
// lm_head

size_t dl_lm_workspace_bytes(int64_t T) {
  // header (status), grid + per-warp unit counters, CTA candidates, pieces (two per warp)
  return 256 + align_up(sizeof(unsigned) * (kWarps + 1), 256) + align_up(sizeof(float2) * kGrid * (size_t)T, 256) +
         sizeof(float) * (size_t)kWarps * 2 * T * 16;
}

int dl_lm_head(const QW& e, const bf16* norm, float eps, const bf16* x, int64_t T, float cap, float* logits,
               int32_t* next_ids, int64_t* pos_dev, void* ws, cudaStream_t st) {
  const int H = e.in;
  if (e.out % 16 || H % 128 || H > kMaxHidden || (e.bits != 4 && e.bits != 6 && e.bits != 8))
    return set_error(FMOE_ERR_UNSUPPORTED, "lm_head: %d-bit [%d, %d] (4/6/8-bit, rows a multiple of 16)", e.bits,
                     e.out, H);
  uint8_t* base = static_cast<uint8_t*>(ws);
  unsigned* ctr = reinterpret_cast<unsigned*>(base + 256);
  float2* cand = reinterpret_cast<float2*>(base + 256 + align_up(sizeof(unsigned) * (kWarps + 1), 256));
  float* piece = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(cand) + align_up(sizeof(float2) * kGrid * T, 256));
  LmArgs a = {};
  const int nw = kWarps;
  a.f = mat_fam(e.bits, H, &e, 1, 0, nw, 2);
  a.f.piece = piece;
  a.f.maxp = split_maxp(a.f.tiles, nw, a.f.us);
  if ((long)a.f.maxp * std::min(a.f.tiles, nw) > 2l * kWarps)
    return set_error(FMOE_ERR_UNSUPPORTED, "lm_head: too few rows for the piece buffer");
  a.f.uctr = ctr + 1;
  a.f.frag_off = kRingBytes;
  const int G = H / 64;
  a.f.xsum_off = kRingBytes + G * 128 * (int)T;
  if (!fits32((long)a.f.tiles * a.f.us, nw)) return set_error(FMOE_ERR_UNSUPPORTED, "lm_head: vocabulary too large");
  a.x = x;
  a.norm = norm;
  a.eps = eps;
  a.cap = cap;
  a.T = (int)T;
  a.H = H;
  a.V = e.out;
  a.logits = logits;
  a.cand = cand;
  a.next_ids = next_ids;
  a.pos = pos_dev;
  a.grid_ctr = ctr;
  const unsigned grid = (unsigned)((nw + NW - 1) / NW);
  const size_t smem = kRingBytes + (size_t)G * 128 * T + G * 32;
  return DL_DISPATCH(e.bits, lm_kernel, a, smem, st, "dl_lm_kernel", grid);
}

}  // namespace fmoe
