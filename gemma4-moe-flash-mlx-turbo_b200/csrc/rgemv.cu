// Resident-weight quantised GEMV for decode (T <= 8 tokens):
//   y[t, r] = x[t] . W[r]^T   over up to four weight matrices ("segments")
// that share one input (q / k / v), MLX-affine 4 / 6 / 8-bit codes.
//
// Work item = one 16-row tile x one chunk of 8 64-column groups (512 inputs).
// Items are numbered chunk-major (all tiles of chunk 0, then chunk 1, ...) and
// every CTA (one per SM) owns a contiguous, balanced range of them, so a CTA
// touches one or two chunks and prepares only those chunks' input fragments.
//
// Latency plan (a decode layer is a chain of small dependent kernels):
//  * before griddepcontrol.wait every warp issues the cp.async copies (16-byte
//    code pieces into padded rows, 4-byte scale / bias pieces) of its share of
//    as many of the CTA's items as the shared-memory ring holds — all of them
//    for the attention-output and MLP projections — and the input norm's
//    weights come in alongside: weights never depend on the preceding kernel,
//    so under programmatic dependent launch they stream in while it finishes.
//    The copies are spread over all nine warps (one warp alone cannot keep
//    enough requests in flight, and per-row bulk copies of a few hundred bytes
//    queue in the copy engine);
//  * after the wait, one global round trip for the input row (RMSNorm over
//    the whole row, GELU gating of the gate / up slices, or plain bf16) builds
//    the f16 B fragments of the CTA's chunks in shared memory;
//  * each warp owns whole items (8 groups = 8 MMA chains, two in flight),
//    applies the per-group affine fixup, issues the item nst places later into
//    the stage it just freed, and stores its 16 rows x T partial sums straight
//    to the item's chunk slice of the fp32 output (out[chunk][t][ld]); the
//    consumer adds the slices in chunk order, so the result is deterministic
//    and no counters, atomics or zeroing are needed;
//  * the shared-memory budget (~110 KB, 9 warps, <= 112 registers) leaves room
//    on each SM for the next kernel of the chain to start its own prefetch.
//
// Tensor-core math as in the other decode GEMVs: mma.sync m16n8k16, A = f16
// (1024 + code) built from the codes in registers, B = the input in f16, fp32
// accumulate; per group y += s * C + (b - 1024 s) * sum(x), C = sum (1024+q) x.
#include "internal.h"
#include "common.cuh"
#include "stage.cuh"
#include "qfrag.cuh"

namespace fmoe {
namespace rg {

constexpr int NW = 9;           // warps: every one consumes items and issues copies
constexpr int NTHR = NW * 32;
constexpr int CG = kRgChunkGroups;   // 64-column groups per item

__device__ __forceinline__ uint32_t ldg_u16(const bf16* p) {
  unsigned short r;
  asm volatile("ld.global.nc.u16 %0, [%1];\n" : "=h"(r) : "l"(p));
  return r;
}

__host__ __device__ __forceinline__ int gmax_of(const RgLayout& L) { return L.maxch * kRgChunkGroups; }

struct Item {
  int sg, c, tile, ng;  // segment, chunk, tile within the segment, groups in the chunk
};
__device__ __forceinline__ Item item_of(const RgArgs& a, int it) {
  const int c = it / a.tiles, tl = it - c * a.tiles;
  int sg = 0;
#pragma unroll
  for (int i = 1; i < kQgMaxSeg; ++i)
    if (i < a.nseg && tl >= a.seg[i].tile0) sg = i;
  const int ng = a.G - c * CG < CG ? a.G - c * CG : CG;
  return Item{sg, c, tl - a.seg[sg].tile0, ng};
}

// Copy helpers.  A stage = [16 rows][rs] codes (padded rows, conflict-free
// A-fragment reads) + [2 arrays][16 rows][8 groups] bf16 scales / biases.
__device__ __forceinline__ void cpa16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cpa4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;\n" ::"r"(dst), "l"(src) : "memory");
}
// The stage's barrier tracks this thread's earlier cp.async copies (counts as
// one of the expected arrivals once they land).
__device__ __forceinline__ void cpa_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];\n" ::"r"(smem_u32(bar)) : "memory");
}

// One warp issues item `it` into stage st: its 16 row pieces as 16-byte
// cp.async copies spread over the lanes, its scales / biases as 4-byte copies
// (K / 64 even; odd: plain loads and stores, then a second, plain arrival of
// every lane), then every lane's async arrival.  Any warp may issue any item:
// the stage's full barrier expects 32 (or 64) arrivals per phase, and
// issued[st] (the phase last issued) tells consumers which phase to wait for.
template <int BITS>
__device__ __forceinline__ void issue(const RgArgs& a, const RgLayout& L, uint8_t* smem, uint64_t* full,
                                      volatile int* issued, int it, int st, int lane) {
  constexpr int GB = 8 * BITS;  // bytes of one 64-column group in a row
  const Item q = item_of(a, it);
  const RgSeg& s = a.seg[q.sg];
  const int64_t rowbytes = (int64_t)a.K * BITS / 8;
  const int npr = q.ng * GB / 16;  // 16-byte pieces per row
  const uint8_t* src = s.w + (int64_t)q.tile * 16 * rowbytes + (int64_t)q.c * CG * GB;
  uint8_t* sb = smem + L.ring + (size_t)st * L.stage;
  const uint32_t dst = smem_u32(sb);
  // piece p = lane + 32 i -> (row r, piece o of the row), stepped without divisions
  int r = 0, o = lane;
  while (o >= npr) {
    o -= npr;
    ++r;
  }
  for (; r < 16;) {
    cpa16(dst + r * L.rs + o * 16, src + r * rowbytes + o * 16);
    o += 32;
    while (o >= npr) {
      o -= npr;
      ++r;
    }
  }
  // scales / biases of the item: lane = (array, row pair half): 16 rows x 2 arrays
  uint16_t* sc = reinterpret_cast<uint16_t*>(sb + L.soff);  // [2][16][8]
  const int64_t e0 = ((int64_t)q.tile * 16) * a.G + q.c * CG;
  if ((a.G & 1) == 0) {
    // 2 arrays x 16 rows x ceil(ng / 2) words; lane handles (array, row) = (lane >> 4, lane & 15)
    const int ar = lane >> 4, r = lane & 15;
    const bf16* base = (ar ? s.b : s.s) + e0 + (int64_t)r * a.G;
    const uint32_t d = smem_u32(sc + (ar * 16 + r) * CG);
    for (int w = 0; 2 * w < q.ng; ++w) cpa4(d + 4 * w, base + 2 * w);
    cpa_arrive(&full[st]);
  } else {
    const int ar = lane >> 4, r = lane & 15;
    const bf16* base = (ar ? s.b : s.s) + e0 + (int64_t)r * a.G;
    uint32_t v[CG];
#pragma unroll
    for (int k = 0; k < CG; ++k) v[k] = k < q.ng ? ldg_u16(base + k) : 0u;
    cpa_arrive(&full[st]);
#pragma unroll
    for (int k = 0; k < CG; ++k) sc[(ar * 16 + r) * CG + k] = (uint16_t)v[k];
    mbar_arrive(&full[st]);  // release: the stores above before the phase completes
  }
  __syncwarp();
  if (lane == 0) {
    __threadfence_block();
    *(issued + st) = it;  // the item now in flight in stage st
  }
}

// Bounded wait until item `it` has been issued into stage st.
__device__ __forceinline__ bool wait_issued(volatile int* issued, int st, int it, int* flag, int* status) {
  for (int i = 0; i < kMaxWaitIters; ++i) {
    if (*(issued + st) >= it) return true;
    if (*(volatile int*)flag) return false;
    __nanosleep(32);
  }
  if (status) atomicCAS(status, 0, 72);
  return false;
}

template <int BITS>
__global__ void __launch_bounds__(NTHR, 2) rgemv_kernel(const __grid_constant__ RgArgs a,
                                                          const __grid_constant__ RgLayout L) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar);
  volatile int* issued = reinterpret_cast<volatile int*>(smem + L.bar + L.nst * 8);
  uint4* frag = reinterpret_cast<uint4*>(smem + L.frag);
  float* xsum = reinterpret_cast<float*>(smem + L.xsum);
  float* rms = reinterpret_cast<float*>(smem + L.misc);
  int* flag = reinterpret_cast<int*>(smem + L.misc + 8 * 4);
  bf16* nw = reinterpret_cast<bf16*>(smem + L.normw);
  bf16* xs = reinterpret_cast<bf16*>(smem + L.xs);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int T = a.T, K = a.K;
  const int i0 = (int)((int64_t)a.items * blockIdx.x / gridDim.x);
  const int i1 = (int)((int64_t)a.items * (blockIdx.x + 1) / gridDim.x);
  const int n = i1 - i0;
  const int c_lo = i0 / a.tiles;
  const int c_hi = n > 0 ? (i1 - 1) / a.tiles : c_lo;
  const int g0 = c_lo * CG;                                                // first group of the CTA's chunks
  const int gn = (c_hi + 1) * CG < a.G ? (c_hi + 1) * CG - g0 : a.G - g0;  // groups prepared

  if (tid == 0) {
    const uint32_t cnt = (a.G & 1) ? 64u : 32u;
    for (int s = 0; s < L.nst; ++s) {
      mbar_init(&full[s], cnt);
      *(issued + s) = -1;
    }
    mbar_fence_init();
    flag[0] = 0;
  }
  __syncthreads();
  // ---- before the wait: every warp issues its share of the first items, the
  // input norm's weights come in alongside
  for (int j = warp; j < n && j < L.nst; j += NW) issue<BITS>(a, L, smem, full, issued, i0 + j, j, lane);
  const bool rmsn = a.in_kind == QG_IN_RMSNORM;
  uint4 nv = make_uint4(0, 0, 0, 0), nv2 = nv;  // gn * 8 <= 2 * NTHR pieces, in flight across the wait
  if (rmsn && tid < gn * 8) nv = ld_u4(a.norm_w + g0 * 64 + tid * 8);
  if (rmsn && tid + NTHR < gn * 8) nv2 = ld_u4(a.norm_w + g0 * 64 + (tid + NTHR) * 8);

  griddep_wait();  // the input belongs to earlier kernels
  griddep_launch_dependents();
  if (rmsn && tid < gn * 8) reinterpret_cast<uint4*>(nw)[tid] = nv;
  if (rmsn && tid + NTHR < gn * 8) reinterpret_cast<uint4*>(nw)[tid + NTHR] = nv2;
  // ---- input prologue: f16 B fragments + per-group sums of the CTA's chunks
  const int xst = gmax_of(L) * 64;  // raw-x stash stride per token (elements)
  if (a.in_kind == QG_IN_RMSNORM) {
    // every thread loads up to two 16-byte pieces of each token row (all loads
    // in flight together), keeps the CTA's groups raw in shared memory, and the
    // per-token sums of squares meet in a fixed-order reduction
    const int np = K / 8;  // pieces per row (<= 2 * NTHR)
    float* red = reinterpret_cast<float*>(smem + L.red);  // [8 tokens][NW warps]
    for (int tb = 0; tb < T; tb += 2) {  // two tokens per round trip
      uint4 wv[2][2];
#pragma unroll
      for (int u = 0; u < 2; ++u)
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int p = tid + h * NTHR, tk = tb + u;
          wv[u][h] = tk < T && p < np ? ld_u4(a.x + (int64_t)tk * a.ldx + p * 8) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int tk = tb + u;
        if (tk >= T) break;
        float ss = 0.f;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t ww[4] = {wv[u][h].x, wv[u][h].y, wv[u][h].z, wv[u][h].w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float lo = bf16lo(ww[e]), hi = bf16hi(ww[e]);
            ss = fmaf(lo, lo, fmaf(hi, hi, ss));
          }
          const int i = (tid + h * NTHR) * 8;
          if (i >= g0 * 64 && i < (g0 + gn) * 64) *reinterpret_cast<uint4*>(xs + tk * xst + i - g0 * 64) = wv[u][h];
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (lane == 0) red[tk * NW + warp] = ss;
      }
    }
    __syncthreads();
    if (tid < T) {
      float ss = 0.f;
      for (int w = 0; w < NW; ++w) ss += red[tid * NW + w];
      rms[tid] = rsqrtf(ss / (float)K + a.eps);
    }
    __syncthreads();
  }
  const int nitems = gn * T * 4;
  for (int item0 = 0; item0 < nitems; item0 += NTHR) {
    // every lane runs the shuffles below; items come in aligned groups of 4
    const int item = item0 + tid;
    const bool live = item < nitems;
    const int tq = item & 3, tk = live ? (item >> 2) % T : 0, gr = live ? (item >> 2) / T : 0;
    const int c0 = (g0 + gr) * 64 + 16 * tq;
    float v[16];
    if (!live) {
#pragma unroll
      for (int e = 0; e < 16; ++e) v[e] = 0.f;
    } else if (a.in_kind == QG_IN_GELU) {
      const float* gp = a.g + (int64_t)tk * a.ldgu + c0;
      const float* up = a.u + (int64_t)tk * a.ldgu + c0;
      float gs[16], us[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) gs[e] = us[e] = 0.f;
      for (int pp = 0; pp < a.gu_parts; ++pp) {  // partial slices in order; a slice's 8 loads in flight together
        float4 gg[4], uu[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          gg[e] = __ldcg(reinterpret_cast<const float4*>(gp + pp * a.gu_part_stride + 4 * e));
          uu[e] = __ldcg(reinterpret_cast<const float4*>(up + pp * a.gu_part_stride + 4 * e));
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          gs[4 * e] += gg[e].x, gs[4 * e + 1] += gg[e].y, gs[4 * e + 2] += gg[e].z, gs[4 * e + 3] += gg[e].w;
          us[4 * e] += uu[e].x, us[4 * e + 1] += uu[e].y, us[4 * e + 2] += uu[e].z, us[4 * e + 3] += uu[e].w;
        }
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) v[e] = round_bf(gelu_tanh(round_bf(gs[e])) * round_bf(us[e]));
    } else {
      uint4 w0, w1;
      if (a.in_kind == QG_IN_RMSNORM) {
        const bf16* xr = xs + tk * xst + gr * 64 + 16 * tq;
        w0 = *reinterpret_cast<const uint4*>(xr);
        w1 = *reinterpret_cast<const uint4*>(xr + 8);
      } else {
        const bf16* xr = a.x + (int64_t)tk * a.ldx + c0;
        w0 = ld_u4(xr);
        w1 = ld_u4(xr + 8);
      }
      const uint32_t ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[2 * e] = bf16lo(ww[e]);
        v[2 * e + 1] = bf16hi(ww[e]);
      }
      if (a.in_kind == QG_IN_RMSNORM) {
        const float r = rms[tk];
        const bf16* nr = nw + gr * 64 + 16 * tq;
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = round_bf(v[e] * r * bf2f(nr[e]));
      }
    }
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      v[e] = f16r(v[e]);
      s += v[e];
    }
    uint32_t b[8];
    make_b_frags<BITS>(v, b);
    if (live) {
      uint4* dst = frag + ((int64_t)gr * 4 * T + 4 * tk + tq) * 2;
      dst[0] = make_uint4(b[0], b[1], b[2], b[3]);
      dst[1] = make_uint4(b[4], b[5], b[6], b[7]);
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (live && tq == 0) xsum[gr * 8 + tk] = s;
  }
  for (int i = tid; i < gn * 8; i += NTHR)
    if ((i & 7) >= T) xsum[i] = 0.f;
  __syncthreads();


  // ---- consumers: warp w owns the CTA's items w, w + NW, ...; after an item
  // it issues the item nst places later into the stage it just freed
  for (int j = warp; j < n; j += NW) {
    const int st = j % L.nst;
    const Item q = item_of(a, i0 + j);
    const RgSeg& sg = a.seg[q.sg];
    // the stage serves items j - nst, j, j + nst ...: wait until item j is
    // issued (its previous phase is then complete), then for its bytes
    if (!wait_issued(issued, st, i0 + j, flag, a.status)) *(volatile int*)flag = 1;
    if (*(volatile int*)flag) break;
    if (!mbar_wait(&full[st], (uint32_t)(j / L.nst) & 1u, a.status, 71)) *(volatile int*)flag = 1;
    if (*(volatile int*)flag) break;
    const uint8_t* sb = smem + L.ring + (size_t)st * L.stage;
    const uint8_t* sc = sb + L.soff;  // [2][16][8] bf16
    const uint4 s_lo = *reinterpret_cast<const uint4*>(sc + g * 16);
    const uint4 s_hi = *reinterpret_cast<const uint4*>(sc + (g + 8) * 16);
    const uint4 b_lo = *reinterpret_cast<const uint4*>(sc + (16 + g) * 16);
    const uint4 b_hi = *reinterpret_cast<const uint4*>(sc + (24 + g) * 16);
    const uint32_t sl[4] = {s_lo.x, s_lo.y, s_lo.z, s_lo.w}, sh[4] = {s_hi.x, s_hi.y, s_hi.z, s_hi.w};
    const uint32_t bl[4] = {b_lo.x, b_lo.y, b_lo.z, b_lo.w}, bh[4] = {b_hi.x, b_hi.y, b_hi.z, b_hi.w};
    const uint8_t* rbase = sb + g * L.rs + t * (2 * BITS);
    const int grb = (q.c - c_lo) * CG;  // the item's first group among the prepared ones
    float y[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int gl = 0; gl < CG; gl += 2) {
      if (gl >= q.ng) break;
      // per group two accumulators (MMAs 0, 2 and 1, 3): four short chains in flight
      float cc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      float cd[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
      float q0[2] = {0.f, 0.f}, q1[2] = {0.f, 0.f};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (gl + h >= q.ng) break;
        const int gr = grb + gl + h;
        uint4 b0 = make_uint4(0, 0, 0, 0), b1 = b0;
        if (g < T) {
          const uint4* fp = frag + ((int64_t)gr * 4 * T + lane) * 2;
          b0 = fp[0];
          b1 = fp[1];
        }
        q0[h] = xsum[gr * 8 + 2 * t];
        q1[h] = xsum[gr * 8 + 2 * t + 1];
        const uint32_t bb0[4] = {b0.x, b0.y, b0.z, b0.w}, bb1[4] = {b1.x, b1.y, b1.z, b1.w};
        const uint8_t* rl = rbase + (gl + h) * (8 * BITS);
        uint32_t af[4][4];
        load_a_frags<BITS>(rl, rl + 8 * L.rs, af);
#pragma unroll
        for (int jj = 0; jj < 4; jj += 2) {
          mma16816_f16(cc[h], af[jj][0], af[jj][1], af[jj][2], af[jj][3], bb0[jj], bb1[jj]);
          mma16816_f16(cd[h], af[jj + 1][0], af[jj + 1][1], af[jj + 1][2], af[jj + 1][3], bb0[jj + 1], bb1[jj + 1]);
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int e = 0; e < 4; ++e) cc[h][e] += cd[h][e];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        if (gl + h >= q.ng) break;
        const int e = gl + h, w = e >> 1, sft = (e & 1) * 16;
        const float s0 = __uint_as_float(((sl[w] >> sft) & 0xFFFFu) << 16);
        const float s1 = __uint_as_float(((sh[w] >> sft) & 0xFFFFu) << 16);
        const float o0 = fmaf(-1024.f, s0, __uint_as_float(((bl[w] >> sft) & 0xFFFFu) << 16));
        const float o1 = fmaf(-1024.f, s1, __uint_as_float(((bh[w] >> sft) & 0xFFFFu) << 16));
        y[0] += fmaf(s0, cc[h][0], o0 * q0[h]);
        y[1] += fmaf(s0, cc[h][1], o0 * q1[h]);
        y[2] += fmaf(s1, cc[h][2], o1 * q0[h]);
        y[3] += fmaf(s1, cc[h][3], o1 * q1[h]);
      }
    }
    __syncwarp();  // every lane is done with the stage
    if (j + L.nst < n) issue<BITS>(a, L, smem, full, issued, i0 + j + L.nst, st, lane);
    // the item's partial sums: rows g / g + 8, tokens 2t / 2t + 1, chunk slice q.c
    float* out = sg.out + (int64_t)q.c * sg.pstride + sg.col0 + q.tile * 16 + g;
    if (2 * t < T) {
      out[(int64_t)(2 * t) * sg.ld] = y[0];
      out[(int64_t)(2 * t) * sg.ld + 8] = y[2];
    }
    if (2 * t + 1 < T) {
      out[(int64_t)(2 * t + 1) * sg.ld] = y[1];
      out[(int64_t)(2 * t + 1) * sg.ld + 8] = y[3];
    }
  }
  // copies still in flight (a wait gave up) must land before the CTA exits
  if (*(volatile int*)flag) asm volatile("cp.async.wait_all;\n" ::: "memory");
}

}  // namespace rg

// ---------------------------------------------------------------------------

int rgemv_plan(RgArgs& a, int bits, RgLayout* L, int smem_budget) {
  const int K = a.K;
  if (bits != 4 && bits != 6 && bits != 8) return set_error(FMOE_ERR_UNSUPPORTED, "rgemv: bits %d", bits);
  if (K % 64 || K <= 0 || a.T < 1 || a.T > 8 || (a.in_kind == QG_IN_RMSNORM && K > 16 * rg::NTHR))
    return set_error(FMOE_ERR_UNSUPPORTED, "rgemv: K %d (multiple of 64; <= %d with RMSNorm), T %d (1..8)", K,
                     16 * rg::NTHR, a.T);
  if (a.nseg < 1 || a.nseg > kQgMaxSeg) return set_error(FMOE_ERR_INVALID, "rgemv: %d segments", a.nseg);
  if (a.in_kind == QG_IN_RMSNORM && (!a.norm_w || !aligned(a.norm_w, 16) || !aligned(a.x, 16) || a.ldx % 8))
    return set_error(FMOE_ERR_ALIGN, "rgemv: input / norm weights not 16-byte aligned");
  a.G = K / 64;
  a.nck = (a.G + kRgChunkGroups - 1) / kRgChunkGroups;
  int tiles = 0;
  for (int i = 0; i < a.nseg; ++i) {
    RgSeg& s = a.seg[i];
    if (s.rows % 16 || s.rows <= 0) return set_error(FMOE_ERR_UNSUPPORTED, "rgemv: rows %d not a multiple of 16", s.rows);
    if (!s.w || !s.s || !s.b || !s.out || !aligned(s.w, 16))
      return set_error(FMOE_ERR_ALIGN, "rgemv: segment %d pointers null or codes not 16-byte aligned", i);
    s.tile0 = tiles;
    s.pstride = (int64_t)a.T * s.ld;
    tiles += s.rows / 16;
  }
  a.tiles = tiles;
  a.items = tiles * a.nck;
  const int grid = a.items < kNumSMs ? a.items : kNumSMs;
  // chunks any CTA spans
  int maxch = 1, per = 0;
  for (int b = 0; b < grid; ++b) {
    const int i0 = (int)((int64_t)a.items * b / grid), i1 = (int)((int64_t)a.items * (b + 1) / grid);
    if (i1 > i0) {
      const int ch = (i1 - 1) / tiles - i0 / tiles + 1;
      maxch = ch > maxch ? ch : maxch;
    }
    per = i1 - i0 > per ? i1 - i0 : per;
  }
  if (maxch > kRgMaxChunks)
    return set_error(FMOE_ERR_UNSUPPORTED, "rgemv: %d items over %d CTAs span %d chunks (max %d)", a.items, grid,
                     maxch, kRgMaxChunks);
  const int gb = 8 * bits;
  L->rs = qgemv_row_stride(kRgChunkGroups * gb, bits);
  L->soff = 16 * L->rs;
  L->stage = (int)align_up((size_t)L->soff + 2 * 16 * kRgChunkGroups * 2, 128);
  const int T = a.T, gmax = maxch * kRgChunkGroups;
  L->maxch = maxch;
  size_t off = 0;
  L->frag = (int)off;
  off += align_up((size_t)gmax * 4 * T * 32, 128);
  L->xsum = (int)off;
  off += align_up((size_t)gmax * 8 * 4, 128);
  L->misc = (int)off;
  off += 128;
  L->normw = (int)off;
  off += a.in_kind == QG_IN_RMSNORM ? align_up((size_t)gmax * 64 * 2, 128) : 0;
  L->xs = (int)off;
  off += a.in_kind == QG_IN_RMSNORM ? align_up((size_t)T * gmax * 64 * 2, 128) : 0;
  L->red = (int)off;
  off += align_up((size_t)8 * rg::NW * 4, 128);
  const size_t fixed = off;
  int nst = (int)(((size_t)smem_budget - fixed - 256) / ((size_t)L->stage + 16));
  if (nst > per) nst = per;
  if (nst < 2) nst = 2;
  if (fixed + 256 + (size_t)nst * (L->stage + 16) > (size_t)smem_budget && smem_budget < 220 * 1024)
    return rgemv_plan(a, bits, L, 220 * 1024);
  if (fixed + 256 + (size_t)nst * (L->stage + 16) > 220 * 1024)
    return set_error(FMOE_ERR_UNSUPPORTED, "rgemv: K %d, T %d exceed shared memory", K, T);
  L->nst = nst;
  L->bar = (int)off;  // nst full barriers, then nst "item issued" words
  off += align_up((size_t)nst * 12, 128);
  L->ring = (int)off;
  off += (size_t)nst * L->stage;
  L->bytes = (int)off;
  L->grid = grid;
  return FMOE_OK;
}

template <int BITS>
static int launch_rgemv_t(const RgArgs& a, const RgLayout& L, bool pdl, cudaStream_t st) {
  static int attr_dev = -1;
  int dev = 0;
  cudaGetDevice(&dev);
  if (attr_dev != dev) {
    cudaFuncSetAttribute(rg::rgemv_kernel<BITS>, cudaFuncAttributeMaxDynamicSharedMemorySize, 220 * 1024);
    attr_dev = dev;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(L.grid);
  cfg.blockDim = dim3(rg::NTHR);
  cfg.dynamicSmemBytes = L.bytes;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  ProfScope prof_(BITS == 4 ? "rgemv_kernel<4>" : BITS == 6 ? "rgemv_kernel<6>" : "rgemv_kernel<8>", st);
  cudaLaunchKernelEx(&cfg, rg::rgemv_kernel<BITS>, a, L);
  return check_launch("rgemv_kernel");
}

int launch_rgemv(const RgArgs& a, const RgLayout& L, int bits, bool pdl, cudaStream_t st) {
  if (a.items == 0) return FMOE_OK;
  if (bits == 4) return launch_rgemv_t<4>(a, L, pdl, st);
  if (bits == 6) return launch_rgemv_t<6>(a, L, pdl, st);
  return launch_rgemv_t<8>(a, L, pdl, st);
}

}  // namespace fmoe
