// Routed-expert kernels for decode-sized token counts (the GEMV form).
//
//   route_build  ids [T, k]            -> per-expert pair lists (device-side
//                                         replacement of the host sync + sort +
//                                         dedup at src/model/moe.rs:355-380)
//   gate_up      x, experts            -> act[pair] = bf16(gelu_tanh(bf16(g)) * bf16(u))
//                                         (src/model/moe.rs:428-437)
//   down         act, weights, experts -> y[t] = sum_j w[t,j] * down_e(act)
//                                         (src/model/moe.rs:438-453)
//
// Work is organised expert-major: every selected expert's weights are
// streamed from HBM once per call no matter how many tokens chose it.  All
// operands of a CTA are staged in shared memory up front (stage.cuh).
#include "internal.h"
#include "gemv.cuh"
#include "route.cuh"
#include "stage.cuh"

namespace fmoe {

constexpr int kRouteWarps = 8;

__global__ void __launch_bounds__(kRouteWarps * 32)
    route_build_kernel(const int32_t* __restrict__ ids, int P, int first, int E, int32_t* __restrict__ start,
                       int32_t* __restrict__ pairs, int32_t* __restrict__ unique, int32_t* __restrict__ num_unique,
                       int4* __restrict__ work, int work_len) {
  extern __shared__ int sm[];
  route_build_block(ids, P, first, E, start, pairs, unique, num_unique, work, work_len, sm);
}

// ---------------------------------------------------------------------------
// gate_up: CTA = (16-row tile of the intermediate dim, one selected expert).
// At CTA start one warp issues TMA bulk copies of the whole working set — the
// 16 gate rows and 16 up rows (~45 KB at H = 2816, one copy per row), the
// tile's four 16-row scale/bias blocks and the x rows of up to 8 of the
// expert's pairs — all tracked by one mbarrier.  The bf16 scales/biases are
// then turned into per-(row, group) fp32 pairs (scale, bias - 128*scale): the
// constants of the affine fixup y += scale*C + (bias - 128*scale)*sum(x).
// kGuWarps warps split the hidden dim into contiguous group ranges; gate and
// up share the x fragments; the warps' partial sums meet in shared memory
// (overlaid on the consumed raw-scale / x area) for the GELU epilogue.
constexpr int kGuWarps = 8;

struct GuLayout {
  int RS, XS;
  size_t f_off, s_off, x_off, bytes;
};
__host__ __device__ inline GuLayout gu_layout(int H, int nvmax) {
  GuLayout L;
  const int G = H / 64;
  L.RS = smem_stride(H / 2, 8);
  L.XS = smem_stride(H * 2, 16);
  L.f_off = 2 * 16 * (size_t)L.RS;                          // float2 [2][16][G]
  L.s_off = align16(L.f_off + 2 * 16 * (size_t)G * sizeof(float2));  // raw bf16 [4][16][G]
  L.x_off = align16(L.s_off + 4 * 16 * (size_t)G * 2);      // x [nvmax][XS]
  size_t end = L.x_off + (size_t)nvmax * L.XS;
  const size_t red_end = L.s_off + sizeof(float) * kGuWarps * 2 * 16 * 8;  // reduction overlay
  L.bytes = end > red_end ? end : red_end;
  return L;
}

// fix[i] = (scale, bias - off*scale) from raw bf16 scales / biases in shared memory.
__device__ __forceinline__ void make_fixup(float2* fix, const bf16* sc, const bf16* bi, int n, float off, int tid,
                                           int nthr) {
  for (int i = tid; i < n; i += nthr) {
    const float s = __bfloat162float(sc[i]);
    fix[i] = make_float2(s, fmaf(-off, s, __bfloat162float(bi[i])));
  }
}

// y[4] += s*C + b'*xs for the lane's rows g (fix_lo) and g+8 (fix_hi).
__device__ __forceinline__ void apply_fix(float (&y)[4], const float (&c)[4], const float (&xs)[4], float2 lo,
                                          float2 hi) {
  y[0] = fmaf(lo.x, c[0], fmaf(lo.y, xs[0], y[0]));
  y[1] = fmaf(lo.x, c[1], fmaf(lo.y, xs[1], y[1]));
  y[2] = fmaf(hi.x, c[2], fmaf(hi.y, xs[2], y[2]));
  y[3] = fmaf(hi.x, c[3], fmaf(hi.y, xs[3], y[3]));
}

// Warp 0: bulk-copy the x rows of pairs [p0, p0 + nv) (lanes `lane0`.. issue
// them), the caller having armed the barrier for these bytes.
__device__ __forceinline__ void bulk_x_rows(uint8_t* xsm, int XS, const bf16* x, int H, const int32_t* pairs, int p0,
                                            int nv, int k, int lane, int lane0, uint64_t* bar) {
  for (int n = lane - lane0; n >= 0 && n < nv; n += 32)
    bulk_g2s(xsm + n * XS, x + (int64_t)(pairs[p0 + n] / k) * H, H * 2, bar);
}

__global__ void __launch_bounds__(kGuWarps * 32, 3)
    moe_gate_up_kernel(const bf16* __restrict__ x, int k, ExpertsDev ex, const int4* __restrict__ work,
                       const int32_t* __restrict__ pairs, bf16* __restrict__ act, int nvmax, int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar;
  griddep_wait();  // routing lists come from the preceding router kernel
  griddep_launch_dependents();
  const int4 wk = work[blockIdx.y];
  if (wk.z == 0) return;
  const int e = wk.x, pbeg = wk.y, np = wk.z;
  const int H = ex.H, I = ex.I, G = H / 64;
  const GuLayout L = gu_layout(H, nvmax);
  const int RB = H / 2, RS = L.RS;
  uint8_t* wsm = smem;                                      // [2][16][RS]
  float2* fix = reinterpret_cast<float2*>(smem + L.f_off);  // [2][16][G]
  bf16* raw = reinterpret_cast<bf16*>(smem + L.s_off);      // [4][16][G]: gs, gb, us, ub
  uint8_t* xsm = smem + L.x_off;                            // [nvmax][XS]
  float* red = reinterpret_cast<float*>(smem + L.s_off);    // [kGuWarps][2][16][8] after use
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int row0 = blockIdx.x * 16;
  const uint8_t* eb = expert_base(ex, e);
  const int gbeg = G * warp / kGuWarps, gend = G * (warp + 1) / kGuWarps;

  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  int nv = min(nvmax, np);
  if (warp == 0) {
    const int sb = 16 * G * 2;  // one 16-row scale block
    if (lane == 0) mbar_arrive_expect_tx(&bar, 32u * RB + 4u * sb + (uint32_t)nv * H * 2);
    __syncwarp();
    {  // lane l: weight row l (gate rows 0..15, up rows 16..31)
      const int mat = lane >> 4, r = lane & 15;
      bulk_g2s(wsm + lane * RS, eb + ex.off[mat ? 3 : 0] + (int64_t)(row0 + r) * RB, RB, &bar);
    }
    if (lane < 4) {
      const int off = lane == 0 ? ex.off[1] : lane == 1 ? ex.off[2] : lane == 2 ? ex.off[4] : ex.off[5];
      bulk_g2s(reinterpret_cast<uint8_t*>(raw) + lane * sb, eb + off + (int64_t)row0 * G * 2, sb, &bar);
    }
    bulk_x_rows(xsm, L.XS, x, H, pairs, pbeg, nv, k, lane, 4, &bar);
  }
  uint32_t phase = 0;
  if (!mbar_wait(&bar, phase, status, 1)) return;
  phase ^= 1;
  make_fixup(fix, raw, raw + 16 * G, 16 * G, 128.0f, threadIdx.x, blockDim.x);
  make_fixup(fix + 16 * G, raw + 32 * G, raw + 48 * G, 16 * G, 128.0f, threadIdx.x, blockDim.x);
  __syncthreads();

  const uint8_t* wg = wsm;
  const uint8_t* wu = wsm + 16 * RS;
  const float2* fg = fix;
  const float2* fu = fix + 16 * G;
  for (int c0 = 0; c0 < np; c0 += nvmax) {
    nv = min(nvmax, np - c0);
    if (c0 > 0) {
      __syncthreads();  // the previous chunk's reduction overlay is no longer read
      if (warp == 0) {
        if (lane == 0) mbar_arrive_expect_tx(&bar, (uint32_t)nv * H * 2);
        __syncwarp();
        bulk_x_rows(xsm, L.XS, x, H, pairs, pbeg + c0, nv, k, lane, 0, &bar);
      }
      if (!mbar_wait(&bar, phase, status, 2)) return;
      phase ^= 1;
    }
    {  // nvmax <= 8: the chunk is one 8-column MMA block
      float yg[4] = {0.f, 0.f, 0.f, 0.f}, yu[4] = {0.f, 0.f, 0.f, 0.f};
      for (int gi = gbeg; gi < gend; ++gi) {
        const BFrag4 b = stage_bfrag4(xsm, L.XS, nv, gi, g, t);
        const uint2 gl = lds_u2(wg + g * RS + gi * 32 + 8 * t);
        const uint2 gh = lds_u2(wg + (g + 8) * RS + gi * 32 + 8 * t);
        const uint2 ul = lds_u2(wu + g * RS + gi * 32 + 8 * t);
        const uint2 uh = lds_u2(wu + (g + 8) * RS + gi * 32 + 8 * t);
        float cg[4] = {0.f, 0.f, 0.f, 0.f}, cu[4] = {0.f, 0.f, 0.f, 0.f}, xs[4] = {0.f, 0.f, 0.f, 0.f};
        mma_group_q4(cg, gl, gh, b);
        mma_group_q4(cu, ul, uh, b);
        mma_group_ones(xs, b);
        apply_fix(yg, cg, xs, fg[g * G + gi], fg[(g + 8) * G + gi]);
        apply_fix(yu, cu, xs, fu[g * G + gi], fu[(g + 8) * G + gi]);
      }
      __syncthreads();  // x rows are read by every warp before the overlay is written
      float* rw = red + warp * 256;  // [2][16][8]
      rw[g * 8 + 2 * t] = yg[0];
      rw[g * 8 + 2 * t + 1] = yg[1];
      rw[(g + 8) * 8 + 2 * t] = yg[2];
      rw[(g + 8) * 8 + 2 * t + 1] = yg[3];
      rw[128 + g * 8 + 2 * t] = yu[0];
      rw[128 + g * 8 + 2 * t + 1] = yu[1];
      rw[128 + (g + 8) * 8 + 2 * t] = yu[2];
      rw[128 + (g + 8) * 8 + 2 * t + 1] = yu[3];
      __syncthreads();
      if (threadIdx.x < 128) {
        const int c = threadIdx.x >> 4, r = threadIdx.x & 15;
        if (c < nv) {
          float sg = 0.f, su = 0.f;
#pragma unroll
          for (int w = 0; w < kGuWarps; ++w) {
            sg += red[w * 256 + r * 8 + c];
            su += red[w * 256 + 128 + r * 8 + c];
          }
          const float gv = round_bf(sg), uv = round_bf(su);
          act[(int64_t)(pbeg + c0 + c) * I + row0 + r] = __float2bfloat16_rn(gelu_tanh(gv) * uv);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// down + combine: CTA = (16-row tile of the hidden dim, group of kDnSlots
// selected experts); each expert slot is served by two warps that split its
// intermediate dim (K) in halves.  Per slot, lane 0 of the first warp issues
// TMA bulk copies of the contiguous 16-row down tile (5.5 KB at I = 704) and
// its two scale/bias blocks before the kernel waits on the preceding gate_up
// kernel (the work list was complete before gate_up ran), then the slot's act
// rows.  Per-warp fp32 sums per (token, row) are added in warp order; with
// more than one expert group the groups' partials go through the workspace
// and the last CTA of each row tile (completion counter) adds them in group
// order, so the result is deterministic.  Slots per CTA: 8 up to 16 tokens; 4
// above (the per-warp (token, row) sums grow with T: at 32 tokens a CTA of 8
// slots would no longer leave room for a second on its SM).
constexpr int kDnSlots = 8;
constexpr int kDnPairs = 2;
inline int dn_slots(int64_t T) { return T > 16 ? 4 : kDnSlots; }

struct DnLayout {
  int RS, AS, gmax;
  size_t slot_bytes, s_off, f_off, a_off, y_off, bytes;
};
__host__ __device__ inline DnLayout dn_layout(int I, int T, int slots) {
  DnLayout L;
  const int Gi = I / 64;
  L.gmax = (Gi + 1) / 2;                                           // groups per half
  L.RS = I / 2;                                                    // rows stay contiguous: one copy per tile
  L.AS = smem_stride(I * 2, 16);
  L.s_off = 16 * (size_t)L.RS;                                     // raw bf16 [2][16][Gi]
  L.f_off = align16(L.s_off + 2 * 16 * (size_t)Gi * 2);            // float2 [2 halves][16][gmax]
  L.a_off = align16(L.f_off + 2 * 16 * (size_t)L.gmax * sizeof(float2));
  L.slot_bytes = align16(L.a_off + (size_t)kDnPairs * L.AS);
  L.y_off = slots * L.slot_bytes;
  L.bytes = L.y_off + sizeof(float) * 2 * slots * (size_t)T * 16;
  return L;
}

template <int SLOTS>
__global__ void __launch_bounds__(2 * SLOTS * 32, SLOTS == 8 ? 2 : 3)
    moe_down_kernel(const bf16* __restrict__ act, int T, int k, const float* __restrict__ wts, ExpertsDev ex,
                    const int4* __restrict__ work, int work_len, const int32_t* __restrict__ pairs,
                    float* __restrict__ part, unsigned* __restrict__ tile_ctr, bf16* __restrict__ y,
                    float* __restrict__ y32, int* status) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int kDnWarps = 2 * SLOTS;
  __shared__ __align__(8) uint64_t bars[SLOTS][2];  // [slot][0: weights + scales, 1: act rows]
  __shared__ int s_last;
  const int H = ex.H, I = ex.I, Gi = I / 64;
  const DnLayout L = dn_layout(I, T, SLOTS);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int half = warp & 1, slot = warp >> 1;
  const int gh0 = half ? L.gmax : 0, gh1 = half ? Gi : L.gmax, ng = gh1 - gh0;
  const int row0 = blockIdx.x * 16;
  uint8_t* ss = smem + slot * L.slot_bytes;
  const bf16* raw = reinterpret_cast<const bf16*>(ss + L.s_off);
  float2* fix = reinterpret_cast<float2*>(ss + L.f_off) + half * 16 * L.gmax;  // [16][gmax]
  uint8_t* asm_ = ss + L.a_off;
  float* ysm = reinterpret_cast<float*>(smem + L.y_off);  // [kDnWarps][T][16]
  uint64_t* bw = &bars[slot][0];
  uint64_t* ba = &bars[slot][1];
  const int u = blockIdx.y * SLOTS + slot;
  const int RB = I / 2, sb = 16 * Gi * 2;
  const bool leader = half == 0 && lane == 0;
  if (threadIdx.x < SLOTS * 2) {
    mbar_init(&bars[threadIdx.x >> 1][threadIdx.x & 1], 1);
    mbar_fence_init();
  }
  __syncthreads();
  // The work list was complete before the preceding kernel ran (it waited on
  // the router), so it can be read before griddep_wait.
  const int4 wk = u < work_len ? work[u] : make_int4(0, 0, 0, 0);
  const int pbeg = wk.y, np = wk.z;
  if (np > 0 && leader) {
    const uint8_t* eb = expert_base(ex, wk.x);
    mbar_arrive_expect_tx(bw, 16u * RB + 2u * sb);
    bulk_g2s(ss, eb + ex.off[6] + (int64_t)row0 * RB, 16 * RB, bw);
    bulk_g2s(ss + L.s_off, eb + ex.off[7] + (int64_t)row0 * Gi * 2, sb, bw);
    bulk_g2s(ss + L.s_off + sb, eb + ex.off[8] + (int64_t)row0 * Gi * 2, sb, bw);
  }
  griddep_wait();  // act comes from the preceding gate_up kernel
  griddep_launch_dependents();
  for (int i = threadIdx.x; i < kDnWarps * T * 16; i += blockDim.x) ysm[i] = 0.f;
  __syncthreads();
  float* my = ysm + warp * T * 16;
  // Both warps of a slot run the same iterations (same np), so the named
  // barrier below is always reached by both; a timed-out wait only skips work.
  bool ok = true;
  uint32_t aphase = 0;
  for (int c0 = 0; c0 < np; c0 += kDnPairs) {
    const int nv = min(kDnPairs, np - c0);
    if (c0 > 0) asm volatile("bar.sync %0, 64;\n" ::"r"(1 + slot) : "memory");  // both warps done with the rows
    if (leader && ok) {
      mbar_arrive_expect_tx(ba, (uint32_t)nv * I * 2);
      for (int n = 0; n < nv; ++n) bulk_g2s(asm_ + n * L.AS, act + (int64_t)(pbeg + c0 + n) * I, I * 2, ba);
    }
    if (c0 == 0 && ok) {
      ok = mbar_wait(bw, 0, status, 11);
      if (ok) {
        for (int i = lane; i < 16 * ng; i += 32) {
          const int r = i / ng, j = i % ng;
          const float s = __bfloat162float(raw[r * Gi + gh0 + j]);
          fix[r * L.gmax + j] = make_float2(s, fmaf(-128.0f, s, __bfloat162float(raw[16 * Gi + r * Gi + gh0 + j])));
        }
      }
      __syncwarp();
    }
    if (ok) ok = mbar_wait(ba, aphase, status, 12);
    aphase ^= 1;
    if (!ok) continue;
    float d[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < ng; ++j) {
      const BFrag4 b = stage_bfrag4(asm_, L.AS, nv, gh0 + j, g, t);
      const uint2 wl = lds_u2(ss + g * L.RS + (gh0 + j) * 32 + 8 * t);
      const uint2 wh = lds_u2(ss + (g + 8) * L.RS + (gh0 + j) * 32 + 8 * t);
      float c[4] = {0.f, 0.f, 0.f, 0.f}, xs[4] = {0.f, 0.f, 0.f, 0.f};
      mma_group_q4(c, wl, wh, b);
      mma_group_ones(xs, b);
      apply_fix(d, c, xs, fix[g * L.gmax + j], fix[(g + 8) * L.gmax + j]);
    }
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int col = 2 * t + j;
      if (col < nv) {
        const int p = pairs[pbeg + c0 + col];
        const int tok = p / k;
        const float wv = wts[p];
        // atomic only so that duplicate ids within a token stay correct
        atomicAdd(&my[tok * 16 + g], wv * d[j]);
        atomicAdd(&my[tok * 16 + g + 8], wv * d[2 + j]);
      }
    }
  }
  __syncthreads();
  const int ngroups = gridDim.y;
  if (ngroups == 1) {
    for (int i = threadIdx.x; i < T * 16; i += blockDim.x) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kDnWarps; ++w) s += ysm[w * T * 16 + i];
      const int64_t o = (int64_t)(i >> 4) * H + row0 + (i & 15);
      if (y32)
        y32[o] = s;
      else
        y[o] = __float2bfloat16_rn(s);
    }
    return;
  }
  for (int i = threadIdx.x; i < T * 16; i += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kDnWarps; ++w) s += ysm[w * T * 16 + i];
    part[((int64_t)blockIdx.y * T + (i >> 4)) * H + row0 + (i & 15)] = s;
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&tile_ctr[blockIdx.x], 1u) == (unsigned)ngroups - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = threadIdx.x; i < T * 16; i += blockDim.x) {
    float s = 0.f;
    for (int q = 0; q < ngroups; ++q) s += __ldcg(part + ((int64_t)q * T + (i >> 4)) * H + row0 + (i & 15));
    const int64_t o = (int64_t)(i >> 4) * H + row0 + (i & 15);
    if (y32)
      y32[o] = s;
    else
      y[o] = __float2bfloat16_rn(s);
  }
  if (threadIdx.x == 0) tile_ctr[blockIdx.x] = 0;
}

// ---------------------------------------------------------------------------
// host launchers

int down_groups(int64_t T, int k, int E) {
  const int64_t maxu = T * k < E ? T * k : E;
  const int slots = dn_slots(T);
  return (int)((maxu + slots - 1) / slots);
}

// ---------------------------------------------------------------------------
// The same lists for many pairs, spread over CTAs: units u = (CTA, warp) own
// consecutive chunks of kRbUnit pairs.  count: per-unit expert counts;
// scan (one CTA): per-expert totals -> start / unique / work, and each
// (unit, expert) count becomes that unit's first output slot; scatter: each
// warp places its chunk in index order.  The result is identical to
// route_build_block's (pairs ascending within an expert).
constexpr int kRbUnit = 256;  // pairs per warp
constexpr int kRbWarps = 8;
constexpr int64_t kRbSingleMax = 4096;  // up to this many pairs one CTA builds the lists

int64_t route_scratch_ints(int64_t P, int E) {
  return P <= kRbSingleMax ? 0 : ((P + kRbUnit - 1) / kRbUnit) * (int64_t)E;
}

__global__ void __launch_bounds__(kRbWarps * 32)
    route_count_kernel(const int32_t* __restrict__ ids, int P, int first, int E, int32_t* __restrict__ cnt) {
  extern __shared__ int wc[];  // [kRbWarps][E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kRbWarps * E; i += blockDim.x) wc[i] = 0;
  __syncthreads();
  const int u = blockIdx.x * kRbWarps + warp;
  const int pb = u * kRbUnit, pe = min(P, pb + kRbUnit);
  for (int p = pb + lane; p < pe; p += 32) {
    const int e = ids[p] - first;
    if (e >= 0 && e < E) atomicAdd(&wc[warp * E + e], 1);
  }
  __syncthreads();
  const int U = (P + kRbUnit - 1) / kRbUnit;
  for (int i = threadIdx.x; i < kRbWarps * E; i += blockDim.x) {
    const int uu = blockIdx.x * kRbWarps + i / E;
    if (uu < U) cnt[(int64_t)uu * E + i % E] = wc[i];
  }
}

__global__ void __launch_bounds__(1024)
    route_scan_kernel(int32_t* __restrict__ cnt, int U, int E, int32_t* __restrict__ start,
                      int32_t* __restrict__ unique, int32_t* __restrict__ num_unique, int4* __restrict__ work,
                      int work_len) {
  __shared__ int tot[1024];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int c = 0;
    for (int u = 0; u < U; ++u) c += cnt[(int64_t)u * E + e];
    tot[e] = c;
  }
  __syncthreads();
  if (warp == 0) {  // exclusive scan over experts, compaction of the non-empty ones
    int run = 0, urun = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int c = e < E ? tot[e] : 0;
      int incl = c, uincl = c > 0;
      for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, incl, o), b = __shfl_up_sync(0xffffffffu, uincl, o);
        if (lane >= o) {
          incl += a;
          uincl += b;
        }
      }
      if (e < E) {
        start[e] = run + incl - c;
        tot[e] = run + incl - c;
        if (c > 0) {
          unique[urun + uincl - 1] = e;
          if (urun + uincl - 1 < work_len) work[urun + uincl - 1] = make_int4(e, run + incl - c, c, 0);
        }
      }
      run += __shfl_sync(0xffffffffu, incl, 31);
      urun += __shfl_sync(0xffffffffu, uincl, 31);
    }
    if (lane == 0) {
      start[E] = run;
      *num_unique = urun;
    }
    for (int u = urun + lane; u < work_len; u += 32) work[u] = make_int4(0, 0, 0, 0);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {  // (unit, expert) first slots
    int o = tot[e];
    for (int u = 0; u < U; ++u) {
      const int c = cnt[(int64_t)u * E + e];
      cnt[(int64_t)u * E + e] = o;
      o += c;
    }
  }
}

__global__ void __launch_bounds__(kRbWarps * 32)
    route_scatter_kernel(const int32_t* __restrict__ ids, int P, int first, int E, const int32_t* __restrict__ off,
                         int32_t* __restrict__ pairs) {
  extern __shared__ int wo[];  // [kRbWarps][E] next slot per (warp, expert)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int U = (P + kRbUnit - 1) / kRbUnit;
  for (int i = threadIdx.x; i < kRbWarps * E; i += blockDim.x) {
    const int uu = blockIdx.x * kRbWarps + i / E;
    wo[i] = uu < U ? off[(int64_t)uu * E + i % E] : 0;
  }
  __syncthreads();
  const int u = blockIdx.x * kRbWarps + warp;
  const int pb = u * kRbUnit, pe = min(P, pb + kRbUnit);
  const unsigned lt = (1u << lane) - 1u;
  for (int p0 = pb; p0 < pe; p0 += 32) {
    const int p = p0 + lane;
    int e = -1;
    if (p < pe) {
      e = ids[p] - first;
      if (e < 0 || e >= E) e = -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0) pairs[wo[warp * E + e] + __popc(peers & lt)] = p;
    __syncwarp();
    if (e >= 0 && (peers & lt) == 0) wo[warp * E + e] += __popc(peers);
    __syncwarp();
  }
}

int launch_route_build(const int32_t* ids, int64_t P, const ExpertsDev& ex, const RouteMeta& m, cudaStream_t st) {
  if (P > kRbSingleMax && m.scratch && ex.E <= 1024) {
    const int U = (int)((P + kRbUnit - 1) / kRbUnit), blocks = (U + kRbWarps - 1) / kRbWarps;
    const size_t sm = sizeof(int) * (size_t)kRbWarps * ex.E;
    {
      ProfScope prof_("route_count_kernel", st);
      route_count_kernel<<<blocks, kRbWarps * 32, sm, st>>>(ids, (int)P, ex.first, ex.E, m.scratch);
    }
    int rc = check_launch("route_count_kernel");
    if (rc) return rc;
    {
      ProfScope prof_("route_scan_kernel", st);
      route_scan_kernel<<<1, 1024, 0, st>>>(m.scratch, U, ex.E, m.start, m.unique, m.num_unique, m.work, m.work_len);
    }
    if ((rc = check_launch("route_scan_kernel"))) return rc;
    {
      ProfScope prof_("route_scatter_kernel", st);
      route_scatter_kernel<<<blocks, kRbWarps * 32, sm, st>>>(ids, (int)P, ex.first, ex.E, m.scratch, m.pairs);
    }
    return check_launch("route_scatter_kernel");
  }
  const size_t smem = sizeof(int) * (size_t)(kRouteWarps + 1) * ex.E;
  if (smem > 200 * 1024) return set_error(FMOE_ERR_UNSUPPORTED, "route_build: %d experts too many", ex.E);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(route_build_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  {
    ProfScope prof_("route_build_kernel", st);
    route_build_kernel<<<1, kRouteWarps * 32, smem, st>>>(ids, (int)P, ex.first, ex.E, m.start, m.pairs, m.unique,
                                                           m.num_unique, m.work, m.work_len);
  }
  return check_launch("route_build_kernel");
}

static cudaLaunchConfig_t pdl_config(dim3 grid, dim3 block, size_t smem, cudaStream_t st, bool pdl,
                                     cudaLaunchAttribute* attr) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  return cfg;
}

int launch_moe_gate_up(const bf16* x, int64_t T, int k, const ExpertsDev& ex, const RouteMeta& m, bf16* act,
                       int* status, bool pdl, cudaStream_t st) {
  const int64_t pairs = T * k;
  const int maxu = m.work_len;
  (void)pairs;
  const int nvmax = (int)(T < 8 ? T : 8);
  const GuLayout L = gu_layout(ex.H, nvmax);
  if (L.bytes > 200 * 1024) return set_error(FMOE_ERR_UNSUPPORTED, "gate_up: hidden %d too large", ex.H);
  cudaFuncSetAttribute(moe_gate_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.bytes);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = pdl_config(dim3(ex.I / 16, maxu), dim3(kGuWarps * 32), L.bytes, st, pdl, attr);
  {
    ProfScope prof_("moe_gate_up_kernel", st);
    cudaLaunchKernelEx(&cfg, moe_gate_up_kernel, x, k, ex, (const int4*)m.work, (const int32_t*)m.pairs, act, nvmax,
                       status);
  }
  return check_launch("moe_gate_up_kernel");
}

int launch_moe_down(const bf16* act, int64_t T, int k, const float* wts, const ExpertsDev& ex, const RouteMeta& m,
                    float* part, unsigned* tile_ctr, bf16* y, int* status, bool pdl, cudaStream_t st, float* y32) {
  const int slots = dn_slots(T);
  const DnLayout L = dn_layout(ex.I, (int)T, slots);
  if (L.bytes > 227 * 1024)
    return set_error(FMOE_ERR_UNSUPPORTED, "down: T=%lld / I=%d exceed shared memory", (long long)T, ex.I);
  auto kern = slots == 8 ? moe_down_kernel<8> : moe_down_kernel<4>;
  cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.bytes);
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg =
      pdl_config(dim3(ex.H / 16, (m.work_len + slots - 1) / slots), dim3(2 * slots * 32), L.bytes, st, pdl, attr);
  {
    ProfScope prof_("moe_down_kernel", st);
    cudaLaunchKernelEx(&cfg, kern, act, (int)T, k, wts, ex, (const int4*)m.work, m.work_len,
                       (const int32_t*)m.pairs, part, tile_ctr, y, y32, status);
  }
  return check_launch("moe_down_kernel");
}

}  // namespace fmoe
