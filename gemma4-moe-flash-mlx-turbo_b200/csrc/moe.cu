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
// streamed from HBM once per call no matter how many tokens chose it.
#include "internal.h"
#include "gemv.cuh"

namespace fmoe {

// ---------------------------------------------------------------------------
// route_build: one CTA of kRouteWarps warps.  Pairs p = t*k + slot are split
// into kRouteWarps contiguous chunks; each warp counts its chunk per expert,
// offsets are (expert, warp)-major exclusive prefixes, and each warp scatters
// its chunk in index order (stable), so pairs[] is ascending within an expert.
constexpr int kRouteWarps = 8;

__global__ void __launch_bounds__(kRouteWarps * 32)
    route_build_kernel(const int32_t* __restrict__ ids, int P, int first, int E, int32_t* __restrict__ start,
                       int32_t* __restrict__ pairs, int32_t* __restrict__ unique, int32_t* __restrict__ num_unique) {
  extern __shared__ int sm[];
  int* wcnt = sm;                     // [kRouteWarps][E] counts, later offsets
  int* tot = sm + kRouteWarps * E;    // [E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < kRouteWarps * E; i += blockDim.x) wcnt[i] = 0;
  __syncthreads();
  const int chunk = (P + kRouteWarps - 1) / kRouteWarps;
  const int pb = warp * chunk, pe = min(P, pb + chunk);
  for (int p = pb + lane; p < pe; p += 32) {
    const int e = ids[p] - first;
    if (e >= 0 && e < E) atomicAdd(&wcnt[warp * E + e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int s = 0;
    for (int w = 0; w < kRouteWarps; ++w) s += wcnt[w * E + e];
    tot[e] = s;
  }
  __syncthreads();
  if (warp == 0) {
    // Exclusive scan of tot[] and compaction of non-empty experts, 32 experts per step.
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
        if (c > 0) unique[urun + uincl - 1] = e;
      }
      run += __shfl_sync(0xffffffffu, incl, 31);
      urun += __shfl_sync(0xffffffffu, uincl, 31);
    }
    if (lane == 0) {
      start[E] = run;
      *num_unique = urun;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int o = tot[e];
    for (int w = 0; w < kRouteWarps; ++w) {
      const int c = wcnt[w * E + e];
      wcnt[w * E + e] = o;
      o += c;
    }
  }
  __syncthreads();
  const unsigned lt = (1u << lane) - 1u;
  for (int p0 = pb; p0 < pe; p0 += 32) {
    const int p = p0 + lane;
    int e = -1;
    if (p < pe) {
      e = ids[p] - first;
      if (e < 0 || e >= E) e = -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0) {
      const int base = wcnt[warp * E + e];
      pairs[base + __popc(peers & lt)] = p;
    }
    __syncwarp();
    if (e >= 0 && (peers & lt) == 0) wcnt[warp * E + e] += __popc(peers);
    __syncwarp();
  }
}

// ---------------------------------------------------------------------------
// gate_up: CTA = (16-row tile of the intermediate dim, one selected expert).
// kGuWarps warps split the hidden dim (64-wide groups, interleaved); each warp
// runs gate and up on the same x fragments; a CTA handles the expert's pairs
// 8 at a time.
constexpr int kGuWarps = 4;

__global__ void __launch_bounds__(kGuWarps * 32)
    moe_gate_up_kernel(const bf16* __restrict__ x, int k, ExpertsDev ex, const int32_t* __restrict__ start,
                       const int32_t* __restrict__ pairs, const int32_t* __restrict__ unique,
                       const int32_t* __restrict__ num_unique, bf16* __restrict__ act) {
  __shared__ float red[kGuWarps][2][16][8];
  const int u = blockIdx.y;
  if (u >= *num_unique) return;
  const int H = ex.H, I = ex.I, G = H / 64, wpr = H / 8;
  const int e = unique[u];
  const int pbeg = start[e], np = start[e + 1] - pbeg;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int row0 = blockIdx.x * 16;
  const uint8_t* eb = ex.base + (int64_t)e * ex.stride;
  const uint32_t* gw = reinterpret_cast<const uint32_t*>(eb + ex.off[0]);
  const bf16* gs = reinterpret_cast<const bf16*>(eb + ex.off[1]);
  const bf16* gb = reinterpret_cast<const bf16*>(eb + ex.off[2]);
  const uint32_t* uw = reinterpret_cast<const uint32_t*>(eb + ex.off[3]);
  const bf16* us = reinterpret_cast<const bf16*>(eb + ex.off[4]);
  const bf16* ub = reinterpret_cast<const bf16*>(eb + ex.off[5]);
  const int64_t rl = row0 + g, rh = row0 + g + 8;

  for (int c0 = 0; c0 < np; c0 += 8) {
    const int nv = min(8, np - c0);
    const bf16* xrow = nullptr;
    if (g < nv) xrow = x + (int64_t)(pairs[pbeg + c0 + g] / k) * H;
    float yg[4] = {0.f, 0.f, 0.f, 0.f}, yu[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
    for (int gi = warp; gi < G; gi += kGuWarps) {
      const uint2 gl = ldg_stream_u2(gw + rl * wpr + gi * 8 + 2 * t);
      const uint2 gh = ldg_stream_u2(gw + rh * wpr + gi * 8 + 2 * t);
      const uint2 ul = ldg_stream_u2(uw + rl * wpr + gi * 8 + 2 * t);
      const uint2 uh = ldg_stream_u2(uw + rh * wpr + gi * 8 + 2 * t);
      const float gsl = bfbits2f(ldg_u16(gs + rl * G + gi)), gbl = bfbits2f(ldg_u16(gb + rl * G + gi));
      const float gsh = bfbits2f(ldg_u16(gs + rh * G + gi)), gbh = bfbits2f(ldg_u16(gb + rh * G + gi));
      const float usl = bfbits2f(ldg_u16(us + rl * G + gi)), ubl = bfbits2f(ldg_u16(ub + rl * G + gi));
      const float ush = bfbits2f(ldg_u16(us + rh * G + gi)), ubh = bfbits2f(ldg_u16(ub + rh * G + gi));
      uint4 xl, xh;
      load_x16(xrow, gi, t, xl, xh);
      const BFrag4 b = make_bfrag4(xl, xh);
      float cg[4] = {0.f, 0.f, 0.f, 0.f}, cu[4] = {0.f, 0.f, 0.f, 0.f}, xs[4] = {0.f, 0.f, 0.f, 0.f};
      mma_group_q4(cg, gl, gh, b);
      mma_group_q4(cu, ul, uh, b);
      mma_group_ones(xs, b);
      affine_fixup(yg, cg, xs, gsl, gbl, gsh, gbh, 128.0f);
      affine_fixup(yu, cu, xs, usl, ubl, ush, ubh, 128.0f);
    }
    red[warp][0][g][2 * t] = yg[0];
    red[warp][0][g][2 * t + 1] = yg[1];
    red[warp][0][g + 8][2 * t] = yg[2];
    red[warp][0][g + 8][2 * t + 1] = yg[3];
    red[warp][1][g][2 * t] = yu[0];
    red[warp][1][g][2 * t + 1] = yu[1];
    red[warp][1][g + 8][2 * t] = yu[2];
    red[warp][1][g + 8][2 * t + 1] = yu[3];
    __syncthreads();
    for (int i = threadIdx.x; i < 128; i += blockDim.x) {
      const int c = i >> 4, r = i & 15;
      if (c < nv) {
        float sg = 0.f, su = 0.f;
#pragma unroll
        for (int w = 0; w < kGuWarps; ++w) {
          sg += red[w][0][r][c];
          su += red[w][1][r][c];
        }
        const float gv = round_bf(sg), uv = round_bf(su);
        act[(int64_t)(pbeg + c0 + c) * I + row0 + r] = __float2bfloat16_rn(gelu_tanh(gv) * uv);
      }
    }
    __syncthreads();
  }
}

// ---------------------------------------------------------------------------
// down + combine: CTA = 16-row tile of the hidden dim; kDnWarps warps take the
// selected experts round-robin; per-warp fp32 partial sums per (token, row)
// are added in warp order at the end (deterministic).
constexpr int kDnWarps = 8;

__global__ void __launch_bounds__(kDnWarps * 32)
    moe_down_kernel(const bf16* __restrict__ act, int T, int k, const float* __restrict__ wts, ExpertsDev ex,
                    const int32_t* __restrict__ start, const int32_t* __restrict__ pairs,
                    const int32_t* __restrict__ unique, const int32_t* __restrict__ num_unique,
                    bf16* __restrict__ y) {
  extern __shared__ float ysm[];  // [kDnWarps][T][16]
  const int H = ex.H, I = ex.I, G = I / 64, wpr = I / 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int row0 = blockIdx.x * 16;
  for (int i = threadIdx.x; i < kDnWarps * T * 16; i += blockDim.x) ysm[i] = 0.f;
  __syncthreads();
  const int U = *num_unique;
  float* my = ysm + warp * T * 16;
  const int64_t rl = row0 + g, rh = row0 + g + 8;
  for (int u = warp; u < U; u += kDnWarps) {
    const int e = unique[u];
    const int pbeg = start[e], np = start[e + 1] - pbeg;
    const uint8_t* eb = ex.base + (int64_t)e * ex.stride;
    const uint32_t* dw = reinterpret_cast<const uint32_t*>(eb + ex.off[6]);
    const bf16* ds = reinterpret_cast<const bf16*>(eb + ex.off[7]);
    const bf16* db = reinterpret_cast<const bf16*>(eb + ex.off[8]);
    for (int c0 = 0; c0 < np; c0 += 8) {
      const int nv = min(8, np - c0);
      const bf16* arow = g < nv ? act + (int64_t)(pbeg + c0 + g) * I : nullptr;
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
      for (int gi = 0; gi < G; ++gi) {
        const uint2 wl = ldg_stream_u2(dw + rl * wpr + gi * 8 + 2 * t);
        const uint2 wh = ldg_stream_u2(dw + rh * wpr + gi * 8 + 2 * t);
        const float sl = bfbits2f(ldg_u16(ds + rl * G + gi)), bl = bfbits2f(ldg_u16(db + rl * G + gi));
        const float sh = bfbits2f(ldg_u16(ds + rh * G + gi)), bh = bfbits2f(ldg_u16(db + rh * G + gi));
        uint4 xl, xh;
        load_x16(arow, gi, t, xl, xh);
        const BFrag4 b = make_bfrag4(xl, xh);
        float c[4] = {0.f, 0.f, 0.f, 0.f}, xs[4] = {0.f, 0.f, 0.f, 0.f};
        mma_group_q4(c, wl, wh, b);
        mma_group_ones(xs, b);
        affine_fixup(d, c, xs, sl, bl, sh, bh, 128.0f);
      }
      // d: (row g | g+8, chunk column 2t | 2t+1)
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
  }
  __syncthreads();
  for (int i = threadIdx.x; i < T * 16; i += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kDnWarps; ++w) s += ysm[w * T * 16 + i];
    y[(int64_t)(i >> 4) * H + row0 + (i & 15)] = __float2bfloat16_rn(s);
  }
}

// ---------------------------------------------------------------------------
// host launchers

int launch_route_build(const int32_t* ids, int64_t P, const ExpertsDev& ex, const RouteMeta& m, cudaStream_t st) {
  const size_t smem = sizeof(int) * (size_t)(kRouteWarps + 1) * ex.E;
  if (smem > 200 * 1024) return set_error(FMOE_ERR_UNSUPPORTED, "route_build: %d experts too many", ex.E);
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(route_build_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  {
    ProfScope prof_("route_build_kernel", st);
    route_build_kernel<<<1, kRouteWarps * 32, smem, st>>>(ids, (int)P, ex.first, ex.E, m.start, m.pairs, m.unique,
                                                         m.num_unique);
  }
  return check_launch("route_build_kernel");
}

int launch_moe_gate_up(const bf16* x, int64_t T, int k, const ExpertsDev& ex, const RouteMeta& m, bf16* act,
                       cudaStream_t st) {
  const int64_t pairs = T * k;
  const int maxu = (int)(pairs < ex.E ? pairs : ex.E);
  dim3 grid(ex.I / 16, maxu);
  {
    ProfScope prof_("moe_gate_up_kernel", st);
    moe_gate_up_kernel<<<grid, kGuWarps * 32, 0, st>>>(x, k, ex, m.start, m.pairs, m.unique, m.num_unique, act);
  }
  return check_launch("moe_gate_up_kernel");
}

int max_decode_tokens() { return 256; }

int launch_moe_down(const bf16* act, int64_t T, int k, const float* wts, const ExpertsDev& ex, const RouteMeta& m,
                    bf16* y, cudaStream_t st) {
  const size_t smem = sizeof(float) * kDnWarps * 16 * (size_t)T;
  if (smem > 48 * 1024)
    cudaFuncSetAttribute(moe_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  {
    ProfScope prof_("moe_down_kernel", st);
    moe_down_kernel<<<ex.H / 16, kDnWarps * 32, smem, st>>>(act, (int)T, k, wts, ex, m.start, m.pairs, m.unique,
                                                          m.num_unique, y);
  }
  return check_launch("moe_down_kernel");
}

}  // namespace fmoe
