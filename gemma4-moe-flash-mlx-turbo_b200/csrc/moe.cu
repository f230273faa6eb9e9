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
#include "route.cuh"

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
  route_build_block(ids, P, first, E, start, pairs, unique, num_unique, sm);
}

// Shared-memory row stride for a tile whose rows are `row_bytes` long: the
// fragment loads read 8 bytes per lane from rows g = 0..7, so a row stride of
// 8 or 24 words (mod 32 banks) keeps each half-warp conflict-free.
__host__ __device__ inline int smem_row_stride(int row_bytes) {
  const int words = row_bytes / 4;
  return (words % 32 == 8 || words % 32 == 24) ? row_bytes : row_bytes + 32;
}

// ---------------------------------------------------------------------------
// gate_up: CTA = (16-row tile of the intermediate dim, one selected expert).
// The CTA's whole weight tile (16 gate rows, 16 up rows, their scales and
// biases: ~50 KB at H = 2816) is put in flight at CTA start with 16-byte
// cp.async copies into shared memory, so every resident CTA keeps its full
// tile outstanding against HBM.  kGuWarps warps split the hidden dim into
// contiguous group ranges, each copying and then consuming its own range;
// gate and up share the x fragments; pairs are processed 8 at a time.
constexpr int kGuWarps = 4;

__global__ void __launch_bounds__(kGuWarps * 32)
    moe_gate_up_kernel(const bf16* __restrict__ x, int k, ExpertsDev ex, const int32_t* __restrict__ start,
                       const int32_t* __restrict__ pairs, const int32_t* __restrict__ unique,
                       const int32_t* __restrict__ num_unique, bf16* __restrict__ act) {
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ float red[kGuWarps][2][16][8];
  const int u = blockIdx.y;
  if (u >= *num_unique) return;
  const int H = ex.H, I = ex.I, G = H / 64;
  const int RB = H / 2, RS = smem_row_stride(RB);
  uint8_t* wsm = smem;                                          // [2][16][RS]
  bf16* ssm = reinterpret_cast<bf16*>(smem + 2 * 16 * RS);      // [4][16][G]: gs, gb, us, ub
  const int e = unique[u];
  const int pbeg = start[e], np = start[e + 1] - pbeg;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int row0 = blockIdx.x * 16;
  const uint8_t* eb = ex.base + (int64_t)e * ex.stride;
  const int gbeg = G * warp / kGuWarps, gend = G * (warp + 1) / kGuWarps;

  // issue: this warp's K range of the 32 weight rows, then its share of the scale blocks
  {
    const uint8_t* gate_w = eb + ex.off[0];
    const uint8_t* up_w = eb + ex.off[3];
    const int chunks = (gend - gbeg) * 2;  // 16-byte chunks per row
    for (int i = lane; i < 32 * chunks; i += 32) {
      const int rr = i / chunks, c = i % chunks, mat = rr >> 4, r = rr & 15;
      const uint8_t* src = (mat ? up_w : gate_w) + (int64_t)(row0 + r) * RB + gbeg * 32 + c * 16;
      cp_async16(wsm + (mat * 16 + r) * RS + gbeg * 32 + c * 16, src);
    }
    const int sb = 16 * G * 2;  // bytes of one 16-row scale block
    uint8_t* sdst = reinterpret_cast<uint8_t*>(ssm);
    const int64_t soff = (int64_t)row0 * G * 2;
    cp_async_block(sdst, eb + ex.off[1] + soff, sb, threadIdx.x, blockDim.x);
    cp_async_block(sdst + sb, eb + ex.off[2] + soff, sb, threadIdx.x, blockDim.x);
    cp_async_block(sdst + 2 * sb, eb + ex.off[4] + soff, sb, threadIdx.x, blockDim.x);
    cp_async_block(sdst + 3 * sb, eb + ex.off[5] + soff, sb, threadIdx.x, blockDim.x);
    cp_async_commit();
    cp_async_wait_all();
    __syncthreads();
  }

  const uint8_t* wg = wsm;
  const uint8_t* wu = wsm + 16 * RS;
  const bf16* gs = ssm;
  const bf16* gb = ssm + 16 * G;
  const bf16* us = ssm + 32 * G;
  const bf16* ub = ssm + 48 * G;
  for (int c0 = 0; c0 < np; c0 += 8) {
    const int nv = min(8, np - c0);
    const bf16* xrow = nullptr;
    if (g < nv) xrow = x + (int64_t)(pairs[pbeg + c0 + g] / k) * H;
    float yg[4] = {0.f, 0.f, 0.f, 0.f}, yu[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
    for (int gi = gbeg; gi < gend; ++gi) {
      uint4 xl, xh;
      load_x16(xrow, gi, t, xl, xh);
      const uint2 gl = lds_u2(wg + g * RS + gi * 32 + 8 * t);
      const uint2 gh = lds_u2(wg + (g + 8) * RS + gi * 32 + 8 * t);
      const uint2 ul = lds_u2(wu + g * RS + gi * 32 + 8 * t);
      const uint2 uh = lds_u2(wu + (g + 8) * RS + gi * 32 + 8 * t);
      const BFrag4 b = make_bfrag4(xl, xh);
      float cg[4] = {0.f, 0.f, 0.f, 0.f}, cu[4] = {0.f, 0.f, 0.f, 0.f}, xs[4] = {0.f, 0.f, 0.f, 0.f};
      mma_group_q4(cg, gl, gh, b);
      mma_group_q4(cu, ul, uh, b);
      mma_group_ones(xs, b);
      affine_fixup(yg, cg, xs, lds_bf(gs + g * G + gi), lds_bf(gb + g * G + gi), lds_bf(gs + (g + 8) * G + gi),
                   lds_bf(gb + (g + 8) * G + gi), 128.0f);
      affine_fixup(yu, cu, xs, lds_bf(us + g * G + gi), lds_bf(ub + g * G + gi), lds_bf(us + (g + 8) * G + gi),
                   lds_bf(ub + (g + 8) * G + gi), 128.0f);
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

size_t gate_up_smem_bytes(int H) { return 2 * 16 * (size_t)smem_row_stride(H / 2) + 4 * 16 * (size_t)(H / 64) * 2; }

// ---------------------------------------------------------------------------
// down + combine: CTA = 16-row tile of the hidden dim; kDnWarps warps take the
// selected experts round-robin.  Each warp double-buffers its experts' 16-row
// down tiles (+ scales, biases) in shared memory with cp.async, so the next
// expert's tile is in flight while the current one is consumed.  Per-warp fp32
// partial sums per (token, row) are added in warp order at the end
// (deterministic).
constexpr int kDnWarps = 8;

__device__ __forceinline__ void down_issue(uint8_t* stage, const uint8_t* eb, const ExpertsDev& ex, int row0, int I,
                                           int RS, int lane) {
  const int RB = I / 2, Gi = I / 64, chunks = RB / 16;
  for (int i = lane; i < 16 * chunks; i += 32) {
    const int r = i / chunks, c = i % chunks;
    cp_async16(stage + r * RS + c * 16, eb + ex.off[6] + (int64_t)(row0 + r) * RB + c * 16);
  }
  const int sb = 16 * Gi * 2;
  cp_async_block(stage + 16 * RS, eb + ex.off[7] + (int64_t)row0 * Gi * 2, sb, lane, 32);
  cp_async_block(stage + 16 * RS + sb, eb + ex.off[8] + (int64_t)row0 * Gi * 2, sb, lane, 32);
}

__global__ void __launch_bounds__(kDnWarps * 32)
    moe_down_kernel(const bf16* __restrict__ act, int T, int k, const float* __restrict__ wts, ExpertsDev ex,
                    const int32_t* __restrict__ start, const int32_t* __restrict__ pairs,
                    const int32_t* __restrict__ unique, const int32_t* __restrict__ num_unique,
                    bf16* __restrict__ y) {
  extern __shared__ __align__(16) uint8_t smem[];
  const int H = ex.H, I = ex.I, Gi = I / 64;
  const int RS = smem_row_stride(I / 2);
  const int stage_bytes = 16 * RS + 2 * 16 * Gi * 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  uint8_t* my_stage = smem + (size_t)warp * 2 * stage_bytes;
  float* ysm = reinterpret_cast<float*>(smem + (size_t)kDnWarps * 2 * stage_bytes);  // [kDnWarps][T][16]
  const int row0 = blockIdx.x * 16;
  const int U = *num_unique;
  for (int i = threadIdx.x; i < kDnWarps * T * 16; i += blockDim.x) ysm[i] = 0.f;
  __syncthreads();
  float* my = ysm + warp * T * 16;

  if (warp < U) down_issue(my_stage, ex.base + (int64_t)unique[warp] * ex.stride, ex, row0, I, RS, lane);
  cp_async_commit();
  int it = 0;
  for (int u = warp; u < U; u += kDnWarps, ++it) {
    const int un = u + kDnWarps;
    if (un < U)
      down_issue(my_stage + ((it + 1) & 1) * stage_bytes, ex.base + (int64_t)unique[un] * ex.stride, ex, row0, I, RS,
                 lane);
    cp_async_commit();
    cp_async_wait_group<1>();
    __syncwarp();
    const uint8_t* wt = my_stage + (it & 1) * stage_bytes;
    const bf16* ds = reinterpret_cast<const bf16*>(wt + 16 * RS);
    const bf16* db = ds + 16 * Gi;
    const int e = unique[u];
    const int pbeg = start[e], np = start[e + 1] - pbeg;
    for (int c0 = 0; c0 < np; c0 += 8) {
      const int nv = min(8, np - c0);
      const bf16* arow = g < nv ? act + (int64_t)(pbeg + c0 + g) * I : nullptr;
      float d[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
      for (int gi = 0; gi < Gi; ++gi) {
        uint4 xl, xh;
        load_x16(arow, gi, t, xl, xh);
        const uint2 wl = lds_u2(wt + g * RS + gi * 32 + 8 * t);
        const uint2 wh = lds_u2(wt + (g + 8) * RS + gi * 32 + 8 * t);
        const BFrag4 b = make_bfrag4(xl, xh);
        float c[4] = {0.f, 0.f, 0.f, 0.f}, xs[4] = {0.f, 0.f, 0.f, 0.f};
        mma_group_q4(c, wl, wh, b);
        mma_group_ones(xs, b);
        affine_fixup(d, c, xs, lds_bf(ds + g * Gi + gi), lds_bf(db + g * Gi + gi), lds_bf(ds + (g + 8) * Gi + gi),
                     lds_bf(db + (g + 8) * Gi + gi), 128.0f);
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
    __syncwarp();
  }
  cp_async_wait_all();
  __syncthreads();
  for (int i = threadIdx.x; i < T * 16; i += blockDim.x) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kDnWarps; ++w) s += ysm[w * T * 16 + i];
    y[(int64_t)(i >> 4) * H + row0 + (i & 15)] = __float2bfloat16_rn(s);
  }
}

size_t down_smem_bytes(int I, int64_t T) {
  const size_t stage = 16 * (size_t)smem_row_stride(I / 2) + 2 * 16 * (size_t)(I / 64) * 2;
  return kDnWarps * 2 * stage + sizeof(float) * kDnWarps * 16 * (size_t)T;
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
  const size_t smem = gate_up_smem_bytes(ex.H);
  if (smem > 200 * 1024) return set_error(FMOE_ERR_UNSUPPORTED, "gate_up: hidden %d too large", ex.H);
  cudaFuncSetAttribute(moe_gate_up_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  dim3 grid(ex.I / 16, maxu);
  {
    ProfScope prof_("moe_gate_up_kernel", st);
    moe_gate_up_kernel<<<grid, kGuWarps * 32, smem, st>>>(x, k, ex, m.start, m.pairs, m.unique, m.num_unique, act);
  }
  return check_launch("moe_gate_up_kernel");
}

int launch_moe_down(const bf16* act, int64_t T, int k, const float* wts, const ExpertsDev& ex, const RouteMeta& m,
                    bf16* y, cudaStream_t st) {
  const size_t smem = down_smem_bytes(ex.I, T);
  if (smem > 227 * 1024) return set_error(FMOE_ERR_UNSUPPORTED, "down: T=%lld / I=%d exceed shared memory", (long long)T, ex.I);
  cudaFuncSetAttribute(moe_down_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  {
    ProfScope prof_("moe_down_kernel", st);
    moe_down_kernel<<<ex.H / 16, kDnWarps * 32, smem, st>>>(act, (int)T, k, wts, ex, m.start, m.pairs, m.unique,
                                                            m.num_unique, y);
  }
  return check_launch("moe_down_kernel");
}

}  // namespace fmoe
