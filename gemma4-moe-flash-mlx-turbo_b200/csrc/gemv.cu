// GEMV-shaped kernels: quantised linear (decode / small T), router logits and
// router top-k.
//
// gemv_partial_kernel computes y = x . W^T for a 16-row x 8-token tile per
// CTA and one of `ksplit` contiguous slices of the reduction dimension, so a
// single-token GEMV still spreads its weight bytes over >= 2 CTAs per SM.
// The slices' fp32 partial sums are added in fixed order by the consumer
// (reduce_partials_kernel or router_topk_kernel), so results are
// deterministic run to run.
#include <cooperative_groups.h>
#include "internal.h"
#include "gemv.cuh"
#include "route.cuh"
#include "stage.cuh"

namespace fmoe {

constexpr int kGemvWarps = 4;

template <int BITS>
__global__ void __launch_bounds__(kGemvWarps * 32)
    gemv_partial_kernel(const bf16* __restrict__ x, int T, int in, int out, const void* __restrict__ w,
                        const bf16* __restrict__ sc, const bf16* __restrict__ bi, int ksplit,
                        float* __restrict__ partial) {
  __shared__ float red[kGemvWarps][16][8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int row0 = blockIdx.x * 16, tok0 = blockIdx.y * 8, kz = blockIdx.z;
  const int G = in / 64;
  const int gbeg = (int)((int64_t)G * kz / ksplit), gend = (int)((int64_t)G * (kz + 1) / ksplit);
  const int wpr = in * BITS / 32, spr = G;
  const bf16* xrow = (tok0 + g < T) ? x + (int64_t)(tok0 + g) * in : nullptr;
  float y[4] = {0.f, 0.f, 0.f, 0.f};
  warp_tile_gemv<BITS>(y, w, sc, bi, row0 + g, row0 + g + 8, wpr, spr, xrow, gbeg + warp, gend, kGemvWarps, t);
  red[warp][g][2 * t] = y[0];
  red[warp][g][2 * t + 1] = y[1];
  red[warp][g + 8][2 * t] = y[2];
  red[warp][g + 8][2 * t + 1] = y[3];
  __syncthreads();
  // 128 outputs: thread i -> token i/16, row i%16 (16 consecutive rows per token).
  const int i = threadIdx.x, tk = i >> 4, r = i & 15;
  if (tok0 + tk < T) {
    float s = 0.f;
#pragma unroll
    for (int wi = 0; wi < kGemvWarps; ++wi) s += red[wi][r][tk];
    partial[((int64_t)kz * T + tok0 + tk) * out + row0 + r] = s;
  }
}

// out[t, o] = sum_kz partial[kz, t, o]  (bf16 and/or f32 outputs).
__global__ void reduce_partials_kernel(const float* __restrict__ partial, int ksplit, int64_t n,
                                       bf16* __restrict__ out_bf16, float* __restrict__ out_f32) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float s = 0.f;
    for (int k = 0; k < ksplit; ++k) s += partial[k * n + i];
    if (out_bf16) out_bf16[i] = __float2bfloat16_rn(s);
    if (out_f32) out_f32[i] = s;
  }
}

// Router pre-normalisation (src/model/moe.rs:325-329, 473-479):
// xs = bf16(bf16(bf16(x * rsqrt(mean(x^2) + eps)) * bf16(root)) * router_scale).
__global__ void router_prenorm_kernel(const bf16* __restrict__ x, int H, float root, float eps,
                                      const bf16* __restrict__ rscale, bf16* __restrict__ xs) {
  const int tkn = blockIdx.x;
  const bf16* xr = x + (int64_t)tkn * H;
  float ss = 0.f;
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    const float v = bf2f(xr[h]);
    ss += v * v;
  }
  __shared__ float red[32];
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float rms = rsqrtf(red[0] / H + eps);
  const float rb = round_bf(root);
  for (int h = threadIdx.x; h < H; h += blockDim.x) {
    float v = round_bf(bf2f(xr[h]) * rms);
    v = round_bf(v * rb);
    if (rscale) v = round_bf(v * bf2f(rscale[h]));
    xs[(int64_t)tkn * H + h] = __float2bfloat16_rn(v);
  }
}

// Top-k of `nv` tokens by the whole CTA over logits already rounded to bf16
// (the router projection's output dtype in the reference, moe.rs:330-334):
// each thread takes one (token, expert) and counts the logits that beat it
// (descending value, ties -> lower id) with 16-byte shared-memory reads — independent compares, no serial
// reduction chain.  Then weights = softmax over the k selected logits (equal
// to softmax(all)[ids] / sum softmax(all)[ids], src/model/moe.rs:331-340),
// times per_expert_scale (moe.rs:341-345).  lg: shared [nv][E], E % 4 == 0.
// Output rows tok0 .. tok0+nv-1 of ids / wts; sel_e receives [nv][16] ids.
constexpr int kTopkMaxK = 16;
__device__ void topk_block(const float* lg, int nv, int E, int k, int tok0, const bf16* pes, int32_t* ids, float* wts,
                           int* sel_e, float* sel_v) {
  for (int i = threadIdx.x; i < nv * E; i += blockDim.x) {
    const int n = i / E, e = i % E;
    const float* row = lg + n * E;
    const float v = row[e];
    int r0 = 0, r1 = 0, r2 = 0, r3 = 0;
#pragma unroll 8
    for (int j = 0; j < E; j += 4) {
      const float4 u = *reinterpret_cast<const float4*>(row + j);
      r0 += (u.x > v || (u.x == v && j < e)) ? 1 : 0;
      r1 += (u.y > v || (u.y == v && j + 1 < e)) ? 1 : 0;
      r2 += (u.z > v || (u.z == v && j + 2 < e)) ? 1 : 0;
      r3 += (u.w > v || (u.w == v && j + 3 < e)) ? 1 : 0;
    }
    const int rank = r0 + r1 + r2 + r3;
    if (rank < k) {
      sel_e[n * kTopkMaxK + rank] = e;
      sel_v[n * kTopkMaxK + rank] = v;
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < nv * kTopkMaxK; i += blockDim.x) {
    const int n = i / kTopkMaxK, r = i % kTopkMaxK;
    if (r < k) {
      const float m = sel_v[n * kTopkMaxK];
      float den = 0.f;
      for (int j = 0; j < k; ++j) den += expf(sel_v[n * kTopkMaxK + j] - m);
      float wv = expf(sel_v[n * kTopkMaxK + r] - m) / den;
      const int e = sel_e[n * kTopkMaxK + r];
      if (pes) wv *= bf2f(pes[e]);
      ids[(int64_t)(tok0 + n) * k + r] = e;
      wts[(int64_t)(tok0 + n) * k + r] = wv;
    }
  }
  __syncthreads();
}

// Routing lists for a single token (T == 1) inside one warp: the k selected
// experts are distinct, so expert j's slot in the ascending list is the number
// of selected ids below it.  Lane j < k holds (id, slot j).
__device__ __forceinline__ void route_single_token(int my_e, int k, int E, RouteMeta m) {
  const int lane = threadIdx.x & 31;
  int rank = 0;
  for (int i = 0; i < k; ++i) {
    const int ei = __shfl_sync(0xffffffffu, my_e, i);
    rank += (lane < k && ei < my_e) ? 1 : 0;
  }
  if (lane < k) {
    m.unique[rank] = my_e;
    m.pairs[rank] = lane;
    m.start[my_e] = rank;
    m.start[my_e + 1] = rank + 1;  // agrees with the next selected expert's own entry when adjacent
    if (rank < m.work_len) m.work[rank] = make_int4(my_e, rank, 1, 0);
  }
  for (int u = k + lane; u < m.work_len; u += 32) m.work[u] = make_int4(0, 0, 0, 0);
  if (lane == 0) {
    m.start[E] = k;
    *m.num_unique = k;
  }
}

// Fused router.  One thread-block cluster per 8-token chunk covers all
// experts: CTA rank r computes the 16-expert tile r % RT over the hidden-dim
// slice r / RT (RT = ceil(E/16) tiles, KS slices, RT*KS <= 16 CTAs).  Each
// CTA stages its weight slice (and scales) before waiting on the preceding
// kernel (programmatic dependent launch), then its slice of the chunk's x rows.
// The rank-0 CTA gathers the partial tiles through distributed shared memory
// in slice order (deterministic), adds the bias, and runs the chunk's top-k
// from shared memory.  With a single chunk it also builds the routing lists;
// with several, the last chunk (completion counter, reset every call) does.
constexpr int kRtWarps = 4;
constexpr int kRtMaxCluster = 16;

struct RtLayout {
  int RS, XS, gmax;
  size_t s_off, f_off, x_off, l_off, bytes;
};
__host__ __device__ inline RtLayout rt_layout(int H, int bits, int E, int ks) {
  RtLayout L;
  const int G = H / 64;
  L.gmax = (G + ks - 1) / ks;  // groups per slice
  L.RS = smem_stride(L.gmax * 64 * bits / 8, bits == 4 ? 8 : 16);
  L.XS = smem_stride(L.gmax * 128, 16);
  L.s_off = 16 * (size_t)L.RS;                                              // raw bf16 [2][16][gmax]
  L.f_off = align16(L.s_off + (bits == 16 ? 0 : 2 * 16 * (size_t)L.gmax * 2));  // float2 [16][gmax]
  L.x_off = align16(L.f_off + (bits == 16 ? 0 : 16 * (size_t)L.gmax * sizeof(float2)));
  L.l_off = align16(L.x_off + 8 * (size_t)L.XS);                           // logits [8][E] (rank 0)
  L.bytes = L.l_off + 8 * (size_t)E * sizeof(float);
  const size_t route = sizeof(int) * (kRtWarps + 1) * (size_t)E;  // route build reuses the tile area
  if (L.l_off < route) {
    L.l_off = align16(route);
    L.bytes = L.l_off + 8 * (size_t)E * sizeof(float);
  }
  return L;
}

template <int BITS>
__global__ void __launch_bounds__(kRtWarps * 32)
    router_fused_kernel(const bf16* __restrict__ x, int T, int H, int E, int RT, int KS, const void* __restrict__ w,
                        const bf16* __restrict__ sc, const bf16* __restrict__ bi, const float* __restrict__ bias,
                        const bf16* __restrict__ pes, int k, int32_t* ids, float* wts, float* logits_out,
                        unsigned* counters, RouteMeta meta, int* status) {
  namespace cg = cooperative_groups;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar;
  __shared__ float red[kRtWarps][16][8];
  __shared__ float part[16][8];
  __shared__ int s_last;
  __shared__ int sel_e[8 * kTopkMaxK];
  __shared__ float sel_v[8 * kTopkMaxK];
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = (int)cluster.block_rank();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int tile = rank % RT, slice = rank / RT;
  const int row0 = tile * 16, tok0 = blockIdx.y * 8;
  const int nv = min(8, T - tok0);
  const int G = H / 64, RB = H * BITS / 8, GB = 64 * BITS / 8;  // bytes per group of a row
  const RtLayout L = rt_layout(H, BITS, E, KS);
  const int g0 = min(G, slice * L.gmax), g1 = min(G, g0 + L.gmax), ng = g1 - g0;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
  }
  __syncthreads();
  // weight slice: independent of the preceding kernel (one bulk copy per row)
  if (warp == 0) {
    if (lane == 0) mbar_arrive_expect_tx(&bar, 16u * ng * GB + (uint32_t)nv * ng * 128);
    __syncwarp();
    if (lane < 16 && ng > 0) {
      const int row = min(row0 + lane, E - 1);
      bulk_g2s(smem + lane * L.RS, static_cast<const uint8_t*>(w) + (int64_t)row * RB + g0 * GB, ng * GB, &bar);
    }
  }
  if (BITS != 16) {
    bf16* raw = reinterpret_cast<bf16*>(smem + L.s_off);
    for (int i = threadIdx.x; i < 16 * ng; i += blockDim.x) {
      const int r = i / ng, j = i % ng, row = min(row0 + r, E - 1);
      raw[r * L.gmax + j] = sc[(int64_t)row * G + g0 + j];
      raw[16 * L.gmax + r * L.gmax + j] = bi[(int64_t)row * G + g0 + j];
    }
  }
  griddep_wait();  // x may come from the preceding kernel
  griddep_launch_dependents();
  if (warp == 0 && lane >= 16 && lane - 16 < nv && ng > 0)
    bulk_g2s(smem + L.x_off + (lane - 16) * L.XS, x + (int64_t)(tok0 + lane - 16) * H + g0 * 64, ng * 128, &bar);
  const bool ok = mbar_wait(&bar, 0, status, 21);
  __syncthreads();
  float2* fix = reinterpret_cast<float2*>(smem + L.f_off);
  if (BITS != 16) {
    const bf16* raw = reinterpret_cast<const bf16*>(smem + L.s_off);
    const float off = BITS == 4 ? 128.0f : 2176.0f;
    for (int i = threadIdx.x; i < 16 * L.gmax; i += blockDim.x) {
      const float s = __bfloat162float(raw[i]);
      fix[i] = make_float2(s, fmaf(-off, s, __bfloat162float(raw[16 * L.gmax + i])));
    }
    __syncthreads();
  }
  const uint8_t* wsm = smem;
  const uint8_t* xsm = smem + L.x_off;
  float y[4] = {0.f, 0.f, 0.f, 0.f};
  for (int j = warp; j < ng; j += kRtWarps) {
    if constexpr (BITS == 16) {
      const BFrag4 b = stage_bfrag4(xsm, L.XS, nv, j, g, t);
      const uint8_t* plo = wsm + g * L.RS + j * 128 + 32 * t;
      const uint8_t* phi = wsm + (g + 8) * L.RS + j * 128 + 32 * t;
      const BFrag4 alo = make_bfrag4(lds_u4(plo), lds_u4(plo + 16)), ahi = make_bfrag4(lds_u4(phi), lds_u4(phi + 16));
#pragma unroll
      for (int s = 0; s < 4; ++s) mma16816(y, alo.b0[s], ahi.b0[s], alo.b1[s], ahi.b1[s], b.b0[s], b.b1[s]);
    } else if constexpr (BITS == 4) {
      const BFrag4 b = stage_bfrag4(xsm, L.XS, nv, j, g, t);
      const uint2 wl = lds_u2(wsm + g * L.RS + j * 32 + 8 * t);
      const uint2 wh = lds_u2(wsm + (g + 8) * L.RS + j * 32 + 8 * t);
      float c[4] = {0.f, 0.f, 0.f, 0.f}, xs[4] = {0.f, 0.f, 0.f, 0.f};
      mma_group_q4(c, wl, wh, b);
      mma_group_ones(xs, b);
      const float2 lo = fix[g * L.gmax + j], hi = fix[(g + 8) * L.gmax + j];
      y[0] = fmaf(lo.x, c[0], fmaf(lo.y, xs[0], y[0]));
      y[1] = fmaf(lo.x, c[1], fmaf(lo.y, xs[1], y[1]));
      y[2] = fmaf(hi.x, c[2], fmaf(hi.y, xs[2], y[2]));
      y[3] = fmaf(hi.x, c[3], fmaf(hi.y, xs[3], y[3]));
    } else {
      const uint8_t* px = xsm + g * L.XS + j * 128 + 32 * t;
      uint4 xl = make_uint4(0, 0, 0, 0), xh = xl;
      if (g < nv) {
        xl = lds_u4(px);
        xh = lds_u4(px + 16);
      }
      const BFrag8 b8 = make_bfrag8(xl, xh);
      const uint4 wl = lds_u4(wsm + g * L.RS + j * 64 + 16 * t);
      const uint4 wh = lds_u4(wsm + (g + 8) * L.RS + j * 64 + 16 * t);
      float c[4] = {0.f, 0.f, 0.f, 0.f}, xs[4] = {0.f, 0.f, 0.f, 0.f};
      mma_group_q8(c, wl, wh, b8);
      mma_group_ones8(xs, b8);
      const float2 lo = fix[g * L.gmax + j], hi = fix[(g + 8) * L.gmax + j];
      y[0] = fmaf(lo.x, c[0], fmaf(lo.y, xs[0], y[0]));
      y[1] = fmaf(lo.x, c[1], fmaf(lo.y, xs[1], y[1]));
      y[2] = fmaf(hi.x, c[2], fmaf(hi.y, xs[2], y[2]));
      y[3] = fmaf(hi.x, c[3], fmaf(hi.y, xs[3], y[3]));
    }
  }
  red[warp][g][2 * t] = y[0];
  red[warp][g][2 * t + 1] = y[1];
  red[warp][g + 8][2 * t] = y[2];
  red[warp][g + 8][2 * t + 1] = y[3];
  __syncthreads();
  {
    const int r = threadIdx.x >> 3, c = threadIdx.x & 7;  // 128 threads = 16 x 8
    float s = 0.f;
#pragma unroll
    for (int wi = 0; wi < kRtWarps; ++wi) s += red[wi][r][c];
    part[r][c] = s;
  }
  cluster.sync();  // every CTA's partial tile is in its shared memory
  float* lg = reinterpret_cast<float*>(smem + L.l_off);  // [8][E] on rank 0
  if (rank == 0) {
    for (int i = threadIdx.x; i < nv * E; i += blockDim.x) {
      const int c = i / E, e = i % E;
      float s = 0.f;
      for (int q = 0; q < KS; ++q) s += cluster.map_shared_rank(&part[0][0], q * RT + e / 16)[(e % 16) * 8 + c];
      if (bias) s += bias[e];
      lg[i] = round_bf(s);  // ranked and softmaxed in the router's bf16 output precision
      if (logits_out && c < nv) logits_out[(int64_t)(tok0 + c) * E + e] = s;
    }
  }
  cluster.sync();  // peers keep their shared memory until rank 0 has read it
  if (rank != 0 || !ok) return;
  __syncthreads();
  topk_block(lg, nv, E, k, tok0, pes, ids, wts, sel_e, sel_v);
  if (T == 1 && meta.start) {
    if (warp == 0) route_single_token(lane < k ? sel_e[lane] : 0, k, E, meta);
    return;
  }
  if (!meta.start) return;
  if (gridDim.y > 1) {
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(&counters[0], 1u) == gridDim.y - 1;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
  } else {
    __threadfence();  // ids reach L2 before route_build_block reads them through it
    __syncthreads();
  }
  route_build_block(ids, T * k, 0, E, meta.start, meta.pairs, meta.unique, meta.num_unique, meta.work, meta.work_len,
                    reinterpret_cast<int*>(smem));
  if (threadIdx.x == 0 && gridDim.y > 1) counters[0] = 0;
}

// ---------------------------------------------------------------------------
// host launchers

int gemv_ksplit(int64_t T, int out, int in) {
  const int G = in / 64;
  const int64_t tiles = (int64_t)(out / 16) * ((T + 7) / 8);
  int ks = (int)((2 * kNumSMs + tiles - 1) / tiles);
  ks = ks < 1 ? 1 : ks;
  const int gmax = G / kGemvWarps > 0 ? G / kGemvWarps : 1;  // >= 4 groups per CTA slice
  return ks > gmax ? gmax : ks;
}

int launch_gemv_partial(const bf16* x, int64_t T, const QW& w, int ksplit, float* partial, cudaStream_t st) {
  dim3 grid(w.out / 16, (unsigned)((T + 7) / 8), ksplit);
  switch (w.bits) {
    case 16:
      {
        ProfScope prof_("gemv_partial_kernel<16>", st);
        gemv_partial_kernel<16><<<grid, kGemvWarps * 32, 0, st>>>(x, (int)T, w.in, w.out, w.w, w.s, w.b, ksplit, partial);
      }
      break;
    case 4:
      {
        ProfScope prof_("gemv_partial_kernel<4>", st);
        gemv_partial_kernel<4><<<grid, kGemvWarps * 32, 0, st>>>(x, (int)T, w.in, w.out, w.w, w.s, w.b, ksplit, partial);
      }
      break;
    case 8:
      {
        ProfScope prof_("gemv_partial_kernel<8>", st);
        gemv_partial_kernel<8><<<grid, kGemvWarps * 32, 0, st>>>(x, (int)T, w.in, w.out, w.w, w.s, w.b, ksplit, partial);
      }
      break;
    default:
      return set_error(FMOE_ERR_UNSUPPORTED, "gemv: bits=%d has no kernel", w.bits);
  }
  return check_launch("gemv_partial_kernel");
}

int launch_reduce_partials(const float* partial, int ksplit, int64_t n, bf16* out_bf16, float* out_f32,
                           cudaStream_t st) {
  const int threads = 256;
  int64_t blocks = (n + threads - 1) / threads;
  if (blocks > 4 * kNumSMs) blocks = 4 * kNumSMs;
  {
    ProfScope prof_("reduce_partials_kernel", st);
    reduce_partials_kernel<<<(unsigned)blocks, threads, 0, st>>>(partial, ksplit, n, out_bf16, out_f32);
  }
  return check_launch("reduce_partials_kernel");
}

int launch_router_prenorm(const bf16* x, int64_t T, int H, float root, float eps, const bf16* rscale, bf16* xs,
                          cudaStream_t st) {
  {
    ProfScope prof_("router_prenorm_kernel", st);
    router_prenorm_kernel<<<(unsigned)T, 256, 0, st>>>(x, H, root, eps, rscale, xs);
  }
  return check_launch("router_prenorm_kernel");
}

int launch_router_fused(const bf16* x, int64_t T, const QW& w, const float* bias, const bf16* pes, int k,
                        int32_t* ids, float* wts, float* logits_out, unsigned* counters, const RouteMeta* meta,
                        int* status, bool pdl, cudaStream_t st) {
  const int E = w.out, G = w.in / 64;
  if (E > 256 || E % 4) return set_error(FMOE_ERR_UNSUPPORTED, "router: num_experts %d (kernels: <= 256, multiple of 4)", E);
  if (k < 1 || k > kTopkMaxK || k > E) return set_error(FMOE_ERR_INVALID, "router: top_k %d out of range", k);
  const int RT = (E + 15) / 16;
  int KS = kRtMaxCluster / RT;
  if (KS > G) KS = G;
  if (KS < 1) KS = 1;
  const RtLayout L = rt_layout(w.in, w.bits, E, KS);
  if (L.bytes > 227 * 1024) return set_error(FMOE_ERR_UNSUPPORTED, "router: hidden %d too large", w.in);
  RouteMeta m = meta ? *meta : RouteMeta{nullptr, nullptr, nullptr, nullptr, nullptr, 0};
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[2];
  cfg.gridDim = dim3(RT * KS, (unsigned)((T + 7) / 8));
  cfg.blockDim = dim3(kRtWarps * 32);
  cfg.dynamicSmemBytes = L.bytes;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = RT * KS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
#define FMOE_ROUTER_LAUNCH(B)                                                                                        \
  {                                                                                                                  \
    cudaFuncSetAttribute(router_fused_kernel<B>, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);                 \
    cudaFuncSetAttribute(router_fused_kernel<B>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.bytes);         \
    ProfScope prof_("router_fused_kernel<" #B ">", st);                                                              \
    cudaLaunchKernelEx(&cfg, router_fused_kernel<B>, x, (int)T, w.in, E, RT, KS, w.w, w.s, w.b, bias, pes, k, ids,   \
                       wts, logits_out, counters, m, status);                                                        \
  }
  switch (w.bits) {
    case 16: FMOE_ROUTER_LAUNCH(16) break;
    case 4: FMOE_ROUTER_LAUNCH(4) break;
    case 8: FMOE_ROUTER_LAUNCH(8) break;
    default: return set_error(FMOE_ERR_UNSUPPORTED, "router: bits=%d has no kernel", w.bits);
  }
#undef FMOE_ROUTER_LAUNCH
  return check_launch("router_fused_kernel");
}

}  // namespace fmoe
