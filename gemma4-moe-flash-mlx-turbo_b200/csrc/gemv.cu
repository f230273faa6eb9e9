// GEMV-shaped kernels: quantised linear (decode / small T), router logits and
// router top-k.
//
// gemv_partial_kernel computes y = x . W^T for a 16-row x 8-token tile per
// CTA and one of `ksplit` contiguous slices of the reduction dimension, so a
// single-token GEMV still spreads its weight bytes over >= 2 CTAs per SM.
// The slices' fp32 partial sums are added in fixed order by the consumer
// (reduce_partials_kernel or router_topk_kernel), so results are
// deterministic run to run.
#include "internal.h"
#include "gemv.cuh"
#include "route.cuh"

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

// Top-k of one token, one warp: logits = sum of the K-slice partials (+ bias);
// top-k by value (ties -> lower id); weights = softmax over the k selected
// logits (equal to softmax(all)[ids] / sum softmax(all)[ids],
// src/model/moe.rs:331-340), times per_expert_scale (moe.rs:341-345).
// Partials are read through L2: other CTAs of the same kernel wrote them.
constexpr int kTopkPerLane = 8;  // E <= 256
__device__ void topk_token(const float* partial, int ksplit, int T, int E, int tkn, const float* bias, const bf16* pes,
                           int k, int first_id, int32_t* ids, float* wts, float* logits_out) {
  const int lane = threadIdx.x & 31;
  float v[kTopkPerLane];
#pragma unroll
  for (int j = 0; j < kTopkPerLane; ++j) {
    const int e = lane + 32 * j;
    float s = -INFINITY;
    if (e < E) {
      s = 0.f;
      for (int kz = 0; kz < ksplit; ++kz) s += __ldcg(partial + ((int64_t)kz * T + tkn) * E + e);
      if (bias) s += bias[e];
      if (logits_out) logits_out[(int64_t)tkn * E + e] = s;
    }
    v[j] = s;
  }
  float mx = 0.f, den = 0.f, my_v = 0.f;
  int my_e = 0;
  for (int r = 0; r < k; ++r) {
    float bv = -INFINITY;
    int be = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kTopkPerLane; ++j) {
      const int e = lane + 32 * j;
      if (e < E && (v[j] > bv || (v[j] == bv && e < be))) {
        bv = v[j];
        be = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oe = __shfl_xor_sync(0xffffffffu, be, o);
      if (ov > bv || (ov == bv && oe < be)) {
        bv = ov;
        be = oe;
      }
    }
    if (r == 0) mx = bv;
    den += expf(bv - mx);
    if (lane == r) {
      my_v = bv;
      my_e = be;
    }
#pragma unroll
    for (int j = 0; j < kTopkPerLane; ++j)
      if (lane + 32 * j == be) v[j] = -INFINITY;
  }
  if (lane < k) {
    float wv = expf(my_v - mx) / den;
    if (pes) wv *= bf2f(pes[my_e]);
    ids[(int64_t)tkn * k + lane] = my_e + first_id;
    wts[(int64_t)tkn * k + lane] = wv;
  }
}

// Fused router: CTA (16-expert tile, 8-token chunk, K slice) computes its
// partial logits; the last CTA to finish a token chunk (completion counter)
// runs the chunk's top-k; the last chunk to finish builds the per-expert pair
// lists for the expert kernels when `meta.start` is set.  Counters return to
// zero at the end of every call.
template <int BITS>
__global__ void __launch_bounds__(kGemvWarps * 32)
    router_fused_kernel(const bf16* __restrict__ x, int T, int in, int E, const void* __restrict__ w,
                        const bf16* __restrict__ sc, const bf16* __restrict__ bi, int ksplit, float* partial,
                        const float* __restrict__ bias, const bf16* __restrict__ pes, int k, int32_t* ids, float* wts,
                        float* logits_out, unsigned* counters, RouteMeta meta) {
  extern __shared__ int rsm[];
  __shared__ float red[kGemvWarps][16][8];
  __shared__ int s_last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const int row0 = blockIdx.x * 16, tok0 = blockIdx.y * 8, kz = blockIdx.z;
  const int G = in / 64;
  const int gbeg = (int)((int64_t)G * kz / ksplit), gend = (int)((int64_t)G * (kz + 1) / ksplit);
  const int wpr = in * BITS / 32;
  const bf16* xrow = (tok0 + g < T) ? x + (int64_t)(tok0 + g) * in : nullptr;
  float y[4] = {0.f, 0.f, 0.f, 0.f};
  warp_tile_gemv<BITS>(y, w, sc, bi, min(row0 + g, E - 1), min(row0 + g + 8, E - 1), wpr, G, xrow, gbeg + warp, gend,
                       kGemvWarps, t);
  red[warp][g][2 * t] = y[0];
  red[warp][g][2 * t + 1] = y[1];
  red[warp][g + 8][2 * t] = y[2];
  red[warp][g + 8][2 * t + 1] = y[3];
  __syncthreads();
  {
    const int i = threadIdx.x, tk = i >> 4, r = i & 15;
    if (tok0 + tk < T && row0 + r < E) {
      float s = 0.f;
#pragma unroll
      for (int wi = 0; wi < kGemvWarps; ++wi) s += red[wi][r][tk];
      partial[((int64_t)kz * T + tok0 + tk) * E + row0 + r] = s;
    }
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&counters[1 + blockIdx.y], 1u) == gridDim.x * gridDim.z - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int tk = warp; tk < 8; tk += kGemvWarps)
    if (tok0 + tk < T) topk_token(partial, ksplit, T, E, tok0 + tk, bias, pes, k, 0, ids, wts, logits_out);
  if (threadIdx.x == 0) counters[1 + blockIdx.y] = 0;
  if (!meta.start) return;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(&counters[0], 1u) == gridDim.y - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  route_build_block(ids, T * k, 0, E, meta.start, meta.pairs, meta.unique, meta.num_unique, rsm);
  if (threadIdx.x == 0) counters[0] = 0;
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

int launch_router_fused(const bf16* x, int64_t T, const QW& w, int ksplit, float* partial, const float* bias,
                        const bf16* pes, int k, int32_t* ids, float* wts, float* logits, unsigned* counters,
                        const RouteMeta* meta, cudaStream_t st) {
  const int E = w.out;
  if (E > 32 * kTopkPerLane) return set_error(FMOE_ERR_UNSUPPORTED, "router: num_experts %d > %d", E, 32 * kTopkPerLane);
  if (k < 1 || k > 16 || k > E) return set_error(FMOE_ERR_INVALID, "router: top_k %d out of range", k);
  dim3 grid((E + 15) / 16, (unsigned)((T + 7) / 8), ksplit);
  RouteMeta m = meta ? *meta : RouteMeta{nullptr, nullptr, nullptr, nullptr};
  const size_t smem = meta ? sizeof(int) * (kGemvWarps + 1) * (size_t)E : 0;
#define FMOE_ROUTER_LAUNCH(B)                                                                                          \
  {                                                                                                                    \
    ProfScope prof_("router_fused_kernel<" #B ">", st);                                                                \
    router_fused_kernel<B><<<grid, kGemvWarps * 32, smem, st>>>(x, (int)T, w.in, E, w.w, w.s, w.b, ksplit, partial,    \
                                                                bias, pes, k, ids, wts, logits, counters, m);          \
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
