// Gemma-4 decoder layer and tied lm_head for the decode step (one token per
// sequence, T <= 8 sequences), DecoderLayer::forward_gemma4 (src/model/mod.rs:
// 67-119) and Model::forward's lm_head + softcap (src/model/mod.rs:325-363).
//
// Kernel sequence of one layer (all on one stream; the GEMVs and small kernels
// chain through programmatic dependent launch so each one's weight stream
// starts while its predecessor drains):
//   1 qgemv  q|k|v = input_norm(x) . [Wq Wk Wv]^T        (norm fused into the input prologue)
//   2 qkv_post  q/k norms, RoPE, v norm, KV-cache append (kv.cu)
//   3 attention (kv.cu)
//   4 qgemv  o = attn . Wo^T                              (fp32, accumulating)
//   5 ff_in  h = x + post_attn_norm(o); h1 = pre_ff_norm(h); h2 = pre_ff_norm_2(h);
//            router input = rms_norm_no_scale(h2) * root * router_scale
//   6 qgemv  g|u = h1 . [Wg Wu]^T                        (dense MLP)
//   7 router (fused GEMV + top-k + routing lists) on the router input
//   8-9 routed experts on h2 -> moe (moe.cu)
//  10 qgemv  d = (gelu(g) * u) . Wd^T                     (GELU gating fused into the input prologue)
//  11 ff_out x' = (h + post_ff_norm(post_ff_norm_1(d) + post_ff_norm_2(moe))) * layer_scalar
// Every intermediate is rounded to bf16 where the reference holds a bf16 array.
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "internal.h"
#include "common.cuh"
#include "stage.cuh"

namespace fmoe {

constexpr int kRowThreads = 256;
constexpr int kRowMaxPer = 16;  // hidden <= 4096

// The row kernels (ff_in / ff_out) run one CTA of kFfThreads per token, each
// thread kFfPer elements of the hidden row.  Every input is loaded before the
// first reduction — the constant norm weights even before griddepcontrol.wait —
// so a call costs one memory round trip plus three or four CTA reductions.
constexpr int kFfThreads = 1024;
constexpr int kFfPer = kRowThreads * kRowMaxPer / kFfThreads;  // 4: hidden <= 4096
constexpr int kFfSlices = 8;                                   // split-K slices loaded per batch

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();  // red is reused across calls
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < NT / 32; ++w) s += red[w];
  return s;
}

__device__ __forceinline__ void load_row_bf16(const bf16* p, int H, float (&v)[kFfPer]) {
#pragma unroll
  for (int k = 0; k < kFfPer; ++k) {
    const int i = threadIdx.x + k * kFfThreads;
    v[k] = (p && i < H) ? bf2f(p[i]) : 0.f;
  }
}

// The row's bf16 bits, not yet converted: loads issued before a dependency
// wait stay in flight across it (converting them would stall there).
__device__ __forceinline__ void load_row_raw(const bf16* p, int H, unsigned short (&v)[kFfPer]) {
#pragma unroll
  for (int k = 0; k < kFfPer; ++k) {
    const int i = threadIdx.x + k * kFfThreads;
    v[k] = (p && i < H) ? __bfloat16_as_ushort(p[i]) : (unsigned short)0;
  }
}
__device__ __forceinline__ void raw_to_f32(const unsigned short (&r)[kFfPer], float (&v)[kFfPer]) {
#pragma unroll
  for (int k = 0; k < kFfPer; ++k) v[k] = __uint_as_float((uint32_t)r[k] << 16);
}

// acc = sum over the split-K slices in slice order (kFfSlices slices' loads in
// flight together).
__device__ __forceinline__ void add_slices(const float* base, int parts, int64_t stride, int H,
                                           float (&acc)[kFfPer]) {
#pragma unroll
  for (int k = 0; k < kFfPer; ++k) acc[k] = 0.f;
  for (int p0 = 0; p0 < parts; p0 += kFfSlices) {
    float v[kFfSlices][kFfPer];
#pragma unroll
    for (int q = 0; q < kFfSlices; ++q)
#pragma unroll
      for (int k = 0; k < kFfPer; ++k) {
        const int i = threadIdx.x + k * kFfThreads;
        v[q][k] = (p0 + q < parts && i < H) ? __ldcg(base + (p0 + q) * stride + i) : 0.f;
      }
#pragma unroll
    for (int q = 0; q < kFfSlices; ++q)
#pragma unroll
      for (int k = 0; k < kFfPer; ++k)
        if (p0 + q < parts) acc[k] += v[q][k];
  }
}

// One CTA per token.  h = bf16(x + bf16(rms(bf16(o)) * w_post_attn));
// h1 / h2 = bf16(rms(h) * w); xs = bf16(bf16(bf16(rms(h2)) * bf16(root)) * router_scale).
__global__ void __launch_bounds__(kFfThreads) ff_in_kernel(const bf16* __restrict__ x, const float* __restrict__ o_acc,
                                                           int o_parts, int64_t o_stride, int H,
                                                           const bf16* __restrict__ w_post_attn,
                                                           const bf16* __restrict__ w_pre_ff,
                                                           const bf16* __restrict__ w_pre_ff2, float eps, float root,
                                                           const bf16* __restrict__ rscale, bf16* __restrict__ h_out,
                                                           bf16* __restrict__ h1_out, bf16* __restrict__ h2_out,
                                                           bf16* __restrict__ xs_out) {
  __shared__ float red[kFfThreads / 32];
  const int t = blockIdx.x;
  float wpa[kFfPer], wpf[kFfPer], wpf2[kFfPer], rsc[kFfPer], xv[kFfPer], a[kFfPer], h[kFfPer], h2[kFfPer];
  unsigned short rwpa[kFfPer], rwpf[kFfPer], rwpf2[kFfPer], rrsc[kFfPer];
  load_row_raw(w_post_attn, H, rwpa);  // constants: in flight across the dependency wait
  load_row_raw(w_pre_ff, H, rwpf);
  load_row_raw(w_pre_ff2, H, rwpf2);
  load_row_raw(rscale, H, rrsc);
  griddep_wait();
  griddep_launch_dependents();
  load_row_bf16(x + (int64_t)t * H, H, xv);
  add_slices(o_acc + (int64_t)t * H, o_parts, o_stride, H, a);
  raw_to_f32(rwpa, wpa);
  raw_to_f32(rwpf, wpf);
  raw_to_f32(rwpf2, wpf2);
  raw_to_f32(rrsc, rsc);
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kFfPer; ++k) {
    a[k] = round_bf(a[k]);
    ss = fmaf(a[k], a[k], ss);
  }
  const float r1 = rsqrtf(block_sum<kFfThreads>(ss, red) / (float)H + eps);
  ss = 0.f;
#pragma unroll
  for (int k = 0; k < kFfPer; ++k) {
    const int i = threadIdx.x + k * kFfThreads;
    h[k] = i < H ? round_bf(xv[k] + round_bf(a[k] * r1 * wpa[k])) : 0.f;
    ss = fmaf(h[k], h[k], ss);
  }
  const float r2 = rsqrtf(block_sum<kFfThreads>(ss, red) / (float)H + eps);
  ss = 0.f;
#pragma unroll
  for (int k = 0; k < kFfPer; ++k) {
    const int i = threadIdx.x + k * kFfThreads;
    if (i < H) {
      h_out[(int64_t)t * H + i] = __float2bfloat16_rn(h[k]);
      h1_out[(int64_t)t * H + i] = __float2bfloat16_rn(h[k] * r2 * wpf[k]);
      h2[k] = round_bf(h[k] * r2 * wpf2[k]);
      h2_out[(int64_t)t * H + i] = __float2bfloat16_rn(h2[k]);
    } else {
      h2[k] = 0.f;
    }
    ss = fmaf(h2[k], h2[k], ss);
  }
  const float r3 = rsqrtf(block_sum<kFfThreads>(ss, red) / (float)H + eps);
  const float rb = round_bf(root);
#pragma unroll
  for (int k = 0; k < kFfPer; ++k) {
    const int i = threadIdx.x + k * kFfThreads;
    if (i < H) {
      float v = round_bf(round_bf(h2[k] * r3) * rb);
      if (rscale) v = round_bf(v * rsc[k]);
      xs_out[(int64_t)t * H + i] = __float2bfloat16_rn(v);
    }
  }
}

// One CTA per token.  x = bf16(bf16(h + bf16(rms(s) * w_post_ff)) * scalar),
// s = bf16(bf16(rms(bf16(d)) * w1) + bf16(rms(moe) * w2)).
__global__ void __launch_bounds__(kFfThreads) ff_out_kernel(const bf16* __restrict__ h_res,
                                                            const float* __restrict__ d_acc, int d_parts,
                                                            int64_t d_stride,
                                                            const bf16* __restrict__ moe, int H,
                                                            const bf16* __restrict__ w1, const bf16* __restrict__ w2,
                                                            const bf16* __restrict__ w, float eps, float scalar,
                                                            bf16* __restrict__ x_out) {
  __shared__ float red[kFfThreads / 32];
  const int t = blockIdx.x;
  float w1v[kFfPer], w2v[kFfPer], wv[kFfPer], d[kFfPer], m[kFfPer], hr[kFfPer];
  unsigned short rw1[kFfPer], rw2[kFfPer], rw[kFfPer];
  load_row_raw(w1, H, rw1);  // constants: in flight across the dependency wait
  load_row_raw(w2, H, rw2);
  load_row_raw(w, H, rw);
  griddep_wait();
  griddep_launch_dependents();
  load_row_bf16(moe + (int64_t)t * H, H, m);
  load_row_bf16(h_res + (int64_t)t * H, H, hr);
  add_slices(d_acc + (int64_t)t * H, d_parts, d_stride, H, d);
  raw_to_f32(rw1, w1v);
  raw_to_f32(rw2, w2v);
  raw_to_f32(rw, wv);
  float sd = 0.f, sm = 0.f;
#pragma unroll
  for (int k = 0; k < kFfPer; ++k) {
    d[k] = round_bf(d[k]);
    sd = fmaf(d[k], d[k], sd);
    sm = fmaf(m[k], m[k], sm);
  }
  const float rd = rsqrtf(block_sum<kFfThreads>(sd, red) / (float)H + eps);
  const float rm = rsqrtf(block_sum<kFfThreads>(sm, red) / (float)H + eps);
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < kFfPer; ++k) {
    const int i = threadIdx.x + k * kFfThreads;
    d[k] = i < H ? round_bf(round_bf(d[k] * rd * w1v[k]) + round_bf(m[k] * rm * w2v[k])) : 0.f;
    ss = fmaf(d[k], d[k], ss);
  }
  const float rs = rsqrtf(block_sum<kFfThreads>(ss, red) / (float)H + eps);
  const float sc = round_bf(scalar);
#pragma unroll
  for (int k = 0; k < kFfPer; ++k) {
    const int i = threadIdx.x + k * kFfThreads;
    if (i < H) {
      const float o = round_bf(hr[k] + round_bf(d[k] * rs * wv[k]));
      x_out[(int64_t)t * H + i] = __float2bfloat16_rn(o * sc);
    }
  }
}

// Softcap (tanh(l / c) * c in the reference's bf16 steps) and greedy argmax
// (ties -> lowest id).  Grid (kCapCtas, T); the last CTA of a token to finish
// merges the CTAs' candidates; it also advances the decode position counters
// when given (pos[0] = position, pos[1] = attended slots).
constexpr int kCapCtas = 64;
__global__ void __launch_bounds__(kRowThreads) softcap_argmax_kernel(float* __restrict__ logits, int64_t V,
                                                                     float cap, float2* __restrict__ cand,
                                                                     unsigned* __restrict__ ctr,
                                                                     int32_t* __restrict__ next_ids,
                                                                     int64_t* __restrict__ pos) {
  __shared__ float bv[kRowThreads / 32];
  __shared__ int bi[kRowThreads / 32];
  __shared__ int last;
  griddep_wait();
  griddep_launch_dependents();
  const int t = blockIdx.y, c = blockIdx.x;
  float* lr = logits + (int64_t)t * V;
  const int64_t per = (V + kCapCtas - 1) / kCapCtas;
  const int64_t lo = c * per, hi = min(V, lo + per);
  float best = -INFINITY;
  int besti = (int)min(lo, V - 1);  // a valid id even if every logit is NaN
  for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
    float v = round_bf(lr[i]);
    if (cap > 0.f) v = round_bf(round_bf(tanhf(round_bf(v / cap))) * cap);
    lr[i] = v;
    if (v > best) {
      best = v;
      besti = (int)i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, besti, o);
    if (ov > best || (ov == best && oi < besti)) {
      best = ov;
      besti = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    bv[warp] = best;
    bi[warp] = besti;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kRowThreads / 32; ++w)
      if (bv[w] > best || (bv[w] == best && bi[w] < besti)) {
        best = bv[w];
        besti = bi[w];
      }
    cand[t * kCapCtas + c] = make_float2(best, __int_as_float(besti));
    __threadfence();
    const unsigned prev = atomicAdd(&ctr[t], 1u);
    last = prev == kCapCtas - 1;
  }
  __syncthreads();
  if (!last || threadIdx.x != 0) return;
  __threadfence();
  ctr[t] = 0u;
  for (int k = 0; k < kCapCtas; ++k) {
    const float2 cv = __ldcg(cand + t * kCapCtas + k);
    const int ci = __float_as_int(cv.y);
    if (k == 0 || cv.x > best || (cv.x == best && ci < besti)) {
      best = cv.x;
      besti = ci;
    }
  }
  next_ids[t] = besti;
  if (pos && t == 0) {
    // every token of the step has finished: advance the position counters once
    pos[0] += 1;
    pos[1] += 1;
  }
}

static cudaLaunchConfig_t row_cfg(dim3 grid, cudaStream_t st, cudaLaunchAttribute* attr, int threads = kFfThreads) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cfg;
}

// ---------------------------------------------------------------------------
// The dense MLP and the routed experts of a layer depend only on ff_in's
// outputs and meet again in ff_out, so the experts run on a second stream
// (fork / join through events; a CUDA-graph capture of the layer records the
// same two branches).  One side stream and event pair per device, created on
// first use.
struct Branch {
  cudaStream_t side = nullptr;
  cudaEvent_t fork = nullptr, join = nullptr;
};
// which: 0 the dense-MLP branch; 1 the second attention stream of the batched layer.
static int branch_for_device(Branch* out, int which = 0) {
  static Branch per_dev[64][2];
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return set_error(FMOE_ERR_CUDA, "decoder: no current device");
  std::lock_guard<std::mutex> lock(mu);
  Branch& b = per_dev[dev][which];
  if (!b.side) {
    if (cudaStreamCreateWithFlags(&b.side, cudaStreamNonBlocking) != cudaSuccess ||
        cudaEventCreateWithFlags(&b.fork, cudaEventDisableTiming) != cudaSuccess ||
        cudaEventCreateWithFlags(&b.join, cudaEventDisableTiming) != cudaSuccess) {
      b = Branch{};
      return set_error(FMOE_ERR_CUDA, "decoder: side stream: %s", cudaGetErrorString(cudaGetLastError()));
    }
  }
  *out = b;
  return FMOE_OK;
}

// ---------------------------------------------------------------------------
// Layer workspace (the router counter lives in the 256-byte header).
struct DecWs {
  WsHead h;
  RouterWs rw;
  MoeWs mw;
  float *qkv, *o, *gu, *d;
  bf16 *q, *attn, *hres, *h1, *h2, *xs, *moe;
  int32_t* ids;
  float* wts;
  void* attn_ws;
  EpWs ep;  // expert-parallel exchange (fmoe_decoder_layer_forward_ep only)
  bool dl;  // the streaming path applies (local experts): plan + its workspace
  DlPlan dlp;
  DlWs dlw;
  size_t bytes;
};

// Decode path selection (environment FMOE_DECODE_PATH, read per call):
//   unset / "ops"  the per-op kernel sequence below (the default: fastest
//                  measured for the whole step);
//   "stream"       the six-launch streaming layer of dlayer.cu;
// the lm_head always uses the streaming kernel unless "ops" is set.
static bool stream_layer_path() {
  const char* e = std::getenv("FMOE_DECODE_PATH");
  return e && std::strcmp(e, "stream") == 0;
}
static bool force_ops_path() {
  const char* e = std::getenv("FMOE_DECODE_PATH");
  return e && std::strcmp(e, "ops") == 0;
}

static int dec_dims(const fmoe_decoder_layer_t* L, int* qkv_rows) {
  if (!L) return set_error(FMOE_ERR_INVALID, "decoder: null layer");
  const int H = L->q_proj.in_features, D = L->head_dim;
  if (L->num_heads <= 0 || L->num_kv_heads <= 0 || L->num_heads % L->num_kv_heads)
    return set_error(FMOE_ERR_INVALID, "decoder: heads %d / kv heads %d", L->num_heads, L->num_kv_heads);
  if (H % 64 || H > kRowThreads * kRowMaxPer) return set_error(FMOE_ERR_UNSUPPORTED, "decoder: hidden %d", H);
  if (L->q_proj.out_features != L->num_heads * D || L->k_proj.out_features != L->num_kv_heads * D ||
      L->o_proj.in_features != L->num_heads * D || L->o_proj.out_features != H)
    return set_error(FMOE_ERR_INVALID, "decoder: projection shapes do not match heads x head_dim");
  if (!L->k_eq_v && (!L->v_proj.w || L->v_proj.out_features != L->num_kv_heads * D))
    return set_error(FMOE_ERR_INVALID, "decoder: v_proj missing (k_eq_v = 0)");
  if (L->rope_dims <= 0 || L->rope_dims > D || L->rope_dims % (D / 16))
    return set_error(FMOE_ERR_UNSUPPORTED, "decoder: rope_dims %d (a multiple of %d up to %d)", L->rope_dims, D / 16, D);
  *qkv_rows = (L->num_heads + (L->k_eq_v ? 1 : 2) * L->num_kv_heads) * D;
  return FMOE_OK;
}

// Split-K slices a GEMV over K inputs can produce (qgemv keeps >= 8 groups of
// 64 per column chunk).
// fp32 output slices of a decode projection over K inputs (one per 512-input chunk)
static int max_parts(int K) { return (K + 64 * kRgChunkGroups - 1) / (64 * kRgChunkGroups); }

// ep_ranks > 0: add the expert-parallel exchange buffers for ep_cap tokens per rank.
static size_t carve_dec(Carver& c, int64_t T, const fmoe_decoder_layer_t* L, const KvDev& kv, DecWs* w,
                        int ep_ranks = 0, int64_t ep_cap = 0) {
  DecWs d = {};
  int qkv_rows = 0;
  dec_dims(L, &qkv_rows);
  const int H = L->q_proj.in_features, Id = L->mlp_gate.out_features, QD = L->num_heads * L->head_dim;
  ExpertsDev ex = {};
  to_experts(&L->experts, &ex);
  // Everything that must hold its value between calls (status word, router /
  // expert / attention merge counters) sits at offsets every layer shares.
  // The expert-parallel buffers (their expert-kernel counters included) come
  // next: their size depends on the expert shapes only, so they too sit at the
  // same offset for every layer type, never overlapping another layer's
  // attention scratch or counters.
  d.h = carve_head(c);
  carve_router(c, T, &L->router, d.h, &d.rw);
  carve_moe(c, T, L->router.top_k, ex, &d.mw);
  if (ep_ranks > 0) carve_ep(c, ep_ranks, ep_cap, nullptr, L->router.top_k, ex, d.h, &d.ep);
  d.attn_ws = c.take<uint8_t>(attn_workspace_bytes(kv, L->num_heads));
  d.qkv = c.take<float>((size_t)max_parts(L->q_proj.in_features) * T * qkv_rows);
  d.o = c.take<float>((size_t)max_parts(QD) * T * H);
  d.gu = c.take<float>((size_t)max_parts(H) * T * 2 * Id);
  d.d = c.take<float>((size_t)max_parts(Id) * T * H);
  d.q = c.take<bf16>((size_t)T * QD);
  d.attn = c.take<bf16>((size_t)T * QD);
  d.hres = c.take<bf16>((size_t)T * H);
  d.h1 = c.take<bf16>((size_t)T * H);
  d.h2 = c.take<bf16>((size_t)T * H);
  d.xs = c.take<bf16>((size_t)T * H);
  d.moe = c.take<bf16>((size_t)T * H);
  d.ids = c.take<int32_t>((size_t)T * L->router.top_k);
  d.wts = c.take<float>((size_t)T * L->router.top_k);
  d.dl = ep_ranks == 0 && stream_layer_path() && dl_plan(L, kv, T, &d.dlp) == FMOE_OK;
  if (d.dl) dl_carve(c, d.dlp, &d.dlw);
  d.bytes = c.off + 256;
  if (w) *w = d;
  return d.bytes;
}

// Batched decode (9 .. kBatMaxT sequences): the attention half runs per group
// of <= 8 sequences on the group-sized buffers; the feed-forward half runs
// once over all T.  Same shared-offset order as carve_dec.
constexpr int kBatMaxT = 64;
struct BatWs {
  WsHead h;
  RouterWs rw;
  MoeWs mw;
  void* attn_ws;
  float *qkv, *o;
  bf16 *q, *attn;
  bf16 *hres, *h1, *h2, *xs, *moe, *act, *dd;
  int32_t* ids;
  float* wts;
  // the odd groups' attention-half buffers (second stream); the attention
  // counters there are cleared by each call, as their offset varies by layer
  void* attn_ws2;
  size_t attn_ws2_ctr_bytes;
  float *qkv2, *o2;
  bf16 *q2, *attn2;
  size_t bytes;
};
static size_t carve_bat(Carver& c, int64_t T, const fmoe_decoder_layer_t* L, const KvDev& kv, BatWs* w) {
  BatWs d = {};
  int qkv_rows = 0;
  dec_dims(L, &qkv_rows);
  const int H = L->q_proj.in_features, Id = L->mlp_gate.out_features, QD = L->num_heads * L->head_dim;
  const int64_t G = T < 8 ? T : 8;
  ExpertsDev ex = {};
  to_experts(&L->experts, &ex);
  KvDev kg = kv;
  kg.B = (int)G;
  d.h = carve_head(c);
  carve_router(c, T, &L->router, d.h, &d.rw);
  carve_moe(c, T, L->router.top_k, ex, &d.mw);
  d.attn_ws = c.take<uint8_t>(attn_workspace_bytes(kg, L->num_heads));
  d.qkv = c.take<float>((size_t)max_parts(H) * G * qkv_rows);
  d.o = c.take<float>((size_t)max_parts(QD) * G * H);
  d.q = c.take<bf16>((size_t)G * QD);
  d.attn = c.take<bf16>((size_t)G * QD);
  d.hres = c.take<bf16>((size_t)T * H);
  d.h1 = c.take<bf16>((size_t)T * H);
  d.h2 = c.take<bf16>((size_t)T * H);
  d.xs = c.take<bf16>((size_t)T * H);
  d.moe = c.take<bf16>((size_t)T * H);
  d.act = c.take<bf16>((size_t)T * Id);
  d.dd = c.take<bf16>((size_t)T * H);
  d.ids = c.take<int32_t>((size_t)T * L->router.top_k);
  d.wts = c.take<float>((size_t)T * L->router.top_k);
  d.attn_ws2 = c.take<uint8_t>(attn_workspace_bytes(kg, L->num_heads));
  d.attn_ws2_ctr_bytes = 256 + sizeof(unsigned) * (size_t)G * kv.Hkv;  // status word slot + merge counters
  d.qkv2 = c.take<float>((size_t)max_parts(H) * G * qkv_rows);
  d.o2 = c.take<float>((size_t)max_parts(QD) * G * H);
  d.q2 = c.take<bf16>((size_t)G * QD);
  d.attn2 = c.take<bf16>((size_t)G * QD);
  d.bytes = c.off + 256;
  if (w) *w = d;
  return d.bytes;
}

// Sequences [b0, b0 + nb) of a cache as a cache of batch nb (same storage).
static KvDev kv_group(const KvDev& kv, int b0, int nb) {
  KvDev g = kv;
  g.B = nb;
  const int64_t rows = (int64_t)b0 * kv.Hkv * kv.cap;
  const int D = kv.D;
  if (kv.mode == FMOE_KV_BF16) {
    g.k = static_cast<bf16*>(kv.k) + rows * D;
    g.v = static_cast<bf16*>(kv.v) + rows * D;
  } else {  // packed 4-bit K, 8-bit V; bf16 scale / bias per 64 elements
    g.k = static_cast<uint8_t*>(kv.k) + rows * (D / 2);
    g.v = static_cast<uint8_t*>(kv.v) + rows * D;
    g.ks = kv.ks + rows * (D / 64);
    g.kb = kv.kb + rows * (D / 64);
    g.vs = kv.vs + rows * (D / 64);
    g.vb = kv.vb + rows * (D / 64);
  }
  return g;
}

static QgSeg seg_of(const QW& q, void* out, int ld, int col0) {
  return QgSeg{static_cast<const uint8_t*>(q.w), q.s, q.b, out, q.out, ld, col0, 0, q.tiled, q.tiled_kc};
}

static RgSeg rseg_of(const QW& q, float* out, int ld, int col0) {
  RgSeg s = {};
  s.w = static_cast<const uint8_t*>(q.w);
  s.s = q.s;
  s.b = q.b;
  s.out = out;
  s.rows = q.out;
  s.ld = ld;
  s.col0 = col0;
  return s;
}

static int check_stream_w(const QW& q, int group, const char* what) {
  if ((q.bits != 4 && q.bits != 6 && q.bits != 8) || group != 64 || q.in % 64 || q.out % 16 ||
      !aligned(q.w, 16) || !aligned(q.s, 16) || !aligned(q.b, 16))
    return set_error(FMOE_ERR_UNSUPPORTED, "decoder: %s must be 4/6/8-bit, group 64, 16-byte aligned", what);
  return FMOE_OK;
}

}  // namespace fmoe

using namespace fmoe;

extern "C" {

size_t fmoe_decoder_workspace_bytes(int64_t T, const fmoe_decoder_layer_t* layer, const fmoe_kv_cache_t* cache) {
  KvDev kv;
  int qkv_rows;
  if (T <= 0 || T > kBatMaxT || dec_dims(layer, &qkv_rows) || kv_to_dev(cache, &kv)) return 0;
  Carver c(nullptr);
  return T > 8 ? carve_bat(c, T, layer, kv, nullptr) : carve_dec(c, T, layer, kv, nullptr);
}

}  // extern "C"

namespace {

// Expert-parallel arguments of a layer call (comm == nullptr: all experts local).
struct EpCall {
  const fmoe_ep_comm_t* comm;
  int n_ranks;
  int64_t cap;
  const void* prep;
  int mode;
};

// Steps 1-5 of a layer for T <= 8 sequences (kv: their cache, or a view of
// sequences of a larger one): q|k|v, norms / RoPE / append, attention, o, and
// ff_in's residual and feed-forward input norms into h / h1 / h2 / xs.
struct AttnBufs {
  float *qkv, *o;
  bf16 *q, *attn;
  void* attn_ws;
  bf16 *hres, *h1, *h2, *xs;
  int* status;
};
int attn_half(const fmoe_decoder_layer_t* L, const KvDev& kv, const QW& q, const QW& k, const QW& v, const QW& o,
              int qkv_rows, bf16* xb, int64_t T, int64_t pos, const int64_t* pos_dev, const AttnBufs& w,
              cudaStream_t st) {
  const int H = q.in, QD = L->num_heads * L->head_dim;
  const int Ti = (int)T;
  int rc, o_parts = 1;
  // 1 q|k|v = input_norm(x) . W^T  (fp32 slices, one per 512-input chunk)
  int qkv_parts = 1;
  {
    RgArgs a = {};
    a.nseg = L->k_eq_v ? 2 : 3;
    a.seg[0] = rseg_of(q, w.qkv, qkv_rows, 0);
    a.seg[1] = rseg_of(k, w.qkv, qkv_rows, QD);
    if (!L->k_eq_v) a.seg[2] = rseg_of(v, w.qkv, qkv_rows, QD + k.out);
    a.K = H;
    a.T = Ti;
    a.in_kind = QG_IN_RMSNORM;
    a.x = xb;
    a.ldx = H;
    a.norm_w = static_cast<const bf16*>(L->input_norm);
    a.eps = L->eps;
    a.status = w.status;
    RgLayout rl;
    // the whole SM: the next kernel (q/k norms, RoPE, append) is a few CTAs
    // that need no room beside it, and every item of the CTA fits in flight
    if ((rc = rgemv_plan(a, q.bits, &rl, 220 * 1024)) || (rc = launch_rgemv(a, rl, q.bits, true, st))) return rc;
    qkv_parts = a.nck;
  }
  // 2 norms, RoPE, KV append
  if ((rc = launch_qkv_post(kv, w.qkv, qkv_rows, qkv_parts, (int64_t)T * qkv_rows, L->num_heads, L->k_eq_v,
                            static_cast<const bf16*>(L->q_norm), static_cast<const bf16*>(L->k_norm), L->eps,
                            L->rope_dims, L->rope_theta, pos, pos_dev, w.q, kv.turbo, true, st)))
    return rc;
  // 3 attention over the slots written so far (pos_dev[1] when counters live on the device)
  const int64_t nvalid = pos + 1 < kv.cap ? pos + 1 : kv.cap;
  if (L->sparse_v_tau > 0.f) {  // gated softmax weights (gemma4_attention.rs:91-93, 196-234)
    if ((rc = launch_sparse_v(kv, w.q, L->num_heads, nvalid, pos_dev ? pos_dev + 1 : nullptr, L->attn_scale,
                              L->sparse_v_tau, w.attn, st)))
      return rc;
  } else if ((rc = launch_attn_decode(kv, w.q, L->num_heads, nvalid, pos_dev ? pos_dev + 1 : nullptr, L->attn_scale,
                                      w.attn_ws, w.attn, st, true, pos, pos_dev))) {
    return rc;
  }
  // 4 o = attn . Wo^T
  {
    RgArgs a = {};
    a.nseg = 1;
    a.seg[0] = rseg_of(o, w.o, H, 0);
    a.K = QD;
    a.T = Ti;
    a.in_kind = QG_IN_BF16;
    a.x = w.attn;
    a.ldx = QD;
    a.status = w.status;
    RgLayout rl;
    if ((rc = rgemv_plan(a, o.bits, &rl)) || (rc = launch_rgemv(a, rl, o.bits, true, st))) return rc;
    o_parts = a.nck;
  }
  // 5 residual + feed-forward input norms
  {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = row_cfg(dim3(Ti), st, attr);
    ProfScope prof_("ff_in_kernel", st);
    cudaLaunchKernelEx(&cfg, ff_in_kernel, (const bf16*)xb, (const float*)w.o, o_parts, (int64_t)T * H, H,
                       static_cast<const bf16*>(L->post_attn_norm), static_cast<const bf16*>(L->pre_ff_norm),
                       static_cast<const bf16*>(L->pre_ff_norm_2), L->eps, L->router.root_size,
                       static_cast<const bf16*>(L->router.router_scale), w.hres, w.h1, w.h2, w.xs);
    if ((rc = check_launch("ff_in_kernel"))) return rc;
  }
  return FMOE_OK;
}

// T > 8 sequences: the attention half per group of <= 8 (views of the cache),
// then router, routed experts and the dense MLP (tensor-core GEMM, T tokens as
// N) once over all T, and the output norms / residual per token.  Each
// expert's weights are read once per layer instead of once per group.
int decoder_forward_batched(const fmoe_decoder_layer_t* L, const KvDev& kv, const QW& q, const QW& k, const QW& v,
                            const QW& o, const QW& gq, const QW& uq, const QW& dq, const QW& rq,
                            const ExpertsDev& ex, int qkv_rows, bf16* xb, int64_t T, int64_t pos,
                            const int64_t* pos_dev, const BatWs& w, cudaStream_t st) {
  const int H = q.in, Id = gq.out;
  int rc;
  if (!qgemm_supported(gq, L->mlp_gate.group_size, H) || !qgemm_supported(uq, L->mlp_up.group_size, H) ||
      !qgemm_supported(dq, L->mlp_down.group_size, Id))
    return set_error(FMOE_ERR_UNSUPPORTED, "decoder: batched dense MLP needs 4/8-bit group-64 weights");
  // even groups on the caller's stream, odd groups on a second stream with
  // their own buffers: one group's row kernels and attention overlap the other
  // group's projections
  const char* ns = std::getenv("FMOE_BATCHED_STREAMS");
  const bool two = T > 8 && !(ns && ns[0] == '1');
  Branch bg;
  if (two) {
    if ((rc = branch_for_device(&bg, 1))) return rc;
    if (cudaEventRecord(bg.fork, st) != cudaSuccess || cudaStreamWaitEvent(bg.side, bg.fork, 0) != cudaSuccess ||
        cudaMemsetAsync(w.attn_ws2, 0, w.attn_ws2_ctr_bytes, bg.side) != cudaSuccess)
      return set_error(FMOE_ERR_CUDA, "decoder: attention fork: %s", cudaGetErrorString(cudaGetLastError()));
  }
  for (int64_t b0 = 0; b0 < T; b0 += 8) {
    const int nb = (int)(T - b0 < 8 ? T - b0 : 8);
    const bool odd = two && ((b0 / 8) & 1);
    const AttnBufs ab = {odd ? w.qkv2 : w.qkv, odd ? w.o2 : w.o, odd ? w.q2 : w.q, odd ? w.attn2 : w.attn,
                         odd ? w.attn_ws2 : w.attn_ws, w.hres + b0 * H, w.h1 + b0 * H, w.h2 + b0 * H, w.xs + b0 * H,
                         w.h.status};
    if ((rc = attn_half(L, kv_group(kv, (int)b0, nb), q, k, v, o, qkv_rows, xb + b0 * H, nb, pos, pos_dev, ab,
                        odd ? bg.side : st)))
      return rc;
  }
  if (two && (cudaEventRecord(bg.join, bg.side) != cudaSuccess || cudaStreamWaitEvent(st, bg.join, 0) != cudaSuccess))
    return set_error(FMOE_ERR_CUDA, "decoder: attention join: %s", cudaGetErrorString(cudaGetLastError()));
  Branch br;
  if ((rc = branch_for_device(&br))) return rc;
  if (cudaEventRecord(br.fork, st) != cudaSuccess || cudaStreamWaitEvent(br.side, br.fork, 0) != cudaSuccess)
    return set_error(FMOE_ERR_CUDA, "decoder: fork: %s", cudaGetErrorString(cudaGetLastError()));
  {
    fmoe_router_t r = L->router;
    r.use_norm = 0;  // ff_in applied the norm chain
    if ((rc = run_router(w.xs, T, &r, rq, w.rw, w.ids, w.wts, nullptr, &w.mw.m, w.h.status, st))) return rc;
    if ((rc = run_experts(w.h2, T, r.top_k, w.ids, w.wts, ex, w.moe, w.mw, false, w.h.status, st))) return rc;
  }
  {  // dense MLP: gated gate|up GEMM (gelu(g) * u), then down
    const QmOut gu[2] = {{&gq, w.act, Id}, {&uq, w.act, Id}};
    if ((rc = launch_qgemm(w.h1, T, H, gu, 2, true, w.h.status, br.side))) return rc;
    const QmOut dd{&dq, w.dd, H};
    if ((rc = launch_qgemm(w.act, T, Id, &dd, 1, false, w.h.status, br.side))) return rc;
  }
  if (cudaEventRecord(br.join, br.side) != cudaSuccess || cudaStreamWaitEvent(st, br.join, 0) != cudaSuccess)
    return set_error(FMOE_ERR_CUDA, "decoder: join: %s", cudaGetErrorString(cudaGetLastError()));
  return launch_ff_out_rows(xb, w.hres, w.dd, w.moe, T, H, static_cast<const bf16*>(L->post_ff_norm_1),
                            static_cast<const bf16*>(L->post_ff_norm_2), static_cast<const bf16*>(L->post_ff_norm),
                            L->eps, L->layer_scalar, st);
}

int decoder_forward(const fmoe_decoder_layer_t* L, const fmoe_kv_cache_t* cache, const EpCall& epc, void* x,
                    int64_t T, int64_t pos, const int64_t* pos_dev, void* workspace, size_t workspace_bytes,
                    void* stream) {
  int qkv_rows = 0;
  int rc = dec_dims(L, &qkv_rows);
  if (rc) return rc;
  KvDev kv;
  rc = kv_to_dev(cache, &kv);
  if (rc) return rc;
  if (T < 1 || T > (epc.comm ? 8 : kBatMaxT))
    return set_error(FMOE_ERR_UNSUPPORTED, "decoder: T=%lld (1..8 sequences per call; up to %d with all experts local)",
                     (long long)T, kBatMaxT);
  if (kv.B != T || kv.Hkv != L->num_kv_heads || kv.D != L->head_dim)
    return set_error(FMOE_ERR_INVALID, "decoder: cache [%d, %d, ., %d] does not match T=%lld / kv heads / head_dim",
                     kv.B, kv.Hkv, kv.D, (long long)T);
  if (!x || !aligned(x, 16)) return set_error(FMOE_ERR_ALIGN, "decoder: x null or not 16-byte aligned");
  QW q, k, v, o, gq, uq, dq, rq;
  ExpertsDev ex;
  if ((rc = to_qw(&L->q_proj, &q)) || (rc = to_qw(&L->k_proj, &k)) || (rc = to_qw(&L->o_proj, &o)) ||
      (rc = to_qw(&L->mlp_gate, &gq)) || (rc = to_qw(&L->mlp_up, &uq)) || (rc = to_qw(&L->mlp_down, &dq)) ||
      (rc = check_router(&L->router, &rq)) || (rc = to_experts(&L->experts, &ex)))
    return rc;
  if (!L->k_eq_v && (rc = to_qw(&L->v_proj, &v))) return rc;
  if ((rc = check_stream_w(q, L->q_proj.group_size, "q_proj")) || (rc = check_stream_w(k, L->k_proj.group_size, "k_proj")) ||
      (!L->k_eq_v && (rc = check_stream_w(v, L->v_proj.group_size, "v_proj"))) ||
      (rc = check_stream_w(o, L->o_proj.group_size, "o_proj")) ||
      (rc = check_stream_w(gq, L->mlp_gate.group_size, "mlp gate")) ||
      (rc = check_stream_w(uq, L->mlp_up.group_size, "mlp up")) ||
      (rc = check_stream_w(dq, L->mlp_down.group_size, "mlp down")))
    return rc;
  const int H = q.in, Id = gq.out, QD = L->num_heads * L->head_dim;
  if (k.in != H || o.out != H || gq.in != H || uq.out != Id || uq.in != H || dq.in != Id || dq.out != H ||
      ex.H != H || rq.in != H || (!L->k_eq_v && v.in != H))
    return set_error(FMOE_ERR_INVALID, "decoder: hidden / intermediate sizes disagree across weights");
  if (epc.comm && (T > epc.cap || (rc = ep_check(epc.comm, ex, rq.out, nullptr))))
    return rc ? rc : set_error(FMOE_ERR_INVALID, "decoder: T=%lld above the exchange capacity", (long long)T);
  if (!epc.comm && ex.first != 0) return set_error(FMOE_ERR_INVALID, "decoder: expert slice without a communicator");
  if (!(L->sparse_v_tau >= 0.f))
    return set_error(FMOE_ERR_INVALID, "decoder: sparse_v_tau %g", (double)L->sparse_v_tau);
  if (T > 8) {
    Carver bz(nullptr);
    const size_t bneed = carve_bat(bz, T, L, kv, nullptr);
    if (!workspace || workspace_bytes < bneed || !aligned(workspace, 16))
      return set_error(FMOE_ERR_WORKSPACE, "decoder: workspace %zu < %zu", workspace_bytes, bneed);
    Carver bc(workspace);
    BatWs bw;
    carve_bat(bc, T, L, kv, &bw);
    return decoder_forward_batched(L, kv, q, k, v, o, gq, uq, dq, rq, ex, qkv_rows, static_cast<bf16*>(x), T, pos,
                                   pos_dev, bw, static_cast<cudaStream_t>(stream));
  }
  Carver cz(nullptr);
  const size_t need = carve_dec(cz, T, L, kv, nullptr, epc.n_ranks, epc.cap);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 16))
    return set_error(FMOE_ERR_WORKSPACE, "decoder: workspace %zu < %zu", workspace_bytes, need);
  Carver c(workspace);
  DecWs w;
  carve_dec(c, T, L, kv, &w, epc.n_ranks, epc.cap);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  bf16* xb = static_cast<bf16*>(x);
  const int Ti = (int)T;
  int gu_parts = 1, d_parts = 1;
  if (w.dl) {
    if (L->sparse_v_tau > 0.f)
      return set_error(FMOE_ERR_UNSUPPORTED, "decoder: sparse-V gating on the layered path only");
    const DlBufs b = {w.q, w.attn, w.hres, w.h1, w.h2, w.xs, w.moe, w.attn_ws};
    return dl_layer_forward(L, kv, w.dlp, w.dlw, xb, pos, pos_dev, b, st);
  }

  {
    const AttnBufs ab = {w.qkv, w.o, w.q, w.attn, w.attn_ws, w.hres, w.h1, w.h2, w.xs, w.h.status};
    if ((rc = attn_half(L, kv, q, k, v, o, qkv_rows, xb, T, pos, pos_dev, ab, st))) return rc;
  }
  // fork: the dense MLP (6, 10) on the side stream; the router and routed
  // experts (7-9), the longer chain, stay here, so ff_out follows the last
  // expert kernel under programmatic dependent launch
  Branch br;
  if ((rc = branch_for_device(&br))) return rc;
  if (cudaEventRecord(br.fork, st) != cudaSuccess || cudaStreamWaitEvent(br.side, br.fork, 0) != cudaSuccess)
    return set_error(FMOE_ERR_CUDA, "decoder: fork: %s", cudaGetErrorString(cudaGetLastError()));
  // 7-9 router on the prepared input, routed experts on h2
  {
    const cudaStream_t sx = st;
    fmoe_router_t r = L->router;
    r.use_norm = 0;  // ff_in applied the norm chain
    if (epc.comm) {  // routed experts on their owning ranks
      if ((rc = run_router(w.xs, T, &r, rq, w.rw, w.ids, w.wts, nullptr, nullptr, w.h.status, sx))) return rc;
      if ((rc = ep_experts(epc.comm, w.h2, T, epc.cap, r.top_k, w.ids, w.wts, ex, static_cast<const bf16*>(epc.prep),
                           w.moe, w.ep, epc.mode, w.h.status, sx)))
        return rc;
    } else {
      if ((rc = run_router(w.xs, T, &r, rq, w.rw, w.ids, w.wts, nullptr, &w.mw.m, w.h.status, sx))) return rc;
      if ((rc = run_experts(w.h2, T, r.top_k, w.ids, w.wts, ex, w.moe, w.mw, false, w.h.status, sx))) return rc;
    }
  }
  // 6 dense MLP gate | up
  {
    RgArgs a = {};
    a.nseg = 2;
    a.seg[0] = rseg_of(gq, w.gu, 2 * Id, 0);
    a.seg[1] = rseg_of(uq, w.gu, 2 * Id, Id);
    a.K = H;
    a.T = Ti;
    a.in_kind = QG_IN_BF16;
    a.x = w.h1;
    a.ldx = H;
    a.status = w.h.status;
    RgLayout rl;
    if ((rc = rgemv_plan(a, gq.bits, &rl)) || (rc = launch_rgemv(a, rl, gq.bits, true, br.side))) return rc;
    gu_parts = a.nck;
  }
  // 10 dense down on gelu(g) * u
  {
    RgArgs a = {};
    a.nseg = 1;
    a.seg[0] = rseg_of(dq, w.d, H, 0);
    a.K = Id;
    a.T = Ti;
    a.in_kind = QG_IN_GELU;
    a.g = w.gu;
    a.u = w.gu + Id;
    a.ldgu = 2 * Id;
    a.gu_parts = gu_parts;
    a.gu_part_stride = (int64_t)T * 2 * Id;
    a.status = w.h.status;
    RgLayout rl;
    if ((rc = rgemv_plan(a, dq.bits, &rl)) || (rc = launch_rgemv(a, rl, dq.bits, true, br.side))) return rc;
    d_parts = a.nck;
  }
  if (cudaEventRecord(br.join, br.side) != cudaSuccess)
    return set_error(FMOE_ERR_CUDA, "decoder: join: %s", cudaGetErrorString(cudaGetLastError()));
  // join: ff_out needs both branches
  if (cudaStreamWaitEvent(st, br.join, 0) != cudaSuccess)
    return set_error(FMOE_ERR_CUDA, "decoder: join: %s", cudaGetErrorString(cudaGetLastError()));
  // 11 output norms, residual, layer scalar -> x
  {
    cudaLaunchAttribute attr[1];
    cudaLaunchConfig_t cfg = row_cfg(dim3(Ti), st, attr);
    ProfScope prof_("ff_out_kernel", st);
    cudaLaunchKernelEx(&cfg, ff_out_kernel, (const bf16*)w.hres, (const float*)w.d, d_parts, (int64_t)T * H,
                       (const bf16*)w.moe, H,
                       static_cast<const bf16*>(L->post_ff_norm_1), static_cast<const bf16*>(L->post_ff_norm_2),
                       static_cast<const bf16*>(L->post_ff_norm), L->eps, L->layer_scalar, xb);
    if ((rc = check_launch("ff_out_kernel"))) return rc;
  }
  return FMOE_OK;
}

}  // namespace

extern "C" {

int fmoe_decoder_layer_forward(const fmoe_decoder_layer_t* L, const fmoe_kv_cache_t* cache, void* x, int64_t T,
                               int64_t pos, const int64_t* pos_dev, void* workspace, size_t workspace_bytes,
                               void* stream) {
  return decoder_forward(L, cache, EpCall{nullptr, 0, 0, nullptr, 0}, x, T, pos, pos_dev, workspace, workspace_bytes,
                         stream);
}

size_t fmoe_decoder_ep_workspace_bytes(int64_t T, const fmoe_decoder_layer_t* layer, const fmoe_kv_cache_t* cache,
                                       int n_ranks, int64_t cap) {
  KvDev kv;
  int qkv_rows;
  if (T <= 0 || n_ranks < 1 || cap < T || dec_dims(layer, &qkv_rows) || kv_to_dev(cache, &kv)) return 0;
  Carver c(nullptr);
  return carve_dec(c, T, layer, kv, nullptr, n_ranks, cap);
}

int fmoe_decoder_layer_forward_ep(const fmoe_decoder_layer_t* L, const fmoe_kv_cache_t* cache, fmoe_ep_comm_t* comm,
                                  int64_t cap, const void* prepared, int mode, void* x, int64_t T, int64_t pos,
                                  const int64_t* pos_dev, void* workspace, size_t workspace_bytes, void* stream) {
  if (!comm) return set_error(FMOE_ERR_INVALID, "decoder_ep: null communicator");
  ExpertsDev ex;
  QW rq;
  int rc, R = 0;
  if ((rc = to_experts(&L->experts, &ex)) || (rc = check_router(&L->router, &rq)) ||
      (rc = ep_check(comm, ex, rq.out, &R)))
    return rc;
  return decoder_forward(L, cache, EpCall{comm, R, cap, prepared, mode}, x, T, pos, pos_dev, workspace,
                         workspace_bytes, stream);
}

size_t fmoe_lm_head_workspace_bytes(int64_t T) {
  if (T <= 0) return 0;
  const size_t ops = 256 + align_up(sizeof(unsigned) * (size_t)T, 256) + sizeof(float2) * (size_t)T * kCapCtas;
  const size_t streaming = dl_lm_workspace_bytes(T);
  return ops > streaming ? ops : streaming;
}

int fmoe_lm_head(const fmoe_qweight_t* embed, const void* final_norm, float eps, const void* x, int64_t T,
                 float softcap, float* logits, int32_t* next_ids, int64_t* pos_dev, void* workspace,
                 size_t workspace_bytes, void* stream) {
  QW q;
  int rc = to_qw(embed, &q);
  if (rc) return rc;
  if ((rc = check_stream_w(q, embed->group_size, "embedding"))) return rc;
  if (T < 1 || T > 8) return set_error(FMOE_ERR_UNSUPPORTED, "lm_head: T=%lld (1..8)", (long long)T);
  if (!x || !logits || !next_ids || !final_norm) return set_error(FMOE_ERR_INVALID, "lm_head: null pointer");
  if (!workspace || workspace_bytes < fmoe_lm_head_workspace_bytes(T))
    return set_error(FMOE_ERR_WORKSPACE, "lm_head: workspace too small");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (!force_ops_path())
    return dl_lm_head(q, static_cast<const bf16*>(final_norm), eps, static_cast<const bf16*>(x), T, softcap, logits,
                      next_ids, pos_dev, workspace, st);
  uint8_t* base = static_cast<uint8_t*>(workspace);
  int* status = reinterpret_cast<int*>(base);
  unsigned* ctr = reinterpret_cast<unsigned*>(base + 256);
  float2* cand = reinterpret_cast<float2*>(base + 256 + align_up(sizeof(unsigned) * (size_t)T, 256));
  QgArgs a = {};
  a.nseg = 1;
  a.seg[0] = seg_of(q, logits, q.out, 0);
  a.K = q.in;
  a.T = (int)T;
  a.out_kind = QG_OUT_F32;
  a.in_kind = QG_IN_RMSNORM;
  a.x = static_cast<const bf16*>(x);
  a.ldx = q.in;
  a.norm_w = static_cast<const bf16*>(final_norm);
  a.eps = eps;
  a.status = status;
  QgLayout ql;
  if ((rc = qgemv_plan(a, q.bits, false, &ql)) || (rc = launch_qgemv(a, ql, q.bits, true, st))) return rc;
  cudaLaunchAttribute attr[1];
  cudaLaunchConfig_t cfg = row_cfg(dim3(kCapCtas, (unsigned)T), st, attr, kRowThreads);
  ProfScope prof_("softcap_argmax_kernel", st);
  cudaLaunchKernelEx(&cfg, softcap_argmax_kernel, logits, (int64_t)q.out, softcap, cand, ctr, next_ids, pos_dev);
  return check_launch("softcap_argmax_kernel");
}

}  // extern "C"
