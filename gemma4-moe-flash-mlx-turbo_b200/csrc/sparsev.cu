// Sparse-V decode attention: the reference's optional decode path
// (sparse_v_attention, src/model/gemma4_attention.rs:196-234, enabled by the
// threshold flag of src/main.rs:62-64): p = softmax(scale * q . K^T) over the
// attended slots, weights below tau set to zero (no renormalisation), out =
// p . V.  The gate needs the softmax's global maximum and sum before any
// weight is compared, so this is a two-pass kernel of its own rather than a
// mode of the split-KV decode attention: one CTA per (sequence, query head),
//   pass 1  a warp per key (lanes over head_dim): the score, kept in shared
//           memory; the running maximum and sum of exp over the warp's keys
//   merge   the warps' (max, sum) pairs
//   pass 2  one thread per output dimension: sum over the keys of the gated
//           weight times V (V rows read across the threads, coalesced)
// bf16 caches only (the TurboQuant round trip applies on append, as in the
// dense path); at most kSvMaxSlots attended slots.  The decoder layer runs it
// in place of the split-KV attention when its sparse_v_tau is above zero
// (decode only, gemma4_attention.rs:91-93).
#include <cmath>
#include "internal.h"
#include "common.cuh"

namespace fmoe {
namespace sv {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

// n_dev (optional): the attended slot count on the device (CUDA-graph replay),
// clamped to the capacity; otherwise n.
template <int D>
__global__ void __launch_bounds__(kThreads) sparse_v_kernel(KvDev c, const bf16* __restrict__ q, int Hq, int n_host,
                                                            const int64_t* __restrict__ n_dev, float scale, float tau,
                                                            bf16* __restrict__ out) {
  constexpr int P = D / 32;
  const int n = n_dev ? (int)(*n_dev < c.cap ? *n_dev : c.cap) : n_host;
  extern __shared__ float sc[];  // [n] scores
  __shared__ float wm[kWarps], wl[kWarps];
  const int b = blockIdx.x / Hq, h = blockIdx.x % Hq;
  const int g = h / (Hq / c.Hkv);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const bf16* kb = static_cast<const bf16*>(c.k) + ((int64_t)b * c.Hkv + g) * c.cap * D;
  const bf16* vb = static_cast<const bf16*>(c.v) + ((int64_t)b * c.Hkv + g) * c.cap * D;
  float qv[P];
  const bf16* qr = q + ((int64_t)b * Hq + h) * D + lane * P;
#pragma unroll
  for (int i = 0; i < P; ++i) qv[i] = bf2f(qr[i]);
  // pass 1: scores and each warp's running (max, sum of exp)
  float m = -INFINITY, l = 0.f;
  for (int t = warp; t < n; t += kWarps) {
    const bf16* kr = kb + (int64_t)t * D + lane * P;
    float d = 0.f;
#pragma unroll
    for (int i = 0; i < P; ++i) d = fmaf(qv[i], bf2f(kr[i]), d);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) d += __shfl_xor_sync(0xffffffffu, d, o);
    const float s = d * scale;
    if (lane == 0) sc[t] = s;
    const float mn = fmaxf(m, s);
    l = l * expf(m - mn) + expf(s - mn);
    m = mn;
  }
  if (lane == 0) {
    wm[warp] = m;
    wl[warp] = l;
  }
  __syncthreads();
  float M = -INFINITY, Lsum = 0.f;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) M = fmaxf(M, wm[w]);
#pragma unroll
  for (int w = 0; w < kWarps; ++w)
    if (wl[w] > 0.f) Lsum += wl[w] * expf(wm[w] - M);
  const float inv = Lsum > 0.f ? 1.f / Lsum : 0.f;
  // pass 2: thread i owns output dims i, i + 256, ...
  for (int d = threadIdx.x; d < D; d += kThreads) {
    float acc = 0.f;
    for (int t = 0; t < n; ++t) {
      const float p = expf(sc[t] - M) * inv;
      if (p >= tau) acc = fmaf(p, bf2f(vb[(int64_t)t * D + d]), acc);
    }
    out[((int64_t)b * Hq + h) * D + d] = __float2bfloat16_rn(acc);
  }
}

}  // namespace sv

int kv_to_dev(const fmoe_kv_cache_t* c, KvDev* d);

int launch_sparse_v(const KvDev& c, const bf16* q, int q_heads, int64_t n_valid, const int64_t* n_dev, float scale,
                    float tau, bf16* out, cudaStream_t st) {
  if (c.mode != FMOE_KV_BF16) return set_error(FMOE_ERR_UNSUPPORTED, "sparse_v: bf16-storage caches only");
  if (c.D != 256 && c.D != 512) return set_error(FMOE_ERR_UNSUPPORTED, "sparse_v: head_dim %d", c.D);
  if (q_heads < c.Hkv || q_heads % c.Hkv)
    return set_error(FMOE_ERR_INVALID, "sparse_v: %d query heads over %d kv heads", q_heads, c.Hkv);
  if (n_dev ? c.cap > kSvMaxSlots : (n_valid < 1 || n_valid > c.cap || n_valid > kSvMaxSlots))
    return set_error(FMOE_ERR_UNSUPPORTED, "sparse_v: %lld attended slots, capacity %lld (at most %d)",
                     (long long)n_valid, (long long)c.cap, kSvMaxSlots);
  if (!(tau >= 0.f)) return set_error(FMOE_ERR_INVALID, "sparse_v: threshold %g", (double)tau);
  const unsigned grid = (unsigned)(c.B * q_heads);
  const size_t smem = sizeof(float) * (size_t)(n_dev ? c.cap : n_valid);
  if (c.D == 256) {
    cudaFuncSetAttribute(sv::sparse_v_kernel<256>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(4 * kSvMaxSlots));
    ProfScope prof_("sparse_v_kernel<256>", st);
    sv::sparse_v_kernel<256><<<grid, sv::kThreads, smem, st>>>(c, q, q_heads, (int)n_valid, n_dev, scale, tau, out);
  } else {
    cudaFuncSetAttribute(sv::sparse_v_kernel<512>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(4 * kSvMaxSlots));
    ProfScope prof_("sparse_v_kernel<512>", st);
    sv::sparse_v_kernel<512><<<grid, sv::kThreads, smem, st>>>(c, q, q_heads, (int)n_valid, n_dev, scale, tau, out);
  }
  return check_launch("sparse_v_kernel");
}

}  // namespace fmoe

using namespace fmoe;

extern "C" int fmoe_attn_decode_sparse_v(const fmoe_kv_cache_t* cache, const void* q, int q_heads, int64_t n_valid,
                                         float scale, float tau, void* out, void* stream) {
  KvDev c;
  int rc;
  if (!cache || !q || !out) return set_error(FMOE_ERR_INVALID, "sparse_v: null cache / q / out");
  if ((rc = kv_to_dev(cache, &c))) return rc;
  return launch_sparse_v(c, static_cast<const bf16*>(q), q_heads, n_valid, nullptr, scale, tau, static_cast<bf16*>(out),
                         static_cast<cudaStream_t>(stream));
}
