// Next-token sampling on the device: the engine's sample() (src/engine.rs:
// 302-355) for every row of the lm_head's logits, so the decode loop needs no
// host round trip per token (the reference materialises the logits on the host
// for its repetition penalty, engine.rs:305-327).
//
//   1. repetition penalty over the row's recent tokens, each distinct token
//      once: a logit >= 0 is divided by the penalty, a negative one multiplied
//      (engine.rs:314-320; applied when penalty > 1 and the list is non-empty)
//   2. temperature 0: argmax, first maximum (engine.rs:329-331)
//   3. z = logits / temperature (engine.rs:333)
//   4. top_p < 1 (engine.rs:335-350): descending order (stable: ties in token
//      order), p = softmax, cumulative = running sum of p, a token is dropped
//      when cumulative - p > top_p; dropped tokens get probability 0
//   5. categorical draw from log(p + 1e-10) (engine.rs:352-354), as a
//      Gumbel-max: argmax over tokens of log(p + 1e-10) + G with
//      G = -log(-log(u)), evaluated as argmax of (p + 1e-10) / (-log(u))
//      (the same order, one logarithm per token).  u comes from a
//      counter-based generator keyed by (seed, call number, row, token), so a
//      CUDA graph replays fresh draws while any draw can be recomputed on the
//      host.
//
// Kernels (one CTA per 4096 logits of a row, grid.y = rows):
//   sample_prep_kernel     penalty, / temperature, chunk max (argmax at T = 0)
//   sample_exp_kernel      row max, exp, chunk sums; sort keys when top_p < 1
//   (cub radix sort of the 64-bit keys row | descending z, stable)
//   sample_psum_kernel     per chunk of sorted positions: its probability mass
//   sample_cut_kernel      per chunk: running sum from the earlier chunks' mass,
//                          the kept tokens and their mass
//   sample_draw_kernel     per token (p + 1e-10) / E, chunk argmax
//   sample_finish_kernel   row argmax -> token; ring push; call counter + 1
#include <climits>
#include <cmath>
#include <cub/device/device_radix_sort.cuh>

#include "common.cuh"
#include "internal.h"

namespace fmoe {
namespace smp {

constexpr int kThreads = 256, kPer = 16, kChunk = kThreads * kPer;
constexpr int kMaxRecent = 4096;

struct Part {
  float max, sum, score;
  int idx;
};
struct Cut {  // per (row, chunk of sorted positions)
  float psum, kept_e;
  int kept, pad;
};

// splitmix64's output function (Steele, Lea & Flood 2014; Vigna's constants)
__host__ __device__ inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}
__host__ __device__ inline uint64_t row_key(uint64_t seed, uint64_t step, uint64_t row) {
  return mix64(mix64(seed ^ (step * 0x9E3779B97F4A7C15ull)) ^ (row * 0xD1B54A32D192ED03ull));
}
// uniform in (0, 1) from 23 random bits: (k + 0.5) / 2^23, exact in fp32
// (k + 0.5 needs 24 significant bits), so -log(u) > 0 for every k
__device__ inline float uniform(uint64_t key, int idx) {
  const uint64_t b = mix64(key + (uint64_t)(uint32_t)idx * 0xA0761D6478BD642Full);
  return ((float)(uint32_t)(b >> 41) + 0.5f) * (1.0f / 8388608.0f);
}
// order-preserving float <-> uint32
__device__ inline uint32_t mono(float f) {
  const uint32_t b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ inline float unmono(uint32_t m) {
  return __uint_as_float((m & 0x80000000u) ? (m & 0x7fffffffu) : ~m);
}
// (score, idx) order: larger score, then lower index
__device__ inline bool better(float s, int i, float bs, int bi) { return s > bs || (s == bs && i < bi); }

struct Args {
  const float* logits;
  int64_t V;
  int rows, nch;
  const int32_t* recent;
  int n_recent;
  float temperature, top_p, penalty;
  uint64_t seed;
  uint64_t* step;  // device call counter or null (then step 0)
  int push;
  int32_t* out;
  float* z;                  // [rows, V]
  uint64_t *keys, *keys_sorted;  // [rows, V]
  int32_t *vals, *vals_sorted;   // [rows, V]
  Part* parts;               // [rows, nch]
  Cut* cut;                  // [rows, nch]
};

template <int NT>
__device__ inline void block_best(float& s, int& i, float* ss, int* si) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float s2 = __shfl_xor_sync(0xffffffffu, s, o);
    const int i2 = __shfl_xor_sync(0xffffffffu, i, o);
    if (better(s2, i2, s, i)) s = s2, i = i2;
  }
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) ss[w] = s, si[w] = i;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int k = 1; k < NT / 32; ++k)
      if (better(ss[k], si[k], s, i)) s = ss[k], i = si[k];
  }
}

__global__ void __launch_bounds__(kThreads) sample_prep_kernel(const Args a) {
  __shared__ float zs[kChunk];
  __shared__ float ss[kThreads / 32];
  __shared__ int si[kThreads / 32];
  const int row = blockIdx.y;
  const int64_t c0 = (int64_t)blockIdx.x * kChunk;
  const float* lg = a.logits + (int64_t)row * a.V;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = threadIdx.x + j * kThreads;
    zs[e] = c0 + e < a.V ? lg[c0 + e] : -INFINITY;
  }
  __syncthreads();
  if (a.penalty > 1.f && a.n_recent > 0) {
    const int32_t* rc = a.recent + (int64_t)row * a.n_recent;
    for (int j = threadIdx.x; j < a.n_recent; j += kThreads) {
      const int t = rc[j];
      if (t < 0 || t >= a.V || t < c0 || t >= c0 + kChunk) continue;
      bool first = true;
      for (int q = 0; q < j && first; ++q) first = rc[q] != t;
      if (!first) continue;  // each distinct token once (engine.rs:315)
      float& v = zs[t - c0];
      v = v >= 0.f ? v / a.penalty : v * a.penalty;
    }
    __syncthreads();
  }
  float best = -INFINITY;
  int bi = INT_MAX;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int e = threadIdx.x + j * kThreads;
    if (c0 + e >= a.V) continue;
    float v = zs[e];
    if (a.temperature > 0.f) {
      v = v / a.temperature;
      a.z[(int64_t)row * a.V + c0 + e] = v;
    }
    if (better(v, (int)(c0 + e), best, bi)) best = v, bi = (int)(c0 + e);
  }
  block_best<kThreads>(best, bi, ss, si);
  if (threadIdx.x == 0) {
    Part& p = a.parts[(int64_t)row * a.nch + blockIdx.x];
    p.max = best;
    p.score = best;
    p.idx = bi;
  }
}

// row max over the chunk maxima (every CTA of the row computes the same)
__device__ inline float row_max(const Args& a, int row) {
  float m = -INFINITY;
  for (int c = 0; c < a.nch; ++c) m = fmaxf(m, a.parts[(int64_t)row * a.nch + c].max);
  return m;
}
__device__ inline float row_sum(const Args& a, int row) {
  float s = 0.f;
  for (int c = 0; c < a.nch; ++c) s += a.parts[(int64_t)row * a.nch + c].sum;
  return s;
}

__global__ void __launch_bounds__(kThreads) sample_exp_kernel(const Args a) {
  __shared__ float sm, red[kThreads / 32];
  const int row = blockIdx.y;
  const int64_t c0 = (int64_t)blockIdx.x * kChunk;
  if (threadIdx.x == 0) sm = row_max(a, row);
  __syncthreads();
  const float m = sm;
  const bool sort = a.top_p < 1.f;
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int64_t i = c0 + threadIdx.x + j * kThreads;
    if (i >= a.V) continue;
    const int64_t o = (int64_t)row * a.V + i;
    const float z = a.z[o];
    s += expf(z - m);
    if (sort) {
      a.keys[o] = ((uint64_t)row << 32) | (uint64_t)(~mono(z));
      a.vals[o] = (int32_t)i;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) t += red[w];
    a.parts[(int64_t)row * a.nch + blockIdx.x].sum = t;
  }
}

// Sorted positions of a chunk: thread t owns the kPer consecutive positions
// c0 + kPer*t ...; p = exp(z - m) / S in that order.
__device__ inline void sorted_chunk(const Args& a, int row, int64_t c0, float m, float S, float* e, float* p) {
  const uint64_t* ks = a.keys_sorted + (int64_t)row * a.V;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    const int64_t j = c0 + (int64_t)threadIdx.x * kPer + i;
    e[i] = j < a.V ? expf(unmono(~(uint32_t)ks[j]) - m) : 0.f;
    p[i] = e[i] / S;
  }
}

__global__ void __launch_bounds__(kThreads) sample_psum_kernel(const Args a) {
  __shared__ float sm, sS, red[kThreads / 32];
  const int row = blockIdx.y;
  if (threadIdx.x == 0) sm = row_max(a, row), sS = row_sum(a, row);
  __syncthreads();
  float e[kPer], p[kPer];
  sorted_chunk(a, row, (int64_t)blockIdx.x * kChunk, sm, sS, e, p);
  float t = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; ++i) t += p[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = t;
  __syncthreads();
  if (threadIdx.x == 0) {
    float c = 0.f;
    for (int w = 0; w < kThreads / 32; ++w) c += red[w];
    a.cut[(int64_t)row * a.nch + blockIdx.x].psum = c;
  }
}

// cumulative(j) = mass of the earlier chunks + the running sum inside this
// one; a token is kept unless cumulative - p > top_p.  Chunks that start well
// past top_p keep nothing (their first token's cumulative - p is the earlier
// mass, up to rounding).
__global__ void __launch_bounds__(kThreads) sample_cut_kernel(const Args a) {
  __shared__ float sm, sS, soff, wtot[kThreads / 32], ke_w[kThreads / 32];
  __shared__ int kc_w[kThreads / 32];
  const int row = blockIdx.y, c = blockIdx.x, lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  Cut* out = a.cut + (int64_t)row * a.nch + c;
  if (threadIdx.x == 0) {
    sm = row_max(a, row), sS = row_sum(a, row);
    float off = 0.f;
    for (int q = 0; q < c; ++q) off += a.cut[(int64_t)row * a.nch + q].psum;
    soff = off;
  }
  __syncthreads();
  if (soff - a.top_p > 1e-3f) {  // block-uniform
    if (threadIdx.x == 0) out->kept = 0, out->kept_e = 0.f;
    return;
  }
  float e[kPer], p[kPer];
  sorted_chunk(a, row, (int64_t)c * kChunk, sm, sS, e, p);
  float tot = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; ++i) tot += p[i];
  // exclusive scan of the thread totals: within the warp, then over the warps
  float incl = tot;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) wtot[w] = incl;
  __syncthreads();
  float before = soff;
  for (int q = 0; q < w; ++q) before += wtot[q];
  float cum = before + incl - tot;
  int kept = 0;
  float kept_e = 0.f;
#pragma unroll
  for (int i = 0; i < kPer; ++i) {
    cum += p[i];
    const int64_t j = (int64_t)c * kChunk + (int64_t)threadIdx.x * kPer + i;
    if (j < a.V && !(cum - p[i] > a.top_p)) ++kept, kept_e += e[i];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    kept += __shfl_xor_sync(0xffffffffu, kept, o);
    kept_e += __shfl_xor_sync(0xffffffffu, kept_e, o);
  }
  if (lane == 0) kc_w[w] = kept, ke_w[w] = kept_e;
  __syncthreads();
  if (threadIdx.x == 0) {
    int k = 0;
    float ke = 0.f;
    for (int q = 0; q < kThreads / 32; ++q) k += kc_w[q], ke += ke_w[q];
    out->kept = k;
    out->kept_e = ke;
  }
}

__global__ void __launch_bounds__(kThreads) sample_draw_kernel(const Args a) {
  __shared__ float sm, sK;
  __shared__ int sk;
  __shared__ float ss[kThreads / 32];
  __shared__ int si[kThreads / 32];
  const int row = blockIdx.y;
  const int64_t c0 = (int64_t)blockIdx.x * kChunk;
  const bool sort = a.top_p < 1.f;
  if (threadIdx.x == 0) {
    if (sort) {
      int k = 0;
      float ke = 0.f;
      for (int q = 0; q < a.nch; ++q) {
        const Cut& ct = a.cut[(int64_t)row * a.nch + q];
        k += ct.kept, ke += ct.kept_e;
      }
      sm = row_max(a, row), sK = ke, sk = k;
    } else {
      sm = row_max(a, row), sK = row_sum(a, row), sk = INT_MAX;
    }
  }
  __syncthreads();
  const float m = sm, Sk = sK;
  const int kept = sk;
  const uint64_t key = row_key(a.seed, a.step ? *a.step : 0ull, (uint64_t)row);
  float best = -INFINITY;
  int bi = INT_MAX;
#pragma unroll 4
  for (int j = 0; j < kPer; ++j) {
    const int64_t pos = c0 + threadIdx.x + j * kThreads;
    if (pos >= a.V) continue;
    const int64_t o = (int64_t)row * a.V + pos;
    float z;
    int idx;
    if (sort) {
      z = unmono(~(uint32_t)a.keys_sorted[o]);
      idx = a.vals_sorted[o];
    } else {
      z = a.z[o];
      idx = (int)pos;
    }
    const float p = pos < kept ? expf(z - m) / Sk : 0.f;
    const float E = -logf(uniform(key, idx));
    const float s = (p + 1e-10f) / E;
    if (better(s, idx, best, bi)) best = s, bi = idx;
  }
  block_best<kThreads>(best, bi, ss, si);
  if (threadIdx.x == 0) {
    Part& p = a.parts[(int64_t)row * a.nch + blockIdx.x];
    p.score = best;
    p.idx = bi;
  }
}

// One warp per row: the row's best (score, token); ring push; the call counter
// advances once every row has its token.
__global__ void __launch_bounds__(256) sample_finish_kernel(const Args a) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint64_t step = a.step ? *a.step : 0ull;
  for (int row = w; row < a.rows; row += blockDim.x >> 5) {
    float best = -INFINITY;
    int bi = INT_MAX;
    for (int c = lane; c < a.nch; c += 32) {
      const Part p = a.parts[(int64_t)row * a.nch + c];
      if (better(p.score, p.idx, best, bi)) best = p.score, bi = p.idx;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float s2 = __shfl_xor_sync(0xffffffffu, best, o);
      const int i2 = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(s2, i2, best, bi)) best = s2, bi = i2;
    }
    if (lane == 0) {
      a.out[row] = bi;
      if (a.push && a.step && a.n_recent > 0)
        const_cast<int32_t*>(a.recent)[(int64_t)row * a.n_recent + (int64_t)(step % (uint64_t)a.n_recent)] = bi;
    }
  }
  __syncthreads();
  if (threadIdx.x == 0 && a.step) *a.step = step + 1;
}

struct Ws {
  float* z;
  uint64_t *keys, *keys_sorted;
  int32_t *vals, *vals_sorted;
  Part* parts;
  Cut* cut;
  void* cub_tmp;
  size_t cub_bytes, total;
};

int end_bit(int rows) {
  int b = 0;
  while ((1 << b) < rows) ++b;
  return 32 + b;
}

Ws carve(int rows, int64_t V, uint8_t* base) {
  Ws w{};
  const int64_t n = (int64_t)rows * V;
  const int nch = (int)((V + kChunk - 1) / kChunk);
  cub::DeviceRadixSort::SortPairs(nullptr, w.cub_bytes, (uint64_t*)nullptr, (uint64_t*)nullptr, (int32_t*)nullptr,
                                  (int32_t*)nullptr, (int)n, 0, end_bit(rows));
  size_t o = 0;
  auto take = [&](size_t bytes) {
    uint8_t* p = base ? base + o : nullptr;
    o = (o + bytes + 255) & ~size_t(255);
    return p;
  };
  w.z = reinterpret_cast<float*>(take(n * 4));
  w.keys = reinterpret_cast<uint64_t*>(take(n * 8));
  w.keys_sorted = reinterpret_cast<uint64_t*>(take(n * 8));
  w.vals = reinterpret_cast<int32_t*>(take(n * 4));
  w.vals_sorted = reinterpret_cast<int32_t*>(take(n * 4));
  w.parts = reinterpret_cast<Part*>(take((size_t)rows * nch * sizeof(Part)));
  w.cut = reinterpret_cast<Cut*>(take((size_t)rows * nch * sizeof(Cut)));
  w.cub_tmp = take(w.cub_bytes);
  w.total = o;
  return w;
}

bool shape_ok(int64_t rows, int64_t V) {
  return rows >= 1 && rows <= 65535 && V >= 1 && V <= ((int64_t)1 << 30) && rows * V <= INT32_MAX;
}

}  // namespace smp
}  // namespace fmoe

using namespace fmoe;

extern "C" {

size_t fmoe_sample_workspace_bytes(int64_t rows, int64_t vocab) {
  if (!smp::shape_ok(rows, vocab)) return 0;
  return smp::carve((int)rows, vocab, nullptr).total;
}

int fmoe_sample(const float* logits, int64_t rows, int64_t vocab, int32_t* recent, int n_recent, float temperature,
                float top_p, float rep_penalty, uint64_t seed, uint64_t* step_dev, int push_recent, int32_t* out,
                void* workspace, size_t workspace_bytes, void* stream) {
  if (!smp::shape_ok(rows, vocab))
    return set_error(FMOE_ERR_INVALID, "sample: rows %lld (1..65535), vocab %lld", (long long)rows,
                     (long long)vocab);
  if (!logits || !out) return set_error(FMOE_ERR_INVALID, "sample: null logits / out");
  if (!(temperature >= 0.f) || !(top_p >= 0.f) || !(rep_penalty > 0.f) || !std::isfinite(temperature))
    return set_error(FMOE_ERR_INVALID, "sample: temperature %g (>= 0), top_p %g (>= 0), penalty %g (> 0)",
                     (double)temperature, (double)top_p, (double)rep_penalty);
  if (n_recent < 0 || n_recent > smp::kMaxRecent || (n_recent > 0 && !recent))
    return set_error(FMOE_ERR_INVALID, "sample: %d recent tokens (0..%d, non-null)", n_recent, smp::kMaxRecent);
  if (push_recent && (!step_dev || n_recent == 0))
    return set_error(FMOE_ERR_INVALID, "sample: pushing into the recent ring needs the device call counter");
  const smp::Ws w = smp::carve((int)rows, vocab, static_cast<uint8_t*>(workspace));
  if (!workspace || workspace_bytes < w.total)
    return set_error(FMOE_ERR_WORKSPACE, "sample: workspace %zu < %zu bytes", workspace_bytes, w.total);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nch = (int)((vocab + smp::kChunk - 1) / smp::kChunk);
  const smp::Args a{logits, vocab, (int)rows, nch, recent, n_recent, temperature, top_p, rep_penalty, seed,
                    step_dev, push_recent, out, w.z, w.keys, w.keys_sorted, w.vals, w.vals_sorted, w.parts, w.cut};
  const dim3 grid(nch, (unsigned)rows);
  int rc;
  {
    ProfScope prof_("sample_prep_kernel", st);
    smp::sample_prep_kernel<<<grid, smp::kThreads, 0, st>>>(a);
  }
  if ((rc = check_launch("sample_prep_kernel"))) return rc;
  if (temperature > 0.f) {
    {
      ProfScope prof_("sample_exp_kernel", st);
      smp::sample_exp_kernel<<<grid, smp::kThreads, 0, st>>>(a);
    }
    if ((rc = check_launch("sample_exp_kernel"))) return rc;
    if (top_p < 1.f) {
      size_t tb = w.cub_bytes;
      const cudaError_t e = cub::DeviceRadixSort::SortPairs(w.cub_tmp, tb, w.keys, w.keys_sorted, w.vals,
                                                            w.vals_sorted, (int)(rows * vocab), 0,
                                                            smp::end_bit((int)rows), st);
      if (e != cudaSuccess) return set_error(FMOE_ERR_CUDA, "sample: radix sort: %s", cudaGetErrorString(e));
      {
        ProfScope prof_("sample_psum_kernel", st);
        smp::sample_psum_kernel<<<grid, smp::kThreads, 0, st>>>(a);
      }
      if ((rc = check_launch("sample_psum_kernel"))) return rc;
      {
        ProfScope prof_("sample_cut_kernel", st);
        smp::sample_cut_kernel<<<grid, smp::kThreads, 0, st>>>(a);
      }
      if ((rc = check_launch("sample_cut_kernel"))) return rc;
    }
    {
      ProfScope prof_("sample_draw_kernel", st);
      smp::sample_draw_kernel<<<grid, smp::kThreads, 0, st>>>(a);
    }
    if ((rc = check_launch("sample_draw_kernel"))) return rc;
  }
  {
    ProfScope prof_("sample_finish_kernel", st);
    smp::sample_finish_kernel<<<1, 256, 0, st>>>(a);
  }
  return check_launch("sample_finish_kernel");
}

}  // extern "C"
