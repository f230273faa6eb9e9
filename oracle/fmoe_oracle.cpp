// fmoe CPU oracle — TEST INFRASTRUCTURE ONLY.
//
// A plain C++ (OpenMP) restatement of the arithmetic that flash-moe's quantized
// MoE / KV-cache hot path performs through MLX.  It is the checker for the CUDA
// library (libfmoe.so) and the timed CPU baseline in bench.py; nothing in the
// product path may link or call it.
//
// PARITY UNPINNED.  The reference (Rust + mlx-rs 0.25.3 / mlx-sys 0.2.0, Metal)
// ships no tests, no golden vectors and no fixtures, and neither a Rust
// toolchain nor MLX is available to run it.  The arithmetic is restated from
// the reference's call sites (cited per function) and from MLX's published
// semantics of the ops it calls; the pieces that are plain Rust in the
// reference (Hadamard construction, LCG signs, Lloyd-Max tables, routing
// renormalisation) are restated exactly and checked by known-answer tests.
//
// Numeric conventions (the definitions the GPU path must reproduce):
//   * bf16 <-> f32 conversion is round-to-nearest-even (RNE).
//   * MLX-affine quantisation, group g along the input dim:
//       w ~= scale * q + bias, q in [0, 2^bits - 1]; the packed row is a
//       little-endian bit stream, element j at bits [j*bits, (j+1)*bits)
//       (for bits in {2,4,8} this is "32/bits values per uint32, lowest bits
//       first").
//   * dequantize(q) = bf16(fmaf(scale, q, bias)).
//   * quantized matmul computes, per group, scale*sum(q*x) + bias*sum(x)
//     (no intermediate rounding of the dequantised weight; the same
//     factorisation MLX's qmv kernels use), accumulated here in double.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <algorithm>
#include <vector>
#include <numeric>
#ifdef _OPENMP
#include <omp.h>
#endif

namespace {

inline float bf2f(uint16_t h) {
  uint32_t u = static_cast<uint32_t>(h) << 16;
  float f;
  std::memcpy(&f, &u, 4);
  return f;
}

inline uint16_t f2bf(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7fffffffu) > 0x7f800000u) return static_cast<uint16_t>((u >> 16) | 0x40u);  // NaN
  uint32_t lsb = (u >> 16) & 1u;
  u += 0x7fffu + lsb;
  return static_cast<uint16_t>(u >> 16);
}

inline float round_bf(float f) { return bf2f(f2bf(f)); }

// Element j of a packed little-endian bit stream of `bits`-wide values.
inline uint32_t get_q(const uint32_t* row, int64_t j, int bits) {
  int64_t pos = j * bits;
  int64_t w = pos >> 5;
  int sh = static_cast<int>(pos & 31);
  uint64_t v = row[w];
  if (sh + bits > 32) v |= static_cast<uint64_t>(row[w + 1]) << 32;
  return static_cast<uint32_t>((v >> sh) & ((1u << bits) - 1u));
}

inline void put_q(uint32_t* row, int64_t j, int bits, uint32_t q) {
  int64_t pos = j * bits;
  int64_t w = pos >> 5;
  int sh = static_cast<int>(pos & 31);
  uint64_t v = static_cast<uint64_t>(q) << sh;
  row[w] |= static_cast<uint32_t>(v);
  if (sh + bits > 32) row[w + 1] |= static_cast<uint32_t>(v >> 32);
}

inline int64_t words_per_row(int64_t cols, int bits) { return cols * bits / 32; }

// gelu_approximate (Hendrycks & Gimpel tanh form), as called at
// src/model/moe.rs:437 and src/model/mlp.rs:37.
inline double gelu_tanh(double g) {
  const double k0 = 0.7978845608028654;  // sqrt(2/pi)
  return 0.5 * g * (1.0 + std::tanh(k0 * (g + 0.044715 * g * g * g)));
}

// Quantise one group of `group` fp32 values.  MLX-affine: scale spans
// [min, max] over 2^bits - 1 steps, bias = min; both rounded to bf16 and the
// codes computed against the rounded values.
inline void quantize_group(const float* w, int group, int bits, uint32_t* qout, uint16_t* s_out,
                           uint16_t* b_out) {
  float mn = w[0], mx = w[0];
  for (int i = 1; i < group; ++i) {
    mn = std::min(mn, w[i]);
    mx = std::max(mx, w[i]);
  }
  const float nmax = static_cast<float>((1u << bits) - 1u);
  float scale = (mx - mn) / nmax;
  if (!(scale >= 1e-7f)) scale = 1e-7f;
  uint16_t sb = f2bf(scale), bb = f2bf(mn);
  float s = bf2f(sb), b = bf2f(bb);
  for (int i = 0; i < group; ++i) {
    float q = std::nearbyint((w[i] - b) / s);
    q = std::min(std::max(q, 0.0f), nmax);
    qout[i] = static_cast<uint32_t>(q);
  }
  *s_out = sb;
  *b_out = bb;
}

// Normalised-free fast Walsh-Hadamard butterfly (natural / Sylvester order):
// stage h = 1, 2, 4, ..., n/2 maps (a, b) at (i, i+h) to (a + b, a - b).  The
// GPU kernels run the same butterfly network, so fp32 results agree bitwise.
inline void fwht_f32(float* v, int n) {
  for (int h = 1; h < n; h <<= 1)
    for (int i = 0; i < n; i += 2 * h)
      for (int j = i; j < i + h; ++j) {
        float a = v[j], b = v[j + h];
        v[j] = a + b;
        v[j + h] = a - b;
      }
}

}  // namespace

extern "C" {

int orc_num_threads() {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

void orc_f32_to_bf16(const float* x, int64_t n, uint16_t* y) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) y[i] = f2bf(x[i]);
}

void orc_bf16_to_f32(const uint16_t* x, int64_t n, float* y) {
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < n; ++i) y[i] = bf2f(x[i]);
}

// ---------------------------------------------------------------------------
// MLX-affine quantisation (mlx::core::quantize, called by the reference at
// src/model/mod.rs:673 when re-quantising unsupported widths).  w: fp32
// [rows, cols]; outputs wq: uint32 [rows, cols*bits/32], scales/biases: bf16
// [rows, cols/group].
void orc_quantize(const float* w, int64_t rows, int64_t cols, int bits, int group, uint32_t* wq,
                  uint16_t* scales, uint16_t* biases) {
  const int64_t wpr = words_per_row(cols, bits), gpr = cols / group;
#pragma omp parallel
  {
    std::vector<uint32_t> q(group);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
      uint32_t* row = wq + r * wpr;
      std::memset(row, 0, sizeof(uint32_t) * wpr);
      for (int64_t g = 0; g < gpr; ++g) {
        quantize_group(w + r * cols + g * group, group, bits, q.data(), scales + r * gpr + g,
                       biases + r * gpr + g);
        for (int i = 0; i < group; ++i) put_q(row, g * group + i, bits, q[i]);
      }
    }
  }
}

// mlx::core::dequantize (reference: embedding gather src/model/mod.rs:145-160,
// re-quantisation src/model/mod.rs:666-670).  out bf16 [rows, cols].
void orc_dequantize(const uint32_t* wq, const uint16_t* scales, const uint16_t* biases, int64_t rows,
                    int64_t cols, int bits, int group, uint16_t* out) {
  const int64_t wpr = words_per_row(cols, bits), gpr = cols / group;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const uint32_t* row = wq + r * wpr;
    for (int64_t c = 0; c < cols; ++c) {
      float s = bf2f(scales[r * gpr + c / group]), b = bf2f(biases[r * gpr + c / group]);
      out[r * cols + c] = f2bf(std::fmaf(s, static_cast<float>(get_q(row, c, bits)), b));
    }
  }
}

// y[t, o] = sum_i x[t, i] * W[o, i]  with W MLX-affine quantised, i.e.
// mlx::core::quantized_matmul(x, w, scales, biases, transpose=true, group, bits)
// as called at src/model/mlp.rs:16-24 and src/model/moe.rs:428-441.
void orc_qmatmul(const uint16_t* x, int64_t T, const uint32_t* wq, const uint16_t* scales,
                 const uint16_t* biases, int64_t out, int64_t in, int bits, int group, float* y) {
  const int64_t wpr = words_per_row(in, bits), gpr = in / group;
  std::vector<double> xf(static_cast<size_t>(T * in)), xs(static_cast<size_t>(T * gpr));
  for (int64_t t = 0; t < T; ++t)
    for (int64_t g = 0; g < gpr; ++g) {
      double acc = 0;
      for (int i = 0; i < group; ++i) {
        double v = bf2f(x[t * in + g * group + i]);
        xf[t * in + g * group + i] = v;
        acc += v;
      }
      xs[t * gpr + g] = acc;
    }
#pragma omp parallel
  {
    std::vector<uint32_t> q(in);
#pragma omp for schedule(static)
    for (int64_t o = 0; o < out; ++o) {
      const uint32_t* row = wq + o * wpr;
      for (int64_t i = 0; i < in; ++i) q[i] = get_q(row, i, bits);
      for (int64_t t = 0; t < T; ++t) {
        double acc = 0;
        const double* xt = &xf[t * in];
        for (int64_t g = 0; g < gpr; ++g) {
          double qd = 0;
          for (int i = 0; i < group; ++i) qd += q[g * group + i] * xt[g * group + i];
          acc += bf2f(scales[o * gpr + g]) * qd + bf2f(biases[o * gpr + g]) * xs[t * gpr + g];
        }
        y[t * out + o] = static_cast<float>(acc);
      }
    }
  }
}

// y[t, o] = sum_i x[t, i] * W[o, i] for a plain bf16 weight [out, in].
void orc_matmul_bf16(const uint16_t* x, int64_t T, const uint16_t* w, int64_t out, int64_t in,
                     float* y) {
#pragma omp parallel for schedule(static)
  for (int64_t o = 0; o < out; ++o)
    for (int64_t t = 0; t < T; ++t) {
      double acc = 0;
      for (int64_t i = 0; i < in; ++i)
        acc += static_cast<double>(bf2f(x[t * in + i])) * bf2f(w[o * in + i]);
      y[t * out + o] = static_cast<float>(acc);
    }
}

// ---------------------------------------------------------------------------
// Router, src/model/moe.rs:324-345 (+ rms_norm_no_scale moe.rs:473-479):
//   if norm:  xs = bf16(bf16(bf16(x * rsqrt(mean(x^2) + eps)) * bf16(root_size)) * router_scale)
//   logits   = xs . Wr^T  (+ logit_bias[e], a synthetic-input device), fp32 in logits_out
//   ids      = top-k of bf16(logits) (descending value, ties -> lower id): the
//              reference's router output is bf16 (moe.rs:330-334)
//   w        = softmax(bf16 logits)[ids] / sum(...)  == softmax over the k selected
//   w       *= per_expert_scale[ids]   (optional)
// wr_bits == 16 means Wr is plain bf16 [E, H]; otherwise MLX-affine packed.
void orc_router(const uint16_t* x, int T, int H, int E, const void* wr, const uint16_t* wr_s,
                const uint16_t* wr_b, int wr_bits, int group, const float* logit_bias,
                int use_norm, float root_size, float eps, const uint16_t* router_scale,
                const uint16_t* per_expert_scale, int k, int32_t* ids, float* weights,
                float* logits_out) {
  std::vector<uint16_t> xs(static_cast<size_t>(T) * H);
  for (int t = 0; t < T; ++t) {
    const uint16_t* xt = x + static_cast<int64_t>(t) * H;
    if (!use_norm) {
      std::memcpy(&xs[static_cast<size_t>(t) * H], xt, sizeof(uint16_t) * H);
      continue;
    }
    double ss = 0;
    for (int h = 0; h < H; ++h) ss += static_cast<double>(bf2f(xt[h])) * bf2f(xt[h]);
    float rms = static_cast<float>(1.0 / std::sqrt(ss / H + static_cast<double>(eps)));
    float root = round_bf(root_size);
    for (int h = 0; h < H; ++h) {
      float v = round_bf(bf2f(xt[h]) * rms);
      v = round_bf(v * root);
      if (router_scale) v = round_bf(v * bf2f(router_scale[h]));
      xs[static_cast<size_t>(t) * H + h] = f2bf(v);
    }
  }
  std::vector<float> lg(static_cast<size_t>(T) * E);
  if (wr_bits == 16)
    orc_matmul_bf16(xs.data(), T, static_cast<const uint16_t*>(wr), E, H, lg.data());
  else
    orc_qmatmul(xs.data(), T, static_cast<const uint32_t*>(wr), wr_s, wr_b, E, H, wr_bits, group,
                lg.data());
  for (int t = 0; t < T; ++t) {
    float* l = &lg[static_cast<size_t>(t) * E];
    if (logit_bias)
      for (int e = 0; e < E; ++e) l[e] += logit_bias[e];
    if (logits_out) std::memcpy(logits_out + static_cast<int64_t>(t) * E, l, sizeof(float) * E);
    // The router projection's output is bf16 in the reference (quantized_matmul /
    // matmul keep x's dtype, moe.rs:330): rank and softmax the rounded logits;
    // the stable sort keeps the lower id first among equal values.
    for (int e = 0; e < E; ++e) l[e] = round_bf(l[e]);
    std::vector<int> ord(E);
    std::iota(ord.begin(), ord.end(), 0);
    std::stable_sort(ord.begin(), ord.end(), [&](int a, int b) { return l[a] > l[b]; });
    double mx = l[ord[0]], den = 0;
    for (int j = 0; j < k; ++j) den += std::exp(static_cast<double>(l[ord[j]]) - mx);
    for (int j = 0; j < k; ++j) {
      int e = ord[j];
      double w = std::exp(static_cast<double>(l[e]) - mx) / den;
      if (per_expert_scale) w *= bf2f(per_expert_scale[e]);
      ids[t * k + j] = e;
      weights[t * k + j] = static_cast<float>(w);
    }
  }
}

// ---------------------------------------------------------------------------
// Routed experts + weighted combine, src/model/moe.rs:424-466:
//   for each token, for each selected expert in ascending id order:
//     g = bf16(x . Wg^T), u = bf16(x . Wu^T)          (quantized_matmul, bf16 out)
//     a = bf16(gelu_tanh(g) * u)
//     d = a . Wd^T
//     y += w * d
// Expert tensors follow the ECB expert-major layout (src/splitter.rs:405-457):
// expert e's tensor j lives at base + e*stride + offs[j], j in
// [gate.w, gate.s, gate.b, up.w, up.s, up.b, down.w, down.s, down.b].
void orc_moe_experts(const uint16_t* x, int T, int H, int I, int k, const int32_t* ids,
                     const float* w, const uint8_t* base, int64_t stride, const int64_t* offs,
                     int bits, int group, float* y_f32, uint16_t* y_bf16, uint16_t* act_out) {
  const int64_t wpr_h = words_per_row(H, bits), gpr_h = H / group;
  const int64_t wpr_i = words_per_row(I, bits), gpr_i = I / group;
  std::vector<double> acc(H), xf(H), xsg(gpr_h), af(I), asg(gpr_i);
  std::vector<uint16_t> a(I);
  for (int t = 0; t < T; ++t) {
    const uint16_t* xt = x + static_cast<int64_t>(t) * H;
    for (int h = 0; h < H; ++h) xf[h] = bf2f(xt[h]);
    for (int g = 0; g < gpr_h; ++g) {
      double s = 0;
      for (int i = 0; i < group; ++i) s += xf[g * group + i];
      xsg[g] = s;
    }
    std::fill(acc.begin(), acc.end(), 0.0);
    std::vector<std::pair<int, int>> order;
    for (int j = 0; j < k; ++j) order.push_back({ids[t * k + j], j});
    std::sort(order.begin(), order.end());
    for (auto& pr : order) {
      const int e = pr.first, slot = pr.second;
      const uint8_t* eb = base + static_cast<int64_t>(e) * stride;
      const uint32_t* gw = reinterpret_cast<const uint32_t*>(eb + offs[0]);
      const uint16_t* gs = reinterpret_cast<const uint16_t*>(eb + offs[1]);
      const uint16_t* gb = reinterpret_cast<const uint16_t*>(eb + offs[2]);
      const uint32_t* uw = reinterpret_cast<const uint32_t*>(eb + offs[3]);
      const uint16_t* us = reinterpret_cast<const uint16_t*>(eb + offs[4]);
      const uint16_t* ub = reinterpret_cast<const uint16_t*>(eb + offs[5]);
      const uint32_t* dw = reinterpret_cast<const uint32_t*>(eb + offs[6]);
      const uint16_t* ds = reinterpret_cast<const uint16_t*>(eb + offs[7]);
      const uint16_t* db = reinterpret_cast<const uint16_t*>(eb + offs[8]);
#pragma omp parallel for schedule(static)
      for (int r = 0; r < I; ++r) {
        double gacc = 0, uacc = 0;
        for (int g = 0; g < gpr_h; ++g) {
          double gq = 0, uq = 0;
          for (int i = 0; i < group; ++i) {
            const int64_t c = g * group + i;
            gq += get_q(gw + r * wpr_h, c, bits) * xf[c];
            uq += get_q(uw + r * wpr_h, c, bits) * xf[c];
          }
          gacc += bf2f(gs[r * gpr_h + g]) * gq + bf2f(gb[r * gpr_h + g]) * xsg[g];
          uacc += bf2f(us[r * gpr_h + g]) * uq + bf2f(ub[r * gpr_h + g]) * xsg[g];
        }
        const double gb16 = round_bf(static_cast<float>(gacc));
        const double ub16 = round_bf(static_cast<float>(uacc));
        a[r] = f2bf(static_cast<float>(gelu_tanh(gb16) * ub16));
        af[r] = bf2f(a[r]);
      }
      if (act_out) std::memcpy(act_out + (static_cast<int64_t>(t) * k + slot) * I, a.data(), 2 * I);
      for (int g = 0; g < gpr_i; ++g) {
        double s = 0;
        for (int i = 0; i < group; ++i) s += af[g * group + i];
        asg[g] = s;
      }
      const double wt = w[t * k + slot];
#pragma omp parallel for schedule(static)
      for (int h = 0; h < H; ++h) {
        double d = 0;
        for (int g = 0; g < gpr_i; ++g) {
          double dq = 0;
          for (int i = 0; i < group; ++i) dq += get_q(dw + h * wpr_i, g * group + i, bits) * af[g * group + i];
          d += bf2f(ds[h * gpr_i + g]) * dq + bf2f(db[h * gpr_i + g]) * asg[g];
        }
        acc[h] += wt * d;
      }
    }
    for (int h = 0; h < H; ++h) {
      const float v = static_cast<float>(acc[h]);
      if (y_f32) y_f32[static_cast<int64_t>(t) * H + h] = v;
      if (y_bf16) y_bf16[static_cast<int64_t>(t) * H + h] = f2bf(v);
    }
  }
}

// ---------------------------------------------------------------------------
// KV cache: TurboQuant constants and round trip, src/cache.rs:6-129.

// generate_hadamard, src/cache.rs:6-26: normalised Sylvester H_n (H H^T = I).
void orc_hadamard(int n, float* h) {
  std::fill(h, h + static_cast<int64_t>(n) * n, 0.0f);
  h[0] = 1.0f;
  for (int size = 1; size < n; size *= 2)
    for (int i = 0; i < size; ++i)
      for (int j = 0; j < size; ++j) {
        float v = h[i * n + j];
        h[i * n + j + size] = v;
        h[(i + size) * n + j] = v;
        h[(i + size) * n + j + size] = -v;
      }
  const float scale = 1.0f / std::sqrt(static_cast<float>(n));
  for (int64_t i = 0; i < static_cast<int64_t>(n) * n; ++i) h[i] *= scale;
}

// deterministic_signs, src/cache.rs:29-43: 64-bit LCG (Knuth MMIX constants),
// sign = +1 when bit 63 of the advanced state is 0.
void orc_signs(int n, uint64_t seed, float* s) {
  uint64_t state = seed;
  for (int i = 0; i < n; ++i) {
    state = state * 6364136223846793005ull + 1442695040888963407ull;
    s[i] = ((state >> 63) & 1ull) == 0 ? 1.0f : -1.0f;
  }
}

// lloyd_max_codebook, src/cache.rs:67-89 (N(0,1) Lloyd-Max tables).  Returns
// the number of centroids; boundaries has (centroids - 1) entries.
int orc_lloyd_max(int bits, float* centroids, float* boundaries) {
  static const float c2[] = {-1.510f, -0.453f, 0.453f, 1.510f};
  static const float b2[] = {-0.982f, 0.0f, 0.982f};
  static const float c3[] = {-2.152f, -1.344f, -0.756f, -0.245f, 0.245f, 0.756f, 1.344f, 2.152f};
  static const float b3[] = {-1.748f, -1.050f, -0.501f, 0.0f, 0.501f, 1.050f, 1.748f};
  static const float c4[] = {-2.733f, -2.069f, -1.618f, -1.256f, -0.942f, -0.657f, -0.388f, -0.128f,
                             0.128f,  0.388f,  0.657f,  0.942f,  1.256f,  1.618f,  2.069f,  2.733f};
  static const float b4[] = {-2.401f, -1.844f, -1.437f, -1.099f, -0.800f, -0.522f, -0.258f, 0.0f,
                             0.258f,  0.522f,  0.800f,  1.099f,  1.437f,  1.844f,  2.401f};
  const float* c = bits == 2 ? c2 : bits == 3 ? c3 : bits == 4 ? c4 : nullptr;
  const float* b = bits == 2 ? b2 : bits == 3 ? b3 : bits == 4 ? b4 : nullptr;
  if (!c) return 0;
  const int n = 1 << bits;
  std::memcpy(centroids, c, sizeof(float) * n);
  std::memcpy(boundaries, b, sizeof(float) * (n - 1));
  return n;
}

// turbo_round_trip_kv, src/cache.rs:94-129, for `rows` vectors of length D
// (rows = B * 2Hkv * T after the reference's concat of K and V on heads):
//   n = ||v||;  y = (v / (n + 1e-8)) @ R * sqrt(D);  idx = #(y >= boundaries)
//   out = bf16(((c[idx] / sqrt(D)) @ R^T) * n),  R = H diag(signs(seed 42)).
// Matrix products are evaluated in double from the fp32 operands (MLX fp32
// matmul; its summation order is not reproducible here).  idx_out (optional)
// receives the codebook index per element.
void orc_turbo_round_trip(const uint16_t* v, int64_t rows, int D, int bits, uint16_t* out,
                          uint8_t* idx_out, float* norm_out) {
  std::vector<float> H(static_cast<size_t>(D) * D), s(D), c(16), b(15);
  orc_hadamard(D, H.data());
  orc_signs(D, 42, s.data());
  const int nc = orc_lloyd_max(bits, c.data(), b.data());
  const float sqrt_d = std::sqrt(static_cast<float>(D)), inv_sqrt_d = 1.0f / sqrt_d;
#pragma omp parallel
  {
    std::vector<float> xv(D), y(D), vals(D);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
      const uint16_t* vr = v + r * D;
      float ss = 0;
      for (int i = 0; i < D; ++i) {
        xv[i] = bf2f(vr[i]);
        ss += xv[i] * xv[i];
      }
      const float n = std::sqrt(ss);
      const float denom = n + 1e-8f;
      for (int i = 0; i < D; ++i) xv[i] = xv[i] / denom;
      for (int j = 0; j < D; ++j) {
        double acc = 0;
        for (int i = 0; i < D; ++i) acc += static_cast<double>(xv[i]) * H[i * D + j] * s[j];
        y[j] = static_cast<float>(acc) * sqrt_d;
        int idx = 0;
        for (int q = 0; q < nc - 1; ++q) idx += (y[j] >= b[q]) ? 1 : 0;
        if (idx_out) idx_out[r * D + j] = static_cast<uint8_t>(idx);
        vals[j] = c[idx] * inv_sqrt_d;
      }
      if (norm_out) norm_out[r] = n;
      for (int j = 0; j < D; ++j) {
        double acc = 0;
        for (int i = 0; i < D; ++i) acc += static_cast<double>(vals[i]) * H[i * D + j] * s[i];
        out[r * D + j] = f2bf(static_cast<float>(acc) * n);
      }
    }
  }
}

// Normalised WHT of `rows` bf16/fp32 vectors (fp32 butterfly, then * 1/sqrt(D)).
void orc_wht_rows(const float* in, int64_t rows, int D, float* out) {
  const float inv = 1.0f / std::sqrt(static_cast<float>(D));
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    float* o = out + r * D;
    std::memcpy(o, in + r * D, sizeof(float) * D);
    fwht_f32(o, D);
    for (int i = 0; i < D; ++i) o[i] *= inv;
  }
}

// Affine-quantised, WHT-rotated KV append (the quantiser of the benchmark's
// quantized-KV configuration; the reference has no counterpart — its cache
// stores bf16 after the TurboQuant round trip, src/cache.rs:290-308).
// For each of `rows` bf16 vectors of length D: r = WHT(v) (butterfly in fp32,
// then * 1/sqrt(D)), then MLX-affine quantise r with `bits`, group `group`.
void orc_kv_quant_affine(const uint16_t* v, int64_t rows, int D, int bits, int group,
                         uint32_t* wq, uint16_t* scales, uint16_t* biases) {
  std::vector<float> f(static_cast<size_t>(rows) * D), r(static_cast<size_t>(rows) * D);
  for (int64_t i = 0; i < rows * D; ++i) f[i] = bf2f(v[i]);
  orc_wht_rows(f.data(), rows, D, r.data());
  orc_quantize(r.data(), rows, D, bits, group, wq, scales, biases);
}

// Decode attention over an affine-quantised rotated cache for one query token
// per (batch, q-head); GQA with Hq/Hkv query heads per KV head.  Positions
// [t_lo, t_hi) of the stored rows are attended (sliding window / causal
// range chosen by the caller).  q: bf16 [B, Hq, D]; cache rows are indexed
// [(b*Hkv + h)*Tcap + t].  Returns out fp32 [B, Hq, D] in the original
// (un-rotated) basis:  out = WHT(softmax(scale * q'.k'^T) . v').
void orc_attn_decode_affine(const uint16_t* q, int B, int Hq, int Hkv, int D, int64_t Tcap,
                            const int32_t* t_lo, const int32_t* t_hi, const uint32_t* kq,
                            const uint16_t* ks, const uint16_t* kb, int kbits, const uint32_t* vq,
                            const uint16_t* vs, const uint16_t* vb, int vbits, int group,
                            float scale, float* out) {
  const int64_t kwpr = words_per_row(D, kbits), vwpr = words_per_row(D, vbits), gpr = D / group;
  const float inv = 1.0f / std::sqrt(static_cast<float>(D));
#pragma omp parallel for schedule(dynamic) collapse(2)
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < Hq; ++h) {
      const int hk = h / (Hq / Hkv);
      std::vector<float> qr(D);
      for (int i = 0; i < D; ++i) qr[i] = bf2f(q[(static_cast<int64_t>(b) * Hq + h) * D + i]);
      fwht_f32(qr.data(), D);
      for (int i = 0; i < D; ++i) qr[i] *= inv;
      const int lo = t_lo[b], hi = t_hi[b];
      std::vector<double> sc(std::max(hi - lo, 0)), acc(D, 0.0);
      double mx = -INFINITY;
      for (int t = lo; t < hi; ++t) {
        const int64_t row = (static_cast<int64_t>(b) * Hkv + hk) * Tcap + t;
        double dot = 0;
        for (int i = 0; i < D; ++i) {
          double kv = static_cast<double>(bf2f(ks[row * gpr + i / group])) * get_q(kq + row * kwpr, i, kbits) +
                      bf2f(kb[row * gpr + i / group]);
          dot += kv * qr[i];
        }
        sc[t - lo] = dot * scale;
        mx = std::max(mx, sc[t - lo]);
      }
      double den = 0;
      for (int t = lo; t < hi; ++t) {
        const double p = std::exp(sc[t - lo] - mx);
        den += p;
        const int64_t row = (static_cast<int64_t>(b) * Hkv + hk) * Tcap + t;
        for (int i = 0; i < D; ++i) {
          double vv = static_cast<double>(bf2f(vs[row * gpr + i / group])) * get_q(vq + row * vwpr, i, vbits) +
                      bf2f(vb[row * gpr + i / group]);
          acc[i] += p * vv;
        }
      }
      std::vector<float> o(D);
      for (int i = 0; i < D; ++i) o[i] = den > 0 ? static_cast<float>(acc[i] / den) : 0.0f;
      fwht_f32(o.data(), D);
      for (int i = 0; i < D; ++i) out[(static_cast<int64_t>(b) * Hq + h) * D + i] = o[i] * inv;
    }
}

// Plain decode SDPA over bf16 K/V (src/model/gemma4_attention.rs:91-104 with
// the reference's additive masks src/model/mod.rs:682-753, and the sparse-V
// gate of gemma4_attention.rs:196-234 when tau > 0).  k, v: bf16 rows as in
// orc_attn_decode_affine.  out fp32 [B, Hq, D].
void orc_attn_decode_bf16(const uint16_t* q, int B, int Hq, int Hkv, int D, int64_t Tcap,
                          const int32_t* t_lo, const int32_t* t_hi, const uint16_t* k,
                          const uint16_t* v, float scale, float tau, float* out) {
#pragma omp parallel for schedule(dynamic) collapse(2)
  for (int b = 0; b < B; ++b)
    for (int h = 0; h < Hq; ++h) {
      const int hk = h / (Hq / Hkv);
      const uint16_t* qh = q + (static_cast<int64_t>(b) * Hq + h) * D;
      const int lo = t_lo[b], hi = t_hi[b];
      std::vector<double> sc(std::max(hi - lo, 0)), acc(D, 0.0);
      double mx = -INFINITY;
      for (int t = lo; t < hi; ++t) {
        const int64_t row = (static_cast<int64_t>(b) * Hkv + hk) * Tcap + t;
        double dot = 0;
        for (int i = 0; i < D; ++i) dot += static_cast<double>(bf2f(qh[i])) * bf2f(k[row * D + i]);
        sc[t - lo] = dot * scale;
        mx = std::max(mx, sc[t - lo]);
      }
      double den = 0;
      for (int t = lo; t < hi; ++t) den += std::exp(sc[t - lo] - mx);
      for (int t = lo; t < hi; ++t) {
        double p = std::exp(sc[t - lo] - mx) / den;
        if (tau > 0 && p < tau) p = 0;
        const int64_t row = (static_cast<int64_t>(b) * Hkv + hk) * Tcap + t;
        for (int i = 0; i < D; ++i) acc[i] += p * bf2f(v[row * D + i]);
      }
      for (int i = 0; i < D; ++i) out[(static_cast<int64_t>(b) * Hq + h) * D + i] = static_cast<float>(acc[i]);
    }
}

// ---------------------------------------------------------------------------
// Decoder-layer pieces (config: Gemma-4 decode step).

// fast::rms_norm (src/model/norm.rs:11-14) and RMSNormNoScale (norm.rs:17-29):
// y = bf16(x * rsqrt(mean(x^2) + eps) * w) per row of n; w == NULL: no scale.
// The mean and rsqrt are evaluated in double, the products in fp32.
void orc_rms_norm(const uint16_t* x, int64_t rows, int n, const uint16_t* w, float eps, uint16_t* y) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const uint16_t* xr = x + r * n;
    double ss = 0;
    for (int i = 0; i < n; ++i) {
      const double v = bf2f(xr[i]);
      ss += v * v;
    }
    const float rs = static_cast<float>(1.0 / std::sqrt(ss / n + static_cast<double>(eps)));
    for (int i = 0; i < n; ++i) {
      const float v = bf2f(xr[i]) * rs;
      y[r * n + i] = f2bf(w ? v * bf2f(w[i]) : v);
    }
  }
}

// fast::rope as called at src/model/gemma4_attention.rs:74-81 (traditional =
// false, scale 1, offset = cache position): for rows of D values, the first
// `dims` rotate in pairs (i, i + dims/2) by angle pos * theta^(-2i/dims),
// out = bf16(x1 cos - x2 sin), bf16(x1 sin + x2 cos); the rest pass through.
// Angles and products in double.
void orc_rope(const uint16_t* x, int64_t rows, int D, int dims, double theta, int64_t pos, uint16_t* y) {
  const int half = dims / 2;
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const uint16_t* xr = x + r * D;
    uint16_t* yr = y + r * D;
    for (int i = 0; i < D; ++i) yr[i] = xr[i];
    for (int i = 0; i < half; ++i) {
      const double ang = static_cast<double>(pos) * std::pow(theta, -2.0 * i / dims);
      const double c = std::cos(ang), s = std::sin(ang);
      const double a = bf2f(xr[i]), b = bf2f(xr[i + half]);
      yr[i] = f2bf(static_cast<float>(a * c - b * s));
      yr[i + half] = f2bf(static_cast<float>(a * s + b * c));
    }
  }
}

}  // extern "C"
