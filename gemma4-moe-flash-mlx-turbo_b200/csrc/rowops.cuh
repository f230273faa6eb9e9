// Warp-per-row helpers for head vectors of D = 32 * P values (lane l holds
// elements l*P .. l*P+P-1): bf16 row load / store, RMSNorm and MLX fast::rope
// (non-traditional), each result rounded to bf16 like the reference's bf16
// arrays.
#pragma once
#include "common.cuh"

namespace fmoe {

template <int P>
__device__ __forceinline__ void load_row_f32(const bf16* row, int lane, float (&v)[P]) {
  const uint4* p = reinterpret_cast<const uint4*>(row + lane * P);
#pragma unroll
  for (int i = 0; i < P / 8; ++i) {
    const uint4 w = p[i];
    v[8 * i + 0] = bf16lo(w.x);
    v[8 * i + 1] = bf16hi(w.x);
    v[8 * i + 2] = bf16lo(w.y);
    v[8 * i + 3] = bf16hi(w.y);
    v[8 * i + 4] = bf16lo(w.z);
    v[8 * i + 5] = bf16hi(w.z);
    v[8 * i + 6] = bf16lo(w.w);
    v[8 * i + 7] = bf16hi(w.w);
  }
}

template <int P>
__device__ __forceinline__ void store_row_bf16(bf16* row, int lane, const float (&v)[P]) {
  uint4* p = reinterpret_cast<uint4*>(row + lane * P);
#pragma unroll
  for (int i = 0; i < P / 8; ++i)
    p[i] = make_uint4(pack_bf16x2(v[8 * i], v[8 * i + 1]), pack_bf16x2(v[8 * i + 2], v[8 * i + 3]),
                      pack_bf16x2(v[8 * i + 4], v[8 * i + 5]), pack_bf16x2(v[8 * i + 6], v[8 * i + 7]));
}

template <int P>
__device__ __forceinline__ void warp_rms_norm(float (&v)[P], const bf16* w, float eps, int lane) {
  constexpr int D = 32 * P;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < P; ++i) ss = fmaf(v[i], v[i], ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / (float)D + eps);
#pragma unroll
  for (int i = 0; i < P; ++i) v[i] = round_bf(w ? v[i] * r * bf2f(w[lane * P + i]) : v[i] * r);
}

template <int P>
__device__ __forceinline__ void warp_rope(float (&v)[P], int rope_dims, float log2_theta, float pos, int lane) {
  const int half = rope_dims / 2;
  const int ofs = half / P;  // partner lane distance (half is a multiple of P)
  float o[P];
#pragma unroll
  for (int i = 0; i < P; ++i) {
    const float up = __shfl_down_sync(0xffffffffu, v[i], ofs & 31);
    const float dn = __shfl_up_sync(0xffffffffu, v[i], ofs & 31);
    const int e = lane * P + i;
    o[i] = v[i];
    if (e < rope_dims) {
      // inv_freq_j = theta^(-2j / rope_dims), j = e mod half
      const int j = e < half ? e : e - half;
      float sn, cs;
      sincosf(pos * exp2f(-(float)(2 * j) / (float)rope_dims * log2_theta), &sn, &cs);
      o[i] = e < half ? round_bf(v[i] * cs - up * sn) : round_bf(dn * sn + v[i] * cs);
    }
  }
#pragma unroll
  for (int i = 0; i < P; ++i) v[i] = o[i];
}

// The same two steps split so that everything independent of the row can run
// early (before a programmatic-dependent wait): norm weights as floats and the
// lane's RoPE cos / sin.
template <int P>
__device__ __forceinline__ void warp_rms_norm_w(float (&v)[P], const float (&wv)[P], bool has_w, float eps, int lane) {
  constexpr int D = 32 * P;
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < P; ++i) ss = fmaf(v[i], v[i], ss);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float r = rsqrtf(ss / (float)D + eps);
#pragma unroll
  for (int i = 0; i < P; ++i) v[i] = round_bf(has_w ? v[i] * r * wv[i] : v[i] * r);
}
template <int P>
__device__ __forceinline__ void rope_angles(int rope_dims, float log2_theta, float pos, int lane, float (&cs)[P],
                                            float (&sn)[P]) {
  const int half = rope_dims / 2;
#pragma unroll
  for (int i = 0; i < P; ++i) {
    const int e = lane * P + i;
    cs[i] = 1.f;
    sn[i] = 0.f;
    if (e < rope_dims) {
      const int j = e < half ? e : e - half;
      sincosf(pos * exp2f(-(float)(2 * j) / (float)rope_dims * log2_theta), &sn[i], &cs[i]);
    }
  }
}
template <int P>
__device__ __forceinline__ void warp_rope_cs(float (&v)[P], int rope_dims, const float (&cs)[P], const float (&sn)[P],
                                             int lane) {
  const int half = rope_dims / 2;
  const int ofs = half / P;
  float o[P];
#pragma unroll
  for (int i = 0; i < P; ++i) {
    const float up = __shfl_down_sync(0xffffffffu, v[i], ofs & 31);
    const float dn = __shfl_up_sync(0xffffffffu, v[i], ofs & 31);
    const int e = lane * P + i;
    o[i] = v[i];
    if (e < rope_dims) o[i] = e < half ? round_bf(v[i] * cs[i] - up * sn[i]) : round_bf(dn * sn[i] + v[i] * cs[i]);
  }
#pragma unroll
  for (int i = 0; i < P; ++i) v[i] = o[i];
}

}  // namespace fmoe
