// MLX-affine quantise / dequantise kernels (one-off weight preparation and
// the embedding lookup; not on the per-layer decode path).
#include "internal.h"
#include "common.cuh"

namespace fmoe {

__device__ __forceinline__ uint32_t get_code(const uint32_t* row, int64_t j, int bits) {
  const int64_t pos = j * bits;
  const int64_t w = pos >> 5;
  const int sh = (int)(pos & 31);
  uint64_t v = row[w];
  if (sh + bits > 32) v |= (uint64_t)row[w + 1] << 32;
  return (uint32_t)((v >> sh) & ((1u << bits) - 1u));
}

// One thread per group: min/max -> bf16 scale/bias -> codes.  Codes of a
// group occupy group*bits/32 whole words (group*bits is a multiple of 32 for
// every supported width with group 32/64/128), so threads never share a word.
__global__ void quantize_kernel(const void* __restrict__ src, int src_is_bf16, int64_t rows, int64_t cols, int bits,
                                int group, uint32_t* __restrict__ wq, bf16* __restrict__ sc, bf16* __restrict__ bi) {
  const int64_t gpr = cols / group, wpr = cols * bits / 32, wpg = (int64_t)group * bits / 32;
  const int64_t ngroups = rows * gpr;
  for (int64_t gid = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; gid < ngroups;
       gid += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = gid / gpr, gg = gid % gpr;
    const int64_t base = r * cols + gg * group;
    auto load = [&](int i) -> float {
      return src_is_bf16 ? __bfloat162float(static_cast<const bf16*>(src)[base + i])
                         : static_cast<const float*>(src)[base + i];
    };
    float mn = load(0), mx = mn;
    for (int i = 1; i < group; ++i) {
      const float v = load(i);
      mn = fminf(mn, v);
      mx = fmaxf(mx, v);
    }
    const float nmax = (float)((1u << bits) - 1u);
    float scale = __fdiv_rn(__fsub_rn(mx, mn), nmax);
    if (!(scale >= 1e-7f)) scale = 1e-7f;
    const bf16 sb = __float2bfloat16_rn(scale), bb = __float2bfloat16_rn(mn);
    const float s = __bfloat162float(sb), b = __bfloat162float(bb);
    uint32_t* out = wq + r * wpr + gg * wpg;
    uint64_t acc = 0;
    int nacc = 0, wi = 0;
    for (int i = 0; i < group; ++i) {
      float q = rintf(__fdiv_rn(__fsub_rn(load(i), b), s));
      q = fminf(fmaxf(q, 0.0f), nmax);
      acc |= (uint64_t)(uint32_t)q << nacc;
      nacc += bits;
      if (nacc >= 32) {
        out[wi++] = (uint32_t)acc;
        acc >>= 32;
        nacc -= 32;
      }
    }
    sc[r * gpr + gg] = sb;
    bi[r * gpr + gg] = bb;
  }
}

// out[i, c] = bf16(fma(scale, q, bias)) of row ids[i] (or row i when ids is
// null), optionally times bf16(row_scale).  An id outside [0, rows) yields a
// zero row instead of a read outside the table.
__global__ void dequantize_kernel(const uint32_t* __restrict__ wq, const bf16* __restrict__ sc,
                                  const bf16* __restrict__ bi, int64_t rows, int64_t cols, int bits, int group,
                                  const int32_t* __restrict__ ids, int64_t n, float row_scale, int apply_scale,
                                  bf16* __restrict__ out) {
  const int64_t gpr = cols / group, wpr = cols * bits / 32;
  const float rs = round_bf(row_scale);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n * cols; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    const int64_t src = ids ? ids[r] : r;
    if (src < 0 || src >= rows) {
      out[i] = __float2bfloat16_rn(0.f);
      continue;
    }
    const float s = __bfloat162float(sc[src * gpr + c / group]), b = __bfloat162float(bi[src * gpr + c / group]);
    float v = round_bf(fmaf(s, (float)get_code(wq + src * wpr, c, bits), b));
    if (apply_scale) v = v * rs;
    out[i] = __float2bfloat16_rn(v);
  }
}

__global__ void gather_bf16_rows_kernel(const bf16* __restrict__ w, int64_t rows, int64_t cols,
                                        const int32_t* __restrict__ ids, int64_t n, float row_scale, int apply_scale,
                                        bf16* __restrict__ out) {
  const float rs = round_bf(row_scale);
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n * cols; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    const int64_t src = ids[r];
    float v = src >= 0 && src < rows ? __bfloat162float(w[src * cols + c]) : 0.f;
    if (apply_scale) v = v * rs;
    out[i] = __float2bfloat16_rn(v);
  }
}

int launch_quantize(const void* src, int src_is_bf16, int64_t rows, int64_t cols, int bits, int group, uint32_t* wq,
                    bf16* s, bf16* b, cudaStream_t st) {
  const int64_t ng = rows * (cols / group);
  int64_t blocks = (ng + 255) / 256;
  if (blocks > 64 * kNumSMs) blocks = 64 * kNumSMs;
  if (blocks < 1) blocks = 1;
  {
    ProfScope prof_("quantize_kernel", st);
    quantize_kernel<<<(unsigned)blocks, 256, 0, st>>>(src, src_is_bf16, rows, cols, bits, group, wq, s, b);
  }
  return check_launch("quantize_kernel");
}

int launch_dequantize(const QW& w, int group, const int32_t* ids, int64_t n, float row_scale, bf16* out,
                      cudaStream_t st) {
  const int64_t total = n * w.in;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 64 * kNumSMs) blocks = 64 * kNumSMs;
  if (blocks < 1) blocks = 1;
  const int apply = row_scale != 1.0f;
  if (w.bits == 16) {
    if (!ids) return set_error(FMOE_ERR_INVALID, "dequantize: bf16 weight needs row ids");
    {
      ProfScope prof_("gather_bf16_rows_kernel", st);
      gather_bf16_rows_kernel<<<(unsigned)blocks, 256, 0, st>>>(static_cast<const bf16*>(w.w), w.out, w.in, ids, n,
                                                              row_scale, apply, out);
    }
  } else {
    {
      ProfScope prof_("dequantize_kernel", st);
      dequantize_kernel<<<(unsigned)blocks, 256, 0, st>>>(static_cast<const uint32_t*>(w.w), w.s, w.b, w.out, w.in,
                                                        w.bits, group, ids, n, row_scale, apply, out);
    }
  }
  return check_launch("dequantize_kernel");
}

}  // namespace fmoe
