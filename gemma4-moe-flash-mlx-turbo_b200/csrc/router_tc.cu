// Router for many tokens on the tensor cores: the gate projection of
// Gemma4MoeBlock's router (src/model/moe.rs:324-330, logits = x . Wr^T with a
// bf16 router weight) as one tcgen05 GEMM per 128-token tile, with the top-k
// selection, renormalised softmax and per-expert scale (moe.rs:331-345) fused
// into the epilogue.
//
// CTA = 128 tokens x all E experts (E <= 256, a multiple of 16), 6 warps:
//   warp 0     TMA producer: per 64-wide K tile the token tile (128 x 64 bf16)
//              and the router tile (E x 64 bf16), both 128-byte swizzled, into
//              a 4-stage ring
//   warp 1     MMA issuer: 4 tcgen05.mma (K 16) per K tile into one fp32 TMEM
//              accumulator of 128 lanes (tokens) x E columns (experts)
//   warps 2-5  epilogue: one token per thread — its E logits from TMEM in
//              16-column loads, + logit bias, into a shared-memory row (the
//              free stage ring); k rounds of argmax (descending logit, ties to
//              the lower id); softmax over the k selected logits, x
//              per_expert_scale
// Results equal the decode router's (same logits up to fp32 summation order,
// same selection and softmax arithmetic).
#include "tc.cuh"

namespace fmoe {
namespace rtc {

using namespace tc;

constexpr int BM = 128, BK = 64, NS = 4, THREADS = 192, KMAX = 16;

struct Args {
  int T, H, E, k;
  const float* bias;   // [E] or null
  const bf16* pes;     // [E] per-expert scale or null
  int32_t* ids;        // [T, k]
  float* wts;          // [T, k]
  float* logits;       // [T, E] or null
  int* status;
};

__host__ __device__ constexpr int stage_bytes(int E) { return BM * BK * 2 + E * BK * 2; }
inline int smem_bytes(int E) { return NS * stage_bytes(E) + 256 + 1024; }
// the epilogue's logit rows [BM][E + 1] fp32 fit in the stage ring
static_assert(BM * (256 + 1) * 4 <= NS * stage_bytes(256), "logit rows exceed the stage ring");

__global__ void __launch_bounds__(THREADS, 1)
    router_tc_kernel(const __grid_constant__ CUtensorMap mx, const __grid_constant__ CUtensorMap mw, const Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023);
  const int STG = stage_bytes(a.E), A_BYTES = BM * BK * 2;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + NS * STG);
  uint64_t* empty = full + NS;
  uint64_t* accf = empty + NS;
  volatile int* failed = reinterpret_cast<volatile int*>(accf + 1);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1) + 1;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tile0 = blockIdx.x * BM, nk = a.H / BK;
  const uint32_t ncols = a.E <= 32 ? 32u : a.E <= 64 ? 64u : a.E <= 128 ? 128u : 256u;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    *failed = 0;
    mbar_fence_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(tmem_slot)),
                 "r"(ncols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      int issued = 0;
      for (int kt = 0; kt < nk; ++kt) {
        const int s = kt % NS;
        if (kt >= NS && !pwait(&empty[s], (uint32_t)((kt / NS) - 1) & 1u, failed, a.status, 41)) break;
        uint8_t* st = smem + s * STG;
        mbar_arrive_expect_tx(&full[s], (uint32_t)STG);
        tma2d(st, &mx, kt * BK, tile0, &full[s]);
        tma2d(st + A_BYTES, &mw, kt * BK, 0, &full[s]);
        issued = kt + 1;
      }
      // copies still in flight finish before the CTA may exit
      for (int kt = issued > NS ? issued - NS : 0; kt < issued; ++kt)
        drain_wait(&full[kt % NS], (uint32_t)(kt / NS) & 1u);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_n(a.E);
      bool ok = true;
      for (int kt = 0; kt < nk && ok; ++kt) {
        const int s = kt % NS;
        ok = pwait(&full[s], (uint32_t)(kt / NS) & 1u, failed, a.status, 42);
        if (!ok) break;
        tc_fence_after();
        const uint32_t sa = smem_u32(smem + s * STG), sb = sa + A_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 16; ++kk)
          mma_ss(tmem, sw128_desc(sa + 32 * kk), sw128_desc(sb + 32 * kk), idesc, (kt | kk) ? 1u : 0u);
        mma_commit(&empty[s]);
      }
      mma_commit(accf);  // arrives once every MMA issued so far is complete
    }
  } else {
    // epilogue: TMEM lane quarter (warp % 4) x 32 = this warp's tokens
    const int q = warp & 3, row = q * 32 + lane, t = tile0 + row;
    const bool ok = __all_sync(0xffffffffu, pwait(accf, 0, failed, a.status, 43));  // warp-uniform: tcgen05.ld
    tc_fence_after();
    if (ok) {
      // the token's E logits (+ bias) into its own shared-memory row; the
      // stage ring is free once every MMA has completed
      float* lg = reinterpret_cast<float*>(smem) + (size_t)row * (a.E + 1);
      for (int c0 = 0; c0 < a.E; c0 += 16) {
        float v[16];
        tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, v);
        tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          if (a.bias) v[j] += __ldg(a.bias + c0 + j);
          lg[c0 + j] = round_bf(v[j]);  // ranked in the router's bf16 output precision
        }
        if (a.logits && t < a.T) {
          float4* o = reinterpret_cast<float4*>(a.logits + (int64_t)t * a.E + c0);
#pragma unroll
          for (int j = 0; j < 4; ++j) o[j] = make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
      }
      // k rounds of argmax (descending logit, ties -> lower id); four
      // interleaved running maxima per round keep the compares independent
      float tv[KMAX];
      int ti[KMAX];
#pragma unroll
      for (int r = 0; r < KMAX; ++r) {
        tv[r] = -INFINITY;
        ti[r] = 0;
        if (r < a.k) {
          float b0 = -INFINITY, b1 = -INFINITY, b2 = -INFINITY, b3 = -INFINITY;
          int i0 = a.E, i1 = a.E, i2 = a.E, i3 = a.E;
          for (int e = 0; e < a.E; e += 4) {
            const float x0 = lg[e], x1 = lg[e + 1], x2 = lg[e + 2], x3 = lg[e + 3];
            if (x0 > b0) { b0 = x0; i0 = e; }
            if (x1 > b1) { b1 = x1; i1 = e + 1; }
            if (x2 > b2) { b2 = x2; i2 = e + 2; }
            if (x3 > b3) { b3 = x3; i3 = e + 3; }
          }
          // merge: larger value, then lower id
          if (b1 > b0 || (b1 == b0 && i1 < i0)) { b0 = b1; i0 = i1; }
          if (b3 > b2 || (b3 == b2 && i3 < i2)) { b2 = b3; i2 = i3; }
          if (b2 > b0 || (b2 == b0 && i2 < i0)) { b0 = b2; i0 = i2; }
          tv[r] = b0;
          ti[r] = i0;
          if (i0 < a.E) lg[i0] = -INFINITY;  // taken
        }
      }
      if (t < a.T) {
        const float m = tv[0];
        float den = 0.f;
#pragma unroll
        for (int r = 0; r < KMAX; ++r)
          if (r < a.k) den += expf(tv[r] - m);
#pragma unroll
        for (int r = 0; r < KMAX; ++r) {
          if (r < a.k) {
            float wv = expf(tv[r] - m) / den;
            if (a.pes) wv *= __bfloat162float(a.pes[ti[r]]);
            a.ids[(int64_t)t * a.k + r] = ti[r];
            a.wts[(int64_t)t * a.k + r] = wv;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(ncols) : "memory");
  }
}

}  // namespace rtc

bool router_tc_eligible(int64_t T, const QW& w, int k) {
  return T >= kRouterTcMinTokens && w.bits == 16 && w.out % 16 == 0 && w.out <= 256 && w.in % 64 == 0 &&
         k <= rtc::KMAX && k <= w.out && T <= (int64_t)1 << 30;
}

int launch_router_tc(const bf16* x, int64_t T, const QW& w, const float* bias, const bf16* pes, int k, int32_t* ids,
                     float* wts, float* logits, int* status, cudaStream_t st) {
  if (!router_tc_eligible(T, w, k)) return set_error(FMOE_ERR_UNSUPPORTED, "router_tc: configuration");
  if (!aligned(x, 16) || !aligned(w.w, 16) || (logits && !aligned(logits, 16)))
    return set_error(FMOE_ERR_ALIGN, "router_tc: x / weight / logits not 16-byte aligned");
  const int H = w.in, E = w.out;
  CUtensorMap mx, mw;
  const cuuint64_t dx[2] = {(cuuint64_t)H, (cuuint64_t)T}, sx[1] = {(cuuint64_t)H * 2};
  const cuuint32_t bx[2] = {(cuuint32_t)rtc::BK, (cuuint32_t)rtc::BM};
  const cuuint64_t dw[2] = {(cuuint64_t)H, (cuuint64_t)E}, sw[1] = {(cuuint64_t)H * 2};
  const cuuint32_t bw[2] = {(cuuint32_t)rtc::BK, (cuuint32_t)E};
  int rc;
  if ((rc = encode(&mx, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, x, dx, sx, bx, CU_TENSOR_MAP_SWIZZLE_128B, "router x")) ||
      (rc = encode(&mw, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w.w, dw, sw, bw, CU_TENSOR_MAP_SWIZZLE_128B,
                   "router weight")))
    return rc;
  const int smem = rtc::smem_bytes(E);
  cudaFuncSetAttribute(rtc::router_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  const rtc::Args a{(int)T, H, E, k, bias, pes, ids, wts, logits, status};
  {
    ProfScope prof_("router_tc_kernel", st);
    rtc::router_tc_kernel<<<(unsigned)((T + rtc::BM - 1) / rtc::BM), rtc::THREADS, smem, st>>>(mx, mw, a);
  }
  return check_launch("router_tc_kernel");
}

}  // namespace fmoe
