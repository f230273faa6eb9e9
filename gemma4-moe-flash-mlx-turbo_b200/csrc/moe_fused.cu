// Single-kernel MoE layer for decode (T <= 8 tokens): router, top-k, routed
// experts and combine in one cooperative launch (every CTA co-resident),
// replacing Gemma4MoeBlock::forward's routing eval + host sync + per-expert
// loop (src/model/moe.rs:324-466) with three phases separated by grid
// barriers:
//
//   R  router logits: CTAs (tile, slice) < 8 x kFzSlices each stage a 16-row
//      slice of the router weight with TMA bulk copies; every CTA stages the
//      token rows x.  Partial logits go to the workspace.          [barrier 1]
//   T  every CTA adds the partials, runs top-k (rank counting over all
//      experts, one thread per expert, ties -> lower id), the renormalised
//      weights and the per-expert pair lists — identically, so no further
//      barrier is needed to share the routing.
//   G  gate/up items (selected expert, 16-row tile of the intermediate dim)
//      round-robin over CTAs -> act (bf16, workspace).  A CTA that is done
//      issues the bulk copies of its down tiles right away.        [barrier 2]
//   D  down items (16-row tile of the hidden dim, group of 8 selected
//      experts): one warp per expert, fp32 sums added in warp order; with
//      several expert groups the last CTA of a tile adds the group partials
//      in order (deterministic).
//
// Grid barriers and mbarrier waits are bounded: a wait that gives up records
// a site code in the workspace status word and the CTA skips the rest.
#include "internal.h"
#include "gemv.cuh"
#include "stage.cuh"

namespace fmoe {

constexpr int kFzWarps = 8;
constexpr int kFzThreads = kFzWarps * 32;
constexpr int kFzMaxT = 8;
constexpr int kFzSlices = 8;   // hidden-dim slices per 16-expert router tile
constexpr int kFzMaxE = 256;
constexpr int kFzMaxK = 16;

struct FzArgs {
  const bf16* x;
  int T, E, k;
  const void* wr;  // router weight [E, H]: bf16 (rbits 16) or 4-bit affine
  int rbits;
  const bf16* rsc;
  const bf16* rbi;
  const float* bias;
  const bf16* pes;
  ExpertsDev ex;
  int32_t* ids;
  float* wts;
  bf16* y;
  float* rpart;        // [kFzSlices][T][E]
  bf16* act;           // [T*k][I]
  float* dpart;        // [groups][T][H]
  unsigned* tile_ctr;  // [H/16]
  unsigned* gbar;      // [3] grid barrier counters, zero between calls
  int* status;
};

struct FzLayout {
  int XS, RSg, RSd, AS, G, Gi, gmax_r;
  size_t x_off, xsum_off, lg_off, tab_off, w_off, a_off, bytes;
};

__host__ __device__ inline FzLayout fz_layout(int H, int I, int E, int T, int rbits) {
  FzLayout L;
  L.G = H / 64;
  L.Gi = I / 64;
  L.gmax_r = (L.G + kFzSlices - 1) / kFzSlices;
  L.XS = smem_stride(H * 2, 16);
  L.RSg = smem_stride(H / 2, 8);
  L.RSd = I / 2;  // down tiles stay contiguous (one copy per tile)
  L.AS = smem_stride(I * 2, 16);
  L.x_off = 0;                                                        // x rows [T][XS]
  L.xsum_off = align16(L.x_off + (size_t)T * L.XS);                   // f32 [T][G]
  L.lg_off = align16(L.xsum_off + sizeof(float) * T * L.G);           // f32 [T][E]
  // routing tables: sel_e [T][K], sel_v [T][K], sel_w [T][K], cnt/ustart [E+1], uexp [E], upairs [T*K], misc
  L.tab_off = align16(L.lg_off + sizeof(float) * T * E);
  const size_t tab = sizeof(int) * (3 * kFzMaxT * kFzMaxK + 2 * (kFzMaxE + 1) + kFzMaxT * kFzMaxK + 64);
  L.w_off = align16(L.tab_off + tab);
  // region W: router slice | gate/up tile (+ raw scales, bias dots) | 8 down slots
  const size_t r_bytes = 16 * (size_t)smem_stride(L.gmax_r * 64 * rbits / 8, rbits == 4 ? 8 : 16) +
                         (rbits == 16 ? 0 : 2 * 16 * (size_t)L.gmax_r * 2);
  const size_t g_bytes = 2 * 16 * (size_t)L.RSg + 4 * 16 * (size_t)L.G * 2 + sizeof(float) * 2 * 16 * kFzMaxT;
  const size_t d_bytes = 8 * (16 * (size_t)L.RSd + 2 * 16 * (size_t)L.Gi * 2);
  size_t w = r_bytes > g_bytes ? r_bytes : g_bytes;
  w = w > d_bytes ? w : d_bytes;
  L.a_off = align16(L.w_off + w);
  // act staging for D (8 slots x 1 row) — also the reduction overlay for R / G
  size_t a = 8 * (size_t)L.AS;
  const size_t red = sizeof(float) * kFzWarps * 2 * 16 * 8;
  a = a > red ? a : red;
  L.bytes = L.a_off + a;
  return L;
}

// Bounded grid barrier over all CTAs of a cooperative launch.
__device__ __forceinline__ bool fz_grid_barrier(unsigned* ctr, int* status, int site) {
  __syncthreads();
  int ok = 1;
  if (threadIdx.x == 0) {
    __threadfence();
    atomicAdd(ctr, 1u);
    unsigned v;
    int i = 0;
    for (;;) {
      asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(ctr) : "memory");
      if (v >= gridDim.x) break;
      if (++i > kMaxWaitIters) {
        atomicCAS(status, 0, site);
        ok = 0;
        break;
      }
      __nanosleep(64);
    }
    __threadfence();
  }
  return __syncthreads_and(ok) != 0;
}

__global__ void __launch_bounds__(kFzThreads, 3) moe_decode_fused_kernel(FzArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ __align__(8) uint64_t bar[3];  // 0: x + router/gate-up copies, 1: down prefetch, 2: act rows
  const ExpertsDev& ex = a.ex;
  const int H = ex.H, I = ex.I, T = a.T, E = a.E, k = a.k;
  const FzLayout L = fz_layout(H, I, E, T, a.rbits);
  const int G = L.G, Gi = L.Gi;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  uint8_t* xsm = smem + L.x_off;
  float* xsum = reinterpret_cast<float*>(smem + L.xsum_off);
  float* lg = reinterpret_cast<float*>(smem + L.lg_off);
  int* sel_e = reinterpret_cast<int*>(smem + L.tab_off);
  float* sel_v = reinterpret_cast<float*>(sel_e + kFzMaxT * kFzMaxK);
  float* sel_w = sel_v + kFzMaxT * kFzMaxK;
  int* ucnt = reinterpret_cast<int*>(sel_w + kFzMaxT * kFzMaxK);  // [E+1]: counts, then starts
  int* uexp = ucnt + (kFzMaxE + 1);                               // [E] unique experts (ascending)
  int* upairs = uexp + (kFzMaxE + 1);                             // [T*k]
  int* misc = upairs + kFzMaxT * kFzMaxK;                         // [0] = U, [1..8] warp counts
  uint8_t* wsm = smem + L.w_off;
  uint8_t* asm_ = smem + L.a_off;
  float* red = reinterpret_cast<float*>(smem + L.a_off);
  int* status = a.status;
  uint32_t ph0 = 0;
  bool ok = true;

  if (threadIdx.x == 0) {
    mbar_init(&bar[0], 1);
    mbar_init(&bar[1], 1);
    mbar_init(&bar[2], 1);
    mbar_fence_init();
  }
  __syncthreads();

  // ---------------- phase R: x rows (every CTA) + router slice (router CTAs)
  const int RT = (E + 15) / 16, nR = RT * kFzSlices;
  const bool is_router = blockIdx.x < nR;
  const int r_tile = blockIdx.x % RT, r_slice = blockIdx.x / RT;
  const int rg0 = min(G, r_slice * L.gmax_r), rg1 = min(G, rg0 + L.gmax_r), rng = rg1 - rg0;
  const int RBr = H * a.rbits / 8, GBr = 64 * a.rbits / 8;
  const int RSr = smem_stride(L.gmax_r * GBr, a.rbits == 4 ? 8 : 16);
  if (warp == 0) {
    const uint32_t rbytes = is_router ? 16u * rng * GBr : 0u;
    if (lane == 0) mbar_arrive_expect_tx(&bar[0], rbytes + (uint32_t)T * H * 2);
    __syncwarp();
    if (lane < T) bulk_g2s(xsm + lane * L.XS, a.x + (int64_t)lane * H, H * 2, &bar[0]);
    if (is_router && rng > 0 && lane >= 16) {
      const int r = lane - 16, row = min(r_tile * 16 + r, E - 1);
      bulk_g2s(wsm + r * RSr, static_cast<const uint8_t*>(a.wr) + (int64_t)row * RBr + rg0 * GBr, rng * GBr, &bar[0]);
    }
  }
  if (is_router && a.rbits != 16) {
    bf16* raw = reinterpret_cast<bf16*>(wsm + 16 * RSr);
    for (int i = threadIdx.x; i < 16 * rng; i += blockDim.x) {
      const int r = i / rng, j = i % rng, row = min(r_tile * 16 + r, E - 1);
      raw[r * L.gmax_r + j] = a.rsc[(int64_t)row * G + rg0 + j];
      raw[16 * L.gmax_r + r * L.gmax_r + j] = a.rbi[(int64_t)row * G + rg0 + j];
    }
  }
  ok = mbar_wait(&bar[0], ph0, status, 31);
  ph0 ^= 1;
  __syncthreads();
  // per-(token, group) sums of x, used by the affine fixups of G
  for (int i = warp; i < T * G; i += kFzWarps) {
    const int n = i / G, gi = i % G;
    const uint32_t v = *reinterpret_cast<const uint32_t*>(xsm + n * L.XS + gi * 128 + lane * 4);
    float s = bf16lo(v) + bf16hi(v);
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) xsum[n * G + gi] = s;
  }
  if (is_router && ok) {
    float yv[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j = warp; j < rng; j += kFzWarps) {
      const BFrag4 b = stage_bfrag4(xsm, L.XS, T, rg0 + j, g, t);
      if (a.rbits == 16) {
        const uint8_t* plo = wsm + g * RSr + j * 128 + 32 * t;
        const uint8_t* phi = wsm + (g + 8) * RSr + j * 128 + 32 * t;
        const BFrag4 alo = make_bfrag4(lds_u4(plo), lds_u4(plo + 16)), ahi = make_bfrag4(lds_u4(phi), lds_u4(phi + 16));
#pragma unroll
        for (int s = 0; s < 4; ++s) mma16816(yv, alo.b0[s], ahi.b0[s], alo.b1[s], ahi.b1[s], b.b0[s], b.b1[s]);
      } else {
        const bf16* raw = reinterpret_cast<const bf16*>(wsm + 16 * RSr);
        const uint2 wl = lds_u2(wsm + g * RSr + j * 32 + 8 * t);
        const uint2 wh = lds_u2(wsm + (g + 8) * RSr + j * 32 + 8 * t);
        float c[4] = {0.f, 0.f, 0.f, 0.f}, xs[4] = {0.f, 0.f, 0.f, 0.f};
        mma_group_q4(c, wl, wh, b);
        mma_group_ones(xs, b);
        affine_fixup(yv, c, xs, __bfloat162float(raw[g * L.gmax_r + j]),
                     __bfloat162float(raw[16 * L.gmax_r + g * L.gmax_r + j]),
                     __bfloat162float(raw[(g + 8) * L.gmax_r + j]),
                     __bfloat162float(raw[16 * L.gmax_r + (g + 8) * L.gmax_r + j]), 128.0f);
      }
    }
    red[warp * 128 + g * 8 + 2 * t] = yv[0];
    red[warp * 128 + g * 8 + 2 * t + 1] = yv[1];
    red[warp * 128 + (g + 8) * 8 + 2 * t] = yv[2];
    red[warp * 128 + (g + 8) * 8 + 2 * t + 1] = yv[3];
  }
  __syncthreads();
  if (is_router && ok && threadIdx.x < 128) {
    const int r = threadIdx.x >> 3, c = threadIdx.x & 7;
    if (c < T && r_tile * 16 + r < E) {
      float s = 0.f;
#pragma unroll
      for (int w = 0; w < kFzWarps; ++w) s += red[w * 128 + r * 8 + c];
      a.rpart[((int64_t)r_slice * T + c) * E + r_tile * 16 + r] = s;
    }
  }
  ok = fz_grid_barrier(&a.gbar[0], status, 32) && ok;

  // ---------------- phase T: logits, top-k, weights, routing lists (every CTA)
  for (int i = threadIdx.x; i < T * E; i += blockDim.x) {
    float s = 0.f;
    for (int q = 0; q < kFzSlices; ++q) s += __ldcg(a.rpart + (int64_t)q * T * E + i);
    if (a.bias) s += a.bias[i % E];
    lg[i] = s;
  }
  __syncthreads();
  for (int n = 0; n < T; ++n) {
    for (int e = threadIdx.x; e < E; e += blockDim.x) {
      const float v = lg[n * E + e];
      int rank = 0;
      for (int j = 0; j < E; ++j) {
        const float u = lg[n * E + j];
        rank += (u > v || (u == v && j < e)) ? 1 : 0;
      }
      if (rank < k) {
        sel_e[n * kFzMaxK + rank] = e;
        sel_v[n * kFzMaxK + rank] = v;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x < T * kFzMaxK) {
    const int n = threadIdx.x / kFzMaxK, r = threadIdx.x % kFzMaxK;
    if (r < k) {
      const float m = sel_v[n * kFzMaxK];
      float den = 0.f;
      for (int j = 0; j < k; ++j) den += expf(sel_v[n * kFzMaxK + j] - m);
      float wv = expf(sel_v[n * kFzMaxK + r] - m) / den;
      const int e = sel_e[n * kFzMaxK + r];
      if (a.pes) wv *= bf2f(a.pes[e]);
      sel_w[n * kFzMaxK + r] = wv;
      if (blockIdx.x == 0) {
        a.ids[n * k + r] = e;
        a.wts[n * k + r] = wv;
      }
    }
  }
  // per-expert counts -> exclusive starts, unique list, stable pair lists
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int c = 0;
    for (int p = 0; p < T * k; ++p) c += sel_e[(p / k) * kFzMaxK + p % k] == e ? 1 : 0;
    ucnt[e] = c;
  }
  __syncthreads();
  if (warp == 0) {
    int run = 0, urun = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int c = e < E ? ucnt[e] : 0;
      int incl = c, uincl = c > 0;
      for (int o = 1; o < 32; o <<= 1) {
        const int p = __shfl_up_sync(0xffffffffu, incl, o), q = __shfl_up_sync(0xffffffffu, uincl, o);
        if (lane >= o) {
          incl += p;
          uincl += q;
        }
      }
      if (e < E) {
        ucnt[e] = run + incl - c;  // start of e's pairs
        if (c > 0) uexp[urun + uincl - 1] = e;
      }
      run += __shfl_sync(0xffffffffu, incl, 31);
      urun += __shfl_sync(0xffffffffu, uincl, 31);
    }
    if (lane == 0) {
      ucnt[E] = run;
      misc[0] = urun;
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int o = ucnt[e];
    for (int p = 0; p < T * k; ++p)
      if (sel_e[(p / k) * kFzMaxK + p % k] == e) upairs[o++] = p;
  }
  __syncthreads();
  const int U = misc[0];

  // ---------------- phase G: gate/up items
  const int NT = I / 16;
  const int RB = H / 2, sbg = 16 * G * 2;
  const int nitems = U * NT;
  uint8_t* wg = wsm;
  uint8_t* wu = wsm + 16 * L.RSg;
  const bf16* graw = reinterpret_cast<const bf16*>(wsm + 2 * 16 * L.RSg);  // gs, gb, us, ub
  float* bdot = reinterpret_cast<float*>(wsm + 2 * 16 * L.RSg + 4 * sbg);  // [2][16][kFzMaxT]
  const int gbeg = G * warp / kFzWarps, gend = G * (warp + 1) / kFzWarps;
  for (int it = blockIdx.x; it < nitems && ok; it += gridDim.x) {
    const int u = it / NT, row0 = (it % NT) * 16;
    const int e = uexp[u];
    const int pbeg = ucnt[e], nv = ucnt[e + 1] - pbeg;  // <= T <= 8
    const uint8_t* eb = ex.base + (int64_t)e * ex.stride;
    if (warp == 0) {
      if (lane == 0) mbar_arrive_expect_tx(&bar[0], 32u * RB + 4u * sbg);
      __syncwarp();
      bulk_g2s(wsm + lane * L.RSg, eb + ((lane >> 4) ? ex.off[3] : ex.off[0]) + (int64_t)(row0 + (lane & 15)) * RB, RB,
               &bar[0]);
      if (lane < 4) {
        const int64_t off = lane == 0 ? ex.off[1] : lane == 1 ? ex.off[2] : lane == 2 ? ex.off[4] : ex.off[5];
        bulk_g2s(wsm + 2 * 16 * L.RSg + lane * sbg, eb + off + (int64_t)row0 * G * 2, sbg, &bar[0]);
      }
    }
    ok = mbar_wait(&bar[0], ph0, status, 33);
    ph0 ^= 1;
    if (!ok) break;
    // bias dots: bdot[mat][r][n] = sum_g (bias - 128*scale)[r][g] * xsum[tok(n)][g]
    for (int i = threadIdx.x; i < 2 * 16 * nv * 4; i += blockDim.x) {
      const int q = i & 3, n = (i >> 2) % nv, r = (i >> 2) / nv % 16, mat = (i >> 2) / nv / 16;
      const bf16* sc = graw + (2 * mat) * 16 * G + r * G;
      const bf16* bi = graw + (2 * mat + 1) * 16 * G + r * G;
      const float* xs = xsum + (upairs[pbeg + n] / k) * G;
      float s = 0.f;
      for (int gi = q; gi < G; gi += 4) s = fmaf(fmaf(-128.0f, bf2f(sc[gi]), bf2f(bi[gi])), xs[gi], s);
      s += __shfl_xor_sync(0xffffffffu, s, 1);
      s += __shfl_xor_sync(0xffffffffu, s, 2);
      if (q == 0) bdot[(mat * 16 + r) * kFzMaxT + n] = s;
    }
    // token row of B column g (lanes with g >= nv read zeros)
    const int xrow = g < nv ? upairs[pbeg + g] / k : 0;
    float yg[4] = {0.f, 0.f, 0.f, 0.f}, yu[4] = {0.f, 0.f, 0.f, 0.f};
    for (int gi = gbeg; gi < gend; ++gi) {
      uint4 xl = make_uint4(0, 0, 0, 0), xh = xl;
      if (g < nv) {
        const uint8_t* p = xsm + xrow * L.XS + gi * 128 + 32 * t;
        xl = lds_u4(p);
        xh = lds_u4(p + 16);
      }
      const BFrag4 b = make_bfrag4(xl, xh);
      const uint2 gl = lds_u2(wg + g * L.RSg + gi * 32 + 8 * t);
      const uint2 gh = lds_u2(wg + (g + 8) * L.RSg + gi * 32 + 8 * t);
      const uint2 ul = lds_u2(wu + g * L.RSg + gi * 32 + 8 * t);
      const uint2 uh = lds_u2(wu + (g + 8) * L.RSg + gi * 32 + 8 * t);
      float cg[4] = {0.f, 0.f, 0.f, 0.f}, cu[4] = {0.f, 0.f, 0.f, 0.f};
      mma_group_q4(cg, gl, gh, b);
      mma_group_q4(cu, ul, uh, b);
      const float gs0 = bf2f(graw[g * G + gi]), gs1 = bf2f(graw[(g + 8) * G + gi]);
      const float us0 = bf2f(graw[32 * G + g * G + gi]), us1 = bf2f(graw[32 * G + (g + 8) * G + gi]);
      yg[0] = fmaf(gs0, cg[0], yg[0]);
      yg[1] = fmaf(gs0, cg[1], yg[1]);
      yg[2] = fmaf(gs1, cg[2], yg[2]);
      yg[3] = fmaf(gs1, cg[3], yg[3]);
      yu[0] = fmaf(us0, cu[0], yu[0]);
      yu[1] = fmaf(us0, cu[1], yu[1]);
      yu[2] = fmaf(us1, cu[2], yu[2]);
      yu[3] = fmaf(us1, cu[3], yu[3]);
    }
    float* rw = red + warp * 256;
    rw[g * 8 + 2 * t] = yg[0];
    rw[g * 8 + 2 * t + 1] = yg[1];
    rw[(g + 8) * 8 + 2 * t] = yg[2];
    rw[(g + 8) * 8 + 2 * t + 1] = yg[3];
    rw[128 + g * 8 + 2 * t] = yu[0];
    rw[128 + g * 8 + 2 * t + 1] = yu[1];
    rw[128 + (g + 8) * 8 + 2 * t] = yu[2];
    rw[128 + (g + 8) * 8 + 2 * t + 1] = yu[3];
    __syncthreads();
    if (threadIdx.x < 128) {
      const int c = threadIdx.x >> 4, r = threadIdx.x & 15;
      if (c < nv) {
        float sg = bdot[r * kFzMaxT + c], su = bdot[(16 + r) * kFzMaxT + c];
#pragma unroll
        for (int w = 0; w < kFzWarps; ++w) {
          sg += red[w * 256 + r * 8 + c];
          su += red[w * 256 + 128 + r * 8 + c];
        }
        const float gv = round_bf(sg), uv = round_bf(su);
        a.act[(int64_t)(pbeg + c) * I + row0 + r] = __float2bfloat16_rn(gelu_tanh(gv) * uv);
      }
    }
    __syncthreads();  // region W and the overlay are reused by the next item
  }

  // ---------------- prefetch this CTA's first down item (before barrier 2)
  const int ND_t = H / 16, ngroups = (U + 7) / 8, nd = ND_t * ngroups;
  const int RBd = I / 2, sbd = 16 * Gi * 2, slot_bytes = 16 * L.RSd + 2 * sbd;
  const int my_slot = warp;
  auto issue_down = [&](int item) {
    const int tile = item % ND_t, grp = item / ND_t;
    if (warp == 0) {
      uint32_t bytes = 0;
      for (int s = 0; s < 8; ++s)
        if (grp * 8 + s < U) bytes += slot_bytes;
      if (lane == 0) mbar_arrive_expect_tx(&bar[1], bytes);
      __syncwarp();
      if (lane < 8 && grp * 8 + lane < U) {
        const uint8_t* eb = ex.base + (int64_t)uexp[grp * 8 + lane] * ex.stride;
        uint8_t* ss = wsm + lane * slot_bytes;
        bulk_g2s(ss, eb + ex.off[6] + (int64_t)tile * 16 * RBd, 16 * RBd, &bar[1]);
        bulk_g2s(ss + 16 * L.RSd, eb + ex.off[7] + (int64_t)tile * sbd, sbd, &bar[1]);
        bulk_g2s(ss + 16 * L.RSd + sbd, eb + ex.off[8] + (int64_t)tile * sbd, sbd, &bar[1]);
      }
    }
  };
  if (ok && blockIdx.x < nd) issue_down(blockIdx.x);
  ok = fz_grid_barrier(&a.gbar[1], status, 34) && ok;

  // ---------------- phase D: down items
  uint32_t ph1 = 0, ph2 = 0;
  float* ysm = reinterpret_cast<float*>(xsm);  // [kFzWarps][T][16] over the consumed x rows
  for (int item = blockIdx.x; item < nd && ok; item += gridDim.x) {
    if (item != blockIdx.x) {
      __syncthreads();
      issue_down(item);
    }
    const int tile = item % ND_t, grp = item / ND_t, row0 = tile * 16;
    const int u = grp * 8 + my_slot;
    const bool live = u < U;
    const int e = live ? uexp[u] : 0;
    const int pbeg = live ? ucnt[e] : 0, np = live ? ucnt[e + 1] - pbeg : 0;
    for (int i = threadIdx.x; i < kFzWarps * T * 16; i += blockDim.x) ysm[i] = 0.f;
    ok = mbar_wait(&bar[1], ph1, status, 35);
    ph1 ^= 1;
    __syncthreads();
    if (!ok) break;
    const uint8_t* ss = wsm + my_slot * slot_bytes;
    const bf16* dsc = reinterpret_cast<const bf16*>(ss + 16 * L.RSd);
    const bf16* dbi = dsc + 16 * Gi;
    float* my = ysm + my_slot * T * 16;
    uint8_t* arow = asm_ + my_slot * L.AS;
    // One act row per expert slot per round; every warp runs the same rounds
    // (the mbarrier and __syncthreads are shared), idle slots skip the math.
    const int maxnp = T;  // upper bound on the pairs of one expert
    for (int c0 = 0; c0 < maxnp; ++c0) {
      if (c0 > 0) __syncthreads();  // previous act rows consumed
      if (warp == 0) {
        uint32_t bytes = 0;
        for (int s = 0; s < 8; ++s) {
          const int us = grp * 8 + s;
          if (us < U) {
            const int es = uexp[us];
            if (c0 < ucnt[es + 1] - ucnt[es]) bytes += I * 2;
          }
        }
        if (lane == 0) mbar_arrive_expect_tx(&bar[2], bytes);
        __syncwarp();
        if (lane < 8 && grp * 8 + lane < U) {
          const int es = uexp[grp * 8 + lane];
          if (c0 < ucnt[es + 1] - ucnt[es])
            bulk_g2s(asm_ + lane * L.AS, a.act + (int64_t)(ucnt[es] + c0) * I, I * 2, &bar[2]);
        }
      }
      const bool w_ok = mbar_wait(&bar[2], ph2, status, 36);
      ph2 ^= 1;
      ok = ok && w_ok;
      if (ok && c0 < np) {
        float d[4] = {0.f, 0.f, 0.f, 0.f};
        for (int gi = 0; gi < Gi; ++gi) {
          const BFrag4 b = stage_bfrag4(arow, L.AS, 1, gi, g, t);
          const uint2 wl = lds_u2(ss + g * L.RSd + gi * 32 + 8 * t);
          const uint2 wh = lds_u2(ss + (g + 8) * L.RSd + gi * 32 + 8 * t);
          float c[4] = {0.f, 0.f, 0.f, 0.f}, xs[4] = {0.f, 0.f, 0.f, 0.f};
          mma_group_q4(c, wl, wh, b);
          mma_group_ones(xs, b);
          affine_fixup(d, c, xs, bf2f(dsc[g * Gi + gi]), bf2f(dbi[g * Gi + gi]), bf2f(dsc[(g + 8) * Gi + gi]),
                       bf2f(dbi[(g + 8) * Gi + gi]), 128.0f);
        }
        if (t == 0) {  // column 0 holds the pair
          const int p = upairs[pbeg + c0];
          const float wv = sel_w[(p / k) * kFzMaxK + p % k];
          my[(p / k) * 16 + g] += wv * d[0];
          my[(p / k) * 16 + g + 8] += wv * d[2];
        }
      }
      if (c0 + 1 >= maxnp) break;
      // stop early once no slot has more pairs
      int more = 0;
      for (int s = 0; s < 8; ++s) {
        const int us = grp * 8 + s;
        if (us < U) {
          const int es = uexp[us];
          more |= (c0 + 1 < ucnt[es + 1] - ucnt[es]);
        }
      }
      if (!more) break;
    }
    __syncthreads();
    if (!ok) break;
    if (ngroups == 1) {
      for (int i = threadIdx.x; i < T * 16; i += blockDim.x) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kFzWarps; ++w) s += ysm[w * T * 16 + i];
        a.y[(int64_t)(i >> 4) * H + row0 + (i & 15)] = __float2bfloat16_rn(s);
      }
    } else {
      for (int i = threadIdx.x; i < T * 16; i += blockDim.x) {
        float s = 0.f;
#pragma unroll
        for (int w = 0; w < kFzWarps; ++w) s += ysm[w * T * 16 + i];
        a.dpart[((int64_t)grp * T + (i >> 4)) * H + row0 + (i & 15)] = s;
      }
      __threadfence();
      __syncthreads();
      __shared__ int s_last;
      if (threadIdx.x == 0) s_last = atomicAdd(&a.tile_ctr[tile], 1u) == (unsigned)ngroups - 1;
      __syncthreads();
      if (s_last) {
        __threadfence();
        for (int i = threadIdx.x; i < T * 16; i += blockDim.x) {
          float s = 0.f;
          for (int q = 0; q < ngroups; ++q) s += __ldcg(a.dpart + ((int64_t)q * T + (i >> 4)) * H + row0 + (i & 15));
          a.y[(int64_t)(i >> 4) * H + row0 + (i & 15)] = __float2bfloat16_rn(s);
        }
        if (threadIdx.x == 0) a.tile_ctr[tile] = 0;
      }
    }
  }

  // ---------------- barrier counters back to zero for the next call
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(&a.gbar[2], 1u) == gridDim.x - 1) {
      a.gbar[0] = 0;
      a.gbar[1] = 0;
      a.gbar[2] = 0;
      __threadfence();
    }
  }
}

// ---------------------------------------------------------------------------
// host side

size_t fused_smem_bytes(int H, int I, int E, int T, int rbits) { return fz_layout(H, I, E, T, rbits).bytes; }

int fused_supported(int64_t T, int E, int k, int H, int rbits) {
  return T >= 1 && T <= kFzMaxT && E <= kFzMaxE && k <= kFzMaxK && (rbits == 16 || rbits == 4) && H % 64 == 0;
}

int launch_moe_fused(const bf16* x, int64_t T, const QW& wr, const float* bias, const bf16* pes, int k,
                     const ExpertsDev& ex, int32_t* ids, float* wts, bf16* y, float* rpart, bf16* act, float* dpart,
                     unsigned* tile_ctr, unsigned* gbar, int* status, cudaStream_t st) {
  const FzLayout L = fz_layout(ex.H, ex.I, wr.out, (int)T, wr.bits);
  if (L.bytes > 227 * 1024) return set_error(FMOE_ERR_UNSUPPORTED, "fused: shared memory %zu too large", L.bytes);
  static thread_local int cached_dev = -1, cached_blocks = 0;
  static thread_local size_t cached_bytes = 0;
  int dev = 0;
  cudaGetDevice(&dev);
  cudaFuncSetAttribute(moe_decode_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.bytes);
  if (dev != cached_dev || cached_bytes != L.bytes) {
    int per_sm = 0, sms = 0;
    cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, moe_decode_fused_kernel, kFzThreads, L.bytes);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cached_blocks = per_sm * sms;
    cached_dev = dev;
    cached_bytes = L.bytes;
  }
  const int nR = ((wr.out + 15) / 16) * kFzSlices;
  if (cached_blocks < nR) return set_error(FMOE_ERR_UNSUPPORTED, "fused: %d co-resident CTAs < %d", cached_blocks, nR);
  FzArgs a;
  a.x = x;
  a.T = (int)T;
  a.E = wr.out;
  a.k = k;
  a.wr = wr.w;
  a.rbits = wr.bits;
  a.rsc = wr.s;
  a.rbi = wr.b;
  a.bias = bias;
  a.pes = pes;
  a.ex = ex;
  a.ids = ids;
  a.wts = wts;
  a.y = y;
  a.rpart = rpart;
  a.act = act;
  a.dpart = dpart;
  a.tile_ctr = tile_ctr;
  a.gbar = gbar;
  a.status = status;
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(cached_blocks);
  cfg.blockDim = dim3(kFzThreads);
  cfg.dynamicSmemBytes = L.bytes;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  {
    ProfScope prof_("moe_decode_fused_kernel", st);
    cudaLaunchKernelEx(&cfg, moe_decode_fused_kernel, a);
  }
  return check_launch("moe_decode_fused_kernel");
}

}  // namespace fmoe
