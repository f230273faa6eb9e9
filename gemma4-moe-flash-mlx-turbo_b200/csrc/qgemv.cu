// Streaming quantised GEMV for decode (T <= 8 tokens): y[t, r] = x[t] . W[r]^T
// over up to four weight matrices ("segments") that share one input, e.g. the
// q / k / v projections of an attention layer.
//
// Work unit = 16 weight rows x one chunk of kc input columns.  Each CTA owns a
// contiguous range of units and streams them through an NST-stage ring of TMA
// bulk copies (one copy per weight row into a bank-conflict-free padded row,
// plus the rows' scale and bias blocks).  The first stages are issued before
// griddepcontrol.wait: weights never depend on the preceding kernel, so under
// programmatic dependent launch they stream in while that kernel finishes.
//
// Tensor-core math (mma.sync m16n8k16, f16 in, fp32 accumulate), one recipe
// for every width: the A operand is (1024 + code) in f16 — exact for codes
// < 1024 — built in registers from the packed codes (PRMT for 8-bit, LOP3 for
// 4-bit, shifts + LOP3 for the 6-bit bit stream); the B operand is the input
// row in f16, prepared once per CTA in fragment order.  Per 64-column group:
//   y += s * C + (b - 1024 s) * sum(x),   C = sum (1024 + q) x.
// The input prologue applies the producer-side elementwise op while it builds
// the fragments: none (bf16 input), RMSNorm with a weight, or GELU-tanh gating
// of two fp32 projections (the dense MLP's act = gelu(g) * u, rounded like
// the reference's bf16 tensors).
#include "internal.h"
#include "common.cuh"
#include "stage.cuh"
#include "qfrag.cuh"

namespace fmoe {

constexpr int kQgMaxWarps = 16;  // consumer warps per CTA (the count is chosen per launch)

// Unit u -> (segment, block of RT 16-row tiles, column chunk).
struct QgUnit {
  int sg, blk, kci;
};
__device__ __forceinline__ QgUnit qg_unit(const QgArgs& a, int u) {
  int sg = 0;
#pragma unroll
  for (int i = 1; i < kQgMaxSeg; ++i)
    if (i < a.nseg && u >= a.seg[i].unit0) sg = i;
  const int v = u - a.seg[sg].unit0;
  return QgUnit{sg, v / a.nkc, v % a.nkc};
}

// Called by the whole producer warp: lane 0 arms the stage's barrier, then
// the lanes issue the row copies in parallel (one copy per row; issuing them
// from one thread costs a few hundred cycles each).
template <int BITS, int RT>
__device__ __forceinline__ void qg_issue(const QgArgs& a, const QgLayout& L, uint8_t* smem, uint64_t* bar, int u,
                                         int st, int lane) {
  constexpr int R = 16 * RT;
  const QgUnit q = qg_unit(a, u);
  const QgSeg& s = a.seg[q.sg];
  const int64_t rowbytes = (int64_t)a.K * BITS / 8;
  const int kcbytes = a.kc * BITS / 8, G = a.K / 64, gc = a.kc / 64;
  uint8_t* sb = smem + (size_t)st * L.stage;
  const uint8_t* w = s.w + (int64_t)q.blk * R * rowbytes + (int64_t)q.kci * kcbytes;
  const int wbytes = s.tiled ? R * L.rs : R * kcbytes;
  if (lane == 0) mbar_arrive_expect_tx(&bar[st], (uint32_t)(wbytes + 2 * R * (L.sfull ? G : gc) * 2));
  __syncwarp();
  if (s.tiled) {  // the unit's RT tiles are one contiguous run of the tile layout
    if (lane == 0)
      bulk_g2s(sb, s.tiled + (((int64_t)q.blk * RT) * a.nkc + q.kci) * 16 * L.rs, (uint32_t)wbytes, &bar[st]);
  } else {
    for (int r = lane; r < R; r += 32) bulk_g2s(sb + r * L.rs, w + r * rowbytes, kcbytes, &bar[st]);
  }
  const bf16* sc = s.s + (int64_t)q.blk * R * G;
  const bf16* bi = s.b + (int64_t)q.blk * R * G;
  if (L.sfull) {  // the block's whole [R][G] scale / bias arrays (contiguous)
    if (lane == 0) bulk_g2s(sb + L.soff, sc, R * G * 2, &bar[st]);
    if (lane == 1) bulk_g2s(sb + L.soff + R * G * 2, bi, R * G * 2, &bar[st]);
  } else {  // the chunk's [R][gc] columns, one 16-byte-multiple copy per row
    for (int r = lane; r < R; r += 32) {
      bulk_g2s(sb + L.soff + r * gc * 2, sc + (int64_t)r * G + q.kci * gc, gc * 2, &bar[st]);
      bulk_g2s(sb + L.soff + R * gc * 2 + r * gc * 2, bi + (int64_t)r * G + q.kci * gc, gc * 2, &bar[st]);
    }
  }
}

// Warp roles: L.nw consumer warps share every unit (64-column groups dealt
// round robin, any leftover groups rotating from unit to unit) and one
// producer warp issues the copies.  A stage is refilled once all consumers
// have released it (per-stage "empty" mbarrier), so consumers never wait on
// each other.  A consumer loads a group's input fragments once and applies
// them to the unit's RT row tiles.  A block's per-warp partial sums meet in
// shared memory and the last warp to arrive (a shared counter) writes them.
template <int BITS, int RT>
__global__ void __launch_bounds__((kQgMaxWarps + 1) * 32, 1) qgemv_kernel(const QgArgs a, const QgLayout L) {
  constexpr int R = 16 * RT;
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);  // [nst] full, then [nst] empty
  uint64_t* empty = bar + L.nst;
  int* cnt = reinterpret_cast<int*>(smem + L.cnt);
  uint4* frag = reinterpret_cast<uint4*>(smem + L.frag);
  float* xsum = reinterpret_cast<float*>(smem + L.xsum);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* rms = reinterpret_cast<float*>(smem + L.misc);
  int* flag = reinterpret_cast<int*>(smem + L.misc + 8 * 4);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int T = a.T, K = a.K, G = K / 64, gc = a.kc / 64;
  // unit range; outputs that are stored (not accumulated) keep a block's chunks in one CTA
  const bool split_ok = a.out_kind == QG_OUT_F32_ADD || a.out_kind == QG_OUT_F32_PART;
  const int ub = split_ok ? 1 : a.nkc;
  const int nb = a.units / ub;
  const int u0 = (int)((int64_t)nb * blockIdx.x / gridDim.x) * ub;
  const int u1 = (int)((int64_t)nb * (blockIdx.x + 1) / gridDim.x) * ub;
  const int n = u1 - u0;
  const int NW = L.nw;

  if (tid == 0) {
    for (int s = 0; s < L.nst; ++s) {
      mbar_init(&bar[s], 1);
      mbar_init(&empty[s], NW);
    }
    mbar_fence_init();
    flag[0] = 0;
  }
  if (tid < L.nst + 1) cnt[tid] = 0;
  __syncthreads();
  if (warp == NW)
    for (int i = 0; i < n && i < L.nst; ++i) qg_issue<BITS, RT>(a, L, smem, bar, u0 + i, i, lane);

  griddep_wait();  // the input (and the buffers cleared below) belong to earlier kernels
  griddep_launch_dependents();

  // buffers that later kernels accumulate into
  for (int z = 0; z < 4; ++z) {
    float* zp = a.zero_ptr[z];
    if (!zp) continue;
    const int64_t nz = a.zero_n[z];
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + tid; i < nz; i += (int64_t)gridDim.x * blockDim.x) zp[i] = 0.f;
  }

  // ---- input prologue: f16 B fragments + per-group sums
  if (a.in_kind == QG_IN_RMSNORM) {
    for (int tk = warp; tk < T; tk += NW + 1) {
      const bf16* xr = a.x + (int64_t)tk * a.ldx;
      float ss = 0.f;
      // K <= 8192: up to 32 16-byte loads per lane, all issued before use
      uint4 wv[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int i = lane * 8 + j * 256;
        wv[j] = i < K ? ld_u4(xr + i) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const uint32_t ww[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float lo = bf16lo(ww[e]), hi = bf16hi(ww[e]);
          ss = fmaf(lo, lo, fmaf(hi, hi, ss));
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (lane == 0) rms[tk] = rsqrtf(ss / (float)K + a.eps);
    }
    __syncthreads();
  }
  const int nitems = G * T * 4;
  for (int item0 = 0; item0 < nitems; item0 += blockDim.x) {
    // every lane runs the shuffles below; items come in aligned groups of 4
    const int item = item0 + tid;
    const bool live = item < nitems;
    const int tq = item & 3, tk = live ? (item >> 2) % T : 0, gi = live ? (item >> 2) / T : 0;
    const int c0 = gi * 64 + 16 * tq;
    float v[16];
    if (!live) {
#pragma unroll
      for (int e = 0; e < 16; ++e) v[e] = 0.f;
    } else if (a.in_kind == QG_IN_GELU) {
      const float* gp = a.g + (int64_t)tk * a.ldgu + c0;
      const float* up = a.u + (int64_t)tk * a.ldgu + c0;
      float gs[16], us[16];
#pragma unroll
      for (int e = 0; e < 16; ++e) gs[e] = us[e] = 0.f;
      for (int pp = 0; pp < a.gu_parts; ++pp) {  // partial slices in order; a slice's 8 loads in flight together
        float4 gg[4], uu[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          gg[e] = __ldcg(reinterpret_cast<const float4*>(gp + pp * a.gu_part_stride + 4 * e));
          uu[e] = __ldcg(reinterpret_cast<const float4*>(up + pp * a.gu_part_stride + 4 * e));
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          gs[4 * e] += gg[e].x, gs[4 * e + 1] += gg[e].y, gs[4 * e + 2] += gg[e].z, gs[4 * e + 3] += gg[e].w;
          us[4 * e] += uu[e].x, us[4 * e + 1] += uu[e].y, us[4 * e + 2] += uu[e].z, us[4 * e + 3] += uu[e].w;
        }
      }
#pragma unroll
      for (int e = 0; e < 16; e += 4) {
        const float ga[4] = {gs[e], gs[e + 1], gs[e + 2], gs[e + 3]}, ua[4] = {us[e], us[e + 1], us[e + 2], us[e + 3]};
#pragma unroll
        for (int q = 0; q < 4; ++q) v[e + q] = round_bf(gelu_tanh(round_bf(ga[q])) * round_bf(ua[q]));
      }
    } else {
      const bf16* xr = a.x + (int64_t)tk * a.ldx + c0;
      const uint4 w0 = ld_u4(xr), w1 = ld_u4(xr + 8);
      const uint32_t ww[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[2 * e] = bf16lo(ww[e]);
        v[2 * e + 1] = bf16hi(ww[e]);
      }
      if (a.in_kind == QG_IN_RMSNORM) {
        const float r = rms[tk];
        const bf16* nw = a.norm_w + c0;
#pragma unroll
        for (int e = 0; e < 16; ++e) v[e] = round_bf(v[e] * r * bf2f(nw[e]));
      }
    }
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      v[e] = f16r(v[e]);
      s += v[e];
    }
    uint32_t b[8];
    make_b_frags<BITS>(v, b);
    if (live) {
      uint4* dst = frag + ((int64_t)gi * 4 * T + 4 * tk + tq) * 2;
      dst[0] = make_uint4(b[0], b[1], b[2], b[3]);
      dst[1] = make_uint4(b[4], b[5], b[6], b[7]);
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (live && tq == 0) xsum[gi * 8 + tk] = s;
  }
  for (int i = tid; i < G * 8; i += blockDim.x)
    if ((i & 7) >= T) xsum[i] = 0.f;
  __syncthreads();

  // ---- producer: refill each stage once every consumer has released it,
  // then let the last copies land before the warp (and smem) goes away
  if (warp == NW) {
    int i = L.nst;
    for (; i < n; ++i) {
      const int st = i % L.nst;
      int stop = 0;
      if (lane == 0) {
        if (*(volatile int*)flag) {
          stop = 1;
        } else if (!mbar_wait(&empty[st], (uint32_t)((i / L.nst - 1) & 1), a.status, 63)) {
          *(volatile int*)flag = 1;
          stop = 1;
        }
      }
      if (__shfl_sync(0xffffffffu, stop, 0)) break;
      qg_issue<BITS, RT>(a, L, smem, bar, u0 + i, st, lane);
    }
    if (lane == 0)
      for (int k = (i > L.nst ? i - L.nst : 0); k < i && k < n; ++k)
        mbar_wait(&bar[k % L.nst], (uint32_t)(k / L.nst) & 1u, a.status, 64);
    return;
  }

  // ---- consumers
  const int nred = L.nst + 1;
  float y[RT][4];
#pragma unroll
  for (int tt = 0; tt < RT; ++tt) y[tt][0] = y[tt][1] = y[tt][2] = y[tt][3] = 0.f;
  int flushes = 0, run_kc0 = -1;
  const int sst = L.sfull ? G : gc;  // scale row stride in a stage
  for (int i = 0; i < n; ++i) {
    const int st = i % L.nst, u = u0 + i;
    const QgUnit q = qg_unit(a, u);
    if (run_kc0 < 0) run_kc0 = q.kci;
    const uint8_t* sb = smem + (size_t)st * L.stage;
    if (!mbar_wait(&bar[st], (uint32_t)(i / L.nst) & 1u, a.status, 61)) *(volatile int*)flag = 1;
    if (*(volatile int*)flag) break;  // a copy never landed (the status word says so)
    const bf16* scl = reinterpret_cast<const bf16*>(sb + L.soff);
    const bf16* bil = reinterpret_cast<const bf16*>(sb + L.soff + R * sst * 2);
    const int rot = (int)(((int64_t)i * (gc % NW)) % NW);
    const int vw = warp + rot < NW ? warp + rot : warp + rot - NW;
    const uint8_t* rbase = sb + g * L.rs + t * (2 * BITS);
    for (int gl = vw; gl < gc; gl += NW) {
      const int gi = q.kci * gc + gl;
      uint4 b0 = make_uint4(0, 0, 0, 0), b1 = b0;
      if (g < T) {
        const uint4* fp = frag + ((int64_t)gi * 4 * T + lane) * 2;
        b0 = fp[0];
        b1 = fp[1];
      }
      const uint32_t bb0[4] = {b0.x, b0.y, b0.z, b0.w}, bb1[4] = {b1.x, b1.y, b1.z, b1.w};
      const float q0 = xsum[gi * 8 + 2 * t], q1 = xsum[gi * 8 + 2 * t + 1];
      const int sc_ = L.sfull ? gi : gl;
#pragma unroll
      for (int tt = 0; tt < RT; ++tt) {
        const uint8_t* rl = rbase + (tt * 16) * L.rs + gl * (8 * BITS);
        uint32_t af[4][4];
        load_a_frags<BITS>(rl, rl + 8 * L.rs, af);
        float cc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
        for (int j = 0; j < 4; ++j) mma16816_f16(cc, af[j][0], af[j][1], af[j][2], af[j][3], bb0[j], bb1[j]);
        const int r0 = tt * 16 + g;
        const float sl = bf2f(scl[r0 * sst + sc_]), blo = bf2f(bil[r0 * sst + sc_]);
        const float sh = bf2f(scl[(r0 + 8) * sst + sc_]), bhi = bf2f(bil[(r0 + 8) * sst + sc_]);
        const float ol = fmaf(-1024.f, sl, blo), oh = fmaf(-1024.f, sh, bhi);
        y[tt][0] += fmaf(sl, cc[0], ol * q0);
        y[tt][1] += fmaf(sl, cc[1], ol * q1);
        y[tt][2] += fmaf(sh, cc[2], oh * q0);
        y[tt][3] += fmaf(sh, cc[3], oh * q1);
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[st]);  // this warp is done with the stage
    // a run of this block's column chunks ends here?  (F32_PART: the run's sum
    // goes to the slice of its first chunk, the run's other slices get zeros)
    bool flush = i + 1 == n;
    if (!flush) {
      const QgUnit nq = qg_unit(a, u + 1);
      flush = nq.sg != q.sg || nq.blk != q.blk;
    }
    if (flush) {
      const int slot = flushes % nred;
      float* rs = red + (size_t)slot * NW * R * T;  // [NW warps][R rows][T tokens]
      float* rw = rs + warp * R * T;
#pragma unroll
      for (int tt = 0; tt < RT; ++tt) {
        const int r0 = tt * 16 + g;
        if (2 * t < T) {
          rw[r0 * T + 2 * t] = y[tt][0];
          rw[(r0 + 8) * T + 2 * t] = y[tt][2];
        }
        if (2 * t + 1 < T) {
          rw[r0 * T + 2 * t + 1] = y[tt][1];
          rw[(r0 + 8) * T + 2 * t + 1] = y[tt][3];
        }
        y[tt][0] = y[tt][1] = y[tt][2] = y[tt][3] = 0.f;
      }
      __threadfence_block();
      __syncwarp();
      int last = 0;
      if (lane == 0) last = (atomicAdd(&cnt[slot], 1) + 1) % NW == 0;  // counters only grow
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last) {
        __threadfence_block();
        const QgSeg& sg = a.seg[q.sg];
        for (int o = lane; o < R * T; o += 32) {
          const int r = o % R, tk = o / R;
          float sum = 0.f;
          for (int w = 0; w < NW; ++w) sum += rs[(w * R + r) * T + tk];
          int64_t oi = (int64_t)tk * sg.ld + sg.col0 + q.blk * R + r;
          if (a.out_kind == QG_OUT_F32_PART) {
            for (int kz = run_kc0 + 1; kz <= q.kci; ++kz)
              static_cast<float*>(sg.out)[oi + (int64_t)kz * T * sg.ld] = 0.f;
            oi += (int64_t)run_kc0 * T * sg.ld;
          }
          if (a.out_kind == QG_OUT_F32_ADD)
            atomicAdd(static_cast<float*>(sg.out) + oi, sum);
          else if (a.out_kind == QG_OUT_F32 || a.out_kind == QG_OUT_F32_PART)
            static_cast<float*>(sg.out)[oi] = sum;
          else
            static_cast<bf16*>(sg.out)[oi] = __float2bfloat16_rn(sum);
        }
      }
      ++flushes;
      run_kc0 = -1;
    }
  }
}

// ---------------------------------------------------------------------------

// Padded smem row stride: residues (mod 128 B) measured conflict-free for the
// lane access patterns of load_a_frags.
int qgemv_row_stride(int bytes, int bits) {
  const int want = bits == 4 ? 32 : bits == 6 ? 16 : 64;
  int s = (bytes + 15) & ~15;
  while (s % 128 != want) s += 16;
  return s;
}

static int qgemv_plan_rt(QgArgs& a, int bits, bool allow_split, bool try_rt2, bool half_sm, QgLayout* L);

int qgemv_plan(QgArgs& a, int bits, bool allow_split, QgLayout* L, bool half_sm) {
  // 32-row units when they fit, else 16-row units; the whole SM when half of it is too small
  const bool budgets[2] = {half_sm, false};
  for (int b = 0; b < (half_sm ? 2 : 1); ++b) {
    if (qgemv_plan_rt(a, bits, allow_split, true, budgets[b], L) == FMOE_OK) return FMOE_OK;
    if (qgemv_plan_rt(a, bits, allow_split, false, budgets[b], L) == FMOE_OK) return FMOE_OK;
  }
  return set_error(FMOE_ERR_UNSUPPORTED, "qgemv: K %d, T %d exceed shared memory", a.K, a.T);
}

// half_sm: at most ~110 KB of shared memory and 8 + 1 warps, so the next
// kernel of a programmatic-dependent chain fits on the SM beside this one and
// streams its weights while this one finishes.
static int qgemv_plan_rt(QgArgs& a, int bits, bool allow_split, bool try_rt2, bool half_sm, QgLayout* L) {
  const int K = a.K, G = K / 64;
  if (bits != 4 && bits != 6 && bits != 8) return set_error(FMOE_ERR_UNSUPPORTED, "qgemv: bits %d", bits);
  if (K % 64 || a.T < 1 || a.T > 8) return set_error(FMOE_ERR_UNSUPPORTED, "qgemv: K %d, T %d", K, a.T);
  int tiles = 0;
  bool even32 = true;
  for (int i = 0; i < a.nseg; ++i) {
    if (a.seg[i].rows % 16) return set_error(FMOE_ERR_UNSUPPORTED, "qgemv: rows %d not a multiple of 16", a.seg[i].rows);
    tiles += a.seg[i].rows / 16;
    even32 = even32 && a.seg[i].rows % 32 == 0;
  }
  // Large matrices: 32-row units over the whole K (input fragments reused by
  // two row tiles, scales copied once).  Otherwise 16-row units with the
  // fewest column chunks that keep a stage's codes <= 48 KB, and (for
  // accumulating outputs) more chunks while the units split unevenly over the SMs.
  int rt = 1, nkc = 0;
  // tiled segments (all or none) fix the column chunk; their layout keeps the
  // two tiles of a 32-row unit adjacent only without column chunks
  int tiled = 0, tkc = 0;
  for (int i = 0; i < a.nseg; ++i)
    if (a.seg[i].tiled) {
      if (tiled && a.seg[i].tiled_kc != tkc) return set_error(FMOE_ERR_INVALID, "qgemv: segments tiled differently");
      tkc = a.seg[i].tiled_kc;
      ++tiled;
    }
  if (tiled && (tiled != a.nseg || tkc < 64 || tkc % 64 || K % tkc || 16 * tkc * bits / 8 > 64 * 1024))
    return set_error(FMOE_ERR_INVALID, "qgemv: tiled chunk %d (K %d)", tkc, K);
  if (tiled) {
    nkc = K / tkc;
    if (nkc > 1 && !allow_split) return set_error(FMOE_ERR_INVALID, "qgemv: tiled chunk needs split output");
    if (try_rt2 && nkc == 1 && even32 && tiles / 2 >= 4 * kNumSMs && 32 * K * bits / 8 <= 96 * 1024) rt = 2;
  } else if (try_rt2 && even32 && tiles / 2 >= 4 * kNumSMs && 32 * K * bits / 8 <= 96 * 1024) {
    rt = 2;
    nkc = 1;
  } else {
    double best_eff = -1.0;
    for (int c = 1; c <= G; ++c) {
      if (G % c || (c > 1 && G / c < 8)) continue;  // >= 8 groups (512 inputs) per chunk
      if (16 * (K / c) * bits / 8 > 48 * 1024) continue;
      if (nkc && !allow_split) break;
      const int64_t u = (int64_t)tiles * c, per = (u + kNumSMs - 1) / kNumSMs;
      const double eff = u < kNumSMs ? 1.0 : (double)u / (double)(per * kNumSMs);
      if (eff > best_eff + 0.02) {
        best_eff = eff;
        nkc = c;
      }
      if (!allow_split || eff >= 0.9 || u >= 6 * kNumSMs) break;
    }
  }
  if (!nkc) return set_error(FMOE_ERR_UNSUPPORTED, "qgemv: no column chunking of K %d at %d bits", K, bits);
  L->rt = rt;
  a.nkc = nkc;
  a.kc = K / nkc;
  if (a.nkc > 1 && a.out_kind != QG_OUT_F32_ADD && a.out_kind != QG_OUT_F32_PART)
    return set_error(FMOE_ERR_UNSUPPORTED, "qgemv: K %d at %d bits needs column chunks (accumulating output)", K, bits);
  const int R = 16 * rt;
  int u = 0;
  for (int i = 0; i < a.nseg; ++i) {
    a.seg[i].unit0 = u;
    u += a.seg[i].rows / R * a.nkc;
  }
  a.units = u;
  const int kcb = a.kc * bits / 8, gc = a.kc / 64;
  // Scales / biases: the row block's whole [R][G] arrays, one contiguous copy
  // each, also for column-chunked units (a chunk's own [R][gc] columns would be
  // 2 R copies of a few dozen bytes, which the copy engine moves far slower).
  L->sfull = 1;
  L->rs = qgemv_row_stride(kcb, bits);
  L->soff = R * L->rs;
  L->stage = (int)align_up(L->soff + 2 * R * (L->sfull ? G : gc) * 2, 128);
  // consumer warps: the count (8..16) that deals a unit's groups most evenly
  const int maxw = half_sm ? 8 : kQgMaxWarps;
  int nw = maxw;
  double nw_eff = 0.0;
  for (int w = maxw; w >= 8; --w) {
    const double e = (double)gc / (double)(w * ((gc + w - 1) / w));
    if (e > nw_eff + 1e-9) {
      nw_eff = e;
      nw = w;
    }
  }
  L->nw = nw;
  const size_t frag = (size_t)G * 4 * a.T * 32, xs = (size_t)G * 8 * 4, red1 = (size_t)nw * R * a.T * 4;
  const size_t fixed = frag + xs + red1 + 8 * 4 + 16 + 16 * 8 + 64 + 512;
  const int budget = half_sm ? 110 * 1024 : 222 * 1024;
  int nst = (int)((budget - fixed) / (L->stage + red1));
  if (nst > 6) nst = 6;
  if (nst < 2) return set_error(FMOE_ERR_UNSUPPORTED, "qgemv: K %d, T %d exceed shared memory", K, a.T);
  const size_t red = (size_t)(nst + 1) * red1;
  L->nst = nst;
  size_t off = (size_t)nst * L->stage;
  L->frag = (int)off;
  off = align_up(off + frag, 16);
  L->xsum = (int)off;
  off = align_up(off + xs, 16);
  L->red = (int)off;
  off = align_up(off + red, 16);
  L->misc = (int)off;
  off = align_up(off + 8 * 4 + 16, 16);
  L->cnt = (int)off;
  off = align_up(off + 4 * (nst + 1), 16);
  L->bar = (int)off;
  off += 2 * 8 * L->nst;
  L->bytes = (int)align_up(off, 128);
  const int ub = (a.out_kind == QG_OUT_F32_ADD || a.out_kind == QG_OUT_F32_PART) ? 1 : a.nkc;
  const int nb = a.units / ub;
  L->grid = nb < kNumSMs ? nb : kNumSMs;
  return FMOE_OK;
}

template <int BITS, int RT>
static int launch_qgemv_t(const QgArgs& a, const QgLayout& L, bool pdl, cudaStream_t st) {
  static bool attr_done = false;
  if (!attr_done) {
    cudaFuncSetAttribute(qgemv_kernel<BITS, RT>, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
    attr_done = true;
  }
  cudaLaunchConfig_t cfg = {};
  cudaLaunchAttribute attr[1];
  cfg.gridDim = dim3(L.grid);
  cfg.blockDim = dim3((L.nw + 1) * 32);
  cfg.dynamicSmemBytes = L.bytes;
  cfg.stream = st;
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  ProfScope prof_(BITS == 4 ? "qgemv_kernel<4>" : BITS == 6 ? "qgemv_kernel<6>" : "qgemv_kernel<8>", st);
  cudaLaunchKernelEx(&cfg, qgemv_kernel<BITS, RT>, a, L);
  return check_launch("qgemv_kernel");
}

int launch_qgemv(const QgArgs& a, const QgLayout& L, int bits, bool pdl, cudaStream_t st) {
  if (bits == 4) return L.rt == 2 ? launch_qgemv_t<4, 2>(a, L, pdl, st) : launch_qgemv_t<4, 1>(a, L, pdl, st);
  if (bits == 6) return L.rt == 2 ? launch_qgemv_t<6, 2>(a, L, pdl, st) : launch_qgemv_t<6, 1>(a, L, pdl, st);
  return L.rt == 2 ? launch_qgemv_t<8, 2>(a, L, pdl, st) : launch_qgemv_t<8, 1>(a, L, pdl, st);
}

}  // namespace fmoe

// ---------------------------------------------------------------------------
// Tile layout (fmoe_qweight_tile): [16-row tile][column chunk][16 rows][rs]
// bytes, rs = the GEMV's padded row stride for a chunk, padding zero.

namespace fmoe {

int qgemv_chunk(int K, int bits, int64_t rows_total, bool allow_split) {
  if ((bits != 4 && bits != 6 && bits != 8) || K % 64 || rows_total < 16 || rows_total % 16) return 0;
  const int G = K / 64;
  const int64_t tiles = rows_total / 16;
  if (rows_total % 32 == 0 && tiles / 2 >= 4 * kNumSMs && 32 * K * bits / 8 <= 96 * 1024) return K;
  int nkc = 0;
  double best_eff = -1.0;
  for (int c = 1; c <= G; ++c) {
    if (G % c || (c > 1 && G / c < 8)) continue;
    if (16 * (K / c) * bits / 8 > 48 * 1024) continue;
    if (nkc && !allow_split) break;
    const int64_t u = tiles * c, per = (u + kNumSMs - 1) / kNumSMs;
    const double eff = u < kNumSMs ? 1.0 : (double)u / (double)(per * kNumSMs);
    if (eff > best_eff + 0.02) {
      best_eff = eff;
      nkc = c;
    }
    if (!allow_split || eff >= 0.9 || u >= 6 * kNumSMs) break;
  }
  return nkc ? K / nkc : 0;
}

__global__ void qg_tile_kernel(const uint8_t* __restrict__ w, int64_t rows, int64_t rowbytes, int kcb, int nkc, int rs,
                               uint8_t* __restrict__ out) {
  const int wpr = rs / 16;  // 16-byte words per padded row piece
  const int64_t n = rows * nkc * wpr;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int j = (int)(i % wpr);
    const int64_t pr = i / wpr;  // (tile, chunk, row) piece
    const int r = (int)(pr % 16);
    const int64_t tc = pr / 16;
    const int c = (int)(tc % nkc);
    const int64_t tile = tc / nkc;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (j * 16 < kcb) v = *reinterpret_cast<const uint4*>(w + (tile * 16 + r) * rowbytes + (int64_t)c * kcb + j * 16);
    reinterpret_cast<uint4*>(out)[i] = v;
  }
}

}  // namespace fmoe

using namespace fmoe;

extern "C" int32_t fmoe_qgemv_chunk(int32_t in_features, int32_t bits, int64_t rows_total, int32_t accumulate) {
  return qgemv_chunk(in_features, bits, rows_total, accumulate != 0);
}

extern "C" size_t fmoe_qweight_tile_bytes(const fmoe_qweight_t* w, int32_t kc) {
  QW q;
  if (to_qw(w, &q) || (q.bits != 4 && q.bits != 6 && q.bits != 8) || q.out % 16 || kc < 64 || kc % 64 ||
      q.in % kc)
    return 0;
  return (size_t)q.out * (q.in / kc) * qgemv_row_stride(kc * q.bits / 8, q.bits);
}

extern "C" int fmoe_qweight_tile(const fmoe_qweight_t* w, int32_t kc, void* out, size_t bytes, void* stream) {
  QW q;
  int rc;
  if ((rc = to_qw(w, &q))) return rc;
  const size_t need = fmoe_qweight_tile_bytes(w, kc);
  if (!need) return set_error(FMOE_ERR_INVALID, "qweight_tile: %d x %d at %d bits, chunk %d", q.out, q.in, q.bits, kc);
  if (!out || bytes < need || !aligned(out, 16) || !aligned(q.w, 16))
    return set_error(FMOE_ERR_WORKSPACE, "qweight_tile: %zu bytes (16-byte aligned) required", need);
  const int kcb = kc * q.bits / 8, rs = qgemv_row_stride(kcb, q.bits);
  qg_tile_kernel<<<4 * kNumSMs, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(q.w), q.out, (int64_t)q.in * q.bits / 8, kcb, q.in / kc, rs,
      static_cast<uint8_t*>(out));
  return check_launch("qg_tile_kernel");
}
