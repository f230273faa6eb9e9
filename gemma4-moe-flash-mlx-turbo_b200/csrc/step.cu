// Whole decode step of the Gemma-4 decoder for one sequence (batch 1) in ONE
// persistent kernel: embedding row, 30 x DecoderLayer::forward_gemma4
// (src/model/mod.rs:67-119: attention block gemma4_attention.rs:46-112, dense
// GeLU MLP mlp.rs:28-41, router + experts moe.rs:315-470), final norm, tied
// lm_head with softcap and greedy argmax (mod.rs:254, 336-362).
//
// Why one kernel: at batch 1 a layer is ~75 MB of weights, 11 us of HBM time
// at 6.5 TB/s, split over ~11 dependent ops; as separate launches every op
// boundary drains the weight stream.  Here every SM runs one CTA for the whole
// step, with three warp roles:
//   * producer (1 thread): streams the CTA's share of EVERY op's weights (and
//     KV tiles) through a shared-memory ring with TMA bulk copies, in program
//     order, running ahead across op boundaries as far as the ring allows.
//     Weight addresses never depend on data, except the routed experts' (it
//     waits for the router's ids) and the KV tile count (the position).
//   * 8 compute warps: per unit, the tensor-core GEMV over the staged tile
//     (f16 "1024 + code" operands, fp32 accumulation) into per-warp partial
//     sums; the row chains between ops (RMSNorms, residuals) and attention.
//   * epilogue warp: adds the partial sums of each unit, applies the op's
//     epilogue (stores, GELU gating, softcap, argmax) and all inter-CTA
//     signalling and last-arriver work (q/k/v norms + RoPE + KV append per
//     head, router top-k, weighted expert combine per row tile), so no global
//     round trip sits between two units of the compute warps.
// Dependencies between ops are device counters (release: __threadfence +
// atomicAdd; acquire: ld.acquire polling), every wait bounded.  An op is a list
// of "units" in segments; CTA c takes the contiguous slice [n c / G, n (c+1) / G)
// of every segment.
//
// Ops per layer (units at the Gemma-4 26B shapes, sliding layer):
//   QKV  q|k|v = input_norm(x) . [Wq Wk Wv]^T: 16-row units, 8-bit, full K.  512
//   ATTN split-KV attention over the cached positions (the slot written this
//        step excluded) on at most 16 CTAs per KV head; one unit = 32 (D 256)
//        or 16 (D 512) positions of a head; per (head, CTA) softmax states are
//        merged with the new position by the head's last segment.       256
//   O    o = attn . Wo^T: 16 rows x 2048 input columns, fp32 partial sums per
//        column chunk, added in chunk order by the next op.              352
//   GU   ff_in (h, pre-ff norms, router input) in every CTA; the bf16 router
//        (32 units of 16 experts x 704 columns; the last runs softmax / top-8
//        / renorm), the dense gate|up (16+16 rows, GELU-tanh gating in the
//        epilogue), then the 8 routed experts' gate|up.             32+132+352
//   DOWN dense down (32 rows), as soon as the dense gate|up is complete, then
//        the experts' down (32 rows each); the last unit of a 32-row tile
//        forms the weighted top-k combine.                            88+704
// then ff_out (the next layer's QKV prologue, or the lm_head's), and LM: the
// 6-bit tied lm_head, softcap, argmax per CTA and one 64-bit atomicMax.
// Numerics follow the per-op kernels of this library (the same bf16 rounding
// points, operands and fp32 accumulation).
#include <algorithm>
#include <cmath>
#include <mutex>
#include <vector>
#include "internal.h"
#include "common.cuh"
#include "stage.cuh"
#include "qfrag.cuh"
#include "rowops.cuh"

namespace fmoe {
namespace step {

constexpr int NW = 8;                 // compute warps
constexpr int NT = NW * 32;           // compute threads
constexpr int EW = NW;                // epilogue warp
constexpr int PW = NW + 1;            // producer warp
constexpr int THREADS = (NW + 2) * 32;
constexpr int SLOTS = 16;             // ring entries in flight
constexpr int RR = 4;                 // partial-sum buffers between compute and epilogue warps
constexpr int H_MAX = 3072;           // hidden size bound (chain buffers)
constexpr int PER = H_MAX / NT;       // hidden elements per compute thread
constexpr int GMAX = 128;             // 64-column input groups in the fragment buffer
constexpr int SPH = 16;               // attention CTAs per KV head
constexpr int SEG_MAX = SPH + 1;      // attention segments per head
constexpr int KMAX = 8;               // top-k bound
constexpr int EMAX = 256;             // experts bound
constexpr int RQ = 4;                 // router column quarters
// Bytes a producer keeps in flight (issued, not landed).  Near the
// bandwidth-delay product per SM: more only lengthens the memory queues that
// every dependent load of the step waits in.
constexpr int INFLIGHT = 64 * 1024;
constexpr int CL = 256;               // counters per layer
constexpr int SMEM = 232448;          // dynamic shared memory per CTA (227 KB)

// counters of layer l at ctr + l * CL; after the last layer: [0] CTAs done, [1] abort flag
enum {
  C_QKV = 0,     // QKV units done
  C_ASEG = 1,    // [16] attention segments published per KV head
  C_ADONE = 17,  // KV heads merged
  C_ODONE = 18,  // O units done
  C_RTR = 19,    // router units done
  C_ROUTE = 20,  // 1 once ids / wts are written
  C_GUD = 21,    // dense gate|up units done
  C_GUE = 22,    // expert gate|up units done
  C_DOWN = 23,   // 32-row DOWN tiles done (dense + weighted expert combine)
};

// shared-memory map
constexpr int S_BAR = 0;                         // full[SLOTS] empty[SLOTS] rfull[RR] rempty[RR]
constexpr int S_MISC = 512;                      // int[4] broadcast slots
constexpr int S_RED8 = S_MISC + 64;              // float[16] block sums
constexpr int S_LG = S_MISC + 128;               // float[EMAX] router logits (epilogue warp)
constexpr int S_SEL = S_LG + 4 * EMAX;           // int sel_e[16], float sel_v[16]
constexpr int S_RED = S_SEL + 128;               // float[RR][NW][32] per-warp unit sums
constexpr int S_XSUM = S_RED + RR * NW * 32 * 4; // float[GMAX]
constexpr int S_FRAG = S_XSUM + GMAX * 4;        // uint4[GMAX][4 lanes][2]; attention: q f32 [8][512]
constexpr int S_VEC = S_FRAG + GMAX * 128;       // bf16[3][H_MAX]; attention: scores / merge
constexpr int S_QKN = S_VEC + 3 * H_MAX * 2;     // bf16[2][512] q_norm, k_norm of the layer
constexpr int S_RING = (S_QKN + 2048 + 127) / 128 * 128;
constexpr int RING = SMEM - S_RING;
static_assert(S_FRAG % 16 == 0 && S_VEC % 16 == 0, "alignment");

// ---------------------------------------------------------------------------
// device-side description of the model and the workspace (built on the host)

struct DQ {
  const uint8_t* w;
  const bf16* s;
  const bf16* b;
};
struct DLayer {
  DQ q, k, v, o, gate, up, down;
  const bf16* router;  // bf16 [E][H]
  const float* logit_bias;
  const bf16 *q_norm, *k_norm, *in_norm, *post_attn, *pre_ff, *post_ff1, *pre_ff2, *post_ff2, *post_ff;
  const bf16 *rscale, *pes;
  const uint8_t* ex;
  int64_t ex_stride;
  int64_t ex_off[9];
  bf16* kc;  // [Hkv][cap][D]
  bf16* vc;
  int64_t cap;
  int Hq, Hkv, D, rope_dims, k_eq_v, pad;
  float log2_theta, eps, scalar, attn_scale, root;
};
struct DModel {
  const DLayer* layers;
  int L, H, Id, E, Ie, K, V;
  DQ embed;
  const bf16* final_norm;
  float eps, softcap, emb_scale;
  // workspace
  int* status;
  int* abort_flag;
  unsigned* ctr;         // [L][CL] + [CL] (step-wide)
  unsigned long long* best;
  float* qkv;            // [rows]
  float* apart;          // [Hkv][SEG_MAX][16 + 8 * D]
  bf16* att;             // [Hq * D]
  float* opart;          // [nkc][H]
  bf16* x;               // [H]
  bf16* h;               // [H]
  float* rlog;           // [RQ][E]
  int32_t* ids;          // [K]
  float* wts;            // [K]
  bf16* actd;            // [Id]
  bf16* acte;            // [K][Ie]
  float* yd;             // [H]
  float* ym;             // [H] weighted expert combine
  // caller
  float* logits;         // [V]
  int32_t* tok;          // [1] in: current token, out: next token
  int64_t* pos;          // [2] {position, attended slots}
};

// ---------------------------------------------------------------------------
// small device helpers

__device__ __forceinline__ void cbar() { asm volatile("bar.sync 1, %0;\n" ::"n"(NT) : "memory"); }
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ int ld_acquire_i(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ float ldcg_bf(const bf16* p) {
  return bfbits2f(__ldcg(reinterpret_cast<const unsigned short*>(p)));
}
__device__ __forceinline__ bool aborted(const DModel& m) { return *(volatile int*)m.abort_flag != 0; }
__device__ __forceinline__ void fail(const DModel& m, int site) {
  atomicCAS(m.status, 0, site);
  atomicExch(m.abort_flag, 1);
}

constexpr int kSpin = 1 << 22;
// One thread: wait until *p >= target (bounded; gives up on a global abort).
__device__ bool spin_ge(const DModel& m, const unsigned* p, unsigned target, int site) {
  for (int i = 0; i < kSpin; ++i) {
    if (ld_acquire(p) >= target) return true;
    if ((i & 15) == 15 && aborted(m)) return false;
    __nanosleep(i < 64 ? 32 : 256);
  }
  fail(m, site);
  return false;
}
__device__ __forceinline__ bool try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(done)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return done != 0;
}
// Bounded mbarrier wait that also gives up on a global abort.
__device__ bool bar_wait(const DModel& m, uint64_t* bar, uint32_t parity, int site) {
  for (int i = 0; i < kMaxWaitIters; ++i) {
    if (try_wait(bar, parity)) return true;
    if ((i & 255) == 255 && aborted(m)) return false;
  }
  fail(m, site);
  return false;
}

// Compute-warp broadcast of thread 0's value (4 rotating slots: a slot is
// rewritten only after every compute thread passed 3 more barriers).
struct Bc {
  int* slot;
  int n;
  __device__ int operator()(int v) {
    int* s = slot + (n & 3);
    ++n;
    if (threadIdx.x == 0) *s = v;
    cbar();
    return *(volatile int*)s;
  }
};

// Sum over the compute threads (fixed order).
__device__ __forceinline__ float csum(float v, float* red8) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  cbar();
  if (lane == 0) red8[warp] = v;
  cbar();
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) s += red8[w];
  return s;
}

__device__ __forceinline__ int slice0(int n, int c, int G) { return (int)((int64_t)n * c / G); }
// CTA owning unit u of a single-segment op with U units over G CTAs.
__device__ __forceinline__ int cta_of(int u, int U, int G) { return (int)(((int64_t)(u + 1) * G + U - 1) / U) - 1; }

__host__ __device__ inline int row_stride(int bytes, int bits) {
  // bank-conflict-free residues (mod 128 B) for the A-fragment loads of
  // load_a_frags / the bf16 router tiles
  int s = (bytes + 15) & ~15;
  for (;;) {
    const int r = s % 128;
    if (bits == 4 && (r == 32 || r == 96)) return s;
    if (bits == 8 && r == 64) return s;
    if (bits == 6 && r == 16) return s;
    if (bits == 16 && r == 16) return s;
    s += 16;
  }
}

__device__ __forceinline__ void load_w(const bf16* w, int H, float (&v)[PER]) {
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = threadIdx.x + k * NT;
    v[k] = w && i < H ? bf2f(w[i]) : 0.f;
  }
}

// ---------------------------------------------------------------------------
// op geometry shared by the three roles

// OP_PRO / OP_GUP / OP_LMP: one unit per CTA carrying the constant vectors of
// the next row chain (norm weights; the embedding row in layer 0), streamed by
// the producer ahead of time like any weight tile.
enum { OP_PRO = 0, OP_QKV, OP_ATTN, OP_O, OP_GUP, OP_GU, OP_DOWN, OP_LMP, OP_LM };
constexpr int OKC = 2048;  // O-projection input columns per unit

struct Geo {
  int U;        // units
  int nseg;     // segments
  int sb[4];    // segment s = units [sb[s], sb[s+1])
  int NA;       // CTAs taking part
  int nold;     // ATTN: cached positions attended (the slot written this step excluded)
  int PT, NTt;  // ATTN: positions per unit, units per KV head
  int evict;    // ATTN: slot overwritten this step (-1: none)
  int64_t slot; // slot of the new position
  int layer;
};

__device__ __forceinline__ Geo geo(const DModel& m, const DLayer& L, int op, int64_t pos, int G) {
  Geo g{};
  g.nseg = 1;
  g.NA = G;
  switch (op) {
    case OP_QKV:
      g.U = (L.Hq + L.Hkv * (L.k_eq_v ? 1 : 2)) * L.D / 16;
      break;
    case OP_ATTN: {
      const int64_t nold = pos < L.cap ? pos : L.cap;
      g.nold = (int)nold;
      g.PT = 8192 / L.D;
      g.NTt = (g.nold + g.PT - 1) / g.PT;
      g.U = L.Hkv * g.NTt;
      g.NA = min(G, L.Hkv * SPH);
      g.evict = pos >= L.cap ? (int)(pos % L.cap) : -1;
      break;
    }
    case OP_O:
      g.U = (m.H / 16) * (L.Hq * L.D / OKC);
      break;
    case OP_GU:
      g.nseg = 3;
      g.sb[1] = (m.E / 16) * RQ;
      g.sb[2] = g.sb[1] + m.Id / 16;
      g.U = g.sb[2] + m.K * (m.Ie / 16);
      break;
    case OP_DOWN:  // CTA r < H/32 owns 32-row tile r: its dense unit, then its K expert units
      g.U = (m.H / 32) * (1 + m.K);
      g.NA = m.H / 32;
      break;
    case OP_LM:
      g.U = m.V / 16;
      break;
    default:  // OP_PRO, OP_GUP, OP_LMP
      g.U = G;
  }
  g.sb[0] = 0;
  g.sb[g.nseg] = g.U;
  g.slot = pos % L.cap;
  g.layer = (int)(&L - m.layers);
  return g;
}

// Units [i0, i1) of segment s for CTA c.
__device__ __forceinline__ void seg_range(const Geo& g, int s, int c, int& i0, int& i1) {
  const int n = g.sb[s + 1] - g.sb[s];
  if (c >= g.NA) {
    i0 = i1 = g.sb[s];
    return;
  }
  i0 = g.sb[s] + slice0(n, c, g.NA);
  i1 = g.sb[s] + slice0(n, c + 1, g.NA);
}

// Layer prologue unit: in_norm | q_norm | k_norm | then post_ff1 | post_ff2 |
// post_ff of the previous layer, or (layer 0) the embedding row's codes and
// 16-byte windows around its scale and bias rows.
__device__ __forceinline__ int pro_bytes(const DModel& m, const DLayer& L, int l) {
  const int base = m.H * 2 + 4 * L.D;
  return l > 0 ? base + 3 * m.H * 2 : base + m.H * 6 / 8 + 2 * 128;
}

// Ring bytes of one unit.
__device__ __forceinline__ int unit_bytes(const DModel& m, const DLayer& L, int op, int u, const Geo& g) {
  const int H = m.H, G = H / 64;
  switch (op) {
    case OP_QKV: return 16 * row_stride(H, 8) + 64 * G;
    case OP_ATTN: return 2 * (8192 / L.D) * L.D * 2;
    case OP_O: return 16 * row_stride(OKC, 8) + 64 * (OKC / 64);
    case OP_GU: return u < g.sb[1] ? 16 * row_stride(H / RQ * 2, 16) : 32 * row_stride(H / 2, 4) + 128 * G;
    case OP_DOWN:
      return u % (1 + m.K) == 0 ? 32 * (m.Id / 2) + 128 * (m.Id / 64) : 32 * (m.Ie / 2) + 128 * (m.Ie / 64);
    case OP_LM: return 16 * row_stride(H * 6 / 8, 6) + 64 * G;
    case OP_PRO: return pro_bytes(m, L, g.layer);
    default: return 4 * H * 2;  // OP_GUP, OP_LMP
  }
}

// Ring allocation: every role replays the same sequence of sizes.
__device__ __forceinline__ int ring_take(int& head, int bytes) {
  int st = head;
  if (st + bytes > RING) st = 0;
  head = st + bytes;
  return st;
}

// ---------------------------------------------------------------------------
// producer: the copies of one unit

__device__ __forceinline__ void cp(uint8_t* dst, const void* src, int bytes, uint64_t* bar) {
  bulk_g2s(dst, src, (uint32_t)bytes, bar);
}
__device__ __forceinline__ void cp_rows(uint8_t* dst, int dstride, const uint8_t* src, int64_t sstride, int bytes,
                                        int rows, uint64_t* bar) {
  for (int r = 0; r < rows; ++r) cp(dst + r * dstride, src + r * sstride, bytes, bar);
}

__device__ void issue_unit(const DModel& m, const DLayer& L, int op, int u, const Geo& gm, const int* ids,
                           uint8_t* dst, uint64_t* bar) {
  const int H = m.H, G = H / 64;
  switch (op) {
    case OP_QKV: {
      const int row0 = u * 16, qd = L.Hq * L.D, kd = L.Hkv * L.D;
      const DQ& w = row0 < qd ? L.q : row0 < qd + kd ? L.k : L.v;
      const int r = row0 < qd ? row0 : row0 < qd + kd ? row0 - qd : row0 - qd - kd;
      const int RS = row_stride(H, 8);
      mbar_arrive_expect_tx(bar, (uint32_t)(16 * H + 64 * G));
      cp_rows(dst, RS, w.w + (int64_t)r * H, H, H, 16, bar);
      cp(dst + 16 * RS, w.s + (int64_t)r * G, 32 * G, bar);
      cp(dst + 16 * RS + 32 * G, w.b + (int64_t)r * G, 32 * G, bar);
      return;
    }
    case OP_ATTN: {
      const int hk = u / gm.NTt, t = u % gm.NTt, p0 = t * gm.PT;
      const int np = min(gm.PT, gm.nold - p0);
      const int64_t off = ((int64_t)hk * L.cap + p0) * L.D;
      const int rb = np * L.D * 2;
      mbar_arrive_expect_tx(bar, (uint32_t)(2 * rb));
      cp(dst, L.kc + off, rb, bar);
      cp(dst + gm.PT * L.D * 2, L.vc + off, rb, bar);
      return;
    }
    case OP_O: {
      const int K = L.Hq * L.D, nkc = K / OKC, Go = K / 64;
      const int tile = u / nkc, kci = u % nkc, row0 = tile * 16;
      const int RS = row_stride(OKC, 8), gc = OKC / 64;
      mbar_arrive_expect_tx(bar, (uint32_t)(16 * OKC + 64 * gc));
      cp_rows(dst, RS, L.o.w + (int64_t)row0 * K + kci * OKC, K, OKC, 16, bar);
      const uint8_t* s = reinterpret_cast<const uint8_t*>(L.o.s + (int64_t)row0 * Go + kci * gc);
      const uint8_t* b = reinterpret_cast<const uint8_t*>(L.o.b + (int64_t)row0 * Go + kci * gc);
      cp_rows(dst + 16 * RS, 2 * gc, s, 2 * Go, 2 * gc, 16, bar);
      cp_rows(dst + 16 * RS + 32 * gc, 2 * gc, b, 2 * Go, 2 * gc, 16, bar);
      return;
    }
    case OP_GU: {
      if (u < gm.sb[1]) {  // router: 16 experts x a quarter of the hidden columns, bf16
        const int tile = u / RQ, qc = u % RQ, cols = H / RQ;
        const int RS = row_stride(cols * 2, 16);
        mbar_arrive_expect_tx(bar, (uint32_t)(16 * cols * 2));
        cp_rows(dst, RS, reinterpret_cast<const uint8_t*>(L.router + (int64_t)tile * 16 * H + qc * cols),
                (int64_t)H * 2, cols * 2, 16, bar);
        return;
      }
      const int ne = m.Ie / 16;
      const uint8_t *gw, *uw;
      const bf16 *gs, *gb, *us, *ub;
      int i;
      if (u < gm.sb[2]) {
        i = u - gm.sb[1];
        gw = L.gate.w, gs = L.gate.s, gb = L.gate.b, uw = L.up.w, us = L.up.s, ub = L.up.b;
      } else {
        const int j = (u - gm.sb[2]) / ne;
        i = (u - gm.sb[2]) % ne;
        const uint8_t* base = L.ex + (int64_t)ids[j] * L.ex_stride;
        gw = base + L.ex_off[0], gs = reinterpret_cast<const bf16*>(base + L.ex_off[1]);
        gb = reinterpret_cast<const bf16*>(base + L.ex_off[2]);
        uw = base + L.ex_off[3], us = reinterpret_cast<const bf16*>(base + L.ex_off[4]);
        ub = reinterpret_cast<const bf16*>(base + L.ex_off[5]);
      }
      const int RS = row_stride(H / 2, 4), rb = H / 2;
      const int64_t r0 = (int64_t)i * 16;
      mbar_arrive_expect_tx(bar, (uint32_t)(32 * rb + 128 * G));
      cp_rows(dst, RS, gw + r0 * rb, rb, rb, 16, bar);
      cp_rows(dst + 16 * RS, RS, uw + r0 * rb, rb, rb, 16, bar);
      uint8_t* sc = dst + 32 * RS;
      cp(sc, gs + r0 * G, 32 * G, bar);
      cp(sc + 32 * G, gb + r0 * G, 32 * G, bar);
      cp(sc + 64 * G, us + r0 * G, 32 * G, bar);
      cp(sc + 96 * G, ub + r0 * G, 32 * G, bar);
      return;
    }
    case OP_DOWN: {
      const uint8_t* w;
      const bf16 *ws, *wb;
      int K;
      const int r = u / (1 + m.K), sl = u % (1 + m.K);
      if (sl == 0) {
        w = L.down.w, ws = L.down.s, wb = L.down.b, K = m.Id;
      } else {
        const uint8_t* base = L.ex + (int64_t)ids[sl - 1] * L.ex_stride;
        w = base + L.ex_off[6], ws = reinterpret_cast<const bf16*>(base + L.ex_off[7]);
        wb = reinterpret_cast<const bf16*>(base + L.ex_off[8]);
        K = m.Ie;
      }
      const int rb = K / 2, Gk = K / 64;
      const int64_t r0 = (int64_t)r * 32;
      mbar_arrive_expect_tx(bar, (uint32_t)(32 * rb + 128 * Gk));
      cp(dst, w + r0 * rb, 32 * rb, bar);  // the row residue keeps contiguous rows conflict-free
      uint8_t* sc = dst + 32 * rb;
      cp(sc, ws + r0 * Gk, 32 * Gk, bar);
      cp(sc + 32 * Gk, wb + r0 * Gk, 32 * Gk, bar);
      cp(sc + 64 * Gk, ws + (r0 + 16) * Gk, 32 * Gk, bar);
      cp(sc + 96 * Gk, wb + (r0 + 16) * Gk, 32 * Gk, bar);
      return;
    }
    case OP_PRO: {
      const int l = gm.layer, H2 = H * 2, D2 = L.D * 2;
      int bytes = H2 + 2 * D2;
      cp(dst, L.in_norm, H2, bar);
      cp(dst + H2, L.q_norm, D2, bar);
      cp(dst + H2 + D2, L.k_norm, D2, bar);
      uint8_t* d2 = dst + H2 + 2 * D2;
      if (l > 0) {
        const DLayer& Lp = m.layers[l - 1];
        cp(d2, Lp.post_ff1, H2, bar);
        cp(d2 + H2, Lp.post_ff2, H2, bar);
        cp(d2 + 2 * H2, Lp.post_ff, H2, bar);
        bytes += 3 * H2;
      } else {
        const int rb = H * 6 / 8;
        const int tok = ids[0];  // the step's token (row 0 when out of range)
        cp(d2, m.embed.w + (int64_t)tok * rb, rb, bar);
        const int64_t so = (int64_t)tok * G * 2, a = so & ~15ll, e = (so + 2 * G + 15) & ~15ll;
        cp(d2 + rb, reinterpret_cast<const uint8_t*>(m.embed.s) + a, (int)(e - a), bar);
        cp(d2 + rb + 128, reinterpret_cast<const uint8_t*>(m.embed.b) + a, (int)(e - a), bar);
        bytes += rb + 2 * (int)(e - a);
      }
      mbar_arrive_expect_tx(bar, (uint32_t)bytes);
      return;
    }
    case OP_GUP: {
      const int H2 = H * 2;
      mbar_arrive_expect_tx(bar, (uint32_t)((L.rscale ? 4 : 3) * H2));
      cp(dst, L.post_attn, H2, bar);
      cp(dst + H2, L.pre_ff, H2, bar);
      cp(dst + 2 * H2, L.pre_ff2, H2, bar);
      if (L.rscale) cp(dst + 3 * H2, L.rscale, H2, bar);
      return;
    }
    case OP_LMP: {
      const int H2 = H * 2;
      mbar_arrive_expect_tx(bar, (uint32_t)(4 * H2));
      cp(dst, L.post_ff1, H2, bar);
      cp(dst + H2, L.post_ff2, H2, bar);
      cp(dst + 2 * H2, L.post_ff, H2, bar);
      cp(dst + 3 * H2, m.final_norm, H2, bar);
      return;
    }
    default: {  // LM: 16 rows of the 6-bit embedding table
      const int rb = H * 6 / 8, RS = row_stride(rb, 6);
      const int64_t r0 = (int64_t)u * 16;
      mbar_arrive_expect_tx(bar, (uint32_t)(16 * rb + 64 * G));
      cp_rows(dst, RS, m.embed.w + r0 * rb, rb, rb, 16, bar);
      cp(dst + 16 * RS, m.embed.s + r0 * G, 32 * G, bar);
      cp(dst + 16 * RS + 32 * G, m.embed.b + r0 * G, 32 * G, bar);
      return;
    }
  }
}

__device__ __forceinline__ bool routed_unit(const DModel& m, int op, int u, const Geo& g) {
  return (op == OP_GU && u >= g.sb[2]) || (op == OP_DOWN && u % (1 + m.K) != 0);
}

// The producer thread: every unit of every op of this CTA, in order.
__device__ void producer(const DModel& m, uint8_t* smem, int64_t pos) {
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S_BAR);
  uint64_t* empty = full + SLOTS;
  uint8_t* ring = smem + S_RING;
  const int c = blockIdx.x, G = gridDim.x;
  int fst[SLOTS], fen[SLOTS];  // unreleased units (FIFO): ring ranges
  int fhead = 0, fn = 0;       // FIFO front index, count
  int head = 0, seq = 0;       // ring head, unit sequence number
  int lseq = 0, lbytes = 0;    // first unit not known to have landed; bytes issued since
  int ids[KMAX];
  {
    const int tok = *m.tok;  // layer 0's prologue unit carries this token's embedding row
    ids[0] = tok >= 0 && tok < m.V ? tok : 0;
  }
  bool ok = true;
  for (int l = 0; l <= m.L && ok; ++l) {
    const DLayer& L = m.layers[l < m.L ? l : m.L - 1];
    const int op0 = l < m.L ? OP_PRO : OP_LMP, op1 = l < m.L ? OP_DOWN : OP_LM;
    bool have_ids = false;
    for (int op = op0; op <= op1 && ok; ++op) {
      const Geo gm = geo(m, L, op, pos, G);
      for (int s = 0; s < gm.nseg && ok; ++s) {
        int i0, i1;
        seg_range(gm, s, c, i0, i1);
        for (int u = i0; u < i1 && ok; ++u) {
          if (routed_unit(m, op, u, gm) && !have_ids) {
            if (!spin_ge(m, m.ctr + l * CL + C_ROUTE, 1u, 201)) {
              ok = false;
              break;
            }
            for (int j = 0; j < m.K; ++j) {
              const int e = ld_acquire_i(m.ids + j);
              ids[j] = e < 0 ? 0 : e >= m.E ? m.E - 1 : e;
            }
            have_ids = true;
          }
          const int bytes = unit_bytes(m, L, op, u, gm);
          int st = head;
          if (st + bytes > RING) st = 0;
          // free the ring range [st, st + bytes) and a slot: wait for the
          // oldest in-flight units until none overlaps and a slot is free
          for (;;) {
            bool clash = fn == SLOTS;
            for (int k = 0; k < fn && !clash; ++k) {
              const int f = (fhead + k) % SLOTS;
              clash = fst[f] < st + bytes && st < fen[f];
            }
            if (!clash) break;
            const int old = seq - fn;  // sequence number of the FIFO front
            if (!bar_wait(m, &empty[old % SLOTS], (uint32_t)(old / SLOTS) & 1u, 202)) {
              ok = false;
              break;
            }
            if (old >= lseq) {  // released implies landed
              for (int k = lseq; k <= old; ++k) lbytes -= fen[(fhead + k - old) % SLOTS] - fst[(fhead + k - old) % SLOTS];
              lseq = old + 1;
            }
            fhead = (fhead + 1) % SLOTS;
            --fn;
          }
          if (!ok) break;
          // keep the bytes in flight near the bandwidth-delay product
          while (lseq < seq && lbytes + bytes > INFLIGHT) {
            const int f0 = (fhead + lseq - (seq - fn)) % SLOTS;
            if (!bar_wait(m, &full[lseq % SLOTS], (uint32_t)(lseq / SLOTS) & 1u, 203)) {
              ok = false;
              break;
            }
            lbytes -= fen[f0] - fst[f0];
            ++lseq;
          }
          if (!ok) break;
          head = st + bytes;
          const int f = (fhead + fn) % SLOTS;
          fst[f] = st;
          fen[f] = st + bytes;
          ++fn;
          issue_unit(m, L, op, u, gm, ids, ring + st, &full[seq % SLOTS]);
          lbytes += bytes;
          ++seq;
        }
      }
    }
  }
  // let every issued copy land before the CTA (and its shared memory) can end
  for (int k = 0; k < fn; ++k) {
    const int s = seq - fn + k;
    for (int i = 0; i < kMaxWaitIters && !try_wait(&full[s % SLOTS], (uint32_t)(s / SLOTS) & 1u); ++i) {
    }
  }
}

// ---------------------------------------------------------------------------
// compute warps

struct Ctx {
  const DModel* m;
  uint8_t* smem;
  uint64_t* full;
  uint64_t* empty;
  uint64_t* rfull;
  uint64_t* rempty;
  float* red8;
  float* red;         // [RR][NW][32]
  float* xsum;
  uint4* frag;
  bf16* vec;          // [3][H_MAX]
  int head, seq, rseq;
  Bc bc;
  int warp, lane;
  int64_t pos;
};

// Wait for the next unit's tile (and, for GEMV units, a free partial-sum
// buffer); false when a wait gave up (the unit is then skipped, not left:
// the next op's counter wait ends the step uniformly).
__device__ __forceinline__ const uint8_t* unit_begin(Ctx& x, int bytes, bool red, bool& ok) {
  const int off = ring_take(x.head, bytes);
  const int s = x.seq;
  ok = bar_wait(*x.m, &x.full[s % SLOTS], (uint32_t)(s / SLOTS) & 1u, 101);
  if (red && x.rseq >= RR && ok)
    ok = bar_wait(*x.m, &x.rempty[x.rseq % RR], (uint32_t)(x.rseq / RR - 1) & 1u, 103);
  return x.smem + S_RING + off;
}
__device__ __forceinline__ void unit_end(Ctx& x, bool red) {
  __syncwarp();
  if (x.lane == 0) {
    mbar_arrive(&x.empty[x.seq % SLOTS]);
    if (red) mbar_arrive(&x.rfull[x.rseq % RR]);
  }
  ++x.seq;
  if (red) ++x.rseq;
}

// Compute-warp wait on a counter (thread 0 polls); uniform result.
__device__ __forceinline__ bool cwait(Ctx& x, const unsigned* p, unsigned target, int site) {
  int ok = 1;
  if (threadIdx.x == 0) ok = spin_ge(*x.m, p, target, site) ? 1 : 0;
  return x.bc(ok) != 0;
}

// f16 B fragments + group sums of an input row held as bf16 in shared memory.
template <int BITS>
__device__ void build_frags(Ctx& x, const bf16* v, int ncols, int gbase) {
  const int items = ncols / 64 * 4;
  for (int it0 = 0; it0 < items; it0 += NT) {
    const int it = it0 + threadIdx.x;
    const bool live = it < items;
    const int gi = it >> 2, tq = it & 3;
    float f[16];
    float s = 0.f;
    if (live) {
      const uint4 a = *reinterpret_cast<const uint4*>(v + gi * 64 + 16 * tq);
      const uint4 b = *reinterpret_cast<const uint4*>(v + gi * 64 + 16 * tq + 8);
      const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        f[2 * e] = f16r(bf16lo(w[e]));
        f[2 * e + 1] = f16r(bf16hi(w[e]));
      }
    } else {
#pragma unroll
      for (int e = 0; e < 16; ++e) f[e] = 0.f;
    }
#pragma unroll
    for (int e = 0; e < 16; ++e) s += f[e];
    uint32_t b[8];
    make_b_frags<BITS>(f, b);
    if (live) {
      uint4* d = x.frag + ((gbase + gi) * 4 + tq) * 2;
      d[0] = make_uint4(b[0], b[1], b[2], b[3]);
      d[1] = make_uint4(b[4], b[5], b[6], b[7]);
    }
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    if (live && tq == 0) x.xsum[gbase + gi] = s;
  }
}

// One 64-column group of a quantised GEMV unit: RT 16-row tiles.  The four
// MMAs of a tile accumulate into two independent chains.
template <int BITS, int RT>
__device__ __forceinline__ void gemv_group(const Ctx& x, const uint8_t* rbase, int RS, int SG, const uint8_t* sc,
                                           int gl, int gi, float (&y)[RT][2]) {
  const int g = x.lane >> 2, t = x.lane & 3;
  uint4 b0 = make_uint4(0, 0, 0, 0), b1 = b0;
  if (g == 0) {
    const uint4* fp = x.frag + (gi * 4 + t) * 2;
    b0 = fp[0];
    b1 = fp[1];
  }
  const uint32_t bb0[4] = {b0.x, b0.y, b0.z, b0.w}, bb1[4] = {b1.x, b1.y, b1.z, b1.w};
  const float xs = x.xsum[gi];
#pragma unroll
  for (int tt = 0; tt < RT; ++tt) {
    const uint8_t* rl = rbase + tt * 16 * RS + gl * (8 * BITS);
    const bf16* st = reinterpret_cast<const bf16*>(sc + tt * 64 * SG);
    const bf16* bt = st + 16 * SG;
    const float sl = bf2f(st[g * SG + gl]), bl = bf2f(bt[g * SG + gl]);
    const float sh = bf2f(st[(g + 8) * SG + gl]), bh = bf2f(bt[(g + 8) * SG + gl]);
    uint32_t af[4][4];
    load_a_frags<BITS>(rl, rl + 8 * RS, af);
    float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
    mma16816_f16(c0, af[0][0], af[0][1], af[0][2], af[0][3], bb0[0], bb1[0]);
    mma16816_f16(c1, af[1][0], af[1][1], af[1][2], af[1][3], bb0[1], bb1[1]);
    mma16816_f16(c0, af[2][0], af[2][1], af[2][2], af[2][3], bb0[2], bb1[2]);
    mma16816_f16(c1, af[3][0], af[3][1], af[3][2], af[3][3], bb0[3], bb1[3]);
    y[tt][0] += fmaf(sl, c0[0] + c1[0], fmaf(-1024.f, sl, bl) * xs);
    y[tt][1] += fmaf(sh, c0[2] + c1[2], fmaf(-1024.f, sh, bh) * xs);
  }
}

// One unit of a quantised GEMV: RT 16-row tiles x ng groups; per-warp sums
// to the unit's partial-sum buffer.  Two groups per iteration.
template <int BITS, int RT>
__device__ __forceinline__ void gemv_unit(Ctx& x, const uint8_t* base, int RS, int ng, int SG, int fg0, bool run) {
  const int g = x.lane >> 2, t = x.lane & 3;
  float y[RT][2];
#pragma unroll
  for (int tt = 0; tt < RT; ++tt) y[tt][0] = y[tt][1] = 0.f;
  const uint8_t* rbase = base + g * RS + t * (2 * BITS);
  const uint8_t* sc = base + RT * 16 * RS;
  if (run) {
    for (int gl = x.warp; gl < ng; gl += 2 * NW) {
      gemv_group<BITS, RT>(x, rbase, RS, SG, sc, gl, fg0 + gl, y);
      if (gl + NW < ng) gemv_group<BITS, RT>(x, rbase, RS, SG, sc, gl + NW, fg0 + gl + NW, y);
    }
  }
  float* rw = x.red + (x.rseq % RR) * NW * 32 + x.warp * 32;
  if (t == 0) {
#pragma unroll
    for (int tt = 0; tt < RT; ++tt) {
      rw[tt * 16 + g] = y[tt][0];
      rw[tt * 16 + g + 8] = y[tt][1];
    }
  }
}

// bf16 router tile: 16 experts x ng 64-column groups against the router input (bf16 in smem).
__device__ __forceinline__ void router_unit(Ctx& x, const uint8_t* base, int RS, int ng, const bf16* xs, bool run) {
  const int g = x.lane >> 2, t = x.lane & 3;
  float y[4] = {0.f, 0.f, 0.f, 0.f};
  for (int gl = x.warp; gl < ng && run; gl += NW) {
    const uint8_t* plo = base + g * RS + gl * 128 + 32 * t;
    const uint8_t* phi = plo + 8 * RS;
    const uint4 l0 = lds_u4(plo), l1 = lds_u4(plo + 16), h0 = lds_u4(phi), h1 = lds_u4(phi + 16);
    uint4 x0 = make_uint4(0, 0, 0, 0), x1 = x0;
    if (g == 0) {
      x0 = *reinterpret_cast<const uint4*>(xs + gl * 64 + 16 * t);
      x1 = *reinterpret_cast<const uint4*>(xs + gl * 64 + 16 * t + 8);
    }
    const uint32_t lw[8] = {l0.x, l0.y, l0.z, l0.w, l1.x, l1.y, l1.z, l1.w};
    const uint32_t hw[8] = {h0.x, h0.y, h0.z, h0.w, h1.x, h1.y, h1.z, h1.w};
    const uint32_t xw[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
#pragma unroll
    for (int s = 0; s < 4; ++s) mma16816(y, lw[2 * s], hw[2 * s], lw[2 * s + 1], hw[2 * s + 1], xw[2 * s], xw[2 * s + 1]);
  }
  float* rw = x.red + (x.rseq % RR) * NW * 32 + x.warp * 32;
  if (t == 0) {
    rw[g] = y[0];
    rw[g + 8] = y[2];
  }
}

// ---------------------------------------------------------------------------
// row chains (every CTA computes them; element i of thread t: i = t + k*NT)

struct FfOutW {
  float w1[PER], w2[PER], w[PER];
};

// ff_out of a layer: x = bf16(bf16(h + bf16(rms(s) * w)) * scalar),
// s = bf16(bf16(rms(bf16(d)) * w1) + bf16(rms(bf16(moe)) * w2)); into v[].
__device__ void chain_ff_out(Ctx& x, const DLayer& Lp, const FfOutW& fw, float (&v)[PER]) {
  const DModel& m = *x.m;
  const int H = m.H;
  float d[PER], mo[PER], hr[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = threadIdx.x + k * NT;
    d[k] = i < H ? __ldcg(m.yd + i) : 0.f;
    mo[k] = i < H ? __ldcg(m.ym + i) : 0.f;
    hr[k] = i < H ? ldcg_bf(m.h + i) : 0.f;
  }
  float sd = 0.f, sm = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    d[k] = round_bf(d[k]);
    mo[k] = round_bf(mo[k]);
    sd = fmaf(d[k], d[k], sd);
    sm = fmaf(mo[k], mo[k], sm);
  }
  const float rd = rsqrtf(csum(sd, x.red8) / (float)H + Lp.eps);
  const float rm = rsqrtf(csum(sm, x.red8 + 8) / (float)H + Lp.eps);
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    d[k] = round_bf(round_bf(d[k] * rd * fw.w1[k]) + round_bf(mo[k] * rm * fw.w2[k]));
    ss = fmaf(d[k], d[k], ss);
  }
  const float rs = rsqrtf(csum(ss, x.red8) / (float)H + Lp.eps);
  const float sc = round_bf(Lp.scalar);
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = threadIdx.x + k * NT;
    v[k] = i < H ? round_bf(round_bf(hr[k] + round_bf(d[k] * rs * fw.w[k])) * sc) : 0.f;
  }
}

__device__ __forceinline__ uint32_t code6(const uint32_t* row, int i) {
  const int b = 6 * i, wi = b >> 5, sh = b & 31;
  uint32_t v = row[wi] >> sh;
  if (sh > 26) v |= row[wi + 1] << (32 - sh);
  return v & 63u;
}

// x (the input of layer l, or of the lm_head when l == L) into v[]; CTA 0 stores
// it.  Layer 0: the embedding row from the prologue unit `emb` (codes, then
// the scale / bias windows).
__device__ void layer_input(Ctx& x, int l, const FfOutW& fw, const uint8_t* emb, float (&v)[PER]) {
  const DModel& m = *x.m;
  const int H = m.H, G = H / 64;
  if (l == 0) {  // embedding row: bf16(bf16(fma(s, q, b)) * bf16(sqrt(H)))
    const int tok = *m.tok;
    const bool okid = tok >= 0 && tok < m.V;
    const int rb = H * 6 / 8, sh = (int)(((int64_t)(okid ? tok : 0) * G * 2) & 15);
    const uint32_t* row = reinterpret_cast<const uint32_t*>(emb);
    const bf16* sc = reinterpret_cast<const bf16*>(emb + rb + sh);
    const bf16* bi = reinterpret_cast<const bf16*>(emb + rb + 128 + sh);
    const float es = round_bf(m.emb_scale);
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int i = threadIdx.x + k * NT;
      float val = 0.f;
      if (i < H && okid) val = round_bf(round_bf(fmaf(bf2f(sc[i / 64]), (float)code6(row, i), bf2f(bi[i / 64]))) * es);
      v[k] = val;
    }
  } else {
    chain_ff_out(x, m.layers[l - 1], fw, v);
  }
  if (blockIdx.x == 0) {
#pragma unroll
    for (int k = 0; k < PER; ++k) {
      const int i = threadIdx.x + k * NT;
      if (i < H) m.x[i] = __float2bfloat16_rn(v[k]);
    }
  }
}

// v -> bf16(rms(v) * w) into `dst` (shared memory).
__device__ void norm_to_vec(Ctx& x, const float (&v)[PER], const float (&w)[PER], float eps, bf16* dst) {
  const int H = x.m->H;
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) ss = fmaf(v[k], v[k], ss);
  const float r = rsqrtf(csum(ss, x.red8) / (float)H + eps);
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = threadIdx.x + k * NT;
    if (i < H) dst[i] = __float2bfloat16_rn(v[k] * r * w[k]);
  }
}

// ---------------------------------------------------------------------------
// attention (batch 1): per KV head, GQ = Hq / Hkv query heads, D = 32 * P.
// A CTA starting a head post-processes the head's projections itself (q / k
// norms, RoPE, v norm; Gemma4Attention::forward, gemma4_attention.rs:46-84):
// q into shared memory as f32 [gq][i][lane] (element lane * P + i: a warp's
// reads of one i are 32 consecutive words), the new k (same layout) and v;
// the head's first CTA also appends k / v to the cache slot.

struct AttnState {
  float acc[8][2];  // [gq][dims of this lane]: D / 256 dims per lane
};
struct AttnSm {
  float* qs;     // [8][P][32]
  float* sc;     // [8][32] scores / probabilities
  float* ml;     // [8] running max, [8] running sum
  float* alpha;  // [8]
  float* coef;   // [8][SEG_MAX] segment weights, [8] new-position weight, [8] 1/L
  float* kn;     // [P][32] new k
  float* vn;     // [D] new v
  const bf16* qn;  // q_norm, k_norm weights (copied from the layer's prologue unit)
  const bf16* kw;
};

template <int P>
__device__ void head_rows(Ctx& x, const DLayer& L, int hk, const AttnSm& A, bool append, int64_t slot) {
  const DModel& m = *x.m;
  const int D = 32 * P, GQ = L.Hq / L.Hkv, lane = x.lane;
  const int nrows = GQ + (L.k_eq_v ? 1 : 2);
  const float fpos = (float)x.pos;
  for (int r = x.warp; r < nrows; r += NW) {
    const int64_t row = r < GQ ? (int64_t)(hk * GQ + r) : r == GQ ? (int64_t)(L.Hq + hk) : (int64_t)(L.Hq + L.Hkv + hk);
    const float* src = m.qkv + row * D + lane * P;
    float v[P];
#pragma unroll
    for (int i = 0; i < P; ++i) v[i] = round_bf(__ldcg(src + i));
    const int64_t dst = ((int64_t)hk * L.cap + slot) * D;
    if (r < GQ) {
      warp_rms_norm<P>(v, A.qn, L.eps, lane);
      warp_rope<P>(v, L.rope_dims, L.log2_theta, fpos, lane);
#pragma unroll
      for (int i = 0; i < P; ++i) A.qs[(r * P + i) * 32 + lane] = v[i];
    } else if (r == GQ) {
      if (L.k_eq_v) {  // v = v_norm(raw k)
        float vv[P];
#pragma unroll
        for (int i = 0; i < P; ++i) vv[i] = v[i];
        warp_rms_norm<P>(vv, nullptr, L.eps, lane);
#pragma unroll
        for (int i = 0; i < P; ++i) A.vn[lane * P + i] = vv[i];
        if (append) store_row_bf16<P>(L.vc + dst, lane, vv);
      }
      warp_rms_norm<P>(v, A.kw, L.eps, lane);
      warp_rope<P>(v, L.rope_dims, L.log2_theta, fpos, lane);
#pragma unroll
      for (int i = 0; i < P; ++i) A.kn[i * 32 + lane] = v[i];
      if (append) store_row_bf16<P>(L.kc + dst, lane, v);
    } else {
      warp_rms_norm<P>(v, nullptr, L.eps, lane);
#pragma unroll
      for (int i = 0; i < P; ++i) A.vn[lane * P + i] = v[i];
      if (append) store_row_bf16<P>(L.vc + dst, lane, v);
    }
  }
}

template <int P>
__device__ void attn_segment_start(Ctx& x, const DLayer& L, int hk, const AttnSm& A, bool append, int64_t slot,
                                   AttnState& a) {
  head_rows<P>(x, L, hk, A, append, slot);
  if (threadIdx.x < 8) {
    A.ml[threadIdx.x] = -INFINITY;
    A.ml[8 + threadIdx.x] = 0.f;
  }
#pragma unroll
  for (int gq = 0; gq < 8; ++gq) a.acc[gq][0] = a.acc[gq][1] = 0.f;
  cbar();
}

// One tile of np positions starting at slot p0 (K rows at kt, V rows at vt).
template <int P>
__device__ void attn_tile(Ctx& x, const DLayer& L, const bf16* kt, const bf16* vt, int np, int p0, int evict,
                          const AttnSm& A, AttnState& a, bool run) {
  const int D = 32 * P, GQ = L.Hq / L.Hkv;
  // scores: warp w takes positions w, w+NW, ...
  for (int p = x.warp; p < np && run; p += NW) {
    float kf[P];
    load_row_f32<P>(kt + (int64_t)p * D, x.lane, kf);
    for (int gq = 0; gq < GQ; ++gq) {
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < P; ++i) s = fmaf(A.qs[(gq * P + i) * 32 + x.lane], kf[i], s);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
      if (x.lane == 0) A.sc[gq * 32 + p] = (p0 + p == evict) ? -INFINITY : s * L.attn_scale;
    }
  }
  cbar();
  // online softmax: warp gq
  if (x.warp < GQ) {
    const int gq = x.warp;
    const float s = x.lane < np && run ? A.sc[gq * 32 + x.lane] : -INFINITY;
    float mx = s;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float mo = A.ml[gq], mn = fmaxf(mo, mx);
    const float al = mn == -INFINITY ? 1.f : __expf(mo - mn);
    const float p = mn == -INFINITY ? 0.f : __expf(s - mn);
    float ps = p;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
    A.sc[gq * 32 + x.lane] = p;
    if (x.lane == 0) {
      A.ml[gq] = mn;
      A.ml[8 + gq] = A.ml[8 + gq] * al + ps;
      A.alpha[gq] = al;
    }
  }
  cbar();
  // P.V: warp w owns dims [w*D/NW, (w+1)*D/NW), D/256 per lane
  constexpr int DL = P / 8;
  const int d0 = x.warp * (D / NW) + x.lane * DL;
#pragma unroll
  for (int gq = 0; gq < 8; ++gq) {
    if (gq < GQ) {
      const float al = A.alpha[gq];
#pragma unroll
      for (int j = 0; j < DL; ++j) a.acc[gq][j] *= al;
    }
  }
  if (!run) return;
  for (int p = 0; p < np; ++p) {
    float vv[DL];
    if constexpr (DL == 1) {
      vv[0] = bf2f(vt[(int64_t)p * D + d0]);
    } else {
      const uint32_t w = *reinterpret_cast<const uint32_t*>(vt + (int64_t)p * D + d0);
      vv[0] = bf16lo(w);
      vv[1] = bf16hi(w);
    }
#pragma unroll
    for (int gq = 0; gq < 8; ++gq) {
      if (gq < GQ) {
        const float pr = A.sc[gq * 32 + p];
#pragma unroll
        for (int j = 0; j < DL; ++j) a.acc[gq][j] = fmaf(pr, vv[j], a.acc[gq][j]);
      }
    }
  }
}

// Publish the segment state of head hk; the last segment of the head merges
// all of them with the new position (in segment order).
template <int P>
__device__ void attn_segment_end(Ctx& x, const DLayer& L, int l, int hk, const Geo& gm, const AttnSm& A,
                                 AttnState& a) {
  const DModel& m = *x.m;
  const int D = 32 * P, GQ = L.Hq / L.Hkv, STR = 16 + 8 * D;
  constexpr int DL = P / 8;
  const int NA = gm.NA, c = blockIdx.x;
  const int cf = cta_of(hk * gm.NTt, gm.U, NA), cl = cta_of((hk + 1) * gm.NTt - 1, gm.U, NA);
  const int nk = cl - cf + 1;
  float* dst = m.apart + ((int64_t)hk * SEG_MAX + (c - cf)) * STR;
  const int d0 = x.warp * (D / NW) + x.lane * DL;
#pragma unroll
  for (int gq = 0; gq < 8; ++gq)
    if (gq < GQ)
#pragma unroll
      for (int j = 0; j < DL; ++j) dst[16 + gq * D + d0 + j] = a.acc[gq][j];
  if (threadIdx.x < 16) dst[threadIdx.x] = A.ml[threadIdx.x];
  __threadfence();
  // segments of this head = CTAs in [cf, cl] with a non-empty range
  int nseg = 0;
  for (int q = cf; q <= cl; ++q) nseg += slice0(gm.U, q, NA) < slice0(gm.U, q + 1, NA);
  int last = 0;
  cbar();
  if (threadIdx.x == 0) last = atomicAdd(m.ctr + l * CL + C_ASEG + hk, 1u) + 1 == (unsigned)nseg;
  last = x.bc(last);
  if (!last) return;
  __threadfence();
  // merge: warp gq computes the coefficients of its query head
  float* cn = A.coef + 8 * SEG_MAX;
  if (x.warp < GQ) {
    const int gq = x.warp;
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < P; ++i) s = fmaf(A.qs[(gq * P + i) * 32 + x.lane], A.kn[i * 32 + x.lane], s);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    s *= L.attn_scale;
    const bool live = x.lane < nk && slice0(gm.U, cf + x.lane, NA) < slice0(gm.U, cf + x.lane + 1, NA);
    const float* sp = m.apart + ((int64_t)hk * SEG_MAX + x.lane) * STR;
    const float mk = live ? __ldcg(sp + gq) : -INFINITY, lk = live ? __ldcg(sp + 8 + gq) : 0.f;
    float mx = fmaxf(s, mk);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float cf_ = mk == -INFINITY ? 0.f : __expf(mk - mx);
    float lsum = lk * cf_;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lsum += __shfl_xor_sync(0xffffffffu, lsum, o);
    if (x.lane < SEG_MAX) A.coef[gq * SEG_MAX + x.lane] = cf_;
    if (x.lane == 0) {
      const float en = __expf(s - mx);
      cn[gq] = en;
      cn[8 + gq] = 1.f / (lsum + en);
    }
  }
  cbar();
  for (int i = threadIdx.x; i < GQ * D; i += NT) {
    const int gq = i / D, d = i % D;
    float av[SEG_MAX];
#pragma unroll
    for (int k = 0; k < SEG_MAX; ++k)
      av[k] = k < nk ? __ldcg(m.apart + ((int64_t)hk * SEG_MAX + k) * STR + 16 + gq * D + d) : 0.f;
    float o = cn[gq] * A.vn[d];
#pragma unroll
    for (int k = 0; k < SEG_MAX; ++k) o = fmaf(A.coef[gq * SEG_MAX + k], av[k], o);
    m.att[((int64_t)hk * GQ + gq) * D + d] = __float2bfloat16_rn(o * cn[8 + gq]);
  }
  __threadfence();
  cbar();
  if (threadIdx.x == 0) atomicAdd(m.ctr + l * CL + C_ADONE, 1u);
}

template <int P>
__device__ bool op_attn(Ctx& x, const DLayer& L, int l) {
  const DModel& m = *x.m;
  const Geo gm = geo(m, L, OP_ATTN, x.pos, gridDim.x);
  const Geo gq = geo(m, L, OP_QKV, x.pos, gridDim.x);
  const int c = blockIdx.x, D = 32 * P;
  int u0, u1;
  seg_range(gm, 0, c, u0, u1);
  AttnSm A;
  A.qs = reinterpret_cast<float*>(x.smem + S_FRAG);
  A.sc = reinterpret_cast<float*>(x.smem + S_VEC);
  A.ml = A.sc + 256;
  A.alpha = A.ml + 16;
  A.coef = A.alpha + 8;
  A.kn = A.coef + 8 * SEG_MAX + 16;
  A.vn = A.kn + D;
  A.qn = reinterpret_cast<const bf16*>(x.smem + S_QKN);
  A.kw = A.qn + 512;
  const bool merge_only = gm.U == 0 && c < L.Hkv;
  if (u0 == u1 && !merge_only) return true;
  if (!cwait(x, m.ctr + l * CL + C_QKV, (unsigned)gq.U, 102)) return false;
  AttnState a;
  if (merge_only) {  // no cached position: the head's output is its new value row
    const int GQ = L.Hq / L.Hkv;
    head_rows<P>(x, L, c, A, true, gm.slot);
    cbar();
    for (int i = threadIdx.x; i < GQ * D; i += NT)
      m.att[((int64_t)c * GQ + i / D) * D + i % D] = __float2bfloat16_rn(A.vn[i % D]);
    __threadfence();
    cbar();
    if (threadIdx.x == 0) atomicAdd(m.ctr + l * CL + C_ADONE, 1u);
    return true;
  }
  int cur = -1;
  for (int u = u0; u < u1; ++u) {
    const int hk = u / gm.NTt, t = u % gm.NTt, p0 = t * gm.PT;
    if (hk != cur) {
      if (cur >= 0) attn_segment_end<P>(x, L, l, cur, gm, A, a);
      // the head's first CTA appends the new k / v
      attn_segment_start<P>(x, L, hk, A, t == 0, gm.slot, a);
      cur = hk;
    }
    bool ok;
    const uint8_t* base = unit_begin(x, unit_bytes(m, L, OP_ATTN, u, gm), false, ok);
    const int np = min(gm.PT, gm.nold - p0);
    attn_tile<P>(x, L, reinterpret_cast<const bf16*>(base), reinterpret_cast<const bf16*>(base + gm.PT * L.D * 2),
                 np, p0, gm.evict, A, a, ok);
    unit_end(x, false);
    cbar();  // every warp is done with the tile's probabilities before the next tile
  }
  attn_segment_end<P>(x, L, l, cur, gm, A, a);
  return true;
}

// ---------------------------------------------------------------------------
// compute-warp ops

__device__ bool op_qkv(Ctx& x, int l) {
  const DModel& m = *x.m;
  const DLayer& L = m.layers[l];
  const int H = m.H, G = H / 64;
  bool ok;
  const Geo gp = geo(m, L, OP_PRO, x.pos, gridDim.x);
  const uint8_t* pro = unit_begin(x, unit_bytes(m, L, OP_PRO, blockIdx.x, gp), false, ok);
  const bf16* pw = reinterpret_cast<const bf16*>(pro);
  FfOutW fw;
  float wn[PER];
  load_w(pw, H, wn);
  if (l > 0) {
    load_w(pw + H + 2 * L.D, H, fw.w1);
    load_w(pw + 2 * H + 2 * L.D, H, fw.w2);
    load_w(pw + 3 * H + 2 * L.D, H, fw.w);
  }
  for (int i = threadIdx.x; i < 2 * L.D; i += NT)  // q_norm | k_norm for the attention
    reinterpret_cast<bf16*>(x.smem + S_QKN)[i < L.D ? i : 512 + i - L.D] = pw[H + i];
  if (l > 0 && !cwait(x, m.ctr + (l - 1) * CL + C_DOWN, (unsigned)(H / 32), 104)) return false;
  float v[PER];
  layer_input(x, l, fw, pro + 2 * H + 4 * L.D, v);
  norm_to_vec(x, v, wn, L.eps, x.vec);
  cbar();
  unit_end(x, false);
  build_frags<8>(x, x.vec, H, 0);
  cbar();
  const Geo gm = geo(m, L, OP_QKV, x.pos, gridDim.x);
  int u0, u1;
  seg_range(gm, 0, blockIdx.x, u0, u1);
  const int RS = row_stride(H, 8);
  for (int u = u0; u < u1; ++u) {
    bool ok;
    const uint8_t* base = unit_begin(x, unit_bytes(m, L, OP_QKV, u, gm), true, ok);
    gemv_unit<8, 1>(x, base, RS, G, G, 0, ok);
    unit_end(x, true);
  }
  return true;
}

__device__ bool op_o(Ctx& x, int l) {
  const DModel& m = *x.m;
  const DLayer& L = m.layers[l];
  const int K = L.Hq * L.D, nkc = K / OKC;
  if (!cwait(x, m.ctr + l * CL + C_ADONE, (unsigned)L.Hkv, 105)) return false;
  for (int i = threadIdx.x * 8; i < K; i += NT * 8)
    *reinterpret_cast<uint4*>(x.vec + i) = __ldcg(reinterpret_cast<const uint4*>(m.att + i));
  cbar();
  build_frags<8>(x, x.vec, K, 0);
  cbar();
  const Geo gm = geo(m, L, OP_O, x.pos, gridDim.x);
  int u0, u1;
  seg_range(gm, 0, blockIdx.x, u0, u1);
  const int RS = row_stride(OKC, 8), gc = OKC / 64;
  for (int u = u0; u < u1; ++u) {
    bool ok;
    const uint8_t* base = unit_begin(x, unit_bytes(m, L, OP_O, u, gm), true, ok);
    gemv_unit<8, 1>(x, base, RS, gc, gc, (u % nkc) * gc, ok);
    unit_end(x, true);
  }
  return true;
}

__device__ bool op_gu(Ctx& x, int l) {
  const DModel& m = *x.m;
  const DLayer& L = m.layers[l];
  const int H = m.H, G = H / 64;
  float wpa[PER], wpf[PER], wpf2[PER], wrs[PER];
  {
    bool ok;
    const Geo gp = geo(m, L, OP_GUP, x.pos, gridDim.x);
    const bf16* pw = reinterpret_cast<const bf16*>(unit_begin(x, unit_bytes(m, L, OP_GUP, blockIdx.x, gp), false, ok));
    load_w(pw, H, wpa);
    load_w(pw + H, H, wpf);
    load_w(pw + 2 * H, H, wpf2);
    load_w(L.rscale ? pw + 3 * H : nullptr, H, wrs);
    __syncwarp();
    unit_end(x, false);  // the vectors are in registers
  }
  const Geo gmo = geo(m, L, OP_O, x.pos, gridDim.x);
  if (!cwait(x, m.ctr + l * CL + C_ODONE, (unsigned)gmo.U, 106)) return false;
  // ff_in: h = bf16(x + bf16(rms(bf16(o)) * w_post_attn)); h1 / h2 = bf16(rms(h) * w);
  // router input = bf16(bf16(bf16(rms(h2)) * bf16(root)) * router_scale)
  const int nkc = L.Hq * L.D / OKC;
  float o[PER], hv[PER], xr[PER];
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = threadIdx.x + k * NT;
    o[k] = 0.f;
    xr[k] = i < H ? ldcg_bf(m.x + i) : 0.f;
  }
  {
    float t[4][PER];  // <= 4 column chunks, all loads in flight together, added in chunk order
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
      for (int k = 0; k < PER; ++k) {
        const int i = threadIdx.x + k * NT;
        t[p][k] = p < nkc && i < H ? __ldcg(m.opart + (int64_t)p * H + i) : 0.f;
      }
#pragma unroll
    for (int p = 0; p < 4; ++p)
#pragma unroll
      for (int k = 0; k < PER; ++k) o[k] += t[p][k];
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    o[k] = round_bf(o[k]);
    ss = fmaf(o[k], o[k], ss);
  }
  const float r1 = rsqrtf(csum(ss, x.red8) / (float)H + L.eps);
  ss = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = threadIdx.x + k * NT;
    hv[k] = i < H ? round_bf(xr[k] + round_bf(o[k] * r1 * wpa[k])) : 0.f;
    ss = fmaf(hv[k], hv[k], ss);
  }
  const float r2 = rsqrtf(csum(ss, x.red8 + 8) / (float)H + L.eps);
  bf16* h1 = x.vec;
  bf16* h2 = x.vec + H_MAX;
  bf16* xs = x.vec + 2 * H_MAX;
  ss = 0.f;
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = threadIdx.x + k * NT;
    if (i < H) {
      if (blockIdx.x == 0) m.h[i] = __float2bfloat16_rn(hv[k]);
      h1[i] = __float2bfloat16_rn(hv[k] * r2 * wpf[k]);
      o[k] = round_bf(hv[k] * r2 * wpf2[k]);
      h2[i] = __float2bfloat16_rn(o[k]);
    } else {
      o[k] = 0.f;
    }
    ss = fmaf(o[k], o[k], ss);
  }
  const float r3 = rsqrtf(csum(ss, x.red8) / (float)H + L.eps);
  const float rb = round_bf(L.root);
#pragma unroll
  for (int k = 0; k < PER; ++k) {
    const int i = threadIdx.x + k * NT;
    if (i < H) {
      float v = round_bf(round_bf(o[k] * r3) * rb);
      if (L.rscale) v = round_bf(v * wrs[k]);
      xs[i] = __float2bfloat16_rn(v);
    }
  }
  cbar();
  build_frags<4>(x, h1, H, 0);
  build_frags<4>(x, h2, H, G);
  cbar();
  const Geo gm = geo(m, L, OP_GU, x.pos, gridDim.x);
  const int RSr = row_stride(H / RQ * 2, 16), RS4 = row_stride(H / 2, 4), cols = H / RQ;
  for (int s = 0; s < 3; ++s) {
    int u0, u1;
    seg_range(gm, s, blockIdx.x, u0, u1);
    for (int u = u0; u < u1; ++u) {
      bool ok;
      const uint8_t* base = unit_begin(x, unit_bytes(m, L, OP_GU, u, gm), true, ok);
      if (s == 0)
        router_unit(x, base, RSr, cols / 64, xs + (u % RQ) * cols, ok);
      else
        gemv_unit<4, 2>(x, base, RS4, G, G, s == 1 ? 0 : G, ok);
      unit_end(x, true);
    }
  }
  return true;
}

__device__ bool op_down(Ctx& x, int l) {
  const DModel& m = *x.m;
  const DLayer& L = m.layers[l];
  const int Gd = m.Id / 64, Ge = m.Ie / 64;
  const Geo gm = geo(m, L, OP_DOWN, x.pos, gridDim.x);
  int u0, u1;
  seg_range(gm, 0, blockIdx.x, u0, u1);
  if (u0 == u1) return true;
  // the tile's dense unit, as soon as the dense gate|up is complete
  if (!cwait(x, m.ctr + l * CL + C_GUD, (unsigned)(m.Id / 16), 107)) return false;
  for (int i = threadIdx.x * 8; i < m.Id; i += NT * 8)
    *reinterpret_cast<uint4*>(x.vec + i) = __ldcg(reinterpret_cast<const uint4*>(m.actd + i));
  cbar();
  build_frags<4>(x, x.vec, m.Id, 0);
  cbar();
  bool ok;
  const uint8_t* base = unit_begin(x, unit_bytes(m, L, OP_DOWN, u0, gm), true, ok);
  gemv_unit<4, 2>(x, base, m.Id / 2, Gd, Gd, 0, ok);
  unit_end(x, true);
  // its expert units
  if (!cwait(x, m.ctr + l * CL + C_GUE, (unsigned)(m.K * (m.Ie / 16)), 108)) return false;
  const int ne = m.K * m.Ie;
  for (int i = threadIdx.x * 8; i < ne; i += NT * 8)
    *reinterpret_cast<uint4*>(x.vec + m.Id + i) = __ldcg(reinterpret_cast<const uint4*>(m.acte + i));
  cbar();
  build_frags<4>(x, x.vec + m.Id, ne, Gd);
  cbar();
  for (int u = u0 + 1; u < u1; ++u) {
    base = unit_begin(x, unit_bytes(m, L, OP_DOWN, u, gm), true, ok);
    gemv_unit<4, 2>(x, base, m.Ie / 2, Ge, Ge, Gd + (u - u0 - 1) * Ge, ok);
    unit_end(x, true);
  }
  return true;
}

__device__ bool op_lm(Ctx& x) {
  const DModel& m = *x.m;
  const int H = m.H, G = H / 64;
  const DLayer& Lp = m.layers[m.L - 1];
  FfOutW fw;
  float wn[PER];
  {
    bool ok;
    const Geo gp = geo(m, Lp, OP_LMP, x.pos, gridDim.x);
    const bf16* pw = reinterpret_cast<const bf16*>(unit_begin(x, unit_bytes(m, Lp, OP_LMP, blockIdx.x, gp), false, ok));
    load_w(pw, H, fw.w1);
    load_w(pw + H, H, fw.w2);
    load_w(pw + 2 * H, H, fw.w);
    load_w(pw + 3 * H, H, wn);
    __syncwarp();
    unit_end(x, false);
  }
  if (!cwait(x, m.ctr + (m.L - 1) * CL + C_DOWN, (unsigned)(H / 32), 109)) return false;
  float v[PER];
  layer_input(x, m.L, fw, nullptr, v);
  norm_to_vec(x, v, wn, m.eps, x.vec);
  cbar();
  build_frags<6>(x, x.vec, H, 0);
  cbar();
  const Geo gm = geo(m, Lp, OP_LM, x.pos, gridDim.x);
  int u0, u1;
  seg_range(gm, 0, blockIdx.x, u0, u1);
  const int RS = row_stride(H * 6 / 8, 6);
  for (int u = u0; u < u1; ++u) {
    bool ok;
    const uint8_t* base = unit_begin(x, unit_bytes(m, Lp, OP_LM, u, gm), true, ok);
    gemv_unit<6, 1>(x, base, RS, G, G, 0, ok);
    unit_end(x, true);
  }
  return true;
}

// ---------------------------------------------------------------------------
// epilogue warp

struct Ep {
  const DModel* m;
  uint8_t* smem;
  uint64_t* rfull;
  uint64_t* rempty;
  const float* red;
  int r;      // partial-sum buffer sequence number
  int lane;
  bool ok;
};

// Wait for unit r's partial sums; v = the sum over the compute warps of row
// `row` (fixed order), then release the buffer.
__device__ __forceinline__ float ep_take(Ep& e, int row) {
  if (e.ok) e.ok = bar_wait(*e.m, &e.rfull[e.r % RR], (uint32_t)(e.r / RR) & 1u, 120);
  const float* rs = e.red + (e.r % RR) * NW * 32;
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) s += rs[w * 32 + row];
  return s;
}
__device__ __forceinline__ float ep_take2(Ep& e, int row, float& second) {
  const float a = ep_take(e, row);
  const float* rs = e.red + (e.r % RR) * NW * 32;
  float s = 0.f;
#pragma unroll
  for (int w = 0; w < NW; ++w) s += rs[w * 32 + 16 + row];
  second = s;
  return a;
}
__device__ __forceinline__ void ep_release(Ep& e) {
  __syncwarp();
  if (e.lane == 0) mbar_arrive(&e.rempty[e.r % RR]);
  ++e.r;
}

// Router top-k by one warp: logits (quarters added in order) -> rank count
// (descending, ties -> lower id) -> softmax over the k selected logits times
// per_expert_scale (the library's topk_block arithmetic).
__device__ void topk_warp(Ep& e, const DLayer& L, int l) {
  const DModel& m = *e.m;
  const int E = m.E, k = m.K, lane = e.lane;
  float* lg = reinterpret_cast<float*>(e.smem + S_LG);
  int* sel_e = reinterpret_cast<int*>(e.smem + S_SEL);
  float* sel_v = reinterpret_cast<float*>(e.smem + S_SEL + 64);
  {
    constexpr int PE = EMAX / 32;
    float part[PE][RQ];  // every quarter of every expert in flight together
#pragma unroll
    for (int q = 0; q < PE; ++q)
#pragma unroll
      for (int c = 0; c < RQ; ++c) part[q][c] = lane + 32 * q < E ? __ldcg(m.rlog + c * E + lane + 32 * q) : 0.f;
#pragma unroll
    for (int q = 0; q < PE; ++q) {
      const int ex = lane + 32 * q;
      if (ex < E) {
        float s = 0.f;
#pragma unroll
        for (int c = 0; c < RQ; ++c) s += part[q][c];
        if (L.logit_bias) s += L.logit_bias[ex];
        lg[ex] = round_bf(s);  // ranked in the router's bf16 output precision
      }
    }
  }
  if (lane < KMAX) {
    sel_e[lane] = lane;  // valid ids even if every logit is NaN
    sel_v[lane] = 0.f;
  }
  __syncwarp();
  constexpr int PE = EMAX / 32;
  float mine[PE];
  int rank[PE];
#pragma unroll
  for (int q = 0; q < PE; ++q) {
    mine[q] = lane + 32 * q < E ? lg[lane + 32 * q] : INFINITY;
    rank[q] = 0;
  }
  for (int j = 0; j < E; ++j) {
    const float u = lg[j];
#pragma unroll
    for (int q = 0; q < PE; ++q) rank[q] += (u > mine[q] || (u == mine[q] && j < lane + 32 * q)) ? 1 : 0;
  }
#pragma unroll
  for (int q = 0; q < PE; ++q)
    if (lane + 32 * q < E && rank[q] < k) {
      sel_e[rank[q]] = lane + 32 * q;
      sel_v[rank[q]] = mine[q];
    }
  __syncwarp();
  if (lane < k) {
    const float mx = sel_v[0];
    float den = 0.f;
    for (int j = 0; j < k; ++j) den += expf(sel_v[j] - mx);
    float wv = expf(sel_v[lane] - mx) / den;
    const int ex = sel_e[lane];
    if (L.pes) wv *= bf2f(L.pes[ex]);
    m.ids[lane] = ex;
    m.wts[lane] = wv;
  }
  __threadfence();
  __syncwarp();
  if (lane == 0) atomicExch(m.ctr + l * CL + C_ROUTE, 1u);
}

// Release-increment by lane 0 after every lane's stores (fence by all).
__device__ __forceinline__ unsigned ep_signal(const Ep& e, unsigned* c, unsigned n) {
  __threadfence();
  __syncwarp();
  unsigned prev = 0;
  if (e.lane == 0) prev = atomicAdd(c, n);
  return __shfl_sync(0xffffffffu, prev, 0);
}

__device__ void epilogue(const DModel& m, uint8_t* smem, int64_t pos) {
  Ep e;
  e.m = &m;
  e.smem = smem;
  e.rfull = reinterpret_cast<uint64_t*>(smem + S_BAR) + 2 * SLOTS;
  e.rempty = e.rfull + RR;
  e.red = reinterpret_cast<const float*>(smem + S_RED);
  e.r = 0;
  e.lane = threadIdx.x & 31;
  e.ok = true;
  const int c = blockIdx.x, G = gridDim.x, H = m.H, lane = e.lane;
  for (int l = 0; l < m.L && e.ok; ++l) {
    const DLayer& L = m.layers[l];
    unsigned* ctr = m.ctr + l * CL;
    int u0, u1;
    // QKV rows
    {
      const Geo gm = geo(m, L, OP_QKV, pos, G);
      seg_range(gm, 0, c, u0, u1);
      for (int u = u0; u < u1; ++u) {
        const float v = ep_take(e, lane & 15);
        if (!e.ok) return;
        ep_release(e);
        if (lane < 16) m.qkv[u * 16 + lane] = v;
      }
      if (u1 > u0) ep_signal(e, ctr + C_QKV, (unsigned)(u1 - u0));
    }
    // O: partial sums per column chunk
    {
      const Geo gm = geo(m, L, OP_O, pos, G);
      const int nkc = L.Hq * L.D / OKC;
      seg_range(gm, 0, c, u0, u1);
      for (int u = u0; u < u1; ++u) {
        const float v = ep_take(e, lane & 15);
        if (!e.ok) return;
        ep_release(e);
        if (lane < 16) m.opart[(int64_t)(u % nkc) * H + (u / nkc) * 16 + lane] = v;
      }
      if (u1 > u0) ep_signal(e, ctr + C_ODONE, (unsigned)(u1 - u0));
    }
    // GU: router partials (+ top-k), dense / expert gate|up with GELU gating
    {
      const Geo gm = geo(m, L, OP_GU, pos, G);
      const int ne = m.Ie / 16, nrt = gm.sb[1];
      for (int s = 0; s < 3; ++s) {
        seg_range(gm, s, c, u0, u1);
        for (int u = u0; u < u1; ++u) {
          if (s == 0) {
            const float v = ep_take(e, lane & 15);
            if (!e.ok) return;
            ep_release(e);
            if (lane < 16) m.rlog[(u % RQ) * m.E + (u / RQ) * 16 + lane] = v;
            if (ep_signal(e, ctr + C_RTR, 1u) + 1 == (unsigned)nrt) {
              __threadfence();
              topk_warp(e, L, l);
            }
          } else {
            float uv;
            const float gv = round_bf(ep_take2(e, lane & 15, uv));
            if (!e.ok) return;
            ep_release(e);
            const bf16 act = __float2bfloat16_rn(gelu_tanh(gv) * round_bf(uv));
            if (lane < 16) {
              if (s == 1)
                m.actd[(u - gm.sb[1]) * 16 + lane] = act;
              else
                m.acte[(int64_t)((u - gm.sb[2]) / ne) * m.Ie + ((u - gm.sb[2]) % ne) * 16 + lane] = act;
            }
          }
        }
        if (s > 0 && u1 > u0) ep_signal(e, ctr + (s == 1 ? C_GUD : C_GUE), (unsigned)(u1 - u0));
      }
    }
    // DOWN: this CTA's 32-row tile: dense rows and the weighted expert combine
    {
      const Geo gm = geo(m, L, OP_DOWN, pos, G);
      seg_range(gm, 0, c, u0, u1);
      float yd = 0.f, ym = 0.f, wk[KMAX];
#pragma unroll
      for (int j = 0; j < KMAX; ++j) wk[j] = 0.f;
      for (int u = u0; u < u1; ++u) {
        const float v = ep_take(e, lane);
        if (!e.ok) return;
        ep_release(e);
        if (u == u0) {
          yd = v;
#pragma unroll
          for (int j = 0; j < KMAX; ++j) wk[j] = j < m.K ? __ldcg(m.wts + j) : 0.f;  // routed by now
        } else {
          float w = 0.f;
#pragma unroll
          for (int j = 0; j < KMAX; ++j) w = j == u - u0 - 1 ? wk[j] : w;
          ym = fmaf(w, v, ym);  // slots in rank order
        }
      }
      if (u1 > u0) {
        const int r = u0 / (1 + m.K);
        m.yd[r * 32 + lane] = yd;
        m.ym[r * 32 + lane] = ym;
        ep_signal(e, ctr + C_DOWN, 1u);
      }
    }
  }
  // LM: softcap, logits, running argmax (ids ascend per lane: first maximum kept)
  float best = -INFINITY;
  int besti = 0x7fffffff;
  if (e.ok) {
    const Geo gm = geo(m, m.layers[m.L - 1], OP_LM, pos, G);
    int u0, u1;
    seg_range(gm, 0, c, u0, u1);
    for (int u = u0; u < u1; ++u) {
      float lv = round_bf(ep_take(e, lane & 15));
      if (!e.ok) return;
      ep_release(e);
      if (m.softcap > 0.f) lv = round_bf(round_bf(tanhf(round_bf(lv / m.softcap))) * m.softcap);
      if (lane < 16) {
        const int id = u * 16 + lane;
        m.logits[id] = lv;
        if (lv > best) {
          best = lv;
          besti = id;
        }
      }
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
  if (lane == 0 && e.ok && besti != 0x7fffffff && best == best) {
    // order-preserving key: larger value first, then the lower id
    const uint32_t b = __float_as_uint(best);
    const uint32_t key = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    atomicMax(m.best, ((unsigned long long)key << 32) | (0xffffffffu - (uint32_t)besti));
  }
  // the last CTA to finish publishes the token and advances the position
  const unsigned done = ep_signal(e, m.ctr + m.L * CL, 1u) + 1;
  if (lane == 0 && done == (unsigned)G && e.ok && !aborted(m)) {
    __threadfence();
    const unsigned long long k = atomicAdd(m.best, 0ull);
    m.tok[0] = k ? (int)(0xffffffffu - (uint32_t)(k & 0xffffffffu)) : 0;
    m.pos[0] += 1;
    m.pos[1] += 1;
  }
}

__global__ void __launch_bounds__(THREADS, 1) decode_step_kernel(const __grid_constant__ DModel m) {
  extern __shared__ __align__(128) uint8_t smem[];
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + S_BAR);
  uint64_t* empty = full + SLOTS;
  uint64_t* rfull = empty + SLOTS;
  uint64_t* rempty = rfull + RR;
  int* misc = reinterpret_cast<int*>(smem + S_MISC);
  if (threadIdx.x == 0) {
    for (int s = 0; s < SLOTS; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    for (int s = 0; s < RR; ++s) {
      mbar_init(&rfull[s], NW);
      mbar_init(&rempty[s], 1);
    }
    mbar_fence_init();
  }
  if (threadIdx.x < 16) misc[threadIdx.x] = 0;
  __syncthreads();
  const int64_t pos = m.pos[0];
  const int warp = threadIdx.x >> 5;
  if (warp == PW) {
    if ((threadIdx.x & 31) == 0) producer(m, smem, pos);
    return;
  }
  if (warp == EW) {
    epilogue(m, smem, pos);
    return;
  }
  Ctx x;
  x.m = &m;
  x.smem = smem;
  x.full = full;
  x.empty = empty;
  x.rfull = rfull;
  x.rempty = rempty;
  x.red8 = reinterpret_cast<float*>(smem + S_RED8);
  x.red = reinterpret_cast<float*>(smem + S_RED);
  x.xsum = reinterpret_cast<float*>(smem + S_XSUM);
  x.frag = reinterpret_cast<uint4*>(smem + S_FRAG);
  x.vec = reinterpret_cast<bf16*>(smem + S_VEC);
  x.head = 0;
  x.seq = 0;
  x.rseq = 0;
  x.bc = Bc{misc, 0};
  x.warp = warp;
  x.lane = threadIdx.x & 31;
  x.pos = pos;
  bool ok = true;
  for (int l = 0; l < m.L && ok; ++l) {
    const DLayer& L = m.layers[l];
    ok = op_qkv(x, l);
    if (ok) ok = L.D == 256 ? op_attn<8>(x, L, l) : op_attn<16>(x, L, l);
    if (ok) ok = op_o(x, l);
    if (ok) ok = op_gu(x, l);
    if (ok) ok = op_down(x, l);
  }
  if (ok) op_lm(x);
}

}  // namespace step

// ---------------------------------------------------------------------------
// host side

using step::DLayer;
using step::DQ;
using step::DModel;

namespace {

struct StepWs {
  size_t table, ctr, best, qkv, apart, att, opart, x, h, rlog, ids, wts, actd, acte, yd, ym, bytes;
};

int check_q(const fmoe_qweight_t& w, int out, int in, int bits, const char* what) {
  if (!w.w || !w.scales || !w.biases || w.out_features != out || w.in_features != in || w.bits != bits ||
      w.group_size != 64)
    return set_error(FMOE_ERR_INVALID, "decode_step: %s must be [%d, %d] %d-bit, group 64", what, out, in, bits);
  if (!aligned(w.w, 16) || !aligned(w.scales, 16) || !aligned(w.biases, 16))
    return set_error(FMOE_ERR_INVALID, "decode_step: %s arrays must be 16-byte aligned", what);
  return FMOE_OK;
}

int check_model(const fmoe_decode_model_t* md) {
  if (!md || md->n_layers < 1 || !md->layers || !md->caches)
    return set_error(FMOE_ERR_INVALID, "decode_step: model, layers and caches are required");
  const fmoe_decoder_layer_t& l0 = md->layers[0];
  const int H = l0.experts.hidden, Id = l0.mlp_gate.out_features, E = l0.router.proj.out_features;
  const int Ie = l0.experts.intermediate, K = l0.router.top_k;
  if (H % (64 * step::RQ) || H > step::H_MAX)
    return set_error(FMOE_ERR_UNSUPPORTED, "decode_step: hidden %d (multiple of %d, <= %d)", H, 64 * step::RQ,
                     step::H_MAX);
  if (Id % 64 || (Id / 2) % 128 != 32 && (Id / 2) % 128 != 96)
    return set_error(FMOE_ERR_UNSUPPORTED, "decode_step: dense intermediate %d has no conflict-free row layout", Id);
  if (Ie % 64 || (Ie / 2) % 128 != 32 && (Ie / 2) % 128 != 96)
    return set_error(FMOE_ERR_UNSUPPORTED, "decode_step: expert intermediate %d has no conflict-free row layout", Ie);
  if (K < 1 || K > step::KMAX || E < K || E > step::EMAX || E % 16)
    return set_error(FMOE_ERR_UNSUPPORTED, "decode_step: %d experts, top-%d", E, K);
  if (Id + K * Ie > 3 * step::H_MAX || (Id + K * Ie) / 64 > step::GMAX || 2 * H / 64 > step::GMAX)
    return set_error(FMOE_ERR_UNSUPPORTED, "decode_step: MLP inputs exceed the fragment buffer");
  if (check_q(md->embed, md->embed.out_features, H, 6, "embed") || md->embed.out_features % 16 || !md->final_norm ||
      !aligned(md->final_norm, 16))
    return set_error(FMOE_ERR_INVALID, "decode_step: embed must be 6-bit [vocab %% 16 == 0, hidden]; final_norm set");
  for (int i = 0; i < md->n_layers; ++i) {
    const fmoe_decoder_layer_t& L = md->layers[i];
    const fmoe_kv_cache_t& c = md->caches[i];
    const int Hq = L.num_heads, Hkv = L.num_kv_heads, D = L.head_dim;
    if (L.sparse_v_tau != 0.f)
      return set_error(FMOE_ERR_UNSUPPORTED, "decode_step: layer %d: sparse-V gating on the layered path only", i);
    if ((D != 256 && D != 512) || Hkv < 1 || Hq % Hkv || Hq / Hkv > 8 || Hq + 2 * Hkv > 48 || Hkv > 16 ||
        (Hq * D) % step::OKC || Hq * D > 8192 || L.rope_dims < 2 || L.rope_dims > D || L.rope_dims % (2 * (D / 32)))
      return set_error(FMOE_ERR_UNSUPPORTED, "decode_step: layer %d attention shape (heads %d/%d, dim %d)", i, Hq, Hkv,
                       D);
    int rc;
    if ((rc = check_q(L.q_proj, Hq * D, H, 8, "q_proj")) || (rc = check_q(L.k_proj, Hkv * D, H, 8, "k_proj")) ||
        (!L.k_eq_v && (rc = check_q(L.v_proj, Hkv * D, H, 8, "v_proj"))) ||
        (rc = check_q(L.o_proj, H, Hq * D, 8, "o_proj")) || (rc = check_q(L.mlp_gate, Id, H, 4, "mlp_gate")) ||
        (rc = check_q(L.mlp_up, Id, H, 4, "mlp_up")) || (rc = check_q(L.mlp_down, H, Id, 4, "mlp_down")))
      return rc;
    const fmoe_router_t& r = L.router;
    if (r.proj.bits != 16 || r.proj.out_features != E || r.proj.in_features != H || !r.proj.w ||
        !aligned(r.proj.w, 16) || r.top_k != K || !r.use_norm)
      return set_error(FMOE_ERR_UNSUPPORTED, "decode_step: layer %d router must be bf16 [%d, %d], top-%d, use_norm", i,
                       E, H, K);
    const fmoe_experts_t& e = L.experts;
    if (e.bits != 4 || e.group_size != 64 || e.hidden != H || e.intermediate != Ie || e.num_experts != E ||
        e.first_expert != 0 || !e.base || !aligned(e.base, 16) || e.expert_stride % 16 || e.slot_of)
      return set_error(FMOE_ERR_UNSUPPORTED, "decode_step: layer %d experts must be all %d, 4-bit, [%d, %d]", i, E, Ie,
                       H);
    for (int j = 0; j < 9; ++j)
      if (e.offsets[j] % 16) return set_error(FMOE_ERR_INVALID, "decode_step: expert offsets must be 16-byte aligned");
    const void* norms[10] = {L.q_norm, L.k_norm, L.input_norm, L.post_attn_norm, L.pre_ff_norm, L.post_ff_norm_1,
                             L.pre_ff_norm_2, L.post_ff_norm_2, L.post_ff_norm, L.router.router_scale};
    for (int j = 0; j < 10; ++j)
      if ((j < 9 && !norms[j]) || (norms[j] && !aligned(norms[j], 16)))
        return set_error(FMOE_ERR_INVALID, "decode_step: layer %d norms are required, 16-byte aligned", i);
    if (c.mode != FMOE_KV_BF16 || c.turbo_bits != 0 || c.batch != 1 || c.kv_heads != Hkv || c.head_dim != D || c.capacity < 16 ||
        c.capacity % 16 || !c.k || !c.v || !aligned(c.k, 16) || !aligned(c.v, 16))
      return set_error(FMOE_ERR_UNSUPPORTED, "decode_step: layer %d cache must be bf16 (no TurboQuant), batch 1, %d heads x %d", i, Hkv,
                       D);
    if (L.experts.hidden != H || L.mlp_gate.out_features != Id || L.router.proj.out_features != E ||
        L.experts.intermediate != Ie)
      return set_error(FMOE_ERR_UNSUPPORTED, "decode_step: layers must share hidden / MLP / expert shapes");
  }
  return FMOE_OK;
}

StepWs ws_layout(const fmoe_decode_model_t* md) {
  const fmoe_decoder_layer_t& l0 = md->layers[0];
  const int H = l0.experts.hidden, Id = l0.mlp_gate.out_features, E = l0.router.proj.out_features;
  const int Ie = l0.experts.intermediate, K = l0.router.top_k;
  int rows = 0, qd = 0, apart = 0, nkc = 0;
  for (int i = 0; i < md->n_layers; ++i) {
    const fmoe_decoder_layer_t& L = md->layers[i];
    rows = std::max(rows, (L.num_heads + L.num_kv_heads * (L.k_eq_v ? 1 : 2)) * L.head_dim);
    qd = std::max(qd, L.num_heads * L.head_dim);
    apart = std::max(apart, L.num_kv_heads * step::SEG_MAX * (16 + 8 * L.head_dim));
    nkc = std::max(nkc, L.num_heads * L.head_dim / step::OKC);
  }
  Carver c(nullptr);
  StepWs w;
  c.take<uint8_t>(256);  // status word
  w.table = c.off, c.take<DLayer>(md->n_layers);
  w.ctr = c.off, c.take<unsigned>((size_t)(md->n_layers + 1) * step::CL);
  w.best = c.off, c.take<unsigned long long>(1);
  w.qkv = c.off, c.take<float>(rows);
  w.apart = c.off, c.take<float>(apart);
  w.att = c.off, c.take<bf16>(qd);
  w.opart = c.off, c.take<float>((size_t)nkc * H);
  w.x = c.off, c.take<bf16>(H);
  w.h = c.off, c.take<bf16>(H);
  w.rlog = c.off, c.take<float>((size_t)step::RQ * E);
  w.ids = c.off, c.take<int32_t>(K);
  w.wts = c.off, c.take<float>(K);
  w.actd = c.off, c.take<bf16>(Id);
  w.acte = c.off, c.take<bf16>((size_t)K * Ie);
  w.yd = c.off, c.take<float>(H);
  w.ym = c.off, c.take<float>(H);
  w.bytes = align_up(c.off, 256);
  return w;
}

DQ to_dq(const fmoe_qweight_t& w) {
  return DQ{static_cast<const uint8_t*>(w.w), static_cast<const bf16*>(w.scales), static_cast<const bf16*>(w.biases)};
}

DModel make_model(const fmoe_decode_model_t* md, uint8_t* ws, const StepWs& w) {
  const fmoe_decoder_layer_t& l0 = md->layers[0];
  DModel m{};
  m.layers = reinterpret_cast<const DLayer*>(ws + w.table);
  m.L = md->n_layers;
  m.H = l0.experts.hidden;
  m.Id = l0.mlp_gate.out_features;
  m.E = l0.router.proj.out_features;
  m.Ie = l0.experts.intermediate;
  m.K = l0.router.top_k;
  m.V = md->embed.out_features;
  m.embed = to_dq(md->embed);
  m.final_norm = static_cast<const bf16*>(md->final_norm);
  m.eps = md->eps;
  m.softcap = md->softcap;
  m.emb_scale = md->embed_scale;
  m.status = reinterpret_cast<int*>(ws);
  m.ctr = reinterpret_cast<unsigned*>(ws + w.ctr);
  m.abort_flag = reinterpret_cast<int*>(m.ctr + m.L * step::CL + 1);  // cleared with the counters
  m.best = reinterpret_cast<unsigned long long*>(ws + w.best);
  m.qkv = reinterpret_cast<float*>(ws + w.qkv);
  m.apart = reinterpret_cast<float*>(ws + w.apart);
  m.att = reinterpret_cast<bf16*>(ws + w.att);
  m.opart = reinterpret_cast<float*>(ws + w.opart);
  m.x = reinterpret_cast<bf16*>(ws + w.x);
  m.h = reinterpret_cast<bf16*>(ws + w.h);
  m.rlog = reinterpret_cast<float*>(ws + w.rlog);
  m.ids = reinterpret_cast<int32_t*>(ws + w.ids);
  m.wts = reinterpret_cast<float*>(ws + w.wts);
  m.actd = reinterpret_cast<bf16*>(ws + w.actd);
  m.acte = reinterpret_cast<bf16*>(ws + w.acte);
  m.yd = reinterpret_cast<float*>(ws + w.yd);
  m.ym = reinterpret_cast<float*>(ws + w.ym);
  return m;
}

}  // namespace

}  // namespace fmoe

using namespace fmoe;

extern "C" size_t fmoe_decode_step_workspace_bytes(const fmoe_decode_model_t* model) {
  if (check_model(model)) return 0;
  return ws_layout(model).bytes;
}

extern "C" int fmoe_decode_step_prepare(const fmoe_decode_model_t* md, void* workspace, size_t bytes) {
  int rc;
  if ((rc = check_model(md))) return rc;
  const StepWs w = ws_layout(md);
  if (!workspace || bytes < w.bytes || !aligned(workspace, 256))
    return set_error(FMOE_ERR_INVALID, "decode_step: workspace of %zu bytes (256-aligned) required", w.bytes);
  std::vector<DLayer> t(md->n_layers);
  for (int i = 0; i < md->n_layers; ++i) {
    const fmoe_decoder_layer_t& L = md->layers[i];
    const fmoe_kv_cache_t& c = md->caches[i];
    DLayer& d = t[i];
    d = DLayer{};
    d.q = to_dq(L.q_proj), d.k = to_dq(L.k_proj), d.v = L.k_eq_v ? d.k : to_dq(L.v_proj), d.o = to_dq(L.o_proj);
    d.gate = to_dq(L.mlp_gate), d.up = to_dq(L.mlp_up), d.down = to_dq(L.mlp_down);
    d.router = static_cast<const bf16*>(L.router.proj.w);
    d.logit_bias = L.router.logit_bias;
    d.q_norm = static_cast<const bf16*>(L.q_norm), d.k_norm = static_cast<const bf16*>(L.k_norm);
    d.in_norm = static_cast<const bf16*>(L.input_norm), d.post_attn = static_cast<const bf16*>(L.post_attn_norm);
    d.pre_ff = static_cast<const bf16*>(L.pre_ff_norm), d.post_ff1 = static_cast<const bf16*>(L.post_ff_norm_1);
    d.pre_ff2 = static_cast<const bf16*>(L.pre_ff_norm_2), d.post_ff2 = static_cast<const bf16*>(L.post_ff_norm_2);
    d.post_ff = static_cast<const bf16*>(L.post_ff_norm);
    d.rscale = static_cast<const bf16*>(L.router.router_scale);
    d.pes = static_cast<const bf16*>(L.router.per_expert_scale);
    d.ex = static_cast<const uint8_t*>(L.experts.base);
    d.ex_stride = L.experts.expert_stride;
    for (int j = 0; j < 9; ++j) d.ex_off[j] = L.experts.offsets[j];
    d.kc = static_cast<bf16*>(c.k), d.vc = static_cast<bf16*>(c.v), d.cap = c.capacity;
    d.Hq = L.num_heads, d.Hkv = L.num_kv_heads, d.D = L.head_dim, d.rope_dims = L.rope_dims, d.k_eq_v = L.k_eq_v;
    d.log2_theta = std::log2(L.rope_theta), d.eps = L.eps, d.scalar = L.layer_scalar, d.attn_scale = L.attn_scale;
    d.root = L.router.root_size;
  }
  if (cudaMemcpy(static_cast<uint8_t*>(workspace) + w.table, t.data(), t.size() * sizeof(DLayer),
                 cudaMemcpyHostToDevice) != cudaSuccess ||
      cudaMemset(workspace, 0, 256) != cudaSuccess)
    return set_error(FMOE_ERR_CUDA, "decode_step: %s", cudaGetErrorString(cudaGetLastError()));
  return FMOE_OK;
}

extern "C" int fmoe_decode_step(const fmoe_decode_model_t* md, int32_t* tokens, float* logits, int64_t* pos_dev,
                                void* workspace, size_t bytes, void* stream) {
  int rc;
  if ((rc = check_model(md))) return rc;
  const StepWs w = ws_layout(md);
  if (!workspace || bytes < w.bytes || !aligned(workspace, 256) || !tokens || !logits || !pos_dev)
    return set_error(FMOE_ERR_INVALID, "decode_step: tokens, logits, pos_dev and a prepared workspace are required");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  DModel m = make_model(md, ws, w);
  m.logits = logits;
  m.tok = tokens;
  m.pos = pos_dev;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaFuncSetAttribute(step::decode_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, step::SMEM);
  });
  // counters and the argmax key start at zero every step
  if (cudaMemsetAsync(ws + w.ctr, 0, w.qkv - w.ctr, st) != cudaSuccess)
    return set_error(FMOE_ERR_CUDA, "decode_step: memset: %s", cudaGetErrorString(cudaGetLastError()));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(kNumSMs);
  cfg.blockDim = dim3(step::THREADS);
  cfg.dynamicSmemBytes = step::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident: CTAs wait on each other's counters
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  {
    ProfScope prof_("decode_step_kernel", st);
    cudaLaunchKernelEx(&cfg, step::decode_step_kernel, m);
  }
  return check_launch("decode_step_kernel");
}
