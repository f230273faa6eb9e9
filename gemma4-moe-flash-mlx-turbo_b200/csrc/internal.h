// Internal declarations shared by the libfmoe translation units.
#pragma once
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <stddef.h>
#include "fmoe.h"

namespace fmoe {

typedef __nv_bfloat16 bf16;

// B200: 148 SMs.  Grids are sized from this (the ABI checks the device).
constexpr int kNumSMs = 148;

// Error reporting: records a per-thread message and returns `code`.
int set_error(int code, const char* fmt, ...);
int check_launch(const char* what);

// RAII timing scope around one kernel launch (active only while
// fmoe_profile_enable(1); see prof.cu).  Name = the kernel's symbol name.
class ProfScope {
 public:
  ProfScope(const char* name, cudaStream_t st);
  ~ProfScope();

 private:
  const char* name_;
  cudaStream_t st_;
  cudaEvent_t a_, b_;
};

// Device view of a linear weight.
struct QW {
  const void* w;
  const bf16* s;
  const bf16* b;
  int out, in, bits;
  const uint8_t* tiled;  // decode-GEMV tile layout of w, or null
  int tiled_kc;
};

// Device view of an ECB expert table.
struct ExpertsDev {
  const uint8_t* base;
  int64_t stride;
  int64_t off[9];
  int E, first, H, I;
  const int32_t* slot_of;  // null, or the slot of each local expert in base
};
// Start of local expert e's tensors.
__device__ __forceinline__ const uint8_t* expert_base(const ExpertsDev& ex, int e) {
  return ex.base + (int64_t)(ex.slot_of ? __ldg(ex.slot_of + e) : e) * ex.stride;
}

// Routing metadata built on the device from ids [T, k] (see moe.cu).
struct RouteMeta {
  int32_t* start;       // [E + 1] exclusive prefix of per-expert pair counts
  int32_t* pairs;       // [T * k] pair index (t*k + slot), grouped by expert, ascending
  int32_t* unique;      // [E] local ids of experts with >= 1 pair, ascending
  int32_t* num_unique;  // [1]
  int4* work;           // [work_len] per expert slot u: (expert, first pair, pair count, 0); count 0 past the end
  int work_len;         // min(T * k, E): the expert kernels' grid extent
  int32_t* scratch;     // [route_scratch_ints(P, E)] or null: lets many pairs be listed by many CTAs
};
// Scratch ints that let launch_route_build spread P pairs over many CTAs.
int64_t route_scratch_ints(int64_t P, int E);

// gemv.cu
int gemv_ksplit(int64_t T, int out, int in);
int launch_gemv_partial(const bf16* x, int64_t T, const QW& w, int ksplit, float* partial, cudaStream_t st);
int launch_reduce_partials(const float* partial, int ksplit, int64_t n, bf16* out_bf16, float* out_f32,
                           cudaStream_t st);
int launch_router_prenorm(const bf16* x, int64_t T, int H, float root, float eps, const bf16* rscale, bf16* xs,
                          cudaStream_t st);
int launch_router_fused(const bf16* x, int64_t T, const QW& w, const float* bias, const bf16* pes, int k,
                        int32_t* ids, float* wts, float* logits_out, unsigned* counters, const RouteMeta* meta,
                        int* status, bool pdl, cudaStream_t st);

// router_tc.cu: the tensor-core router for many tokens (bf16 router weight).
constexpr int64_t kRouterTcMinTokens = 64;
bool router_tc_eligible(int64_t T, const QW& w, int k);
int launch_router_tc(const bf16* x, int64_t T, const QW& w, const float* bias, const bf16* pes, int k, int32_t* ids,
                     float* wts, float* logits, int* status, cudaStream_t st);

// moe.cu
int launch_route_build(const int32_t* ids, int64_t P, const ExpertsDev& ex, const RouteMeta& m, cudaStream_t st);
int down_groups(int64_t T, int k, int E);
int launch_moe_gate_up(const bf16* x, int64_t T, int k, const ExpertsDev& ex, const RouteMeta& m, bf16* act,
                       int* status, bool pdl, cudaStream_t st);
// y32 != nullptr: the combined rows go there in fp32 instead of bf16 to y.
int launch_moe_down(const bf16* act, int64_t T, int k, const float* wts, const ExpertsDev& ex, const RouteMeta& m,
                    float* part, unsigned* tile_ctr, bf16* y, int* status, bool pdl, cudaStream_t st,
                    float* y32 = nullptr);

// quant.cu
int launch_quantize(const void* src, int src_is_bf16, int64_t rows, int64_t cols, int bits, int group, uint32_t* wq,
                    bf16* s, bf16* b, cudaStream_t st);
int launch_dequantize(const QW& w, int group, const int32_t* ids, int64_t n, float row_scale, bf16* out,
                      cudaStream_t st);

// kv.cu: device view of one layer's KV cache (see fmoe_kv_cache_t).
struct KvDev {
  int mode, B, Hkv, D;
  int turbo;  // bf16 mode: TurboQuant bits applied by the decoder's append (0: none)
  int64_t cap;
  void* k;  // bf16 rows (FMOE_KV_BF16) or packed 4-bit codes (FMOE_KV_AFFINE)
  void* v;  // bf16 rows or packed 8-bit codes
  bf16* ks;
  bf16* kb;
  bf16* vs;
  bf16* vb;
};
// Split-KV plan of one decode-attention launch: S slots per split.
struct AttnPlan {
  int S, nsplit;
};

// qgemv.cu: streaming quantised GEMV (decode, T <= 8) over up to 4 weight
// matrices sharing one input.
constexpr int kQgMaxSeg = 4;
enum { QG_IN_BF16 = 0, QG_IN_RMSNORM = 1, QG_IN_GELU = 2 };
// QG_OUT_F32_PART: column chunk c of the input stores its partial sums in
// slice c of the output ([nkc][T][ld] f32, slice stride T * ld); the consumer
// adds the slices in order (deterministic split-K).
enum { QG_OUT_F32 = 0, QG_OUT_F32_ADD = 1, QG_OUT_BF16 = 2, QG_OUT_F32_PART = 3 };
struct QgSeg {
  const uint8_t* w;  // packed codes [rows][K*bits/32 words]
  const bf16* s;     // [rows][K/64]
  const bf16* b;
  void* out;         // [T][ld]: f32 or bf16 by QgArgs::out_kind
  int rows, ld, col0;
  int unit0;         // set by qgemv_plan
  const uint8_t* tiled = nullptr;  // tile layout of w (fmoe_qweight_tile), or null
  int tiled_kc = 0;
};
struct QgArgs {
  QgSeg seg[kQgMaxSeg];
  int nseg, K, T;
  int kc, nkc, units;  // set by qgemv_plan
  int out_kind;
  int in_kind;
  const bf16* x;       // [T][ldx] (QG_IN_BF16 / QG_IN_RMSNORM)
  int ldx;
  const bf16* norm_w;  // [K] (QG_IN_RMSNORM)
  float eps;
  const float* g;      // [T][ldgu] fp32 gate / up projections (QG_IN_GELU)
  const float* u;
  int ldgu;
  int gu_parts;        // QG_IN_GELU: partial slices of g / u to add (>= 1)
  int64_t gu_part_stride;
  float* zero_ptr[4];  // fp32 buffers cleared after griddepcontrol.wait (for later accumulating kernels)
  int64_t zero_n[4];
  int* status;
};
struct QgLayout {
  int rs, soff, stage, sfull, nst, frag, xsum, red, misc, cnt, bar, bytes, grid, nw, rt;
};
int qgemv_plan(QgArgs& a, int bits, bool allow_split, QgLayout* L, bool half_sm = false);
// Column chunk (inputs) of the plan for rows_total rows of K inputs; 0 if none.
int qgemv_chunk(int K, int bits, int64_t rows_total, bool allow_split);
int qgemv_row_stride(int kc_bytes, int bits);
int launch_qgemv(const QgArgs& a, const QgLayout& L, int bits, bool pdl, cudaStream_t st);

// rgemv.cu: resident-weight decode GEMV (items = 16-row tile x 512-input
// chunk, chunk-major over the CTAs; fp32 output slices out[chunk][t][ld] that
// the consumer adds in chunk order).  Input kinds as QgArgs (QG_IN_*).
constexpr int kRgChunkGroups = 8;  // 64-column groups per chunk
constexpr int kRgMaxChunks = 4;    // chunks one CTA may span
struct RgSeg {
  const uint8_t* w;  // packed codes [rows][K*bits/8 bytes]
  const bf16* s;     // [rows][K/64]
  const bf16* b;
  float* out;        // slice c, token t, row r at out[c * pstride + t * ld + col0 + r]
  int rows, ld, col0;
  int tile0;         // set by rgemv_plan
  int64_t pstride;   // set by rgemv_plan: T * ld
};
struct RgArgs {
  RgSeg seg[kQgMaxSeg];
  int nseg, K, T;
  int G, nck, tiles, items;  // set by rgemv_plan
  int in_kind;
  const bf16* x;       // [T][ldx] (QG_IN_BF16 / QG_IN_RMSNORM)
  int ldx;
  const bf16* norm_w;  // [K] (QG_IN_RMSNORM)
  float eps;
  const float* g;      // [T][ldgu] fp32 gate / up slices (QG_IN_GELU)
  const float* u;
  int ldgu;
  int gu_parts;
  int64_t gu_part_stride;
  int* status;
};
struct RgLayout {
  int rs, soff, stage, nst, maxch, frag, xsum, misc, normw, xs, red, bar, ring, bytes, grid;
};
int rgemv_plan(RgArgs& a, int bits, RgLayout* L, int smem_budget = 110 * 1024);
int launch_rgemv(const RgArgs& a, const RgLayout& L, int bits, bool pdl, cudaStream_t st);

inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

struct Carver;

// abi.cu: argument checks, workspace carving and the router / expert sequence
// shared by the MoE-block and decoder-layer entry points.
bool aligned(const void* p, size_t a);
int to_qw(const fmoe_qweight_t* w, QW* q);

// qgemm.cu: dense 4 / 8-bit group-64 linear layers over many tokens on tcgen05.
// Up to kQmMaxSeg weights of the same K and bits share x (one launch); in the
// gated form o[0] / o[1] are gate / up and o[0].out receives gelu(g) * u.
constexpr int kSvMaxSlots = 32768;  // sparsev.cu: attended slots of one sparse-V call (scores in shared memory)
constexpr int kQmMaxSeg = 3;
struct QmOut {
  const QW* w;
  bf16* out;  // row t at out + t * ld
  int ld;
};
bool qgemm_supported(const QW& w, int group, int K);
int launch_qgemm(const bf16* x, int64_t T, int K, const QmOut* o, int nseg, bool gated, int* status, cudaStream_t st);
// pflayer.cu: output norms / residual / layer scalar of rows (h may equal x)
int launch_ff_out_rows(bf16* x, const bf16* h, const bf16* d, const bf16* moe, int64_t rows, int H, const bf16* w1,
                       const bf16* w2, const bf16* w, float eps, float scalar, cudaStream_t st);
// pflayer.cu: prefill attention of T tokens of one sequence (window 0: causal)
// affine_ok: an affine (rotated K4 / V8) ring is dequantised as it is read; q and
// the staged rows must then be in the rotated basis (the decoder layer's prefill).
int launch_attn_prefill(const KvDev& c, const bf16* q, int Hq, int64_t T, int64_t pos0, int window, const bf16* ks,
                        const bf16* vs, bf16* out, float scale, cudaStream_t st, bool affine_ok = false);
int to_experts(const fmoe_experts_t* e, ExpertsDev* d);
int check_router(const fmoe_router_t* r, QW* q);
// Every workspace starts with a 256-byte header: [0] device status word (0 ok;
// otherwise the site code of a timed-out wait), [1] router completion counter.
struct WsHead {
  int* status;
  unsigned* router_ctr;
};
struct RouterWs {
  unsigned* counters;  // [1]: token chunks done (several chunks), zero between calls
  bf16* xs;            // normalised router input (use_norm)
  float* unused;
};
struct MoeWs {
  RouteMeta m;
  bf16* act;           // [T*k, I] gated intermediate activations
  float* part;         // [groups, T, H] per-expert-group partial outputs
  unsigned* tile_ctr;  // [H/16] completion counters, zero between calls
};
WsHead carve_head(Carver& c);
size_t carve_router(Carver& c, int64_t T, const fmoe_router_t* r, const WsHead& h, RouterWs* w);
size_t carve_moe(Carver& c, int64_t T, int k, const ExpertsDev& ex, MoeWs* w);
int run_router(const bf16* x, int64_t T, const fmoe_router_t* r, const QW& q, const RouterWs& w, int32_t* ids,
               float* wts, float* logits, const RouteMeta* meta, int* status, cudaStream_t st);
// y32 != nullptr: fp32 output rows there instead of bf16 ones in y.
int run_experts(const bf16* x, int64_t T, int k, const int32_t* ids, const float* wts, const ExpertsDev& ex, bf16* y,
                const MoeWs& w, bool build_routes, int* status, cudaStream_t st, float* y32 = nullptr);

// prefill.cu: the expert stage of the tensor-core path on routed tokens (any
// expert table slice; pairs whose id is outside it contribute nothing).
struct PfExWs {
  RouteMeta m;
  int4* tiles;   // [P/BM + E + 1] (expert, first sorted pair, rows, 0)
  int* ntiles;   // [1]
  int32_t* inv;  // [P] sorted position of pair p, -1 when the pair is not local
  bf16* xs;      // [P, H] token rows in expert order
  bf16* act;     // [P, I] gated activations
  bf16* ys;      // [P, H] per-pair expert outputs
};
int check_prefill(const ExpertsDev& d);
size_t carve_pf_ex(Carver& c, int64_t T, int k, const ExpertsDev& d, PfExWs* w);
// ids / wts: [T, k].  build_routes: build w.m from ids (false when the router
// already built it).  prep: fmoe_moe_prefill_prepare's copy for this table.
int run_prefill_experts(const bf16* x, int64_t T, int k, const int32_t* ids, const float* wts, const ExpertsDev& d,
                        const bf16* prep, bf16* y, const PfExWs& w, bool build_routes, int* status, cudaStream_t st,
                        float* y32 = nullptr);

// ep.cu: expert-parallel dispatch -> local experts -> combine over NCCL.
struct EpWs {
  RouterWs rw;                        // router scratch (MoE-block entry point only)
  int32_t *ids, *slots, *counts, *rcounts;
  float* wts;
  bf16* sx;                           // [R][cap] send blocks
  int32_t* sids;
  float* swts;
  bf16* rx;                           // received rows (R * cap at most)
  int32_t* rids;
  float* rwts;
  float *ypart, *ret;                 // fp32 partial sums: computed here | returned from the peers
  MoeWs mw;                           // decode expert kernels, min(R * cap, 128) rows
  PfExWs pw;                          // tensor-core expert stage (R * cap > 128)
  bool gemm;
};
size_t carve_ep(Carver& c, int R, int64_t cap, const fmoe_router_t* r, int k, const ExpertsDev& d, const WsHead& h,
                EpWs* w);
// The slice must be experts [rank*E/n, (rank+1)*E/n) of E_total.
int ep_check(const fmoe_ep_comm_t* c, const ExpertsDev& d, int E_total, int* n_ranks);
int ep_comm_ranks(const fmoe_ep_comm_t* c);  // ranks of the communicator (0 for null)
int ep_experts(const fmoe_ep_comm_t* c, const bf16* x, int64_t T, int64_t cap, int k, const int32_t* ids,
               const float* wts, const ExpertsDev& d, const bf16* prep, bf16* y, const EpWs& w, int mode, int* status,
               cudaStream_t st);

// kv.cu
int kv_to_dev(const fmoe_kv_cache_t* c, KvDev* d);
size_t attn_workspace_bytes(const KvDev& c, int Hq);
// pdl: launched as a programmatic dependent of the preceding kernel (the
// kernel waits for it before reading q or the newest cache row).  newest /
// newest_dev: the position whose row the preceding kernel appended (its slot
// is newest % cap; -1: none): every other chunk is copied before the wait.
// sparsev.cu: gated decode attention (n_dev: attended slots on the device, or null)
int launch_sparse_v(const KvDev& c, const bf16* q, int q_heads, int64_t n_valid, const int64_t* n_dev, float scale,
                    float tau, bf16* out, cudaStream_t st);
int launch_attn_decode(const KvDev& c, const bf16* q, int Hq, int64_t nvalid, const int64_t* nvalid_dev, float scale,
                       void* ws, bf16* out, cudaStream_t st, bool pdl = false, int64_t newest = -1,
                       const int64_t* newest_dev = nullptr);
// qkv: fp32 projections in `parts` slices part_stride floats apart (added in order)
int launch_qkv_post(const KvDev& c, const float* qkv, int ld, int parts, int64_t part_stride, int Hq, int k_eq_v,
                    const bf16* q_norm,
                    const bf16* k_norm, float eps, int rope_dims, float rope_theta, int64_t pos,
                    const int64_t* pos_dev, bf16* q_out, int turbo_bits, bool pdl, cudaStream_t st);

// dlayer.cu: the decode layer as six streaming launches (T <= 8, experts
// local) and the streaming lm_head.
struct DlPlan {
  int T, H, D, Hq, Hkv, QD, Id, Ie, E, k, Umax, qkv_tiles;
  int qbits, obits, rbits;
  int nw_r, nw_g, nw_d, nw_x;                      // warps of the two-family launches
  int mp_qkv, mp_o, mp_r, mp_g, mp_d, mp_x, mp_y;  // pieces per unit (bounds)
  size_t sm_qkv, sm_o, sm_1, sm_2, sm_3;           // dynamic shared memory per launch
};
struct DlWs {  // counters are zero between calls
  unsigned *uc_qkv, *uc_o, *uc_r, *uc_g, *uc_d, *uc_x, *uc_y, *gc_qkv, *gc_y, *grid;
  float *p_qkv, *p_o, *p_r, *p_g, *p_d, *p_x, *p_y;  // pieces
  float *f_qkv, *f_o, *f_r, *f_d, *f_y;              // finished units
  bf16 *act_d, *act_e;
  int32_t *ids, *slot, *uniq, *nuniq;
  float* wts;
};
struct DlBufs {  // layer buffers shared with the per-op path
  bf16 *q, *attn, *h, *h1, *h2, *xs, *moe;
  void* attn_ws;
};
struct Carver;
// FMOE_OK when the layer call can take the streaming path (fills *p).
int dl_plan(const fmoe_decoder_layer_t* L, const KvDev& kv, int64_t T, DlPlan* p);
size_t dl_carve(Carver& c, const DlPlan& p, DlWs* w);
int dl_layer_forward(const fmoe_decoder_layer_t* L, const KvDev& kv, const DlPlan& p, const DlWs& w, bf16* x,
                     int64_t pos, const int64_t* pos_dev, const DlBufs& b, cudaStream_t st);
size_t dl_lm_workspace_bytes(int64_t T);
int dl_lm_head(const QW& e, const bf16* norm, float eps, const bf16* x, int64_t T, float cap, float* logits,
               int32_t* next_ids, int64_t* pos_dev, void* ws, cudaStream_t st);

// Bump allocator over a caller workspace.
struct Carver {
  uint8_t* base;
  size_t off = 0;
  explicit Carver(void* p) : base(static_cast<uint8_t*>(p)) {}
  template <class T>
  T* take(size_t n) {
    off = align_up(off, 256);
    T* p = base ? reinterpret_cast<T*>(base + off) : nullptr;
    off += n * sizeof(T);
    return p;
  }
};

}  // namespace fmoe
