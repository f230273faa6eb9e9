// extern "C" entry points of libfmoe (declared in include/fmoe.h): argument
// validation, workspace carving and kernel sequencing.  No entry point
// synchronises the stream or allocates device memory.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include "internal.h"

namespace fmoe {

static thread_local char g_err[512] = "";

int set_error(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

int check_launch(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return set_error(FMOE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return FMOE_OK;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

int to_qw(const fmoe_qweight_t* w, QW* q) {
  if (!w || !w->w) return set_error(FMOE_ERR_INVALID, "qweight: null weight");
  if (w->out_features <= 0 || w->in_features <= 0) return set_error(FMOE_ERR_INVALID, "qweight: empty shape");
  if (w->bits != 16) {
    if (!w->scales || !w->biases) return set_error(FMOE_ERR_INVALID, "qweight: null scales/biases");
    if (w->group_size <= 0 || w->in_features % w->group_size)
      return set_error(FMOE_ERR_INVALID, "qweight: in_features %d not a multiple of group %d", w->in_features,
                       w->group_size);
  }
  q->w = w->w;
  q->s = static_cast<const bf16*>(w->scales);
  q->b = static_cast<const bf16*>(w->biases);
  q->out = w->out_features;
  q->in = w->in_features;
  q->bits = w->bits;
  q->tiled = static_cast<const uint8_t*>(w->tiled);
  q->tiled_kc = w->tiled ? w->tiled_kc : 0;
  return FMOE_OK;
}

// Shapes the register-dequant GEMV kernels accept.
static int check_gemv_weight(const QW& q, int group) {
  if (q.bits != 16 && q.bits != 4 && q.bits != 8)
    return set_error(FMOE_ERR_UNSUPPORTED, "gemv: bits=%d (kernels: 4, 8, 16=bf16)", q.bits);
  if (q.bits != 16 && group != 64) return set_error(FMOE_ERR_UNSUPPORTED, "gemv: group_size %d (kernels: 64)", group);
  if (q.in % 64 || q.out % 16)
    return set_error(FMOE_ERR_UNSUPPORTED, "gemv: [out=%d, in=%d] needs in %% 64 == 0 and out %% 16 == 0", q.out, q.in);
  if (!aligned(q.w, 16)) return set_error(FMOE_ERR_ALIGN, "gemv: weight not 16-byte aligned");
  return FMOE_OK;
}

int to_experts(const fmoe_experts_t* e, ExpertsDev* d) {
  if (!e || !e->base) return set_error(FMOE_ERR_INVALID, "experts: null table");
  if (e->bits != 4 || e->group_size != 64)
    return set_error(FMOE_ERR_UNSUPPORTED, "experts: bits=%d group=%d (kernels: 4-bit, group 64)", e->bits,
                     e->group_size);
  if (e->hidden <= 0 || e->intermediate <= 0 || e->hidden % 64 || e->intermediate % 64)
    return set_error(FMOE_ERR_UNSUPPORTED, "experts: hidden %d / intermediate %d must be multiples of 64", e->hidden,
                     e->intermediate);
  if (e->num_experts <= 0 || e->num_experts > 1024) return set_error(FMOE_ERR_INVALID, "experts: num_experts %d", e->num_experts);
  if (!aligned(e->base, 16) || e->expert_stride % 16) return set_error(FMOE_ERR_ALIGN, "experts: base/stride not 16-byte aligned");
  for (int j = 0; j < 9; ++j)
    if (e->offsets[j] < 0 || e->offsets[j] % 16)  // TMA bulk copies need 16-byte aligned sources
      return set_error(FMOE_ERR_ALIGN, "experts: offset[%d]=%lld misaligned", j, (long long)e->offsets[j]);
  d->base = static_cast<const uint8_t*>(e->base);
  d->stride = e->expert_stride;
  for (int j = 0; j < 9; ++j) d->off[j] = e->offsets[j];
  d->E = e->num_experts;
  d->first = e->first_expert;
  d->H = e->hidden;
  d->I = e->intermediate;
  d->slot_of = e->slot_of;
  return FMOE_OK;
}

static const int kMaxDecodeTokens = 128;

// Every workspace starts with a 256-byte header: [0] device status word (0 ok;
// otherwise the site code of a timed-out wait), [1] router completion counter.
WsHead carve_head(Carver& c) {
  int* p = c.take<int>(64);
  return WsHead{p, p ? reinterpret_cast<unsigned*>(p + 1) : nullptr};
}


size_t carve_router(Carver& c, int64_t T, const fmoe_router_t* r, const WsHead& h, RouterWs* w) {
  const int H = r->proj.in_features;
  bf16* xs = r->use_norm ? c.take<bf16>((size_t)T * H) : nullptr;
  if (w) *w = RouterWs{h.router_ctr, xs, nullptr};
  return c.off;
}


size_t carve_moe(Carver& c, int64_t T, int k, const ExpertsDev& ex, MoeWs* w) {
  MoeWs m;
  m.tile_ctr = c.take<unsigned>(ex.H / 16);
  m.m.start = c.take<int32_t>(ex.E + 1);
  m.m.pairs = c.take<int32_t>((size_t)T * k);
  m.m.unique = c.take<int32_t>(ex.E);
  m.m.num_unique = c.take<int32_t>(1);
  m.m.work_len = (int)(T * k < ex.E ? T * k : ex.E);
  m.m.work = c.take<int4>(m.m.work_len);
  m.m.scratch = nullptr;  // decode sizes: one CTA builds the lists
  m.act = c.take<bf16>((size_t)T * k * ex.I);
  const int groups = down_groups(T, k, ex.E);
  m.part = groups > 1 ? c.take<float>((size_t)groups * T * ex.H) : nullptr;
  if (w) *w = m;
  return c.off;
}

int check_router(const fmoe_router_t* r, QW* q) {
  if (!r) return set_error(FMOE_ERR_INVALID, "router: null");
  int rc = to_qw(&r->proj, q);
  if (rc) return rc;
  if (q->bits != 16 && q->bits != 4 && q->bits != 8)
    return set_error(FMOE_ERR_UNSUPPORTED, "router: bits=%d (kernels: 4, 8, 16=bf16)", q->bits);
  if (q->bits != 16 && r->proj.group_size != 64)
    return set_error(FMOE_ERR_UNSUPPORTED, "router: group_size %d (kernels: 64)", r->proj.group_size);
  if (q->in % 64) return set_error(FMOE_ERR_UNSUPPORTED, "router: hidden %d not a multiple of 64", q->in);
  if (!aligned(q->w, 16)) return set_error(FMOE_ERR_ALIGN, "router: weight not 16-byte aligned");
  if (r->top_k < 1 || r->top_k > 16 || r->top_k > q->out) return set_error(FMOE_ERR_INVALID, "router: top_k %d", r->top_k);
  return FMOE_OK;
}

// meta != nullptr: the router kernel also builds the per-expert pair lists.
int run_router(const bf16* x, int64_t T, const fmoe_router_t* r, const QW& q, const RouterWs& w, int32_t* ids,
                      float* wts, float* logits, const RouteMeta* meta, int* status, cudaStream_t st) {
  const bf16* xin = x;
  if (r->use_norm) {
    const int rc =
        launch_router_prenorm(x, T, q.in, r->root_size, r->eps, static_cast<const bf16*>(r->router_scale), w.xs, st);
    if (rc) return rc;
    xin = w.xs;
  }
  if (router_tc_eligible(T, q, r->top_k) && aligned(xin, 16) && aligned(q.w, 16) && (!logits || aligned(logits, 16))) {
    // many tokens: tensor-core GEMM + top-k epilogue
    int rc = launch_router_tc(xin, T, q, r->logit_bias, static_cast<const bf16*>(r->per_expert_scale), r->top_k, ids,
                              wts, logits, status, st);
    if (rc || !meta) return rc;
    ExpertsDev all = {};
    all.E = q.out;  // lists over every expert of the router (first 0)
    return launch_route_build(ids, T * r->top_k, all, *meta, st);
  }
  return launch_router_fused(xin, T, q, r->logit_bias, static_cast<const bf16*>(r->per_expert_scale), r->top_k, ids,
                             wts, logits, w.counters, meta, status, true, st);
}

int run_experts(const bf16* x, int64_t T, int k, const int32_t* ids, const float* wts, const ExpertsDev& ex,
                       bf16* y, const MoeWs& w, bool build_routes, int* status, cudaStream_t st, float* y32) {
  int rc;
  if (build_routes) {
    rc = launch_route_build(ids, T * k, ex, w.m, st);
    if (rc) return rc;
  }
  rc = launch_moe_gate_up(x, T, k, ex, w.m, w.act, status, true, st);
  if (rc) return rc;
  return launch_moe_down(w.act, T, k, wts, ex, w.m, w.part, w.tile_ctr, y, status, true, st, y32);
}

}  // namespace fmoe

using namespace fmoe;

extern "C" {

int fmoe_version(void) { return 100; }

int fmoe_last_error(char* buf, size_t len) {
  const size_t n = strlen(g_err);
  if (buf && len) {
    const size_t c = n < len - 1 ? n : len - 1;
    memcpy(buf, g_err, c);
    buf[c] = 0;
  }
  return (int)n;
}

int fmoe_quantize(const void* src, int src_is_bf16, int64_t rows, int64_t cols, int bits, int group_size, void* wq,
                  void* scales, void* biases, void* stream) {
  if (!src || !wq || !scales || !biases) return set_error(FMOE_ERR_INVALID, "quantize: null pointer");
  if (!(bits == 2 || bits == 3 || bits == 4 || bits == 5 || bits == 6 || bits == 8))
    return set_error(FMOE_ERR_INVALID, "quantize: bits=%d", bits);
  if (group_size <= 0 || cols % group_size || (group_size * bits) % 32)
    return set_error(FMOE_ERR_INVALID, "quantize: cols %lld / group %d", (long long)cols, group_size);
  if (rows <= 0) return FMOE_OK;
  return launch_quantize(src, src_is_bf16, rows, cols, bits, group_size, static_cast<uint32_t*>(wq),
                         static_cast<bf16*>(scales), static_cast<bf16*>(biases), static_cast<cudaStream_t>(stream));
}

int fmoe_dequantize(const fmoe_qweight_t* w, void* out, void* stream) {
  QW q;
  int rc = to_qw(w, &q);
  if (rc) return rc;
  if (q.bits == 16) return set_error(FMOE_ERR_INVALID, "dequantize: weight is not quantised");
  if (!out) return set_error(FMOE_ERR_INVALID, "dequantize: null out");
  return launch_dequantize(q, w->group_size, nullptr, q.out, 1.0f, static_cast<bf16*>(out),
                           static_cast<cudaStream_t>(stream));
}

int fmoe_embed_rows(const fmoe_qweight_t* w, const int32_t* ids, int64_t n, float row_scale, void* out, void* stream) {
  QW q;
  int rc = to_qw(w, &q);
  if (rc) return rc;
  if (!ids || !out) return set_error(FMOE_ERR_INVALID, "embed_rows: null ids/out");
  if (n <= 0) return FMOE_OK;
  return launch_dequantize(q, w->group_size, ids, n, row_scale, static_cast<bf16*>(out),
                           static_cast<cudaStream_t>(stream));
}

size_t fmoe_router_workspace_bytes(int64_t T, const fmoe_router_t* r) {
  if (!r || T <= 0) return 0;
  Carver c(nullptr);
  const WsHead h = carve_head(c);
  return carve_router(c, T, r, h, nullptr) + 256;
}

int fmoe_router(const void* x, int64_t T, const fmoe_router_t* r, int32_t* ids, float* weights, float* logits,
                void* workspace, size_t workspace_bytes, void* stream) {
  QW q;
  int rc = check_router(r, &q);
  if (rc) return rc;
  if (!x || !ids || !weights) return set_error(FMOE_ERR_INVALID, "router: null x/ids/weights");
  if (T <= 0) return FMOE_OK;
  if (!aligned(x, 16)) return set_error(FMOE_ERR_ALIGN, "router: x not 16-byte aligned");
  if (!workspace || workspace_bytes < fmoe_router_workspace_bytes(T, r))
    return set_error(FMOE_ERR_WORKSPACE, "router: workspace %zu < %zu", workspace_bytes, fmoe_router_workspace_bytes(T, r));
  Carver c(workspace);
  const WsHead h = carve_head(c);
  RouterWs w;
  carve_router(c, T, r, h, &w);
  return run_router(static_cast<const bf16*>(x), T, r, q, w, ids, weights, logits, nullptr, h.status,
                    static_cast<cudaStream_t>(stream));
}

// Decode-size inputs of 4 / 6 / 8-bit weights go to the streaming tensor-core
// GEMV (qgemv.cu); everything else to the split-K GEMV (gemv.cu).
static bool qlinear_streams(int64_t T, const QW& q, int group) {
  return T >= 1 && T <= 8 && (q.bits == 4 || q.bits == 6 || q.bits == 8) && group == 64 && q.in % 64 == 0 &&
         q.out % 16 == 0 && aligned(q.w, 16) && aligned(q.s, 16) && aligned(q.b, 16);
}

size_t fmoe_qlinear_workspace_bytes(int64_t T, const fmoe_qweight_t* w) {
  if (!w || T <= 0 || w->out_features <= 0 || w->in_features < 64) return 0;
  QW q;
  if (T > 8 && to_qw(w, &q) == FMOE_OK && qgemm_supported(q, w->group_size, q.in)) return 256;
  const int ks = gemv_ksplit(T, w->out_features, w->in_features);
  const size_t split = sizeof(float) * (size_t)ks * T * w->out_features;
  const size_t acc = sizeof(float) * (size_t)T * w->out_features;
  return align_up(split > acc ? split : acc, 256) + 256;
}

int fmoe_qlinear(const void* x, int64_t T, const fmoe_qweight_t* w, void* y, void* workspace, size_t workspace_bytes,
                 void* stream) {
  QW q;
  int rc = to_qw(w, &q);
  if (rc) return rc;
  if (!x || !y) return set_error(FMOE_ERR_INVALID, "qlinear: null x/y");
  if (T <= 0) return FMOE_OK;
  if (!aligned(x, 16)) return set_error(FMOE_ERR_ALIGN, "qlinear: x not 16-byte aligned");
  const size_t need = fmoe_qlinear_workspace_bytes(T, w);
  if (!workspace || workspace_bytes < need) return set_error(FMOE_ERR_WORKSPACE, "qlinear: workspace %zu < %zu", workspace_bytes, need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (qlinear_streams(T, q, w->group_size)) {
    QgArgs a = {};
    a.nseg = 1;
    a.seg[0] = QgSeg{static_cast<const uint8_t*>(q.w), q.s, q.b, y, q.out, q.out, 0, 0, q.tiled, q.tiled_kc};
    a.K = q.in;
    a.T = (int)T;
    a.in_kind = QG_IN_BF16;
    a.x = static_cast<const bf16*>(x);
    a.ldx = q.in;
    a.out_kind = QG_OUT_BF16;
    QgLayout L;
    if (qgemv_plan(a, q.bits, false, &L) == FMOE_OK) return launch_qgemv(a, L, q.bits, false, st);
    // the rows need column chunks: accumulate in fp32, then round
    a.out_kind = QG_OUT_F32_ADD;
    Carver c(workspace);
    float* acc = c.take<float>((size_t)T * q.out);
    a.seg[0].out = acc;
    if (qgemv_plan(a, q.bits, true, &L) == FMOE_OK) {
      if (cudaMemsetAsync(acc, 0, sizeof(float) * (size_t)T * q.out, st) != cudaSuccess)
        return set_error(FMOE_ERR_CUDA, "qlinear: clearing the accumulator failed");
      rc = launch_qgemv(a, L, q.bits, false, st);
      if (rc) return rc;
      return launch_reduce_partials(acc, 1, T * q.out, static_cast<bf16*>(y), nullptr, st);
    }
    // too large for the streaming kernel's shared memory: split-K path below
  }
  if (T > 8 && qgemm_supported(q, w->group_size, q.in)) {
    // many tokens: the tensor-core GEMM (no workspace)
    const QmOut o{&q, static_cast<bf16*>(y), q.out};
    return launch_qgemm(static_cast<const bf16*>(x), T, q.in, &o, 1, false, nullptr, st);
  }
  rc = check_gemv_weight(q, w->group_size);
  if (rc) return rc;
  const int ks = gemv_ksplit(T, q.out, q.in);
  Carver c(workspace);
  float* part = c.take<float>((size_t)ks * T * q.out);
  rc = launch_gemv_partial(static_cast<const bf16*>(x), T, q, ks, part, st);
  if (rc) return rc;
  return launch_reduce_partials(part, ks, T * q.out, static_cast<bf16*>(y), nullptr, st);
}

size_t fmoe_moe_workspace_bytes(int64_t T, int top_k, const fmoe_experts_t* ex) {
  ExpertsDev d;
  if (T <= 0 || to_experts(ex, &d)) return 0;
  Carver c(nullptr);
  carve_head(c);
  return carve_moe(c, T, top_k, d, nullptr) + 256;
}

int fmoe_moe_experts(const void* x, int64_t T, int top_k, const int32_t* ids, const float* weights,
                     const fmoe_experts_t* ex, void* y, void* workspace, size_t workspace_bytes, void* stream) {
  ExpertsDev d;
  int rc = to_experts(ex, &d);
  if (rc) return rc;
  if (!x || !ids || !weights || !y) return set_error(FMOE_ERR_INVALID, "moe_experts: null pointer");
  if (T <= 0) return FMOE_OK;
  if (top_k < 1 || top_k > 16) return set_error(FMOE_ERR_INVALID, "moe_experts: top_k %d", top_k);
  if (T > kMaxDecodeTokens)
    return set_error(FMOE_ERR_UNSUPPORTED, "moe_experts: T=%lld above the decode path's %d", (long long)T, kMaxDecodeTokens);
  if (!aligned(x, 16)) return set_error(FMOE_ERR_ALIGN, "moe_experts: x not 16-byte aligned");
  const size_t need = fmoe_moe_workspace_bytes(T, top_k, ex);
  if (!workspace || workspace_bytes < need) return set_error(FMOE_ERR_WORKSPACE, "moe_experts: workspace %zu < %zu", workspace_bytes, need);
  Carver c(workspace);
  const WsHead h = carve_head(c);
  MoeWs w;
  carve_moe(c, T, top_k, d, &w);
  return run_experts(static_cast<const bf16*>(x), T, top_k, ids, weights, d, static_cast<bf16*>(y), w, true, h.status,
                     static_cast<cudaStream_t>(stream));
}

size_t fmoe_moe_block_workspace_bytes(int64_t T, const fmoe_router_t* r, const fmoe_experts_t* ex) {
  ExpertsDev d;
  if (T <= 0 || !r || to_experts(ex, &d)) return 0;
  Carver c(nullptr);
  const WsHead h = carve_head(c);
  carve_router(c, T, r, h, nullptr);
  c.take<int32_t>((size_t)T * r->top_k);
  c.take<float>((size_t)T * r->top_k);
  return carve_moe(c, T, r->top_k, d, nullptr) + 256;
}

int fmoe_moe_block_forward(const void* x, int64_t T, const fmoe_router_t* r, const fmoe_experts_t* ex, void* y,
                           int32_t* ids, float* weights, void* workspace, size_t workspace_bytes, void* stream) {
  QW q;
  int rc = check_router(r, &q);
  if (rc) return rc;
  ExpertsDev d;
  rc = to_experts(ex, &d);
  if (rc) return rc;
  if (T <= 0) return FMOE_OK;  // no tokens: nothing to route (x / y may be null)
  if (!x || !y) return set_error(FMOE_ERR_INVALID, "moe_block: null x/y");
  if (q.in != d.H) return set_error(FMOE_ERR_INVALID, "moe_block: router in %d != hidden %d", q.in, d.H);
  if (T > kMaxDecodeTokens)
    return set_error(FMOE_ERR_UNSUPPORTED, "moe_block: T=%lld above the decode path's %d", (long long)T, kMaxDecodeTokens);
  if (!aligned(x, 16)) return set_error(FMOE_ERR_ALIGN, "moe_block: x not 16-byte aligned");
  const size_t need = fmoe_moe_block_workspace_bytes(T, r, ex);
  if (!workspace || workspace_bytes < need) return set_error(FMOE_ERR_WORKSPACE, "moe_block: workspace %zu < %zu", workspace_bytes, need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver c(workspace);
  const WsHead h = carve_head(c);
  RouterWs w;
  carve_router(c, T, r, h, &w);
  int32_t* ids_ws = c.take<int32_t>((size_t)T * r->top_k);
  float* w_ws = c.take<float>((size_t)T * r->top_k);
  int32_t* ids_out = ids ? ids : ids_ws;
  float* w_out = weights ? weights : w_ws;
  MoeWs mw;
  carve_moe(c, T, r->top_k, d, &mw);
  if (q.out != d.E || d.first != 0)
    return set_error(FMOE_ERR_INVALID, "moe_block: router has %d experts, table %d (first %d)", q.out, d.E, d.first);
  rc = run_router(static_cast<const bf16*>(x), T, r, q, w, ids_out, w_out, nullptr, &mw.m, h.status, st);
  if (rc) return rc;
  return run_experts(static_cast<const bf16*>(x), T, r->top_k, ids_out, w_out, d, static_cast<bf16*>(y), mw, false,
                     h.status, st);
}

int fmoe_workspace_status(const void* workspace, int clear, void* stream) {
  if (!workspace) return set_error(FMOE_ERR_INVALID, "workspace_status: null workspace");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  int v = 0;
  if (cudaMemcpyAsync(&v, workspace, sizeof(int), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
      cudaStreamSynchronize(st) != cudaSuccess)
    return set_error(FMOE_ERR_CUDA, "workspace_status: %s", cudaGetErrorString(cudaGetLastError()));
  if (v && clear && cudaMemsetAsync(const_cast<void*>(workspace), 0, sizeof(int), st) != cudaSuccess)
    return set_error(FMOE_ERR_CUDA, "workspace_status: clear failed");
  if (v) return set_error(FMOE_ERR_TIMEOUT, "a device wait gave up (site %d)", v);
  return FMOE_OK;
}

}  // extern "C"
