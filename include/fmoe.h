/*
 * libfmoe — C ABI of the B200 (sm_100a) quantised-MoE hot path of flash-moe.
 *
 * This is the seam a host engine binds to in place of flash-moe's MLX calls on
 * the MoE / quantised-KV path and of its only native shim, src/ffi.rs:5-14
 * (extern "C" mlx_array_from_mmap) / src/ffi_zerocopy.cpp:14-55.  Every entry
 * point is a plain C function: device pointers, sizes, an explicit CUDA stream
 * (passed as void*; NULL = legacy default stream) and an int status.
 *
 * Conventions
 *   - bf16 tensors are raw 16-bit bfloat16 (RNE), row-major, no padding.
 *   - MLX-affine quantised weight [out, in]: w uint32 [out, in*bits/32] holding
 *     a little-endian bit stream of codes (value j at bits [j*bits,(j+1)*bits)),
 *     scales / biases bf16 [out, in/group]; w ~= scale*q + bias.
 *   - Status: 0 ok, negative FMOE_ERR_*; fmoe_last_error() gives the text of the
 *     most recent failure on the calling thread.  No exceptions cross the ABI.
 *   - The library never frees caller memory.  Calls are asynchronous on the
 *     given stream; buffers must stay alive until the stream has passed them.
 *   - Thread safety: entry points keep no global mutable state besides the
 *     per-thread error text; concurrent calls are safe on distinct workspaces.
 */
#ifndef FMOE_H_
#define FMOE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define FMOE_OK 0
#define FMOE_ERR_INVALID -1     /* bad argument, shape or bit width */
#define FMOE_ERR_ALIGN -2       /* pointer or stride misaligned for the kernel */
#define FMOE_ERR_WORKSPACE -3   /* workspace NULL or smaller than required */
#define FMOE_ERR_CUDA -4        /* CUDA launch / runtime error */
#define FMOE_ERR_UNSUPPORTED -5 /* configuration outside the compiled kernels */
#define FMOE_ERR_TIMEOUT -6     /* a bounded device wait gave up */
#define FMOE_ERR_NCCL -7        /* NCCL failure (expert parallelism) */
#define FMOE_ERR_ALLOC -8       /* device allocation failed */

/* MLX-affine quantised (bits 2/3/4/5/6/8) or plain bf16 (bits 16) linear
 * weight [out_features, in_features].  Mirrors QuantizedLinear,
 * src/model/mlp.rs:4-12. */
typedef struct fmoe_qweight {
  const void* w;      /* uint32 packed codes, or bf16 [out, in] when bits == 16 */
  const void* scales; /* bf16 [out, in/group]; NULL when bits == 16 */
  const void* biases; /* bf16 [out, in/group]; NULL when bits == 16 */
  int32_t out_features;
  int32_t in_features;
  int32_t bits;
  int32_t group_size;
  /* Optional copy of w in the streaming GEMV's tile layout (fmoe_qweight_tile;
   * NULL: none).  The decode GEMV then moves one contiguous block per 16-row
   * unit instead of one copy per row.  tiled_kc: its column chunk in inputs. */
  const void* tiled;
  int32_t tiled_kc;
  int32_t reserved;
} fmoe_qweight_t;

/* Routed experts of one MoE layer in the ECB expert-major layout written by
 * src/splitter.rs:405-457 and read by src/memory.rs:571-607: expert e's
 * tensor j is at base + e*expert_stride + offsets[j], j in the order
 * gate.w gate.s gate.b up.w up.s up.b down.w down.s down.b.
 * gate/up: [intermediate, hidden]; down: [hidden, intermediate]. */
typedef struct fmoe_experts {
  const void* base;
  int64_t expert_stride;
  int64_t offsets[9];
  int32_t num_experts;  /* experts present in this table (local shard) */
  int32_t first_expert; /* global id of the table's expert 0 (0 unless sharded) */
  int32_t hidden;
  int32_t intermediate;
  int32_t bits;
  int32_t group_size;
  /* NULL: expert e (local index) is at base + e*expert_stride.  Else a device
   * int32 [num_experts] slot map: expert e is at base + slot_of[e]*expert_stride
   * (an HBM cache of slots filled from a pinned host copy; decode expert
   * kernels only — the prefill and whole-step paths reject it). */
  const int32_t* slot_of;
} fmoe_experts_t;

/* Router of Gemma4MoeBlock, src/model/moe.rs:298-312 / 324-345. */
typedef struct fmoe_router {
  fmoe_qweight_t proj;          /* router_proj [num_experts, hidden] */
  const void* router_scale;     /* bf16 [hidden] or NULL (applied only when use_norm) */
  const void* per_expert_scale; /* bf16 [num_experts] or NULL */
  const float* logit_bias;      /* f32 [num_experts] or NULL; added to logits */
  float root_size;              /* hidden^-1/2 (used when use_norm) */
  float eps;                    /* rms_norm_eps (used when use_norm) */
  int32_t use_norm;             /* 1: rms_norm_no_scale -> *root_size -> *router_scale */
  int32_t top_k;                /* experts per token (<= 16) */
} fmoe_router_t;

/* ---- library -------------------------------------------------------- */

/* Version as major*10000 + minor*100 + patch. */
int fmoe_version(void);

/* Copies the calling thread's most recent error text (NUL-terminated, truncated
 * to len) and returns its full length. */
int fmoe_last_error(char* buf, size_t len);

/* Per-kernel device timing (replaces the reference's host-side phase
 * accumulators, src/perf.rs:65-153).  While enabled, each kernel launch is
 * bracketed by CUDA events on its stream (do not enable during stream
 * capture).  fmoe_profile_read synchronises on the recorded events, folds them
 * into per-kernel totals, copies up to max_entries of them and returns the
 * number of distinct kernels (or a negative status); reset != 0 clears them. */
typedef struct fmoe_kernel_stat {
  char name[64];
  int64_t launches;
  double total_ms;
} fmoe_kernel_stat_t;
int fmoe_profile_enable(int on);
int fmoe_profile_read(fmoe_kernel_stat_t* out, int max_entries, int reset);

/* ---- quantisation (mlx::core::quantize / dequantize) ------------------ */

/* MLX-affine quantisation of a row-major [rows, cols] matrix (fp32 when
 * src_is_bf16 == 0, else bf16): per group, scale = (max-min)/(2^bits-1) and
 * bias = min (both rounded to bf16), q = clamp(rint((w-bias)/scale)).
 * Replaces mlx quantize at src/model/mod.rs:673.  bits in {2,3,4,5,6,8}. */
int fmoe_quantize(const void* src, int src_is_bf16, int64_t rows, int64_t cols, int bits,
                  int group_size, void* wq, void* scales, void* biases, void* stream);

/* out bf16 [out, in] = bf16(fma(scale, q, bias)).  Replaces mlx dequantize at
 * src/model/mod.rs:149 and mod.rs:666-670. */
int fmoe_dequantize(const fmoe_qweight_t* w, void* out, void* stream);

/* Embedding lookup: out bf16 [n, in] = dequantize(rows ids[i]) * row_scale.
 * Replaces take + dequantize + (x sqrt(hidden)) at src/model/mod.rs:145-160. */
int fmoe_embed_rows(const fmoe_qweight_t* w, const int32_t* ids, int64_t n, float row_scale,
                    void* out, void* stream);

/* y bf16 [T, out] = x bf16 [T, in] . W^T.  Replaces QuantizedLinear::forward,
 * src/model/mlp.rs:15-25 (mlx quantized_matmul, transpose=true).  Kernels:
 * bits 4, 6 and 8 at T <= 8 (streaming tensor-core GEMV; 16-byte aligned
 * weight, scales and biases), bits 4, 8 and 16 (bf16) at any T, group 64,
 * in % 64 == 0, out % 16 == 0.  The workspace holds fp32 partial sums
 * (fmoe_qlinear_workspace_bytes). */
/* Tile layout of a 4/6/8-bit weight for the decode GEMV: for each 16-row tile
 * and each chunk of kc inputs, the tile's 16 row pieces (kc*bits/8 bytes each)
 * at a padded row stride, contiguous.  fmoe_qgemv_chunk gives the kc the GEMV
 * uses for a launch over rows_total weight rows sharing one input (all the
 * segments of that launch must be tiled with it); accumulate != 0 for launches
 * whose output accumulates split-K slices (the dense MLP, o_proj), 0 otherwise
 * (q|k|v, lm_head).  0: not tileable. */
int32_t fmoe_qgemv_chunk(int32_t in_features, int32_t bits, int64_t rows_total, int32_t accumulate);
size_t fmoe_qweight_tile_bytes(const fmoe_qweight_t* w, int32_t kc);
int fmoe_qweight_tile(const fmoe_qweight_t* w, int32_t kc, void* out, size_t bytes, void* stream);

size_t fmoe_qlinear_workspace_bytes(int64_t T, const fmoe_qweight_t* w);
int fmoe_qlinear(const void* x, int64_t T, const fmoe_qweight_t* w, void* y, void* workspace,
                 size_t workspace_bytes, void* stream);

/* ---- MoE ------------------------------------------------------------ */

/* Router, src/model/moe.rs:324-345.  x bf16 [T, hidden].  Writes ids int32
 * [T, top_k] (global expert ids, descending logit, ties -> lower id) and
 * weights f32 [T, top_k] (softmax over the selected logits, i.e. the
 * renormalised top-k probabilities, times per_expert_scale).  logits (f32
 * [T, num_experts]) may be NULL.  Needs fmoe_router_workspace_bytes(T, r) of
 * workspace that is zero-filled before its first use: the router keeps
 * completion counters there (one fused kernel: logits, top-k, routing lists)
 * and every call leaves them at zero again.  Calls that share a workspace must
 * not overlap on the GPU. */
size_t fmoe_router_workspace_bytes(int64_t T, const fmoe_router_t* r);
int fmoe_router(const void* x, int64_t T, const fmoe_router_t* r, int32_t* ids, float* weights,
                float* logits, void* workspace, size_t workspace_bytes, void* stream);

/* Workspace for fmoe_moe_experts with T tokens (routing lists + the gated
 * intermediate activations); no initialisation needed. */
size_t fmoe_moe_workspace_bytes(int64_t T, int top_k, const fmoe_experts_t* ex);

/* Routed experts + weighted combine, src/model/moe.rs:361-466 (unique/dedup
 * of the selected experts, per-expert 4-bit GELU-gated MLP, weighted sum):
 *   y[t] = sum_j weights[t,j] * down(gelu_tanh(gate.x[t]) * up.x[t]) of expert ids[t,j].
 * x bf16 [T, hidden]; ids int32 [T, top_k] global ids (ids outside the table's
 * [first_expert, first_expert+num_experts) contribute nothing); weights f32;
 * y bf16 [T, hidden].  No host synchronisation. */
int fmoe_moe_experts(const void* x, int64_t T, int top_k, const int32_t* ids, const float* weights,
                     const fmoe_experts_t* ex, void* y, void* workspace, size_t workspace_bytes,
                     void* stream);

/* Gemma4MoeBlock::forward, src/model/moe.rs:315-470: router + experts in one
 * call (3 kernels: fused router + routing lists, gate/up, down + combine).
 * ids / weights (may be NULL) receive the routing.  Workspace:
 * fmoe_moe_block_workspace_bytes, zero-filled before first use (see
 * fmoe_router).  T <= 128 (decode path). */
size_t fmoe_moe_block_workspace_bytes(int64_t T, const fmoe_router_t* r, const fmoe_experts_t* ex);
int fmoe_moe_block_forward(const void* x, int64_t T, const fmoe_router_t* r, const fmoe_experts_t* ex,
                           void* y, int32_t* ids, float* weights, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Variant of fmoe_moe_block_forward for callers that cannot allocate device
 * memory when they run the layer (an engine that gives its whole device budget
 * to its own pool, a plugin host that forbids library allocations, a decode
 * loop that cannot afford cudaMalloc's device synchronisation).  No
 * counterpart in the reference.  Same arguments and results as
 * fmoe_moe_block_forward minus the workspace: the library uses a fixed
 * FMOE_NOALLOC_SCRATCH_BYTES scratch array of its own, in static device memory
 * that every GPU loading the library holds until the process exits.  Calls
 * whose fmoe_moe_block_workspace_bytes exceeds it are rejected with
 * FMOE_ERR_WORKSPACE (for the Gemma-4 shapes: up to 16 tokens).  It calls no
 * cudaMalloc / cudaFree.  The first call on each device looks up the array's
 * device address (cudaGetSymbolAddress); make that first call before any
 * stream capture.  Every call shares the array and clears the part it uses;
 * calls that overlap on the GPU race on it. */
#define FMOE_NOALLOC_SCRATCH_BYTES (4u << 20)
int fmoe_moe_block_forward_noalloc(const void* x, int64_t T, const fmoe_router_t* r,
                                   const fmoe_experts_t* ex, void* y, int32_t* ids, float* weights,
                                   void* stream);
/* Device status word of the no-allocation entry point's scratch array (the
 * fmoe_workspace_status of that array; no counterpart in the reference):
 * FMOE_OK, or FMOE_ERR_TIMEOUT when a bounded device wait in an earlier call
 * gave up (that call's y is then not valid).  The word persists across calls
 * until read with clear != 0.  Synchronises `stream`. */
int fmoe_moe_block_noalloc_status(int clear, void* stream);

/* ---- quantised KV cache + decode attention ---------------------------- */

/* Storage modes of a layer's KV cache.
 *   FMOE_KV_BF16    bf16 rows, the reference's KVCache (src/cache.rs:266-310);
 *                   optionally each appended row passes through the TurboQuant
 *                   round trip first (src/cache.rs:290-308, turbo_bits 2..4).
 *   FMOE_KV_AFFINE  rows rotated by the normalised Walsh-Hadamard transform
 *                   over head_dim, then MLX-affine quantised: K 4-bit, V 8-bit,
 *                   group 64.  No reference counterpart (the benchmark's
 *                   quantised-KV configuration); attention rotates the query the
 *                   same way and returns its output in the original basis.
 * Layout (per array): [batch][kv_heads][capacity][...] row-major; position p
 * of a sequence lives in slot p % capacity (a ring: capacity = sliding window
 * keeps the last `window` positions, src/cache.rs:139-148). */
#define FMOE_KV_BF16 0
#define FMOE_KV_AFFINE 1

typedef struct fmoe_kv_cache {
  int32_t mode;
  int32_t batch;
  int32_t kv_heads;
  int32_t head_dim;   /* 256 or 512 */
  int64_t capacity;   /* slots per (batch, kv head); a multiple of 16 */
  int32_t k_bits;     /* 16 (bf16 mode) or 4 */
  int32_t v_bits;     /* 16 (bf16 mode) or 8 */
  int32_t group_size; /* 64 (affine mode) */
  int32_t turbo_bits; /* bf16 mode: 0, or 2..4: the decoder layer passes each appended
                         K / V row through the TurboQuant round trip first (the
                         reference's quantised cache, src/cache.rs:290-308) */
  void* k;        /* bf16 [.., head_dim], or uint32 codes [.., head_dim/8] */
  void* v;        /* bf16 [.., head_dim], or uint32 codes [.., head_dim/4] */
  void* k_scales; /* affine: bf16 [.., head_dim/64]; NULL in bf16 mode */
  void* k_biases;
  void* v_scales;
  void* v_biases;
} fmoe_kv_cache_t;

/* Bytes of one layer's cache (0 for an unsupported shape), and the carving of
 * a caller buffer of at least that size into *cache (host only, no launch).
 * The contents start undefined; only slots that were appended are read. */
size_t fmoe_kv_cache_bytes(int mode, int batch, int kv_heads, int head_dim, int64_t capacity);
int fmoe_kv_cache_init(fmoe_kv_cache_t* cache, int mode, int batch, int kv_heads, int head_dim,
                       int64_t capacity, void* buffer, size_t buffer_bytes);

/* Append T_new positions: k, v bf16 [batch, kv_heads, T_new, head_dim] for
 * positions pos .. pos+T_new-1 (pos_dev, when not NULL, is a device int64
 * read instead of pos: CUDA-graph friendly).  Replaces the append half of
 * KVCache::update_and_fetch, src/cache.rs:266-310 (the fetch half is the
 * cache itself: attention reads it in place).  turbo_bits 2..4 applies the
 * TurboQuant round trip in bf16 mode; 0 stores the rows as given.  In affine
 * mode rows are rotated and quantised on the way in. */
int fmoe_kv_append(const fmoe_kv_cache_t* cache, const void* k, const void* v, int64_t T_new,
                   int64_t pos, const int64_t* pos_dev, int turbo_bits, void* stream);

/* Decode attention of one query token per sequence over the cache:
 * out[b, h] = softmax(scale * q[b, h] . K^T) . V over the first n_valid slots
 * of kv head h / (q_heads / kv_heads) (GQA), q / out bf16 [batch, q_heads,
 * head_dim].  Replaces fast::scaled_dot_product_attention at
 * src/model/gemma4_attention.rs:95-104 with the causal / sliding masks of
 * src/model/mod.rs:682-753 (all cached slots are attendable: the ring holds
 * exactly the window).  n_valid = min(positions appended, capacity);
 * n_valid_dev (device int64, optional) overrides it at run time.
 * q_heads / kv_heads in {1, 2, 4, 8}.  One kernel (split-KV with an in-kernel
 * merge).  The workspace (fmoe_attn_decode_workspace_bytes) must be
 * zero-filled before first use; each call leaves its merge counters at zero.
 * Calls sharing a workspace must not overlap on the GPU. */
size_t fmoe_attn_decode_workspace_bytes(const fmoe_kv_cache_t* cache, int q_heads);
int fmoe_attn_decode(const fmoe_kv_cache_t* cache, const void* q, int q_heads, int64_t n_valid,
                     const int64_t* n_valid_dev, float scale, void* out, void* workspace,
                     size_t workspace_bytes, void* stream);

/* Sparse-V decode attention, the reference's optional decode path
 * (sparse_v_attention, src/model/gemma4_attention.rs:196-234; threshold flag
 * src/main.rs:62-64): over the first n_valid slots of every sequence's ring,
 * p = softmax(scale * q . K^T); weights p < tau are set to zero (the others
 * are not renormalised); out = p . V.  q / out bf16 [batch, q_heads,
 * head_dim].  tau = 0 gives the dense attention.  bf16-storage caches (with or
 * without the TurboQuant round trip), 1 <= n_valid <= min(capacity, 32768).
 * No workspace; two passes over the keys per (sequence, query head). */
int fmoe_attn_decode_sparse_v(const fmoe_kv_cache_t* cache, const void* q, int q_heads, int64_t n_valid,
                              float scale, float tau, void* out, void* stream);

/* TurboQuant quantise -> dequantise round trip of `rows` bf16 vectors of
 * length head_dim (256 or 512), bits 2..4: turbo_round_trip_kv,
 * src/cache.rs:94-129 (the rotation R = H diag(signs) applied as a fast
 * Walsh-Hadamard transform). */
int fmoe_turbo_round_trip(const void* x, int64_t rows, int head_dim, int bits, void* out,
                          void* stream);

/* ---- decoder layer + lm_head (decode step) ----------------------------- */

/* One Gemma-4 decoder layer, DecoderLayer::forward_gemma4 (src/model/mod.rs:
 * 67-119) with Gemma4Attention (src/model/gemma4_attention.rs:16-112), GeLUMLP
 * (src/model/mlp.rs:28-41) and Gemma4MoeBlock (src/model/moe.rs:298-470).
 * All bf16 norm weights are [hidden] except q_norm / k_norm ([head_dim]).
 * The router's use_norm / root_size / router_scale / eps describe its input
 * chain (rms_norm_no_scale, * root_size, * router_scale) as in fmoe_router. */
typedef struct fmoe_decoder_layer {
  fmoe_qweight_t q_proj, k_proj, v_proj, o_proj; /* v_proj unused when k_eq_v */
  const void* q_norm;
  const void* k_norm;
  const void* input_norm;
  const void* post_attn_norm;
  const void* pre_ff_norm;
  const void* post_ff_norm_1;
  const void* pre_ff_norm_2;
  const void* post_ff_norm_2;
  const void* post_ff_norm;
  fmoe_qweight_t mlp_gate, mlp_up, mlp_down; /* dense GeLU MLP */
  fmoe_router_t router;
  fmoe_experts_t experts;
  int32_t num_heads;
  int32_t num_kv_heads;
  int32_t head_dim;
  int32_t rope_dims;   /* rotated dims (non-traditional RoPE); head_dim * partial factor */
  int32_t k_eq_v;      /* 1: V is the raw K projection (full-attention layers) */
  float sparse_v_tau;  /* > 0: decode attention zeroes softmax weights below it, no
                        * renormalisation (sparse-V gating, gemma4_attention.rs:91-93,
                        * 196-234; bf16 / TurboQuant caches, layered path); 0: off */
  float rope_theta;
  float eps;           /* rms_norm_eps of every norm */
  float layer_scalar;
  float attn_scale;    /* SDPA scale (1.0 in Gemma 4) */
} fmoe_decoder_layer_t;

/* One decode step of a layer for T = cache.batch sequences (1..8; up to 64
 * with every expert local: the attention half then runs per group of 8
 * sequences and the router, routed experts and dense MLP once over all T, the
 * dense MLP on the tensor-core GEMM, so each expert is read once per layer;
 * alternate groups' attention on a second library stream, joined back),
 * one token each, at position pos: x bf16 [T, hidden] is the layer input and receives
 * the layer output.  The new K/V rows go to slot pos % capacity of `cache`;
 * attention covers min(pos + 1, capacity) slots.  pos_dev (optional) points to
 * device int64 {pos, attended slots}, read instead of pos (CUDA-graph replay).
 * Weights: q/k/v/o, dense MLP: 4/6/8-bit, group 64; router as fmoe_router;
 * experts 4-bit.  Workspace: fmoe_decoder_workspace_bytes (the largest over
 * the layers and caches used with it), zero-filled once before first use. */
size_t fmoe_decoder_workspace_bytes(int64_t T, const fmoe_decoder_layer_t* layer,
                                    const fmoe_kv_cache_t* cache);
int fmoe_decoder_layer_forward(const fmoe_decoder_layer_t* layer, const fmoe_kv_cache_t* cache, void* x,
                               int64_t T, int64_t pos, const int64_t* pos_dev, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Prefill of one layer for T prompt tokens of ONE sequence (cache batch 1, or
 * a one-sequence view) at positions pos0 .. pos0 + T - 1: DecoderLayer::
 * forward_gemma4 (src/model/mod.rs:67-119) with l = T.  Attention covers the
 * cached positions and the new ones under the causal mask, and, when
 * window > 0, only positions p - window < j <= p (create_attention_mask /
 * create_sliding_mask, src/model/mod.rs:682-753); the new K/V rows (through
 * the TurboQuant round trip when the cache has it, src/cache.rs:290-308) are
 * appended after attention.  A sliding cache needs capacity >= window; a full
 * one pos0 + T <= capacity.  bf16 caches (with or without TurboQuant) and the
 * rotated affine K4 / V8 cache, whose new rows enter attention as the cache
 * returns them (rotated, quantised, dequantised).  Projections and the
 * dense MLP run on the tensor-core GEMM (4/8-bit, group 64); the routed
 * experts as fmoe_moe_prefill, with expert_prep from fmoe_moe_prefill_prepare.
 * x bf16 [T, hidden] is replaced by the layer output.  Workspace:
 * fmoe_decoder_layer_prefill_workspace_bytes(layer, T), zero-filled once
 * before first use; its first int is the status word (fmoe_workspace_status). */
size_t fmoe_decoder_layer_prefill_workspace_bytes(const fmoe_decoder_layer_t* layer, int64_t T);
int fmoe_decoder_layer_prefill(const fmoe_decoder_layer_t* layer, const fmoe_kv_cache_t* cache, void* x, int64_t T,
                               int64_t pos0, int window, const void* expert_prep, void* workspace,
                               size_t workspace_bytes, void* stream);

/* Prefill attention alone (the step inside fmoe_decoder_layer_prefill): q bf16
 * [T, q_heads, head_dim] (normed, rotated), k_new / v_new bf16 [kv_heads, T,
 * head_dim] the new rows as they will be stored; positions < pos0 are read
 * from the ring.  out bf16 [T, q_heads * head_dim].  The cache is not
 * modified (append the new rows afterwards with fmoe_kv_append).  bf16 caches
 * (the affine cache is prefilled through fmoe_decoder_layer_prefill). */
int fmoe_attn_prefill(const fmoe_kv_cache_t* cache, const void* q, int q_heads, int64_t T, int64_t pos0, int window,
                      const void* k_new, const void* v_new, void* out, float scale, void* stream);

/* GeLUMLP::forward (src/model/mlp.rs:28-41) for T tokens on the tensor-core
 * GEMM: y = down(gelu_tanh(gate(x)) * up(x)), bf16 [T, hidden]; 4/8-bit
 * group-64 weights.  Workspace: fmoe_mlp_workspace_bytes(T, gate). */
size_t fmoe_mlp_workspace_bytes(int64_t T, const fmoe_qweight_t* gate);
int fmoe_mlp_forward(const void* x, int64_t T, const fmoe_qweight_t* gate, const fmoe_qweight_t* up,
                     const fmoe_qweight_t* down, void* y, void* workspace, size_t workspace_bytes, void* stream);

/* Final norm + tied lm_head + logit softcap + greedy next token:
 * TextModel::forward's norm (src/model/mod.rs:254), Model::forward
 * (src/model/mod.rs:336-362): logits f32 [T, vocab] = tanh(l / softcap) *
 * softcap with l = rms_norm(x, final_norm) . embed^T (softcap <= 0: none);
 * next_ids int32 [T] = argmax (ties -> lowest id).  embed: the 4/6/8-bit
 * embedding table [vocab, hidden].  pos_dev (optional): the decode position
 * counters {pos, attended slots}, both advanced by one when the step ends.
 * Workspace: fmoe_lm_head_workspace_bytes, zero-filled once. */
size_t fmoe_lm_head_workspace_bytes(int64_t T);
int fmoe_lm_head(const fmoe_qweight_t* embed, const void* final_norm, float eps, const void* x, int64_t T,
                 float softcap, float* logits, int32_t* next_ids, int64_t* pos_dev, void* workspace,
                 size_t workspace_bytes, void* stream);

/* ---- prefill MoE block (many tokens) -------------------------------------
 * Gemma4MoeBlock::forward (src/model/moe.rs:315-470) for T tokens on the
 * tcgen05 tensor cores: router + top-k as fmoe_moe_block_forward, then grouped
 * 4-bit x bf16 GEMMs over token-sorted expert tiles (gate|up with GELU-tanh
 * gating, down) with fp32 accumulation, and the weighted top-k combine in slot
 * order.  Each expert output is rounded to bf16 before the combine, as the
 * reference's per-expert quantized_matmul output is (moe.rs:438-465).
 * Requirements: hidden a multiple of 256, intermediate a multiple of 64, the
 * whole expert table (first_expert 0), 16-byte aligned tensors.
 * fmoe_moe_prefill_prepare writes a transposed copy of the table's scales and
 * biases ([group][row], fmoe_moe_prefill_prepare_bytes; once per table). */
size_t fmoe_moe_prefill_prepare_bytes(const fmoe_experts_t* experts);
int fmoe_moe_prefill_prepare(const fmoe_experts_t* experts, void* prepared, size_t prepared_bytes, void* stream);
size_t fmoe_moe_prefill_workspace_bytes(int64_t T, const fmoe_router_t* router, const fmoe_experts_t* experts);
int fmoe_moe_prefill(const void* x, int64_t T, const fmoe_router_t* router, const fmoe_experts_t* experts,
                     const void* prepared, void* y, int32_t* ids, float* weights, void* workspace,
                     size_t workspace_bytes, void* stream);

/* The expert stage of fmoe_moe_prefill on given routing (the tensor-core
 * counterpart of fmoe_moe_experts): ids int32 / weights f32 [T, top_k] hold
 * global expert ids; pairs whose id lies outside the table's
 * [first_expert, first_expert + num_experts) contribute nothing, so the table
 * may be one rank's slice.  prepared: fmoe_moe_prefill_prepare of this table. */
size_t fmoe_moe_prefill_experts_workspace_bytes(int64_t T, int top_k, const fmoe_experts_t* experts);
int fmoe_moe_prefill_experts(const void* x, int64_t T, int top_k, const int32_t* ids, const float* weights,
                             const fmoe_experts_t* experts, const void* prepared, void* y, void* workspace,
                             size_t workspace_bytes, void* stream);

/* ---- expert parallelism (one process per GPU, NCCL over NVLink) ----------
 * Not in the reference, which runs on one device (moe.rs:361-466 evaluates
 * every routed expert locally): the E experts of a layer are split
 * contiguously over n_ranks GPUs — rank r passes the fmoe_experts_t of experts
 * [r*E/n, (r+1)*E/n) with first_expert = r*E/n — while router weights are
 * replicated and each rank routes its own T tokens.  One MoE block: router ->
 * dispatch (a token's row, ids and weights cross once to every rank owning
 * one of its experts) -> local experts -> the per-rank partial sums return (fp32) ->
 * y = their sum in ascending rank order.  Transport: grouped ncclSend /
 * ncclRecv from libnccl.so.2, resolved at run time.  Every rank of the
 * communicator must make the same sequence of fmoe_ep_* calls with the same
 * cap and mode (a rank without tokens passes T = 0). */
typedef struct fmoe_ep_comm fmoe_ep_comm_t;

#define FMOE_EP_UNIQUE_ID_BYTES 128
#define FMOE_EP_FIXED 0 /* every rank exchanges cap rows with every rank: no host sync, CUDA-graph capturable */
#define FMOE_EP_EXACT 1 /* counts cross first (one host sync per block), then only the routed rows */
#define FMOE_EP_P2P 2   /* as FIXED, but the rows and partial sums are stored straight into the peers' memory
                           (CUDA IPC over NVLink, flag-synchronised) instead of NCCL send/recv; needs
                           fmoe_ep_p2p_init with the same cap / hidden / top_k */

/* Rank 0 makes the id; the host engine hands it to the other ranks. */
int fmoe_ep_unique_id(void* id, size_t len);
/* Blocking: returns when all n_ranks have joined (current CUDA device). */
int fmoe_ep_comm_init(fmoe_ep_comm_t** comm, int n_ranks, int rank, const void* id, size_t len);
/* Frees comm.  With peer-memory windows (fmoe_ep_p2p_init) it is collective: every
 * rank calls it (two NCCL barriers, so no window is freed while a peer still maps
 * it); after a rank was lost use fmoe_ep_comm_abort instead. */
int fmoe_ep_comm_destroy(fmoe_ep_comm_t* comm);
/* For a host watchdog: ends outstanding NCCL work with an error and frees comm
 * (no collective; peer-memory windows stay allocated until the process exits). */
int fmoe_ep_comm_abort(fmoe_ep_comm_t* comm);
/* FMOE_OK, or FMOE_ERR_NCCL when NCCL has recorded an asynchronous error. */
int fmoe_ep_comm_status(fmoe_ep_comm_t* comm);
/* Collective (all ranks): allocates this rank's exchange window for FMOE_EP_P2P
 * (receive rows, ids, weights and returned partial sums for n_ranks x cap rows;
 * flags) and maps every peer's window into this process.  At most 8 ranks.
 * Released by fmoe_ep_comm_destroy / _abort or a new call (which frees the old
 * windows: destroy any CUDA graph that captured P2P exchanges on them first).  Waits on peers'
 * flags are bounded: a timeout ends with FMOE_ERR_TIMEOUT in the workspace
 * status word. */
int fmoe_ep_p2p_init(fmoe_ep_comm_t* comm, int64_t cap, int hidden, int top_k);

/* cap: the largest T any rank passes (FIXED exchanges cap rows per peer).
 * Received rows are served by the decode expert kernels up to 128 rows, by the
 * tensor-core path above (prepared = fmoe_moe_prefill_prepare of the local
 * slice; required when n_ranks * cap > 128).  ids / weights (optional) receive
 * this rank's routing.  Workspace: zero-filled once before first use. */
size_t fmoe_ep_moe_workspace_bytes(int n_ranks, int64_t cap, const fmoe_router_t* router,
                                   const fmoe_experts_t* local);
int fmoe_ep_moe_forward(fmoe_ep_comm_t* comm, const void* x, int64_t T, int64_t cap, const fmoe_router_t* router,
                        const fmoe_experts_t* local, const void* prepared, void* y, int32_t* ids, float* weights,
                        int mode, void* workspace, size_t workspace_bytes, void* stream);

/* fmoe_decoder_layer_prefill with layer->experts being this rank's slice: the
 * routed experts run through fmoe_ep_moe_forward (FMOE_EP_EXACT, cap = T),
 * everything else on this rank.  Collective: every rank calls it for every
 * layer with the same T (each with its own sequence and cache).  expert_prep:
 * fmoe_moe_prefill_prepare of the local slice.  Workspace:
 * fmoe_decoder_layer_prefill_ep_workspace_bytes, zero-filled once. */
size_t fmoe_decoder_layer_prefill_ep_workspace_bytes(const fmoe_decoder_layer_t* layer, int64_t T, int n_ranks);
int fmoe_decoder_layer_prefill_ep(const fmoe_decoder_layer_t* layer, const fmoe_kv_cache_t* cache,
                                  fmoe_ep_comm_t* comm, void* x, int64_t T, int64_t pos0, int window,
                                  const void* expert_prep, void* workspace, size_t workspace_bytes, void* stream);

/* fmoe_decoder_layer_forward with layer->experts being this rank's slice: the
 * routed experts of the MoE block run on their owning ranks as in
 * fmoe_ep_moe_forward (cap >= T on every rank; prepared as there).  Attention,
 * dense MLP and router stay local. */
size_t fmoe_decoder_ep_workspace_bytes(int64_t T, const fmoe_decoder_layer_t* layer, const fmoe_kv_cache_t* cache,
                                       int n_ranks, int64_t cap);
int fmoe_decoder_layer_forward_ep(const fmoe_decoder_layer_t* layer, const fmoe_kv_cache_t* cache,
                                  fmoe_ep_comm_t* comm, int64_t cap, const void* prepared, int mode, void* x,
                                  int64_t T, int64_t pos, const int64_t* pos_dev, void* workspace,
                                  size_t workspace_bytes, void* stream);

/* ---- whole decode step (batch 1) ----------------------------------------
 * One persistent kernel per generated token: embedding row, every decoder
 * layer (as fmoe_decoder_layer_forward), final norm, tied lm_head, softcap and
 * greedy argmax — Model::forward for one sequence and one token
 * (src/model/mod.rs:145-160, 67-119, 254, 336-362; the per-layer eval
 * barriers of mod.rs:214,244 and moe.rs:356 disappear).  Requirements: bf16
 * KV caches of batch 1; q/k/v/o 8-bit, dense MLP and experts 4-bit, embedding
 * 6-bit (all group 64), bf16 router with use_norm; layers share the hidden,
 * MLP and expert shapes. */
typedef struct fmoe_decode_model {
  int32_t n_layers;
  int32_t reserved;
  const fmoe_decoder_layer_t* layers; /* host array [n_layers] */
  const fmoe_kv_cache_t* caches;      /* host array [n_layers] */
  fmoe_qweight_t embed;               /* tied embedding / lm_head [vocab, hidden] */
  const void* final_norm;             /* bf16 [hidden] */
  float eps;                          /* final norm eps */
  float softcap;                      /* logit softcap (<= 0: none) */
  float embed_scale;                  /* sqrt(hidden) */
} fmoe_decode_model_t;

/* Workspace bytes (0: unsupported model).  fmoe_decode_step_prepare writes the
 * device copy of the model description into the workspace (synchronous; call
 * again whenever a weight or cache pointer changes). */
size_t fmoe_decode_step_workspace_bytes(const fmoe_decode_model_t* model);
int fmoe_decode_step_prepare(const fmoe_decode_model_t* model, void* workspace, size_t workspace_bytes);

/* One step: tokens int32 [1] holds the current token and receives the next
 * one; logits f32 [vocab] (after softcap); pos_dev int64 {position, attended
 * slots} is read for the KV slot / context length and advanced by one.  The
 * launch is capturable in a CUDA graph (a memset node + a cooperative kernel
 * node).  Device-side waits are bounded: a lost dependency ends the step with
 * FMOE_ERR_TIMEOUT in the workspace status word (fmoe_workspace_status). */
int fmoe_decode_step(const fmoe_decode_model_t* model, int32_t* tokens, float* logits, int64_t* pos_dev,
                     void* workspace, size_t workspace_bytes, void* stream);

/* Synchronises `stream` and reads the status word every workspace starts with:
 * FMOE_OK, or FMOE_ERR_TIMEOUT when a kernel's bounded wait on an async copy
 * gave up (fmoe_last_error names the site); clear != 0 resets the word. */
int fmoe_workspace_status(const void* workspace, int clear, void* stream);

/* Self-test of the bounded device waits (no counterpart in the reference):
 * runs the expert-parallel exchange's flag wait (a few hundred milliseconds of
 * polling at most) on a flag in `workspace` (>= 512 bytes, 16-byte aligned,
 * its header cleared here) that holds `flag_value` (0: nothing ever sets it,
 * so the wait runs out; 1: it is already set).  Returns the launch status; a
 * following fmoe_workspace_status reports FMOE_ERR_TIMEOUT after a wait that
 * ran out, FMOE_OK otherwise, and the context stays usable either way. */
int fmoe_wait_selftest(void* workspace, size_t workspace_bytes, int flag_value, void* stream);

/* ---- next-token sampling on the device (the engine's sample(), src/engine.rs:302-355) ----
 * logits: [rows, vocab] fp32 on the device (fmoe_lm_head's output).  Per row:
 *   repetition penalty (rep_penalty > 1 and n_recent > 0): every distinct token of
 *     recent[row, 0..n_recent) inside [0, vocab) once: logit >= 0 divided by the
 *     penalty, negative multiplied (entries < 0 or >= vocab are ignored: empty slots);
 *   temperature 0: out = argmax (first maximum);
 *   else z = logits / temperature; top_p < 1: in descending order (ties in token
 *     order) a token is dropped when (running sum of softmax(z)) - p > top_p;
 *     a categorical draw with P(token) proportional to p' + 1e-10, p' = softmax over the
 *     kept tokens (0 for dropped ones), as the Gumbel-max argmax of (p' + 1e-10) / E,
 *     E = -log(u), u = (k + 0.5) / 2^23, k = top 23 bits of a splitmix64 hash keyed by
 *     (seed, call number, row, token) — reproducible on the host.
 * step_dev: device uint64 call number (null: 0), advanced by one per call, so a CUDA
 * graph replays fresh draws.  push_recent != 0 (needs step_dev): the drawn token is
 * stored into recent[row, call number % n_recent] (a ring of the last n_recent tokens;
 * fill it with -1 first).  n_recent <= 4096; rows <= 65535; rows * vocab < 2^31.
 * Capturable in a CUDA graph (no host sync). */
size_t fmoe_sample_workspace_bytes(int64_t rows, int64_t vocab);
int fmoe_sample(const float* logits, int64_t rows, int64_t vocab, int32_t* recent, int n_recent,
                float temperature, float top_p, float rep_penalty, uint64_t seed, uint64_t* step_dev,
                int push_recent, int32_t* out, void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FMOE_H_ */
