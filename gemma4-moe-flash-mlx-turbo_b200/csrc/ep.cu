// Expert parallelism: the experts of a MoE layer split contiguously over the
// GPUs of one box, one process per GPU, tokens exchanged over NVLink by NCCL.
//
// The reference runs on one device (Gemma4MoeBlock::forward,
// src/model/moe.rs:315-470, evaluates every routed expert locally).  Here rank
// r of n holds experts [r*E/n, (r+1)*E/n); router weights are replicated and
// every rank routes its own tokens.  Per MoE block:
//   plan     one CTA per destination rank: slot of token t in rank r's block =
//            number of earlier tokens with an expert on r, -1 if none (a token
//            crosses to a rank once, however many of its experts live there)
//   pack     token rows + their full id / weight rows into per-rank blocks
//   dispatch grouped ncclSend / ncclRecv (FIXED: every block is cap rows, no
//            host sync, capturable in a CUDA graph; EXACT: counts first, one
//            host sync, then only routed rows cross)
//   experts  the local slice over the received rows (ids outside the slice
//            contribute nothing): decode GEMV kernels up to 128 rows, the
//            tcgen05 grouped GEMMs above
//   return   the per-rank partial sums travel back the same way, in fp32 (the
//            sum over all experts is accumulated in fp32 end to end)
//   combine  y[t] = sum over ranks, ascending, of the partial at slots[r][t]
//            (fp32 accumulation; rank order = ascending expert-id order of
//            the reference's combine, moe.rs:443-465)
// NCCL is resolved from libnccl.so.2 at run time (the copy the host process
// already loaded when there is one), so the library loads without it.
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstring>
#include <cstdio>
#include <mutex>
#include <vector>

#include "common.cuh"
#include "internal.h"

struct fmoe_ep_comm {
  ncclComm_t nc;
  int n_ranks;
  int rank;
  int device;
  int32_t* host_counts;  // pinned [2 * n_ranks]: send counts | receive counts (EXACT mode)
  // peer-memory exchange (fmoe_ep_p2p_init): every rank's window mapped here
  uint8_t* win = nullptr;
  uint8_t* peer_win[8] = {};
  int64_t p2p_cap = 0;
  int p2p_hidden = 0, p2p_k = 0;
  uint32_t* seq = nullptr;     // device: exchanges completed
  unsigned* done = nullptr;    // device [3]: finished CTAs of the dispatch / return / combine kernels
};

namespace fmoe {
namespace ep {

constexpr int kPlanThreads = 1024;
constexpr int kGemvRows = 128;  // rows the decode expert kernels serve per call

__global__ void __launch_bounds__(kPlanThreads) plan_kernel(const int32_t* __restrict__ ids, int T, int k,
                                                             int per_rank, int cap, int32_t* __restrict__ slots,
                                                             int32_t* __restrict__ counts) {
  __shared__ int wsum[kPlanThreads / 32];
  const int r = blockIdx.x, lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
  const int lo = r * per_rank, hi = lo + per_rank;
  int run = 0;
  for (int t0 = 0; t0 < T; t0 += blockDim.x) {
    const int t = t0 + threadIdx.x;
    bool f = false;
    if (t < T)
      for (int j = 0; j < k; ++j) {
        const int e = ids[(int64_t)t * k + j];
        f |= (e >= lo && e < hi);
      }
    const unsigned m = __ballot_sync(0xffffffffu, f);
    if (lane == 0) wsum[warp] = __popc(m);
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < nw; ++w) {
      const int c = wsum[w];
      before += w < warp ? c : 0;
      total += c;
    }
    if (t < T) slots[(int64_t)r * cap + t] = f ? run + before + __popc(m & ((1u << lane) - 1u)) : -1;
    run += total;
    __syncthreads();
  }
  if (threadIdx.x == 0) counts[r] = run;
}

// Block r of the send buffers holds the rows of the tokens routed to rank r in
// slot order; rows from counts[r] to cap carry ids -1 (they select no expert).
__global__ void pack_kernel(const bf16* __restrict__ x, const int32_t* __restrict__ ids,
                            const float* __restrict__ wts, const int32_t* __restrict__ slots,
                            const int32_t* __restrict__ counts, int T, int k, int H, int R, int cap,
                            bf16* __restrict__ sx, int32_t* __restrict__ sids, float* __restrict__ swts) {
  const int words = H / 8;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t n = (int64_t)R * T * words;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int r = (int)(i / ((int64_t)T * words));
    const int rem = (int)(i % ((int64_t)T * words));
    const int t = rem / words, w = rem % words;
    const int s = slots[(int64_t)r * cap + t];
    if (s < 0) continue;
    const int64_t row = (int64_t)r * cap + s;
    *reinterpret_cast<uint4*>(sx + row * H + 8 * w) = *reinterpret_cast<const uint4*>(x + (int64_t)t * H + 8 * w);
    if (w < k) {  // k <= H / 8 (checked on the host)
      sids[row * k + w] = ids[(int64_t)t * k + w];
      swts[row * k + w] = wts[(int64_t)t * k + w];
    }
  }
  const int64_t m = (int64_t)R * cap * k;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < m; i += stride) {
    const int r = (int)(i / ((int64_t)cap * k));
    const int j = (int)((i % ((int64_t)cap * k)) / k);
    if (j >= counts[r]) {
      sids[i] = -1;
      swts[i] = 0.f;
    }
  }
}

// y[t] = bf16(sum over r ascending of ret[r][slots[r][t]]), fp32 partials and sums.
__global__ void combine_kernel(const float* __restrict__ ret, const int32_t* __restrict__ slots, int T, int R, int cap,
                               int H, bf16* __restrict__ y) {
  const int words = H / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)T * words;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / words), w = (int)(i % words);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < R; ++r) {
      const int s = slots[(int64_t)r * cap + t];
      if (s < 0) continue;
      const float4* v = reinterpret_cast<const float4*>(ret + ((int64_t)r * cap + s) * H + 8 * w);
      const float4 a = v[0], b = v[1];
      acc[0] += a.x;
      acc[1] += a.y;
      acc[2] += a.z;
      acc[3] += a.w;
      acc[4] += b.x;
      acc[5] += b.y;
      acc[6] += b.z;
      acc[7] += b.w;
    }
    *reinterpret_cast<uint4*>(y + (int64_t)t * H + 8 * w) =
        make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                   pack_bf16x2(acc[6], acc[7]));
  }
}

// ---------------------------------------------------------------------------
// Peer-memory exchange (FMOE_EP_P2P): every rank owns a window mapped into the
// others (CUDA IPC over NVLink).  The dispatch kernel stores each routed row
// straight into the owning rank's window (block `me` of its receive rows, at
// the token's slot) — pack and send in one pass; the return kernel stores the
// fp32 partial sums into the source rank's window.  The last CTA of each
// publishes a flag per destination (system-scope release after a system fence);
// the receiver's wait kernel polls its flags (acquire, bounded) before the
// expert kernels read the rows.  Flags carry the exchange number (device
// counter `seq`), so nothing is reset between exchanges, and a CUDA graph can
// replay the sequence.  Plain stores only (no TMA, no multicast).

struct WinLayout {
  size_t rx_flag, ret_flag, rx_cnt, rx, rids, rwts, ret, bytes;
};
__host__ __device__ inline size_t al256(size_t v) { return (v + 255) & ~size_t(255); }
inline WinLayout win_layout(int R, int64_t cap, int H, int k) {
  WinLayout L;
  size_t o = 0;
  L.rx_flag = o;
  o += 256;
  L.ret_flag = o;
  o += 256;
  L.rx_cnt = o;  // int32 [8]: rows each source rank routed here
  o += 256;
  L.rx = o;
  o = al256(o + (size_t)R * cap * H * 2);
  L.rids = o;
  o = al256(o + (size_t)R * cap * k * 4);
  L.rwts = o;
  o = al256(o + (size_t)R * cap * k * 4);
  L.ret = o;
  o = al256(o + (size_t)R * cap * H * 4);
  L.bytes = o;
  return L;
}
struct PeerWins {
  uint8_t* w[8];
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;\n" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];\n" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// The last CTA (device counter `done`, reset by it) publishes seq + 1 in the
// flag slot `me` of every rank's window at byte offset `flag_off`.
__device__ __forceinline__ void publish_flags(const PeerWins& pw, size_t flag_off, int R, int me,
                                              const uint32_t* seq, unsigned* done) {
  __shared__ int s_last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (!s_last) return;
  __threadfence_system();
  const uint32_t v = *reinterpret_cast<const volatile uint32_t*>(seq) + 1;
  if (threadIdx.x < R) st_release_sys(reinterpret_cast<uint32_t*>(pw.w[threadIdx.x] + flag_off) + me, v);
  if (threadIdx.x == 0) *done = 0;
}

__global__ void p2p_dispatch_kernel(const bf16* __restrict__ x, const int32_t* __restrict__ ids,
                                    const float* __restrict__ wts, const int32_t* __restrict__ slots,
                                    const int32_t* __restrict__ counts, int T, int k, int H, int R, int cap, int me,
                                    PeerWins pw, WinLayout L, const uint32_t* seq, unsigned* done) {
  const int words = H / 8;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t n = (int64_t)R * T * words;
  if (blockIdx.x == 0 && threadIdx.x < R)
    reinterpret_cast<int32_t*>(pw.w[threadIdx.x] + L.rx_cnt)[me] = counts[threadIdx.x];
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += stride) {
    const int r = (int)(i / ((int64_t)T * words));
    const int rem = (int)(i % ((int64_t)T * words));
    const int t = rem / words, w = rem % words;
    const int s = slots[(int64_t)r * cap + t];
    if (s < 0) continue;
    const int64_t row = (int64_t)me * cap + s;
    uint8_t* win = pw.w[r];
    *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(win + L.rx) + row * H + 8 * w) =
        *reinterpret_cast<const uint4*>(x + (int64_t)t * H + 8 * w);
    if (w < k) {
      reinterpret_cast<int32_t*>(win + L.rids)[row * k + w] = ids[(int64_t)t * k + w];
      reinterpret_cast<float*>(win + L.rwts)[row * k + w] = wts[(int64_t)t * k + w];
    }
  }
  const int64_t m = (int64_t)R * cap * k;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < m; i += stride) {
    const int r = (int)(i / ((int64_t)cap * k));
    const int j = (int)((i % ((int64_t)cap * k)) / k), c = (int)(i % k);
    if (j >= counts[r]) {
      const int64_t o = ((int64_t)me * cap + j) * k + c;
      reinterpret_cast<int32_t*>(pw.w[r] + L.rids)[o] = -1;
      reinterpret_cast<float*>(pw.w[r] + L.rwts)[o] = 0.f;
    }
  }
  publish_flags(pw, L.rx_flag, R, me, seq, done);
}

// Decode-sized exchanges (R * T <= kP2pPlanSlots): every CTA forms the routing
// plan of plan_kernel in shared memory (for each destination rank, its tokens'
// slots in token order) instead of reading it from a separate launch; CTA 0
// also stores it for the combine.  The stores and flags are those of
// p2p_dispatch_kernel.
constexpr int kP2pThreads = 256;
constexpr int kP2pPlanSlots = 4096;
__global__ void __launch_bounds__(kP2pThreads) p2p_plan_dispatch_kernel(
    const bf16* __restrict__ x, const int32_t* __restrict__ ids, const float* __restrict__ wts, int T, int k, int H,
    int R, int cap, int per_rank, int me, int32_t* __restrict__ slots, int32_t* __restrict__ counts, PeerWins pw,
    WinLayout L, const uint32_t* seq, unsigned* done) {
  __shared__ int s_slot[kP2pPlanSlots];
  __shared__ int s_cnt[8];
  __shared__ int wsum[kP2pThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  for (int r = 0; r < R; ++r) {
    const int lo = r * per_rank, hi = lo + per_rank;
    int run = 0;
    for (int t0 = 0; t0 < T; t0 += kP2pThreads) {
      const int t = t0 + threadIdx.x;
      bool f = false;
      if (t < T)
        for (int j = 0; j < k; ++j) {
          const int e = ids[(int64_t)t * k + j];
          f |= (e >= lo && e < hi);
        }
      const unsigned m = __ballot_sync(0xffffffffu, f);
      if (lane == 0) wsum[warp] = __popc(m);
      __syncthreads();
      int before = 0, total = 0;
#pragma unroll
      for (int w = 0; w < kP2pThreads / 32; ++w) {
        const int c = wsum[w];
        before += w < warp ? c : 0;
        total += c;
      }
      if (t < T) s_slot[r * T + t] = f ? run + before + __popc(m & ((1u << lane) - 1u)) : -1;
      run += total;
      __syncthreads();
    }
    if (threadIdx.x == 0) s_cnt[r] = run;
  }
  __syncthreads();
  if (blockIdx.x == 0) {
    for (int i = threadIdx.x; i < R * T; i += kP2pThreads) slots[(int64_t)(i / T) * cap + i % T] = s_slot[i];
    if (threadIdx.x < R) {
      counts[threadIdx.x] = s_cnt[threadIdx.x];
      reinterpret_cast<int32_t*>(pw.w[threadIdx.x] + L.rx_cnt)[me] = s_cnt[threadIdx.x];
    }
  }
  const int words = H / 8;
  const int64_t stride = (int64_t)gridDim.x * kP2pThreads;
  const int64_t n = (int64_t)R * T * words;
  for (int64_t i = (int64_t)blockIdx.x * kP2pThreads + threadIdx.x; i < n; i += stride) {
    const int r = (int)(i / ((int64_t)T * words));
    const int rem = (int)(i % ((int64_t)T * words));
    const int t = rem / words, w = rem % words;
    const int s = s_slot[r * T + t];
    if (s < 0) continue;
    const int64_t row = (int64_t)me * cap + s;
    uint8_t* win = pw.w[r];
    *reinterpret_cast<uint4*>(reinterpret_cast<bf16*>(win + L.rx) + row * H + 8 * w) =
        *reinterpret_cast<const uint4*>(x + (int64_t)t * H + 8 * w);
    if (w < k) {
      reinterpret_cast<int32_t*>(win + L.rids)[row * k + w] = ids[(int64_t)t * k + w];
      reinterpret_cast<float*>(win + L.rwts)[row * k + w] = wts[(int64_t)t * k + w];
    }
  }
  const int64_t m = (int64_t)R * cap * k;
  for (int64_t i = (int64_t)blockIdx.x * kP2pThreads + threadIdx.x; i < m; i += stride) {
    const int r = (int)(i / ((int64_t)cap * k));
    const int j = (int)((i % ((int64_t)cap * k)) / k), c = (int)(i % k);
    if (j >= s_cnt[r]) {
      const int64_t o = ((int64_t)me * cap + j) * k + c;
      reinterpret_cast<int32_t*>(pw.w[r] + L.rids)[o] = -1;
      reinterpret_cast<float*>(pw.w[r] + L.rwts)[o] = 0.f;
    }
  }
  publish_flags(pw, L.rx_flag, R, me, seq, done);
}

// Partial sums of the rows received from rank r (block r of ypart, its first
// rx_cnt[r] rows) go to block `me` of r's returned rows.
__global__ void p2p_return_kernel(const float* __restrict__ ypart, int R, int cap, int H, int me, PeerWins pw,
                                  WinLayout L, const uint32_t* seq, unsigned* done) {
  const int q4 = H / 4;
  const int64_t n = (int64_t)R * cap * q4;
  const int32_t* cnt = reinterpret_cast<const int32_t*>(pw.w[me] + L.rx_cnt);
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / ((int64_t)cap * q4));
    const int64_t rem = i % ((int64_t)cap * q4);
    const int row = (int)(rem / q4), c = (int)(rem % q4);
    if (row >= cnt[r]) continue;
    reinterpret_cast<float4*>(reinterpret_cast<float*>(pw.w[r] + L.ret) + ((int64_t)me * cap + row) * H)[c] =
        reinterpret_cast<const float4*>(ypart + ((int64_t)r * cap + row) * H)[c];
  }
  publish_flags(pw, L.ret_flag, R, me, seq, done);
}

// One warp: lane r waits until flag r reaches seq + 1 (bounded; a timeout sets
// *status).  advance != 0: then seq = seq + 1 (the exchange is complete).
constexpr int kP2pPolls = 1 << 22;
// Polls one flag until it reaches target (acquire, bounded); false on timeout.
__device__ __forceinline__ bool poll_flag(const uint32_t* f, uint32_t target) {
  int it = 0;
  while ((int32_t)(ld_acquire_sys(f) - target) < 0) {
    if (++it > kP2pPolls) return false;
    __nanosleep(64);
  }
  return true;
}

__global__ void p2p_wait_kernel(const uint8_t* win, size_t flag_off, int R, uint32_t* seq, int advance, int* status,
                                int site) {
  const int lane = threadIdx.x;
  const uint32_t target = *reinterpret_cast<volatile uint32_t*>(seq) + 1;
  bool ok = true;
  if (lane < R) ok = poll_flag(reinterpret_cast<const uint32_t*>(win + flag_off) + lane, target);
  if (!ok) atomicCAS(status, 0, site);
  __syncwarp();
  if (advance && lane == 0) *seq = target;
}

// The return wait and the combine in one launch: threads r < R of every CTA
// wait for rank r's return flag (bounded, as p2p_wait_kernel), then the CTA
// sums its rows as combine_kernel does, reading the returned partials from L2
// (peer stores land there).  The last CTA to finish advances seq (the
// exchange is complete) and resets its counter.
__global__ void __launch_bounds__(kP2pThreads) p2p_combine_kernel(const uint8_t* win, size_t flag_off,
                                                                  size_t ret_off, const int32_t* __restrict__ slots,
                                                                  int T, int R, int cap, int H,
                                                                  bf16* __restrict__ y, uint32_t* seq,
                                                                  unsigned* done, int* status, int site) {
  __shared__ uint32_t s_target;
  __shared__ int s_last;
  if (threadIdx.x == 0) s_target = *reinterpret_cast<volatile uint32_t*>(seq) + 1;
  __syncthreads();
  const uint32_t target = s_target;
  if (threadIdx.x < R && !poll_flag(reinterpret_cast<const uint32_t*>(win + flag_off) + threadIdx.x, target))
    atomicCAS(status, 0, site);
  __syncthreads();
  const float* ret = reinterpret_cast<const float*>(win + ret_off);
  const int words = H / 8;
  for (int64_t i = (int64_t)blockIdx.x * kP2pThreads + threadIdx.x; i < (int64_t)T * words;
       i += (int64_t)gridDim.x * kP2pThreads) {
    const int t = (int)(i / words), w = (int)(i % words);
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int r = 0; r < R; ++r) {
      const int s = slots[(int64_t)r * cap + t];
      if (s < 0) continue;
      const float4* v = reinterpret_cast<const float4*>(ret + ((int64_t)r * cap + s) * H + 8 * w);
      const float4 a = __ldcg(v), b = __ldcg(v + 1);
      acc[0] += a.x;
      acc[1] += a.y;
      acc[2] += a.z;
      acc[3] += a.w;
      acc[4] += b.x;
      acc[5] += b.y;
      acc[6] += b.z;
      acc[7] += b.w;
    }
    *reinterpret_cast<uint4*>(y + (int64_t)t * H + 8 * w) =
        make_uint4(pack_bf16x2(acc[0], acc[1]), pack_bf16x2(acc[2], acc[3]), pack_bf16x2(acc[4], acc[5]),
                   pack_bf16x2(acc[6], acc[7]));
  }
  __syncthreads();
  if (threadIdx.x == 0) s_last = atomicAdd(done, 1u) == gridDim.x - 1;
  __syncthreads();
  if (s_last && threadIdx.x == 0) {
    *seq = target;
    *done = 0;
  }
}

// ---------------------------------------------------------------------------
// NCCL, resolved at run time

struct NcclApi {
  decltype(&ncclGetUniqueId) get_unique_id = nullptr;
  decltype(&ncclCommInitRank) comm_init_rank = nullptr;
  decltype(&ncclCommDestroy) comm_destroy = nullptr;
  decltype(&ncclCommAbort) comm_abort = nullptr;
  decltype(&ncclCommGetAsyncError) comm_async_error = nullptr;
  decltype(&ncclGroupStart) group_start = nullptr;
  decltype(&ncclGroupEnd) group_end = nullptr;
  decltype(&ncclSend) send = nullptr;
  decltype(&ncclRecv) recv = nullptr;
  decltype(&ncclGetErrorString) error_string = nullptr;
  decltype(&ncclAllGather) all_gather = nullptr;
};

const NcclApi* nccl() {
  static NcclApi api;
  static bool ok = false;
  static std::once_flag once;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
#define FMOE_NCCL_SYM(field, name)                                   \
  api.field = reinterpret_cast<decltype(api.field)>(dlsym(h, name)); \
  if (!api.field) return;
    FMOE_NCCL_SYM(get_unique_id, "ncclGetUniqueId")
    FMOE_NCCL_SYM(comm_init_rank, "ncclCommInitRank")
    FMOE_NCCL_SYM(comm_destroy, "ncclCommDestroy")
    FMOE_NCCL_SYM(comm_abort, "ncclCommAbort")
    FMOE_NCCL_SYM(comm_async_error, "ncclCommGetAsyncError")
    FMOE_NCCL_SYM(group_start, "ncclGroupStart")
    FMOE_NCCL_SYM(group_end, "ncclGroupEnd")
    FMOE_NCCL_SYM(send, "ncclSend")
    FMOE_NCCL_SYM(recv, "ncclRecv")
    FMOE_NCCL_SYM(error_string, "ncclGetErrorString")
    FMOE_NCCL_SYM(all_gather, "ncclAllGather")
#undef FMOE_NCCL_SYM
    ok = true;
  });
  return ok ? &api : nullptr;
}

int nccl_error(const NcclApi* api, ncclResult_t r, const char* what) {
  return set_error(FMOE_ERR_NCCL, "ep: %s: %s", what, api->error_string(r));
}

// One grouped exchange: to every peer p, send sbytes[p] bytes at sptr[p] and
// receive rbytes[p] bytes into rptr[p], for each of up to three buffers.
struct Xfer {
  const void* sptr[3];
  void* rptr[3];
  size_t sbytes[3], rbytes[3];
};

int exchange(const fmoe_ep_comm* c, const std::vector<Xfer>& peers, int nbuf, cudaStream_t st, const char* what) {
  const NcclApi* api = nccl();
  ncclResult_t r = api->group_start();
  if (r != ncclSuccess) return nccl_error(api, r, what);
  ncclResult_t first = ncclSuccess;
  for (int p = 0; p < c->n_ranks; ++p)
    for (int b = 0; b < nbuf; ++b) {
      const Xfer& x = peers[p];
      if (x.sbytes[b] && (r = api->send(x.sptr[b], x.sbytes[b], ncclUint8, p, c->nc, st)) != ncclSuccess &&
          first == ncclSuccess)
        first = r;
      if (x.rbytes[b] && (r = api->recv(x.rptr[b], x.rbytes[b], ncclUint8, p, c->nc, st)) != ncclSuccess &&
          first == ncclSuccess)
        first = r;
    }
  r = api->group_end();
  if (first != ncclSuccess) return nccl_error(api, first, what);
  if (r != ncclSuccess) return nccl_error(api, r, what);
  return FMOE_OK;
}

}  // namespace ep

size_t carve_ep(Carver& c, int R, int64_t cap, const fmoe_router_t* r, int k, const ExpertsDev& d, const WsHead& h,
                EpWs* w) {
  using ep::kGemvRows;
  EpWs e;
  const int64_t rows = (int64_t)R * cap;
  if (r) carve_router(c, cap, r, h, &e.rw);
  e.ids = c.take<int32_t>((size_t)cap * k);
  e.wts = c.take<float>((size_t)cap * k);
  e.slots = c.take<int32_t>((size_t)rows);
  e.counts = c.take<int32_t>(R);
  e.rcounts = c.take<int32_t>(R);
  e.sx = c.take<bf16>((size_t)rows * d.H);
  e.sids = c.take<int32_t>((size_t)rows * k);
  e.swts = c.take<float>((size_t)rows * k);
  e.rx = c.take<bf16>((size_t)rows * d.H);
  e.rids = c.take<int32_t>((size_t)rows * k);
  e.rwts = c.take<float>((size_t)rows * k);
  e.ypart = c.take<float>((size_t)rows * d.H);
  e.ret = c.take<float>((size_t)rows * d.H);
  carve_moe(c, std::min<int64_t>(rows, kGemvRows), k, d, &e.mw);
  e.gemm = rows > kGemvRows;
  if (e.gemm) carve_pf_ex(c, rows, k, d, &e.pw);
  if (w) *w = e;
  return c.off;
}

int ep_comm_ranks(const fmoe_ep_comm* c) { return c ? c->n_ranks : 0; }

int ep_check(const fmoe_ep_comm* c, const ExpertsDev& d, int E_total, int* n_ranks) {
  if (!c || !c->nc) return set_error(FMOE_ERR_INVALID, "ep: null communicator");
  if (E_total % c->n_ranks || d.E != E_total / c->n_ranks || d.first != c->rank * d.E)
    return set_error(FMOE_ERR_INVALID, "ep: rank %d of %d must hold experts [%d, %d) of %d (table: %d from %d)",
                     c->rank, c->n_ranks, c->rank * (E_total / std::max(c->n_ranks, 1)),
                     (c->rank + 1) * (E_total / std::max(c->n_ranks, 1)), E_total, d.E, d.first);
  if (!ep::nccl()) return set_error(FMOE_ERR_NCCL, "ep: libnccl.so.2 not found");
  if (n_ranks) *n_ranks = c->n_ranks;
  return FMOE_OK;
}

// Dispatch -> local experts -> return -> combine for T routed tokens (ids /
// wts [T, k], global expert ids).  Shared by the MoE-block and decoder-layer
// entry points.
int ep_experts(const fmoe_ep_comm* c, const bf16* x, int64_t T, int64_t cap, int k, const int32_t* ids,
               const float* wts, const ExpertsDev& d, const bf16* prep, bf16* y, const EpWs& w, int mode,
               int* status, cudaStream_t st) {
  using namespace ep;
  const int R = c->n_ranks;
  const int H = d.H;
  int rc;
  if (T > cap) return set_error(FMOE_ERR_INVALID, "ep: T=%lld above the exchange capacity %lld", (long long)T,
                                (long long)cap);
  if (mode != FMOE_EP_FIXED && mode != FMOE_EP_EXACT && mode != FMOE_EP_P2P)
    return set_error(FMOE_ERR_INVALID, "ep: mode %d", mode);
  if (mode == FMOE_EP_P2P && (!c->win || c->p2p_cap != cap || c->p2p_hidden != H || c->p2p_k != k))
    return set_error(FMOE_ERR_INVALID, "ep: peer-memory exchange not set up for cap %lld, hidden %d, top_k %d "
                     "(fmoe_ep_p2p_init)", (long long)cap, H, k);
  if (mode == FMOE_EP_EXACT) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    cudaStreamIsCapturing(st, &cs);
    if (cs != cudaStreamCaptureStatusNone)
      return set_error(FMOE_ERR_INVALID, "ep: EXACT mode synchronises on the host and cannot be captured");
  }
  const bool fused_plan = mode == FMOE_EP_P2P && (int64_t)R * T <= kP2pPlanSlots;
  if (!fused_plan) {
    ProfScope prof_("ep_plan_kernel", st);
    plan_kernel<<<R, kPlanThreads, 0, st>>>(ids, (int)T, k, d.E, (int)cap, w.slots, w.counts);
  }
  if (!fused_plan && (rc = check_launch("ep_plan_kernel"))) return rc;
  if (mode == FMOE_EP_P2P) {  // dispatch and return through the peers' windows
    PeerWins pw;
    for (int r = 0; r < 8; ++r) pw.w[r] = r < R ? c->peer_win[r] : nullptr;
    const WinLayout L = win_layout(R, cap, H, k);
    auto blocks = [](int64_t items) { return (unsigned)std::max<int64_t>(1, std::min<int64_t>(2 * kNumSMs, (items + 255) / 256)); };
    const unsigned dgrid = blocks((int64_t)R * std::max<int64_t>(T, cap) * (H / 8));
    if (fused_plan) {
      ProfScope prof_("ep_p2p_plan_dispatch_kernel", st);
      p2p_plan_dispatch_kernel<<<dgrid, kP2pThreads, 0, st>>>(x, ids, wts, (int)T, k, H, R, (int)cap, d.E, c->rank,
                                                              w.slots, w.counts, pw, L, c->seq, c->done);
    } else {
      ProfScope prof_("ep_p2p_dispatch_kernel", st);
      p2p_dispatch_kernel<<<dgrid, 256, 0, st>>>(x, ids, wts, w.slots, w.counts, (int)T, k, H, R, (int)cap, c->rank,
                                                 pw, L, c->seq, c->done);
    }
    if ((rc = check_launch("ep_p2p_dispatch_kernel"))) return rc;
    {
      ProfScope prof_("ep_p2p_wait_kernel", st);
      p2p_wait_kernel<<<1, 32, 0, st>>>(c->win, L.rx_flag, R, c->seq, 0, status, 71);
    }
    if ((rc = check_launch("ep_p2p_wait_kernel"))) return rc;
    const int64_t rows = (int64_t)R * cap;
    const bf16* rx = reinterpret_cast<const bf16*>(c->win + L.rx);
    const int32_t* rids = reinterpret_cast<const int32_t*>(c->win + L.rids);
    const float* rwts = reinterpret_cast<const float*>(c->win + L.rwts);
    if (rows <= kGemvRows) {
      rc = run_experts(rx, rows, k, rids, rwts, d, nullptr, w.mw, true, status, st, w.ypart);
    } else {
      if (!w.gemm || !prep)
        return set_error(FMOE_ERR_INVALID, "ep: %lld received rows need the tensor-core path (prepared scales)",
                         (long long)rows);
      rc = run_prefill_experts(rx, rows, k, rids, rwts, d, prep, nullptr, w.pw, true, status, st, w.ypart);
    }
    if (rc) return rc;
    {
      ProfScope prof_("ep_p2p_return_kernel", st);
      p2p_return_kernel<<<blocks(rows * (H / 4)), 256, 0, st>>>(w.ypart, R, (int)cap, H, c->rank, pw, L, c->seq,
                                                               c->done + 1);
    }
    if ((rc = check_launch("ep_p2p_return_kernel"))) return rc;
    {
      ProfScope prof_("ep_p2p_combine_kernel", st);
      const unsigned cgrid = (unsigned)std::max<int64_t>(
          1, std::min<int64_t>(4 * kNumSMs, (T * (H / 8) + kP2pThreads - 1) / kP2pThreads));
      p2p_combine_kernel<<<cgrid, kP2pThreads, 0, st>>>(c->win, L.ret_flag, L.ret, w.slots, (int)T, R, (int)cap, H,
                                                        y, c->seq, c->done + 2, status, 72);
    }
    return check_launch("ep_p2p_combine_kernel");
  }
  {
    ProfScope prof_("ep_pack_kernel", st);
    pack_kernel<<<2 * kNumSMs, 256, 0, st>>>(x, ids, wts, w.slots, w.counts, (int)T, k, H, R, (int)cap, w.sx, w.sids,
                                             w.swts);
  }
  if ((rc = check_launch("ep_pack_kernel"))) return rc;

  const size_t row_b = (size_t)H * sizeof(bf16), part_b = (size_t)H * sizeof(float), meta_b = (size_t)k * sizeof(int32_t);
  std::vector<Xfer> px(R), pb(R);
  std::vector<int64_t> scnt(R, cap), rcnt(R, cap), roff(R);
  if (mode == FMOE_EP_EXACT) {
    std::vector<Xfer> pc(R);
    for (int p = 0; p < R; ++p) {
      pc[p] = Xfer{};
      pc[p].sptr[0] = w.counts + p;
      pc[p].rptr[0] = w.rcounts + p;
      pc[p].sbytes[0] = pc[p].rbytes[0] = sizeof(int32_t);
    }
    if ((rc = exchange(c, pc, 1, st, "count exchange"))) return rc;
    if (cudaMemcpyAsync(c->host_counts, w.counts, R * sizeof(int32_t), cudaMemcpyDeviceToHost, st) != cudaSuccess ||
        cudaMemcpyAsync(c->host_counts + R, w.rcounts, R * sizeof(int32_t), cudaMemcpyDeviceToHost, st) !=
            cudaSuccess ||
        cudaStreamSynchronize(st) != cudaSuccess)
      return set_error(FMOE_ERR_CUDA, "ep: count read-back failed: %s", cudaGetErrorString(cudaGetLastError()));
    for (int p = 0; p < R; ++p) {
      scnt[p] = c->host_counts[p];
      rcnt[p] = c->host_counts[R + p];
      if (scnt[p] < 0 || scnt[p] > cap || rcnt[p] < 0 || rcnt[p] > cap)
        return set_error(FMOE_ERR_INVALID, "ep: exchange counts out of range (peer %d: %lld / %lld, cap %lld)", p,
                         (long long)scnt[p], (long long)rcnt[p], (long long)cap);
    }
  }
  int64_t rows = 0;
  for (int p = 0; p < R; ++p) {
    roff[p] = rows;
    rows += rcnt[p];
  }
  for (int p = 0; p < R; ++p) {
    const int64_t so = (int64_t)p * cap;
    px[p] = Xfer{};
    px[p].sptr[0] = w.sx + so * H;
    px[p].sptr[1] = w.sids + so * k;
    px[p].sptr[2] = w.swts + so * k;
    px[p].rptr[0] = w.rx + roff[p] * H;
    px[p].rptr[1] = w.rids + roff[p] * k;
    px[p].rptr[2] = w.rwts + roff[p] * k;
    px[p].sbytes[0] = scnt[p] * row_b;
    px[p].sbytes[1] = px[p].sbytes[2] = scnt[p] * meta_b;
    px[p].rbytes[0] = rcnt[p] * row_b;
    px[p].rbytes[1] = px[p].rbytes[2] = rcnt[p] * meta_b;
    // the way back: partials of the rows p sent here return to p's block of ret
    pb[p] = Xfer{};
    pb[p].sptr[0] = w.ypart + roff[p] * H;
    pb[p].rptr[0] = w.ret + so * H;
    pb[p].sbytes[0] = rcnt[p] * part_b;
    pb[p].rbytes[0] = scnt[p] * part_b;
  }
  if ((rc = exchange(c, px, 3, st, "dispatch"))) return rc;
  if (rows > 0) {
    if (rows <= kGemvRows) {
      rc = run_experts(w.rx, rows, k, w.rids, w.rwts, d, nullptr, w.mw, true, status, st, w.ypart);
    } else {
      if (!w.gemm || !prep)
        return set_error(FMOE_ERR_INVALID, "ep: %lld received rows need the tensor-core path (prepared scales)",
                         (long long)rows);
      rc = run_prefill_experts(w.rx, rows, k, w.rids, w.rwts, d, prep, nullptr, w.pw, true, status, st, w.ypart);
    }
    if (rc) return rc;
  }
  if ((rc = exchange(c, pb, 1, st, "combine"))) return rc;
  {
    ProfScope prof_("ep_combine_kernel", st);
    combine_kernel<<<2 * kNumSMs * 4, 256, 0, st>>>(w.ret, w.slots, (int)T, R, (int)cap, H, y);
  }
  return check_launch("ep_combine_kernel");
}

}  // namespace fmoe

using namespace fmoe;

extern "C" {

int fmoe_wait_selftest(void* workspace, size_t workspace_bytes, int flag_value, void* stream) {
  if (!workspace || workspace_bytes < 512 || !aligned(workspace, 16))
    return set_error(FMOE_ERR_WORKSPACE, "wait_selftest: workspace needs 512 bytes, 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* w = static_cast<uint8_t*>(workspace);
  // [0, 256): header (status word); 256: exchange sequence word (0); 272: the flag
  if (cudaMemsetAsync(w, 0, 512, st) != cudaSuccess ||
      (flag_value && cudaMemsetAsync(w + 272, 1, 1, st) != cudaSuccess))
    return set_error(FMOE_ERR_CUDA, "wait_selftest: %s", cudaGetErrorString(cudaGetLastError()));
  {
    ProfScope prof_("p2p_wait_kernel", st);
    ep::p2p_wait_kernel<<<1, 32, 0, st>>>(w, 272, 1, reinterpret_cast<uint32_t*>(w + 256), 0,
                                          reinterpret_cast<int*>(w), 99);
  }
  return check_launch("p2p_wait_kernel");
}

int fmoe_ep_unique_id(void* id, size_t len) {
  const ep::NcclApi* api = ep::nccl();
  if (!api) return set_error(FMOE_ERR_NCCL, "ep: libnccl.so.2 not found");
  if (!id || len < sizeof(ncclUniqueId))
    return set_error(FMOE_ERR_INVALID, "ep: unique id buffer needs %zu bytes", sizeof(ncclUniqueId));
  ncclUniqueId u;
  const ncclResult_t r = api->get_unique_id(&u);
  if (r != ncclSuccess) return ep::nccl_error(api, r, "ncclGetUniqueId");
  memcpy(id, &u, sizeof(u));
  return FMOE_OK;
}

int fmoe_ep_comm_init(fmoe_ep_comm_t** comm, int n_ranks, int rank, const void* id, size_t len) {
  const ep::NcclApi* api = ep::nccl();
  if (!api) return set_error(FMOE_ERR_NCCL, "ep: libnccl.so.2 not found");
  if (!comm || !id || len < sizeof(ncclUniqueId) || n_ranks < 1 || rank < 0 || rank >= n_ranks)
    return set_error(FMOE_ERR_INVALID, "ep: comm_init(n_ranks=%d, rank=%d)", n_ranks, rank);
  *comm = nullptr;
  auto* c = new fmoe_ep_comm{};
  c->n_ranks = n_ranks;
  c->rank = rank;
  cudaGetDevice(&c->device);
  if (cudaHostAlloc(&c->host_counts, 2 * n_ranks * sizeof(int32_t), cudaHostAllocDefault) != cudaSuccess) {
    delete c;
    return set_error(FMOE_ERR_CUDA, "ep: pinned count buffer: %s", cudaGetErrorString(cudaGetLastError()));
  }
  ncclUniqueId u;
  memcpy(&u, id, sizeof(u));
  const ncclResult_t r = api->comm_init_rank(&c->nc, n_ranks, u, rank);
  if (r != ncclSuccess) {
    cudaFreeHost(c->host_counts);
    delete c;
    return ep::nccl_error(api, r, "ncclCommInitRank");
  }
  *comm = c;
  return FMOE_OK;
}

// All-gather of n host bytes per rank (rank order) through a device buffer.
static int gather_bytes(const ep::NcclApi* api, fmoe_ep_comm_t* c, const void* mine, size_t n, void* all) {
  uint8_t* d = nullptr;
  cudaStream_t s = nullptr;
  int rc = FMOE_OK;
  if (cudaMalloc(&d, n * (c->n_ranks + 1)) != cudaSuccess ||
      cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMemcpy(d, mine, n, cudaMemcpyHostToDevice) != cudaSuccess) {
    rc = set_error(FMOE_ERR_CUDA, "ep: gather buffer: %s", cudaGetErrorString(cudaGetLastError()));
  } else {
    const ncclResult_t r = api->all_gather(d, d + n, n, ncclUint8, c->nc, s);
    if (r != ncclSuccess)
      rc = ep::nccl_error(api, r, "all-gather");
    else if (cudaStreamSynchronize(s) != cudaSuccess || cudaMemcpy(all, d + n, n * c->n_ranks,
                                                                   cudaMemcpyDeviceToHost) != cudaSuccess)
      rc = set_error(FMOE_ERR_CUDA, "ep: gather copy: %s", cudaGetErrorString(cudaGetLastError()));
  }
  if (d) cudaFree(d);
  if (s) cudaStreamDestroy(s);
  return rc;
}

// Releases the peer-memory window.  A peer's mapping of this rank's window is
// closed before the window is freed (freeing exported memory that another
// process still maps is undefined), so the collective modes take two
// barriers; all ranks call them together.
//   kP2pBarrier  this rank's work done; barrier (every rank's exchanges are
//                complete); close the mappings of the peers' windows;
//                barrier; free
//   kP2pAgreed   set-up that all ranks agreed failed after some mapped:
//                close; barrier; free
//   kP2pLocal    set-up failures before any rank mapped a window: free
//   kP2pAbort    frees nothing (a peer may still be storing into the window):
//                it stays allocated, and the peers' windows mapped, until the
//                process exits
enum P2pRelease { kP2pAbort, kP2pLocal, kP2pAgreed, kP2pBarrier };
static int p2p_barrier(const ep::NcclApi* api, fmoe_ep_comm_t* c) {
  if (c->n_ranks < 2) return FMOE_OK;
  if (!api) return set_error(FMOE_ERR_NCCL, "ep: libnccl.so.2 not found");
  int32_t mine = 0;
  std::vector<int32_t> all(c->n_ranks);
  return gather_bytes(api, c, &mine, sizeof mine, all.data());
}
static int p2p_release(fmoe_ep_comm_t* c, P2pRelease how) {
  if (!c->win) return FMOE_OK;
  int rc = FMOE_OK;
  const ep::NcclApi* api = ep::nccl();
  if (how == kP2pBarrier) {
    cudaDeviceSynchronize();
    rc = p2p_barrier(api, c);
  }
  if (how != kP2pAbort) {
    for (int r = 0; r < c->n_ranks && r < 8; ++r)
      if (r != c->rank && c->peer_win[r]) cudaIpcCloseMemHandle(c->peer_win[r]);
    if (how == kP2pBarrier || how == kP2pAgreed) {
      const int rc2 = p2p_barrier(api, c);
      if (!rc) rc = rc2;
    }
    cudaFree(c->win);
    cudaFree(c->seq);
  }
  c->win = nullptr;
  c->seq = nullptr;
  c->done = nullptr;
  for (int r = 0; r < 8; ++r) c->peer_win[r] = nullptr;
  c->p2p_cap = 0;
  return rc;
}

int fmoe_ep_p2p_init(fmoe_ep_comm_t* c, int64_t cap, int hidden, int top_k) {
  const ep::NcclApi* api = ep::nccl();
  if (!api) return set_error(FMOE_ERR_NCCL, "ep: libnccl.so.2 not found");
  if (!c || !c->nc) return set_error(FMOE_ERR_INVALID, "ep: null communicator");
  if (c->n_ranks > 8 || cap < 1 || cap > (1 << 20) || hidden < 64 || hidden % 8 || top_k < 1 || top_k > 16 ||
      hidden / 8 < top_k)
    return set_error(FMOE_ERR_INVALID, "ep_p2p_init: ranks %d (<= 8), cap %lld, hidden %d, top_k %d", c->n_ranks,
                     (long long)cap, hidden, top_k);
  int rc = p2p_release(c, kP2pBarrier);
  if (rc) return rc;
  // Every rank takes both all-gathers below, failed or not, and all ranks
  // agree on the outcome (a rank that failed to allocate or map makes every
  // rank free its window and return an error).
  struct Rec {
    int32_t ok, hidden, top_k, pad;
    int64_t cap;
    cudaIpcMemHandle_t h;
  };
  const ep::WinLayout L = ep::win_layout(c->n_ranks, cap, hidden, top_k);
  Rec mine{};
  char why[160] = "";
  if (cudaMalloc(&c->win, L.bytes) != cudaSuccess || cudaMemset(c->win, 0, L.bytes) != cudaSuccess ||
      cudaMalloc(&c->seq, 16) != cudaSuccess || cudaMemset(c->seq, 0, 16) != cudaSuccess ||
      cudaDeviceSynchronize() != cudaSuccess ||  // zeroed flags before any peer can see the window
      (c->n_ranks > 1 && cudaIpcGetMemHandle(&mine.h, c->win) != cudaSuccess))
    snprintf(why, sizeof why, "window of %zu bytes: %s", L.bytes, cudaGetErrorString(cudaGetLastError()));
  mine.ok = why[0] == 0;
  mine.hidden = hidden;
  mine.top_k = top_k;
  mine.cap = cap;
  std::vector<Rec> all(c->n_ranks);
  all[c->rank] = mine;
  if (c->n_ranks > 1 && (rc = gather_bytes(api, c, &mine, sizeof(Rec), all.data()))) {
    p2p_release(c, kP2pLocal);
    return rc;
  }
  for (int p = 0; p < c->n_ranks && !why[0]; ++p) {
    if (!all[p].ok) snprintf(why, sizeof why, "rank %d could not allocate its window", p);
    else if (all[p].cap != cap || all[p].hidden != hidden || all[p].top_k != top_k)  // window layouts must agree
      snprintf(why, sizeof why, "rank %d asked for cap %lld, hidden %d, top_k %d; this rank cap %lld, hidden %d, "
               "top_k %d", p, (long long)all[p].cap, all[p].hidden, all[p].top_k, (long long)cap, hidden, top_k);
  }
  if (!why[0]) {
    c->done = reinterpret_cast<unsigned*>(c->seq + 1);
    c->peer_win[c->rank] = c->win;
    for (int p = 0; p < c->n_ranks && !why[0]; ++p) {
      if (p == c->rank) continue;
      void* ptr = nullptr;
      if (cudaIpcOpenMemHandle(&ptr, all[p].h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
        snprintf(why, sizeof why, "map rank %d's window: %s", p, cudaGetErrorString(cudaGetLastError()));
      else
        c->peer_win[p] = static_cast<uint8_t*>(ptr);
    }
    std::vector<int32_t> oks(c->n_ranks, 1);
    int32_t ok = why[0] == 0;
    oks[c->rank] = ok;
    if (c->n_ranks > 1 && (rc = gather_bytes(api, c, &ok, sizeof ok, oks.data()))) {
      p2p_release(c, kP2pLocal);
      return rc;
    }
    for (int p = 0; p < c->n_ranks && !why[0]; ++p)
      if (!oks[p]) snprintf(why, sizeof why, "rank %d could not map every window", p);
    if (why[0]) {  // every rank agreed; some may hold mappings of this window
      p2p_release(c, kP2pAgreed);
      return set_error(FMOE_ERR_CUDA, "ep_p2p_init: %s", why);
    }
  }
  if (why[0]) {  // no rank mapped any window
    p2p_release(c, kP2pLocal);
    return set_error(FMOE_ERR_CUDA, "ep_p2p_init: %s", why);
  }
  c->p2p_cap = cap;
  c->p2p_hidden = hidden;
  c->p2p_k = top_k;
  return FMOE_OK;
}

int fmoe_ep_comm_destroy(fmoe_ep_comm_t* c) {
  if (!c) return FMOE_OK;
  p2p_release(c, kP2pBarrier);
  const ep::NcclApi* api = ep::nccl();
  ncclResult_t r = ncclSuccess;
  if (c->nc && api) r = api->comm_destroy(c->nc);
  cudaFreeHost(c->host_counts);
  delete c;
  return r == ncclSuccess ? FMOE_OK : ep::nccl_error(api, r, "ncclCommDestroy");
}

int fmoe_ep_comm_abort(fmoe_ep_comm_t* c) {
  if (!c) return FMOE_OK;
  p2p_release(c, kP2pAbort);
  const ep::NcclApi* api = ep::nccl();
  ncclResult_t r = ncclSuccess;
  if (c->nc && api) r = api->comm_abort(c->nc);
  cudaFreeHost(c->host_counts);
  delete c;
  return r == ncclSuccess ? FMOE_OK : ep::nccl_error(api, r, "ncclCommAbort");
}

int fmoe_ep_comm_status(fmoe_ep_comm_t* c) {
  if (!c || !c->nc) return set_error(FMOE_ERR_INVALID, "ep: null communicator");
  const ep::NcclApi* api = ep::nccl();
  ncclResult_t state = ncclSuccess;
  const ncclResult_t r = api->comm_async_error(c->nc, &state);
  if (r != ncclSuccess) return ep::nccl_error(api, r, "ncclCommGetAsyncError");
  if (state != ncclSuccess && state != ncclInProgress) return ep::nccl_error(api, state, "asynchronous error");
  return FMOE_OK;
}

size_t fmoe_ep_moe_workspace_bytes(int n_ranks, int64_t cap, const fmoe_router_t* r, const fmoe_experts_t* local) {
  ExpertsDev d;
  if (n_ranks < 1 || cap < 1 || !r || r->top_k < 1 || r->top_k > 16 || to_experts(local, &d)) return 0;
  Carver c(nullptr);
  const WsHead h = carve_head(c);
  return carve_ep(c, n_ranks, cap, r, r->top_k, d, h, nullptr) + 256;
}

int fmoe_ep_moe_forward(fmoe_ep_comm_t* comm, const void* x, int64_t T, int64_t cap, const fmoe_router_t* r,
                        const fmoe_experts_t* local, const void* prep, void* y, int32_t* ids, float* weights, int mode,
                        void* workspace, size_t workspace_bytes, void* stream) {
  QW q;
  int rc;
  if ((rc = check_router(r, &q))) return rc;
  ExpertsDev d;
  if ((rc = to_experts(local, &d)) || (rc = ep_check(comm, d, q.out, nullptr))) return rc;
  if (!x || !y) return set_error(FMOE_ERR_INVALID, "ep: null x / y");
  if (T < 0 || cap < 1 || cap > (1 << 24)) return set_error(FMOE_ERR_INVALID, "ep: T=%lld cap=%lld", (long long)T,
                                                           (long long)cap);
  if (q.in != d.H || d.H % 8 || d.H / 8 < r->top_k)
    return set_error(FMOE_ERR_INVALID, "ep: router in %d vs hidden %d", q.in, d.H);
  if (!aligned(x, 16) || !aligned(y, 16)) return set_error(FMOE_ERR_ALIGN, "ep: x / y not 16-byte aligned");
  const size_t need = fmoe_ep_moe_workspace_bytes(comm->n_ranks, cap, r, local);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 16))
    return set_error(FMOE_ERR_WORKSPACE, "ep: workspace %zu < %zu (16-byte aligned)", workspace_bytes, need);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver c(workspace);
  const WsHead h = carve_head(c);
  EpWs w;
  carve_ep(c, comm->n_ranks, cap, r, r->top_k, d, h, &w);
  int32_t* ids_out = ids ? ids : w.ids;
  float* w_out = weights ? weights : w.wts;
  if (T > 0 &&
      (rc = run_router(static_cast<const bf16*>(x), T, r, q, w.rw, ids_out, w_out, nullptr, nullptr, h.status, st)))
    return rc;
  // Every rank takes part in both exchanges, also with no tokens of its own.
  return ep_experts(comm, static_cast<const bf16*>(x), T, cap, r->top_k, ids_out, w_out, d,
                    static_cast<const bf16*>(prep), static_cast<bf16*>(y), w, mode, h.status, st);
}

}  // extern "C"
