// Device-side routing metadata: per-expert lists of (token, slot) pairs built
// from top-k ids, replacing the host sync + sort + dedup of
// src/model/moe.rs:355-380.  Pairs p = t*k + slot are split into one
// contiguous chunk per warp; each warp counts its chunk per expert, offsets
// are (expert, warp)-major exclusive prefixes, and each warp scatters its chunk
// in index order, so pairs[] is ascending within an expert (deterministic).
#pragma once
#include "common.cuh"

namespace fmoe {

// Block-wide build of the per-expert pair lists (see the file comment).  ids
// are read through L2 (they may have been written earlier in the same kernel
// by other CTAs).  sm: (nwarps + 1) * E ints of shared memory.
__device__ __forceinline__ void route_build_block(const int32_t* ids, int P, int first, int E, int32_t* start, int32_t* pairs,
                                  int32_t* unique, int32_t* num_unique, int4* work, int work_len, int* sm) {
  const int nw = blockDim.x >> 5;
  int* wcnt = sm;           // [nw][E] counts, later offsets
  int* tot = sm + nw * E;   // [E]
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int i = threadIdx.x; i < nw * E; i += blockDim.x) wcnt[i] = 0;
  __syncthreads();
  const int chunk = (P + nw - 1) / nw;
  const int pb = min(P, warp * chunk), pe = min(P, pb + chunk);
  for (int p = pb + lane; p < pe; p += 32) {
    const int e = __ldcg(ids + p) - first;
    if (e >= 0 && e < E) atomicAdd(&wcnt[warp * E + e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int c = 0;
    for (int w = 0; w < nw; ++w) c += wcnt[w * E + e];
    tot[e] = c;
  }
  __syncthreads();
  if (warp == 0) {
    // Exclusive scan of tot[] and compaction of non-empty experts, 32 experts per step.
    int run = 0, urun = 0;
    for (int e0 = 0; e0 < E; e0 += 32) {
      const int e = e0 + lane;
      const int c = e < E ? tot[e] : 0;
      int incl = c, uincl = c > 0;
      for (int o = 1; o < 32; o <<= 1) {
        const int a = __shfl_up_sync(0xffffffffu, incl, o), b = __shfl_up_sync(0xffffffffu, uincl, o);
        if (lane >= o) {
          incl += a;
          uincl += b;
        }
      }
      if (e < E) {
        start[e] = run + incl - c;
        tot[e] = run + incl - c;
        if (c > 0) {
          unique[urun + uincl - 1] = e;
          if (urun + uincl - 1 < work_len) work[urun + uincl - 1] = make_int4(e, run + incl - c, c, 0);
        }
      }
      run += __shfl_sync(0xffffffffu, incl, 31);
      urun += __shfl_sync(0xffffffffu, uincl, 31);
    }
    if (lane == 0) {
      start[E] = run;
      *num_unique = urun;
    }
    for (int u = urun + lane; u < work_len; u += 32) work[u] = make_int4(0, 0, 0, 0);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) {
    int o = tot[e];
    for (int w = 0; w < nw; ++w) {
      const int c = wcnt[w * E + e];
      wcnt[w * E + e] = o;
      o += c;
    }
  }
  __syncthreads();
  const unsigned lt = (1u << lane) - 1u;
  for (int p0 = pb; p0 < pe; p0 += 32) {
    const int p = p0 + lane;
    int e = -1;
    if (p < pe) {
      e = __ldcg(ids + p) - first;
      if (e < 0 || e >= E) e = -1;
    }
    const unsigned peers = __match_any_sync(0xffffffffu, e);
    if (e >= 0) pairs[wcnt[warp * E + e] + __popc(peers & lt)] = p;
    __syncwarp();
    if (e >= 0 && (peers & lt) == 0) wcnt[warp * E + e] += __popc(peers);
    __syncwarp();
  }
  __syncthreads();
}

}  // namespace fmoe
