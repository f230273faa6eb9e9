// fmoe_moe_block_forward_noalloc: the MoE block forward for callers that
// cannot hand the library a workspace.
//
// Some hosts cannot allocate device memory at the point where they run the MoE
// layer: an engine that gives its whole device budget to its own memory pool
// (a cudaMalloc behind its back fails or fragments that pool), a plugin host
// that forbids libraries from allocating, or a latency-critical decode loop
// where cudaMalloc / cudaFree may synchronise the device.  For them this entry
// point runs the same three kernels as fmoe_moe_block_forward on a fixed
// scratch array that lives in the library itself (static device memory, held
// by every GPU that loads the library until the process exits).  The caller
// still provides x, y and the routing outputs.
//
// The array is shared by every call on a device and keeps whatever the last
// call left in it: each call clears the part it uses before launching, and
// calls that overlap on the GPU (two streams, two threads) race on it.
#include <mutex>
#include "internal.h"

namespace fmoe {

constexpr size_t kNoallocScratchBytes = FMOE_NOALLOC_SCRATCH_BYTES;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoallocScratchBytes];

// Host code only sees a host-side stand-in for g_noalloc_scratch; the device
// address is looked up once per device, with that device current.
static int noalloc_scratch_ptr(void** out) {
  static std::mutex mu;
  static void* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return set_error(FMOE_ERR_CUDA, "moe_block_forward_noalloc: no current device");
  std::lock_guard<std::mutex> lk(mu);
  if (!ptrs[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p)
      return set_error(FMOE_ERR_CUDA, "moe_block_forward_noalloc: cudaGetSymbolAddress failed: %s",
                       cudaGetErrorString(e));
    ptrs[dev] = p;
  }
  *out = ptrs[dev];
  return FMOE_OK;
}

}  // namespace fmoe

using namespace fmoe;

extern "C" int fmoe_moe_block_forward_noalloc(const void* x, int64_t T, const fmoe_router_t* r,
                                              const fmoe_experts_t* ex, void* y, int32_t* ids, float* weights,
                                              void* stream) {
  if (T <= 0) return FMOE_OK;  // nothing to do, nothing queued on the shared array
  // Cheap argument checks first, so a call that is going to be rejected queues
  // nothing on the array every call shares.
  if (!x || !y) return set_error(FMOE_ERR_INVALID, "moe_block_forward_noalloc: null x/y");
  if (!aligned(x, 16)) return set_error(FMOE_ERR_ALIGN, "moe_block_forward_noalloc: x not 16-byte aligned");
  const size_t need = fmoe_moe_block_workspace_bytes(T, r, ex);
  if (need == 0) return set_error(FMOE_ERR_INVALID, "moe_block_forward_noalloc: bad router or expert table");
  if (need > kNoallocScratchBytes)
    return set_error(FMOE_ERR_WORKSPACE,
                     "moe_block_forward_noalloc: T=%lld needs %zu bytes of scratch, the static array holds %zu "
                     "(use fmoe_moe_block_forward with a caller workspace)",
                     (long long)T, need, kNoallocScratchBytes);
  void* scratch = nullptr;
  int rc = noalloc_scratch_ptr(&scratch);
  if (rc) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // The router's completion counter and the down kernel's tile counters must
  // start at zero.  Word 0 (the device status word) is left alone: a bounded
  // device wait that gave up in an earlier call stays visible to
  // fmoe_moe_block_noalloc_status until the caller clears it.
  const cudaError_t e =
      cudaMemsetAsync(static_cast<uint8_t*>(scratch) + sizeof(int), 0, need - sizeof(int), st);
  if (e != cudaSuccess)
    return set_error(FMOE_ERR_CUDA, "moe_block_forward_noalloc: clearing the scratch failed: %s",
                     cudaGetErrorString(e));
  return fmoe_moe_block_forward(x, T, r, ex, y, ids, weights, scratch, kNoallocScratchBytes, stream);
}

extern "C" int fmoe_moe_block_noalloc_status(int clear, void* stream) {
  void* scratch = nullptr;
  const int rc = noalloc_scratch_ptr(&scratch);
  if (rc) return rc;
  return fmoe_workspace_status(scratch, clear, stream);
}
