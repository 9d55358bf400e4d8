// ossm_cheby_ema_fwd_noalloc: the forward for callers that cannot allocate
// device memory.
//
// Some hosts cannot call cudaMalloc at the point where they run the forward:
// code that runs under a caching or arena allocator that owns all device
// memory, plugins whose host only hands them input and output buffers, and
// code paths that must not allocate for latency reasons.  This entry point
// takes the forward's scratch (the look-back records and the launch header)
// from a fixed array inside the library instead of a caller workspace.
//
// Limits, stated for the caller:
//  * the scratch is OSSM_NOALLOC_SCRATCH_BYTES per GPU, held from the moment
//    the library's module loads on a GPU until the process exits; a call whose
//    workspace (ossm_fwd_workspace_bytes) would exceed it is rejected with
//    OSSM_EWORKSPACE before anything is launched;
//  * every call on a GPU shares that one array: calls whose kernels overlap on
//    the GPU (different streams without ordering, or other host threads) race
//    on it and may return wrong results or time out;
//  * the first call on each GPU does the set-up (finds the array's device
//    address and clears it on the caller's stream); make that first call
//    before any other work that could overlap it, and before any stream
//    capture;
//  * a call that takes the generic kernel (fp32 x or output, other head
//    sizes, LUT) also clears that kernel's look-back flags in the array on
//    the caller's stream first, because an earlier call of another shape may
//    have left data there.
#include <cuda_runtime.h>

#include <mutex>

#include "orthossm_b200.h"

size_t ossm_fwd_flag_region(const ossm_fwd_args* a, size_t* offset);

namespace {

// The shared scratch.  Only device code and cudaGetSymbolAddress may use the
// name: in host code it denotes a host-side stand-in, not device memory.
__device__ __align__(256) unsigned char g_noalloc_scratch[OSSM_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices];  // device address of g_noalloc_scratch, per device, after set-up

}  // namespace

extern "C" int ossm_cheby_ema_fwd_noalloc(const ossm_fwd_args* a, ossm_stream_t stream, void** scratch) {
  if (!a) return OSSM_EINVAL;
  // everything on the caller's stream: no side streams are created or used.
  // The size check is made on these arguments, since the flag changes how
  // the bf16 path lays out its scratch.
  ossm_fwd_args one = *a;
  one.flags |= OSSM_F_ONE_STREAM;
  const size_t need = ossm_fwd_workspace_bytes(&one);
  if (need == 0) return OSSM_EINVAL;
  if (need > (size_t)OSSM_NOALLOC_SCRATCH_BYTES) return OSSM_EWORKSPACE;  // over the fixed maximum

  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return OSSM_ELAUNCH;
  if (dev >= kMaxDevices) return OSSM_EINVAL;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  void* ptr = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_setup_mu);
    if (!g_scratch_ptr[dev]) {
      // set-up, once per device with that device current: the array's device
      // address, then a clear (the launch header's counters must start at
      // zero; every launch leaves them at zero again)
      void* p = nullptr;
      if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || p == nullptr) return OSSM_ELAUNCH;
      if (cudaMemsetAsync(p, 0, OSSM_NOALLOC_SCRATCH_BYTES, st) != cudaSuccess) return OSSM_ELAUNCH;
      g_scratch_ptr[dev] = p;
    }
    ptr = g_scratch_ptr[dev];
  }
  if (scratch) *scratch = ptr;
  size_t flag_off = 0;
  const size_t flag_bytes = ossm_fwd_flag_region(&one, &flag_off);
  if (flag_bytes > 0 && cudaMemsetAsync(static_cast<char*>(ptr) + flag_off, 0, flag_bytes, st) != cudaSuccess)
    return OSSM_ELAUNCH;
  return ossm_cheby_ema_fwd(&one, ptr, (size_t)OSSM_NOALLOC_SCRATCH_BYTES, stream);
}
