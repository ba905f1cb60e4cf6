// fa_fwd_sm100_noalloc: the forward for callers that cannot allocate device memory.
//
// fa_fwd_sm100 with workspace == NULL allocates its scheduler workspace with
// cudaMalloc the first time it sees a (device, stream).  Some callers cannot
// allow that: runtimes that hand out all device memory through their own pool
// and forbid allocations behind its back, plug-in hosts that give a library its
// input and output buffers and nothing else, and latency-bound loops in which the
// implicit synchronisation of a cudaMalloc is not acceptable.  This entry point
// takes its scratch from a fixed array in the library's own device memory
// instead: every GPU that loads the library holds kScratchBytes of it until the
// process exits.
//
// The scratch holds the persistent tile scheduler's counter, which must be zero
// when a launch starts; it is cleared with cudaMemsetAsync on the caller's stream
// before every launch, which allocates nothing.  All calls on a device share the
// one array, so calls whose kernels overlap on the GPU (for example on two
// streams without ordering between them) race on the counter and compute wrong
// results: order them, or use fa_fwd_sm100 with one workspace per stream.
//
// The array's device address is looked up once per device (the first call on
// that device, with it current) and cached; a cudaDeviceReset of that device
// makes the cached address stale, so the entry point must not be called on a
// device after resetting it in the same process.
#include <cuda_runtime.h>

#include <cstring>
#include <mutex>

#include "fa_launch.h"
#include "../../include/fa_sm100.h"

namespace {

// Size of the static scratch: one scheduler workspace (fa_fwd_workspace_bytes()).
constexpr size_t kScratchBytes = 256;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

// In host code g_noalloc_scratch names a host-side stand-in, not device memory:
// the kernel must get the address cudaGetSymbolAddress returns for the current
// device.  Resolved once per device, with that device current.
std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};

int scratch_address(int dev, void** out) {
  if (dev < 0 || dev >= kMaxDevices) {
    fa::set_last_error("fa_fwd_sm100_noalloc: device index out of range");
    return FA_ERR_UNSUPPORTED;
  }
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    void* ptr = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&ptr, g_noalloc_scratch);
    if (e != cudaSuccess || ptr == nullptr) {
      fa::set_last_error("fa_fwd_sm100_noalloc: cudaGetSymbolAddress of the static scratch failed");
      return FA_ERR_LAUNCH;
    }
    g_scratch_ptr[dev] = ptr;
  }
  *out = g_scratch_ptr[dev];
  return FA_OK;
}

}  // namespace

extern "C" {

int fa_fwd_sm100_noalloc(const fa_fwd_params* p, void* stream) {
  // The argument checks come first, as in fa_fwd_sm100: a bad call is rejected
  // before any CUDA runtime call.
  const int vrc = fa::validate_params(p);
  if (vrc != FA_OK) return vrc;
  if (p->workspace != nullptr) {
    fa::set_last_error("fa_fwd_sm100_noalloc: params->workspace must be NULL (this entry point uses its own static scratch)");
    return FA_ERR_BAD_PARAM;
  }
  if (fa_fwd_workspace_bytes() > kScratchBytes) {
    fa::set_last_error("fa_fwd_sm100_noalloc: the scheduler needs more scratch than the static array holds");
    return FA_ERR_BAD_SHAPE;
  }
  // The device check comes before the symbol lookup, so a device that is not an
  // sm_100 part is reported as FA_ERR_UNSUPPORTED, as fa_fwd_sm100 reports it.
  int dev = 0;
  const int drc = fa::current_sm100_device(&dev, nullptr);
  if (drc != FA_OK) return drc;
  void* scratch = nullptr;
  const int rc = scratch_address(dev, &scratch);
  if (rc != FA_OK) return rc;
  fa_fwd_params q;
  std::memcpy(&q, p, sizeof(q));
  q.workspace = scratch;
  q.workspace_bytes = kScratchBytes;
  return fa_fwd_sm100(&q, stream);
}

}  // extern "C"
