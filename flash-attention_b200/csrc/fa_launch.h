// Internal interface between the C-ABI front end (fa_sm100.cu) and the per-head-dim
// translation units that instantiate the kernel (fa_fwd_d{32,64,128}.cu).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

#include "fa_fwd_kernel.cuh"
#include "fa_sm100.h"

namespace fa {

struct LaunchSpec {
  CUtensorMap tq, tk, tv;
  KernelParams kp;
  int grid;
  cudaStream_t stream;
  bool bf16;
  bool causal;
};

// Sets the message fa_last_error() returns on this host thread.
void set_last_error(const char* msg);
// fa_fwd_sm100's device-free argument checks alone (status code, message in
// fa_last_error()).
int validate_params(const fa_fwd_params* p);
// The current device, if it is an sm_100 part (FA_OK), else FA_ERR_UNSUPPORTED /
// FA_ERR_LAUNCH with the message set; also gives its SM count.
int current_sm100_device(int* dev, int* sms);

cudaError_t launch_d32(const LaunchSpec& s);
cudaError_t launch_d64(const LaunchSpec& s);
cudaError_t launch_d128(const LaunchSpec& s);

// Devices whose "attribute set" flags are cached; on a device past this the
// attribute is set on every launch (correct, only slower).
constexpr int kAttrDevices = 64;

// Sets the dynamic-smem attribute of one kernel instantiation once per device
// (done[dev] records it).
template <typename Kernel>
cudaError_t ensure_smem_attr(Kernel k, int smem_bytes, int (&done)[kAttrDevices]) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const bool cached = dev >= 0 && dev < kAttrDevices;
  if (cached && __atomic_load_n(&done[dev], __ATOMIC_ACQUIRE)) return cudaSuccess;
  e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_bytes);
  if (e != cudaSuccess) return e;
  if (cached) __atomic_store_n(&done[dev], 1, __ATOMIC_RELEASE);
  return cudaSuccess;
}

template <int D>
cudaError_t launch_for_dim(const LaunchSpec& s) {
  constexpr int smem = static_cast<int>(Cfg<D>::SMEM_BYTES);
  static int done[4][kAttrDevices] = {};
  const int v = (s.bf16 ? 1 : 0) | (s.causal ? 2 : 0);
  // Programmatic dependent launch: this grid's CTAs may start (barrier setup,
  // TMEM allocation) while the previous kernel on the stream finishes; they wait
  // in griddepcontrol.wait for it to complete before touching global memory.
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(s.grid));
  cfg.blockDim = dim3(kNumThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s.stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e;
  switch (v) {
#define FA_CASE(IDX, BF, CA)                                                       \
  case IDX:                                                                        \
    e = ensure_smem_attr(fa_fwd_sm100_kernel<D, BF, CA>, smem, done[IDX]);        \
    if (e != cudaSuccess) return e;                                                \
    e = cudaLaunchKernelEx(&cfg, fa_fwd_sm100_kernel<D, BF, CA>, s.tq, s.tk, s.tv, s.kp); \
    if (e != cudaSuccess) return e;                                                \
    break;
    FA_CASE(0, false, false)
    FA_CASE(1, true, false)
    FA_CASE(2, false, true)
    FA_CASE(3, true, true)
#undef FA_CASE
    default:
      return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace fa
