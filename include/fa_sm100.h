/*
 * fa_sm100.h - C ABI of the B200 (sm_100a) FlashAttention-2 forward.
 *
 * Plain C: pointers, sizes and ints only, so it binds from ctypes, cgo, JNI or a
 * C++ driver without any PyTorch type.  One call = one asynchronous kernel launch
 * on the caller's stream and the caller's current CUDA device.
 *
 * Replaces the reference's C++ launch entry: `config::ForwardKernelArgs`
 * (wenssir/flash-attention src/config/config.cuh:20-45) plus
 * `forward::forward_smem_bytes<Cfg>()` (src/utils/util_func.cuh:12-21) plus the
 * launch `flash_attention_forward_v6_mma<Cfg><<<(N/64,H,B),128,smem>>>(args)`
 * (src/forward/forward_v6_mma.cuh:325-412, launched at
 * python/flash_attention_runtime/_ext.cu:59-122 and
 * benchmark/cpp/correctness_v6.cu:144-188).
 */
#ifndef FA_SM100_H
#define FA_SM100_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FA_API __attribute__((visibility("default")))
#else
#define FA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes.  The reference raised through TORCH_CHECK
 * (python/flash_attention_runtime/_ext.cu:19-57,109-120,146-147) or returned
 * silently from the kernel (src/forward/forward_v6_mma.cuh:330-339); here every
 * rejected call returns a code and never launches. */
enum fa_status {
  FA_OK = 0,
  FA_ERR_BAD_SHAPE = 1,      /* batch/heads/seq_len < 1, or a stride that does not fit the shape */
  FA_ERR_BAD_ALIGN = 2,      /* base pointer not 16-byte aligned, or a stride not a multiple of 8 elements */
  FA_ERR_UNSUPPORTED = 3,    /* head_dim not in {32, 64, 128}, unknown dtype, or no sm_100 device */
  FA_ERR_LAUNCH = 4,         /* a CUDA runtime call failed; see fa_last_error() */
  FA_ERR_DEVICE_TIMEOUT = 5, /* reported through the status word: a pipeline wait timed out */
  FA_ERR_BAD_PARAM = 6       /* null pointer, non-positive or non-finite softmax_scale, bad workspace */
};

enum fa_dtype { FA_DTYPE_F16 = 0, FA_DTYPE_BF16 = 1 };

typedef struct fa_fwd_params {
  /* ---- the reference's ForwardKernelArgs, same names, order and meaning
   *      (src/config/config.cuh:20-45).  Tensors are [B, H, N, d] with the head
   *      dimension contiguous; strides are in elements. */
  void* Q;
  void* K;
  void* V;
  void* O;
  int stride_batch_q;
  int stride_seq_q;
  int stride_head_q;
  int stride_batch_k;
  int stride_seq_k;
  int stride_head_k;
  int stride_batch_v;
  int stride_seq_v;
  int stride_head_v;
  int stride_batch_o;
  int stride_seq_o;
  int stride_head_o;
  int seq_len;
  int heads;
  int head_dim;
  float softmax_scale;
  int causal; /* 0: disabled, 1: key j masked for query i when j > i */

  /* ---- appended (no counterpart in ForwardKernelArgs) */
  float* LSE;    /* optional fp32 [B, H, N] contiguous: natural-log logsumexp of scale*QK^T rows */
  int dtype;     /* enum fa_dtype; Q, K, V and O share it */
  int batch;     /* B (the reference derived it from the grid) */
  /* 64-bit batch / head strides for tensors past 2^31 elements; a non-zero entry
   * overrides the int field.  Index 0..3 = q, k, v, o. */
  int64_t stride_batch64[4];
  int64_t stride_head64[4];
  /* Scratch for the persistent tile scheduler: at least fa_fwd_workspace_bytes(),
   * 16-byte aligned device memory, or NULL to let the library use a buffer it
   * allocates once per (device, stream) - per host thread for
   * cudaStreamPerThread - and keeps until exit.  Launches that overlap on the
   * GPU must not share a workspace. */
  void* workspace;
  size_t workspace_bytes;
  int* status;                 /* optional device int: set to 0x100|site if a wait times out */
  unsigned long long timeout_ns; /* per-wait limit inside the kernel; 0 = 2 s */
} fa_fwd_params;

/* Launch O = softmax(softmax_scale * Q K^T [causal]) V (and LSE) on `stream`
 * (a cudaStream_t; NULL = legacy default stream).  Asynchronous. */
FA_API int fa_fwd_sm100(const fa_fwd_params* params, void* stream);

/* Same computation as fa_fwd_sm100, for callers that cannot allocate device
 * memory: runtimes whose memory pool forbids allocations behind its back,
 * plug-in hosts that hand a library only its input and output buffers, and
 * latency-bound loops that cannot take a cudaMalloc's implicit synchronisation.
 * No counterpart in the reference.  params->workspace must be NULL: the
 * scheduler's scratch is a fixed 256-byte array inside this library's device
 * memory (one per GPU, held until the process exits), cleared with
 * cudaMemsetAsync before every launch; a scheduler needing more than 256 bytes
 * is rejected with FA_ERR_BAD_SHAPE.  No cudaMalloc / cudaFree is called.  The
 * first call on a device looks up the array's address (cudaGetSymbolAddress)
 * with that device current and caches it; after a cudaDeviceReset of that
 * device the cached address is stale.  All calls
 * on a device share the array: calls whose kernels overlap on the GPU race on it. */
FA_API int fa_fwd_sm100_noalloc(const fa_fwd_params* params, void* stream);

/* Dynamic shared memory one CTA of the kernel uses for this head_dim / dtype
 * (the reference's forward_smem_bytes<Cfg>(), src/utils/util_func.cuh:12-21).
 * Returns 0 for an unsupported combination. */
FA_API size_t fa_fwd_smem_bytes(int head_dim, int dtype);

/* Bytes of device workspace fa_fwd_sm100 needs when params->workspace is set. */
FA_API size_t fa_fwd_workspace_bytes(void);

/* Human-readable name of a status code. */
FA_API const char* fa_status_string(int status);

/* Detail message of the last failing call on this host thread ("" if none). */
FA_API const char* fa_last_error(void);

#ifdef __cplusplus
}
#endif

#endif /* FA_SM100_H */
