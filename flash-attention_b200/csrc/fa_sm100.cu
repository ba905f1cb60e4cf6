// C-ABI front end of the sm_100a forward: validates a fa_fwd_params, encodes the
// TMA tensor maps, picks the persistent grid and launches the kernel.
//
// Mirrors the reference's host launcher (python/flash_attention_runtime/_ext.cu:30-122):
// the same checks (shapes, dtypes, head_dim), the ForwardKernelArgs fill with
// scale = 1/sqrt(d) by default, and a launch on the caller's stream; but every
// check returns a status code instead of throwing, and nothing here depends on
// PyTorch.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <tuple>
#include <utility>

#include "fa_launch.h"
#include "../../include/fa_sm100.h"

namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

struct DeviceInfo {
  int sms = 0;
  int major = 0;
  int minor = 0;
};

// Per-device properties, queried once.
bool device_info(int dev, DeviceInfo* out) {
  static std::mutex mu;
  static std::map<int, DeviceInfo> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(dev);
  if (it != cache.end()) {
    *out = it->second;
    return true;
  }
  DeviceInfo di;
  if (cudaDeviceGetAttribute(&di.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&di.major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess) return false;
  if (cudaDeviceGetAttribute(&di.minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) return false;
  cache[dev] = di;
  *out = di;
  return true;
}

// Library-owned scheduler workspace, one per (device, stream), allocated on first
// use and kept until the process exits (256 bytes each: a process that creates
// many short-lived streams should pass its own workspace instead).  The handle
// cudaStreamPerThread names a different stream in every host thread, so for it
// the calling thread is part of the key: two threads' kernels may overlap and must
// not share a tile counter.  Like every CUDA allocation, the buffers die with
// their context: after cudaDeviceReset the cached pointers are stale, so calls
// with workspace == NULL must not follow a reset of the device in this process.
void* default_workspace(int dev, cudaStream_t stream) {
  struct Key {
    int dev;
    cudaStream_t stream;
    std::thread::id thread;
    bool operator<(const Key& o) const {
      return std::tie(dev, stream, thread) < std::tie(o.dev, o.stream, o.thread);
    }
  };
  static std::mutex mu;
  static std::map<Key, void*> cache;
  const Key key{dev, stream, stream == cudaStreamPerThread ? std::this_thread::get_id() : std::thread::id()};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) return it->second;
  void* p = nullptr;
  if (cudaMalloc(&p, fa_fwd_workspace_bytes()) != cudaSuccess) return nullptr;
  // Zeroed once; every launch leaves it zeroed again (its last CTA resets it).
  if (cudaMemset(p, 0, fa_fwd_workspace_bytes()) != cudaSuccess) {
    cudaFree(p);
    return nullptr;
  }
  cache[key] = p;
  return p;
}

int64_t pick(int64_t wide, int narrow) { return wide != 0 ? wide : static_cast<int64_t>(narrow); }

// Largest stride, in elements, that a TMA tensor map takes: strides are below 2^40 bytes.
constexpr int64_t kMaxStride = int64_t(1) << 39;
// Largest extent of a tensor, in elements (2^48 bytes, above any device memory);
// it keeps the kernel's 64-bit O and LSE addressing far from overflow.
constexpr int64_t kMaxExtent = int64_t(1) << 47;

int encode_map(CUtensorMap* map, void* base, int d, int n, int h, int b, int64_t s_seq, int64_t s_head,
               int64_t s_batch, bool bf16, const char* name) {
  const uint32_t sw = fa::swizzle_bytes(d);
  // A stride of a size-1 dimension is never followed; give TMA a valid one (a
  // multiple of 16 bytes below 2^40 bytes).
  if (h == 1) s_head = s_seq * n < kMaxStride ? s_seq * n : s_seq;
  if (b == 1) s_batch = s_head * h < kMaxStride ? s_head * h : s_head;
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(h),
                        static_cast<cuuint64_t>(b)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(s_seq) * 2, static_cast<cuuint64_t>(s_head) * 2,
                           static_cast<cuuint64_t>(s_batch) * 2};
  cuuint32_t box[4] = {sw / 2, 128, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  auto fn = get_encode_fn();
  if (!fn) return fail(FA_ERR_LAUNCH, "cuTensorMapEncodeTiled is not available from the driver");
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, base, dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  sw == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FA_ERR_BAD_ALIGN, "cuTensorMapEncodeTiled(%s) failed with CUresult %d", name, int(r));
  return FA_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

struct Strides {
  int64_t seq[4], head[4], batch[4];  // elements; index 0..3 = Q, K, V, O
};

// Every check that needs no device, in a fixed order; the first failure is
// returned.  Fills the effective 64-bit strides of Q, K, V, O.
int validate(const fa_fwd_params* p, Strides* st) {
  if (p == nullptr) return fail(FA_ERR_BAD_PARAM, "params is NULL");
  if (!p->Q || !p->K || !p->V || !p->O) return fail(FA_ERR_BAD_PARAM, "Q, K, V and O must be non-NULL");
  if (p->dtype != FA_DTYPE_F16 && p->dtype != FA_DTYPE_BF16)
    return fail(FA_ERR_UNSUPPORTED, "dtype %d is not FA_DTYPE_F16 or FA_DTYPE_BF16", p->dtype);
  const int d = p->head_dim;
  if (d != 32 && d != 64 && d != 128) return fail(FA_ERR_UNSUPPORTED, "head_dim %d not in {32, 64, 128}", d);
  if (p->batch < 1 || p->heads < 1 || p->seq_len < 1)
    return fail(FA_ERR_BAD_SHAPE, "batch (%d), heads (%d) and seq_len (%d) must be >= 1", p->batch, p->heads,
                p->seq_len);
  if (!(std::isfinite(p->softmax_scale) && p->softmax_scale > 0.f))
    return fail(FA_ERR_BAD_PARAM, "softmax_scale must be finite and > 0 (got %g)", double(p->softmax_scale));
  if (p->causal != 0 && p->causal != 1) return fail(FA_ERR_BAD_PARAM, "causal must be 0 or 1");
  const int n = p->seq_len, h = p->heads, b = p->batch;
  const void* bases[4] = {p->Q, p->K, p->V, p->O};
  const char* names[4] = {"Q", "K", "V", "O"};
  const int seq_s[4] = {p->stride_seq_q, p->stride_seq_k, p->stride_seq_v, p->stride_seq_o};
  const int head_s[4] = {p->stride_head_q, p->stride_head_k, p->stride_head_v, p->stride_head_o};
  const int batch_s[4] = {p->stride_batch_q, p->stride_batch_k, p->stride_batch_v, p->stride_batch_o};
  int64_t* ss = st->seq;
  int64_t* hs = st->head;
  int64_t* bs = st->batch;
  for (int i = 0; i < 4; ++i) {
    if (!aligned16(bases[i])) return fail(FA_ERR_BAD_ALIGN, "%s is not 16-byte aligned", names[i]);
    ss[i] = seq_s[i];
    hs[i] = pick(p->stride_head64[i], head_s[i]);
    bs[i] = pick(p->stride_batch64[i], batch_s[i]);
    if (ss[i] < d) return fail(FA_ERR_BAD_SHAPE, "stride_seq of %s (%lld) < head_dim", names[i], (long long)ss[i]);
    if ((h > 1 && hs[i] < 1) || (b > 1 && bs[i] < 1))
      return fail(FA_ERR_BAD_SHAPE, "head/batch strides of %s must be positive", names[i]);
    const int64_t chk[3] = {ss[i], h > 1 ? hs[i] : 8, b > 1 ? bs[i] : 8};
    for (int k = 0; k < 3; ++k)
      if (chk[k] % 8 != 0)
        return fail(FA_ERR_BAD_ALIGN, "strides of %s must be multiples of 8 elements (16 bytes)", names[i]);
    for (int k = 0; k < 3; ++k)
      if (chk[k] >= kMaxStride)
        return fail(FA_ERR_BAD_SHAPE, "a stride of %s is 2^40 bytes or more (the TMA limit)", names[i]);
    const __int128 extent = __int128(b - 1) * (b > 1 ? bs[i] : 0) + __int128(h - 1) * (h > 1 ? hs[i] : 0) +
                            __int128(n - 1) * ss[i] + d;
    if (extent > kMaxExtent) return fail(FA_ERR_BAD_SHAPE, "%s spans more than 2^48 bytes", names[i]);
  }
  if (p->LSE && (reinterpret_cast<uintptr_t>(p->LSE) & 3u)) return fail(FA_ERR_BAD_ALIGN, "LSE not 4-byte aligned");
  return FA_OK;
}


}  // namespace

namespace fa {
void set_last_error(const char* msg) { g_last_error = msg; }

int validate_params(const fa_fwd_params* p) {
  g_last_error.clear();
  Strides st;
  return validate(p, &st);
}

int current_sm100_device(int* dev_out, int* sms_out) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(FA_ERR_UNSUPPORTED, "no CUDA device");
  DeviceInfo di;
  if (!device_info(dev, &di)) return fail(FA_ERR_LAUNCH, "cudaDeviceGetAttribute failed on device %d", dev);
  if (di.major != 10 || di.minor != 0)
    return fail(FA_ERR_UNSUPPORTED, "device %d is sm_%d%d; this library is built for sm_100a only", dev, di.major,
                di.minor);
  *dev_out = dev;
  if (sms_out) *sms_out = di.sms;
  return FA_OK;
}
}  // namespace fa

extern "C" {

size_t fa_fwd_workspace_bytes(void) { return 256; }

size_t fa_fwd_smem_bytes(int head_dim, int dtype) {
  if (dtype != FA_DTYPE_F16 && dtype != FA_DTYPE_BF16) return 0;
  switch (head_dim) {
    case 32: return fa::Cfg<32>::SMEM_BYTES;
    case 64: return fa::Cfg<64>::SMEM_BYTES;
    case 128: return fa::Cfg<128>::SMEM_BYTES;
    default: return 0;
  }
}

const char* fa_status_string(int status) {
  switch (status) {
    case FA_OK: return "FA_OK";
    case FA_ERR_BAD_SHAPE: return "FA_ERR_BAD_SHAPE";
    case FA_ERR_BAD_ALIGN: return "FA_ERR_BAD_ALIGN";
    case FA_ERR_UNSUPPORTED: return "FA_ERR_UNSUPPORTED";
    case FA_ERR_LAUNCH: return "FA_ERR_LAUNCH";
    case FA_ERR_DEVICE_TIMEOUT: return "FA_ERR_DEVICE_TIMEOUT";
    case FA_ERR_BAD_PARAM: return "FA_ERR_BAD_PARAM";
    default: return "FA_ERR_UNKNOWN";
  }
}

const char* fa_last_error(void) { return g_last_error.c_str(); }

int fa_fwd_sm100(const fa_fwd_params* p, void* stream_ptr) {
  g_last_error.clear();
  Strides st;
  const int vrc = validate(p, &st);
  if (vrc != FA_OK) return vrc;
  const int d = p->head_dim;
  const int n = p->seq_len, h = p->heads, b = p->batch;
  const int64_t* ss = st.seq;
  const int64_t* hs = st.head;
  const int64_t* bs = st.batch;

  int dev = 0, sms = 0;
  const int drc = fa::current_sm100_device(&dev, &sms);
  if (drc != FA_OK) return drc;
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);

  void* ws = p->workspace;
  const bool caller_ws = ws != nullptr;
  if (caller_ws) {
    if (p->workspace_bytes < fa_fwd_workspace_bytes() || !aligned16(ws))
      return fail(FA_ERR_BAD_PARAM, "workspace must be >= %zu bytes and 16-byte aligned", fa_fwd_workspace_bytes());
  } else {
    ws = default_workspace(dev, stream);
    if (!ws) return fail(FA_ERR_LAUNCH, "could not allocate the scheduler workspace");
  }

  const bool bf16 = p->dtype == FA_DTYPE_BF16;
  fa::LaunchSpec s;
  std::memset(&s, 0, sizeof(s));
  int rc;
  if ((rc = encode_map(&s.tq, p->Q, d, n, h, b, ss[0], hs[0], bs[0], bf16, "Q")) != FA_OK) return rc;
  if ((rc = encode_map(&s.tk, p->K, d, n, h, b, ss[1], hs[1], bs[1], bf16, "K")) != FA_OK) return rc;
  if ((rc = encode_map(&s.tv, p->V, d, n, h, b, ss[2], hs[2], bs[2], bf16, "V")) != FA_OK) return rc;

  fa::KernelParams& kp = s.kp;
  kp.O = p->O;
  kp.LSE = p->LSE;
  kp.o_stride_b = bs[3];
  kp.o_stride_h = hs[3];
  kp.o_stride_s = ss[3];
  kp.batch = b;
  kp.heads = h;
  kp.seq_len = n;
  kp.scale_log2 = p->softmax_scale * 1.4426950408889634f;
  const fa::SchedPlan plan = fa::plan_schedule(b, h, n, d, fa::kBlockN, sms, p->causal != 0);
  if (plan.num_tiles < 0)
    return fail(FA_ERR_BAD_SHAPE, "batch*heads*ceil(N/256) = %lld tiles is too many",
                static_cast<long long>(b) * h * plan.n_pairs);
  kp.n_pairs = plan.n_pairs;
  kp.n_kv = plan.n_kv;
  kp.num_tiles = plan.num_tiles;
  kp.group_bh = plan.group_bh;
  kp.tile_counter = static_cast<int*>(ws);
  kp.status = p->status;
  kp.timeout_ns = p->timeout_ns ? p->timeout_ns : 2000000000ull;
  s.grid = plan.grid;
  s.stream = stream;
  s.bf16 = bf16;
  s.causal = p->causal != 0;

  // The scheduler's two counter words start at zero.  A library-owned workspace
  // is zeroed at allocation and every launch leaves it zeroed; a caller's
  // workspace is cleared here, on the caller's stream, as the interface promises.
  cudaError_t e = cudaSuccess;
  if (caller_ws) {
    e = cudaMemsetAsync(ws, 0, 2 * sizeof(int), stream);
    if (e != cudaSuccess) return fail(FA_ERR_LAUNCH, "cudaMemsetAsync(workspace): %s", cudaGetErrorString(e));
  }
  switch (d) {
    case 32: e = fa::launch_d32(s); break;
    case 64: e = fa::launch_d64(s); break;
    default: e = fa::launch_d128(s); break;
  }
  if (e != cudaSuccess) return fail(FA_ERR_LAUNCH, "kernel launch failed: %s", cudaGetErrorString(e));
  return FA_OK;
}

}  // extern "C"
