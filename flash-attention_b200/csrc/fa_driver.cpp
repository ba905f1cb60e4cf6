// fa_driver: a C++-only driver for fa_fwd_sm100 (no Python, no torch).
//
// It replaces the reference's C++ drivers, which fill a config::ForwardKernelArgs
// and launch the v6 kernel themselves (benchmark/cpp/benchmark_v6.cu:120-155,
// benchmark/cpp/correctness_v6.cu:144-188), and keeps their command line:
//
//   fa_driver [config|BxHxNxD] [--mode benchmark|ncu] [--warmup-iters N] [--benchmark-iters N]
//             [--dtype f16|bf16] [--causal|--non-causal] [--scale S] [--seed S] [--flush] [--dump DIR]
//
// config is one of the benchmark workloads (cfg0, cfg1, cfg2, cfg3, cfg4_d32,
// cfg4_d64, cfg4_d128) and sets shape, dtype and mask; a BxHxNxD shape takes
// --dtype (default f16) and --causal (default non-causal); --dtype, --causal
// and --non-causal also override a named workload's.  Inputs are N(0,1) from a
// counter-based generator (seeded, the same on every machine), rounded to the
// dtype on the host and copied to the device once.  Each timed iteration is one launch between
// two CUDA events on the driver's stream; --flush writes 256 MiB (twice the L2)
// before every launch so that small workloads do not run from L2.  --mode ncu
// defaults to 0 warm-up and 1 timed iteration, for a profiler capture.
//
// It prints one JSON line: shape, dtype, mask, per-launch times (median, mean,
// min), TFLOPS (4*B*H*N^2*d, halved for causal), the kernel's status word, and
// the number of non-finite outputs.  --dump DIR also writes q.bin, k.bin and
// v.bin (raw 16-bit inputs), o.bin (16-bit output), lse.bin (fp32) and
// meta.json, so that a test can check the driver's results against a CPU
// attention.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cerrno>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "fa_sm100.h"

namespace {

struct Workload {
  const char* name;
  int b, h, n, d, dtype, causal;
};

// The benchmark workloads: shape, dtype and mask.
constexpr Workload kWorkloads[] = {
    {"cfg0", 1, 4, 256, 64, FA_DTYPE_F16, 0},      {"cfg1", 4, 16, 1024, 64, FA_DTYPE_F16, 0},
    {"cfg2", 8, 32, 4096, 128, FA_DTYPE_BF16, 1},  {"cfg3", 2, 32, 16384, 128, FA_DTYPE_BF16, 1},
    {"cfg4_d32", 16, 16, 2048, 32, FA_DTYPE_F16, 0}, {"cfg4_d64", 16, 16, 2048, 64, FA_DTYPE_F16, 0},
    {"cfg4_d128", 16, 16, 2048, 128, FA_DTYPE_F16, 0},
};

struct Options {
  Workload w{"custom", 0, 0, 0, 0, FA_DTYPE_F16, 0};
  bool ncu = false;
  int warmup = -1, iters = -1;  // -1: the mode's default
  float scale = 0.0f;           // 0: 1/sqrt(d)
  uint64_t seed = 0;
  bool flush = false;
  std::string dump;
};

void usage(const char* argv0) {
  std::printf(
      "Usage: %s [config|BxHxNxD] [--mode benchmark|ncu] [--warmup-iters N] [--benchmark-iters N]\n"
      "          [--dtype f16|bf16] [--causal|--non-causal] [--scale S] [--seed S] [--flush] [--dump DIR]\n"
      "  config: cfg0 cfg1 cfg2 cfg3 cfg4_d32 cfg4_d64 cfg4_d128 (default cfg2)\n"
      "  mode=benchmark default: warmup=10, benchmark=100\n"
      "  mode=ncu default: warmup=0, benchmark=1\n",
      argv0);
}

[[noreturn]] void die(const char* fmt, const char* arg) {
  std::fprintf(stderr, fmt, arg);
  std::fputc('\n', stderr);
  std::exit(2);
}

bool parse_int(const char* s, long long lo, long long hi, long long* out) {
  char* end = nullptr;
  errno = 0;
  const long long v = std::strtoll(s, &end, 10);
  if (errno != 0 || end == s || *end != '\0' || v < lo || v > hi) return false;
  *out = v;
  return true;
}

bool parse_shape(const char* s, Workload* w) {
  long long v[4];
  std::string str(s);
  size_t pos = 0;
  for (int i = 0; i < 4; ++i) {
    const size_t x = str.find('x', pos);
    if ((i < 3) != (x != std::string::npos)) return false;
    const std::string part = str.substr(pos, i < 3 ? x - pos : std::string::npos);
    if (!parse_int(part.c_str(), 1, 1ll << 30, &v[i])) return false;
    pos = x + 1;
  }
  w->name = "custom";
  w->b = int(v[0]);
  w->h = int(v[1]);
  w->n = int(v[2]);
  w->d = int(v[3]);
  return true;
}

Options parse(int argc, char** argv) {
  Options o;
  bool have_shape = false, dtype_set = false, causal_set = false;
  for (int i = 1; i < argc; ++i) {
    const std::string a = argv[i];
    auto value = [&](const char* flag) -> const char* {
      if (i + 1 >= argc) die("%s needs a value", flag);
      return argv[++i];
    };
    long long n = 0;
    if (a == "-h" || a == "--help") {
      usage(argv[0]);
      std::exit(0);
    } else if (a == "--mode") {
      const std::string m = value("--mode");
      if (m == "ncu") o.ncu = true;
      else if (m != "benchmark") die("invalid --mode %s (expected benchmark|ncu)", m.c_str());
    } else if (a == "--warmup-iters") {
      if (!parse_int(value("--warmup-iters"), 0, 1000000, &n)) die("bad --warmup-iters %s", argv[i]);
      o.warmup = int(n);
    } else if (a == "--benchmark-iters") {
      if (!parse_int(value("--benchmark-iters"), 1, 1000000, &n)) die("bad --benchmark-iters %s", argv[i]);
      o.iters = int(n);
    } else if (a == "--dtype") {
      const std::string t = value("--dtype");
      if (t == "f16" || t == "fp16") o.w.dtype = FA_DTYPE_F16;
      else if (t == "bf16") o.w.dtype = FA_DTYPE_BF16;
      else die("invalid --dtype %s (expected f16|bf16)", t.c_str());
      dtype_set = true;
    } else if (a == "--causal" || a == "--non-causal") {
      o.w.causal = a == "--causal";
      causal_set = true;
    } else if (a == "--scale") {
      char* end = nullptr;
      const char* s = value("--scale");
      o.scale = std::strtof(s, &end);
      if (end == s || *end != '\0' || !(o.scale > 0.0f) || !std::isfinite(o.scale)) die("bad --scale %s", s);
    } else if (a == "--seed") {
      if (!parse_int(value("--seed"), 0, (1ll << 62), &n)) die("bad --seed %s", argv[i]);
      o.seed = uint64_t(n);
    } else if (a == "--flush") {
      o.flush = true;
    } else if (a == "--dump") {
      o.dump = value("--dump");
    } else if (!a.empty() && a[0] == '-') {
      die("unknown option %s", a.c_str());
    } else if (have_shape) {
      die("unexpected extra argument %s", a.c_str());
    } else {
      have_shape = true;
      bool found = false;
      for (const Workload& w : kWorkloads) {
        if (a == w.name) {
          const int dt = o.w.dtype, c = o.w.causal;
          o.w = w;
          if (dtype_set) o.w.dtype = dt;
          if (causal_set) o.w.causal = c;
          found = true;
        }
      }
      if (!found) {
        if (!parse_shape(a.c_str(), &o.w)) die("not a workload name or BxHxNxD shape: %s", a.c_str());
      }
    }
  }
  if (!have_shape) {
    const int dt = o.w.dtype, c = o.w.causal;
    o.w = kWorkloads[2];
    if (dtype_set) o.w.dtype = dt;
    if (causal_set) o.w.causal = c;
  }
  if (o.warmup < 0) o.warmup = o.ncu ? 0 : 10;
  if (o.iters < 0) o.iters = o.ncu ? 1 : 100;
  if (o.scale == 0.0f) o.scale = 1.0f / std::sqrt(float(o.w.d));
  return o;
}

// Counter-based N(0,1): element i of tensor t is a function of (seed, t, i)
// alone, so threads can fill disjoint ranges in any order.  splitmix64 mixing,
// Box-Muller on two 53-bit uniforms.
uint64_t mix(uint64_t x) {
  x += 0x9e3779b97f4a7c15ull;
  x = (x ^ (x >> 30)) * 0xbf58476d1ce4e5b9ull;
  x = (x ^ (x >> 27)) * 0x94d049bb133111ebull;
  return x ^ (x >> 31);
}

float normal_at(uint64_t seed, uint64_t tensor, uint64_t i) {
  const uint64_t base = mix(seed ^ mix(tensor * 0x100000001b3ull + 1)) + 2 * i;
  const double u1 = (double((mix(base) >> 11) + 1)) * 0x1.0p-53;  // (0, 1]
  const double u2 = double(mix(base + 1) >> 11) * 0x1.0p-53;       // [0, 1)
  return float(std::sqrt(-2.0 * std::log(u1)) * std::cos(6.283185307179586 * u2));
}

uint16_t to_bits(float x, int dtype) {
  uint16_t b;
  if (dtype == FA_DTYPE_BF16) {
    const __nv_bfloat16 v = __float2bfloat16_rn(x);
    std::memcpy(&b, &v, 2);
  } else {
    const __half v = __float2half_rn(x);
    std::memcpy(&b, &v, 2);
  }
  return b;
}

float from_bits(uint16_t b, int dtype) {
  if (dtype == FA_DTYPE_BF16) {
    const uint32_t u = uint32_t(b) << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
  }
  __half v;
  std::memcpy(&v, &b, 2);
  return __half2float(v);
}

template <typename F>
void parallel_for(size_t n, F f) {
  const unsigned t = std::max(1u, std::min(32u, std::thread::hardware_concurrency()));
  std::vector<std::thread> pool;
  const size_t chunk = (n + t - 1) / t;
  for (unsigned k = 0; k < t; ++k) {
    const size_t lo = std::min(n, size_t(k) * chunk), hi = std::min(n, lo + chunk);
    if (lo < hi) pool.emplace_back([=] { f(lo, hi); });
  }
  for (auto& th : pool) th.join();
}

#define CHECK_CUDA(call)                                                                             \
  do {                                                                                               \
    const cudaError_t e_ = (call);                                                                   \
    if (e_ != cudaSuccess) {                                                                         \
      std::fprintf(stderr, "%s failed: %s\n", #call, cudaGetErrorString(e_));                        \
      std::exit(1);                                                                                  \
    }                                                                                                \
  } while (0)

bool write_file(const std::string& path, const void* data, size_t bytes) {
  FILE* f = std::fopen(path.c_str(), "wb");
  if (!f) return false;
  const bool ok = std::fwrite(data, 1, bytes, f) == bytes;
  return std::fclose(f) == 0 && ok;
}

}  // namespace

int main(int argc, char** argv) {
  const Options o = parse(argc, argv);
  const Workload& w = o.w;
  const size_t elems = size_t(w.b) * w.h * w.n * w.d;
  const size_t rows = size_t(w.b) * w.h * w.n;
  const char* dtype_name = w.dtype == FA_DTYPE_BF16 ? "bf16" : "f16";

  int dev_count = 0;
  if (cudaGetDeviceCount(&dev_count) != cudaSuccess || dev_count == 0) {
    std::fprintf(stderr, "fa_driver: no CUDA device\n");
    return 1;
  }

  std::vector<uint16_t> host[3];
  for (int t = 0; t < 3; ++t) {
    host[t].resize(elems);
    uint16_t* dst = host[t].data();
    parallel_for(elems, [&, dst, t](size_t lo, size_t hi) {
      for (size_t i = lo; i < hi; ++i) dst[i] = to_bits(normal_at(o.seed, uint64_t(t), i), w.dtype);
    });
  }

  cudaStream_t stream;
  CHECK_CUDA(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking));
  void* dev[4];
  float* lse = nullptr;
  int* status = nullptr;
  void* flush_buf = nullptr;
  const size_t flush_bytes = size_t(256) << 20;
  for (int t = 0; t < 4; ++t) CHECK_CUDA(cudaMalloc(&dev[t], elems * 2));
  CHECK_CUDA(cudaMalloc(&lse, rows * sizeof(float)));
  CHECK_CUDA(cudaMalloc(&status, sizeof(int)));
  CHECK_CUDA(cudaMemset(status, 0, sizeof(int)));
  if (o.flush) CHECK_CUDA(cudaMalloc(&flush_buf, flush_bytes));
  for (int t = 0; t < 3; ++t) CHECK_CUDA(cudaMemcpy(dev[t], host[t].data(), elems * 2, cudaMemcpyHostToDevice));

  // The reference drivers' ForwardKernelArgs, field for field, plus the appended fields.
  fa_fwd_params p;
  std::memset(&p, 0, sizeof(p));
  p.Q = dev[0];
  p.K = dev[1];
  p.V = dev[2];
  p.O = dev[3];
  const long long sb = (long long)w.h * w.n * w.d, sh = (long long)w.n * w.d;
  int* strides[4][3] = {{&p.stride_batch_q, &p.stride_head_q, &p.stride_seq_q},
                        {&p.stride_batch_k, &p.stride_head_k, &p.stride_seq_k},
                        {&p.stride_batch_v, &p.stride_head_v, &p.stride_seq_v},
                        {&p.stride_batch_o, &p.stride_head_o, &p.stride_seq_o}};
  for (int t = 0; t < 4; ++t) {
    // int fields where they fit, the 64-bit overrides where they do not
    *strides[t][0] = sb <= INT32_MAX ? int(sb) : 0;
    *strides[t][1] = sh <= INT32_MAX ? int(sh) : 0;
    *strides[t][2] = w.d;
    if (sb > INT32_MAX) p.stride_batch64[t] = sb;
    if (sh > INT32_MAX) p.stride_head64[t] = sh;
  }
  p.seq_len = w.n;
  p.heads = w.h;
  p.head_dim = w.d;
  p.softmax_scale = o.scale;
  p.causal = w.causal;
  p.LSE = lse;
  p.dtype = w.dtype;
  p.batch = w.b;
  p.status = status;

  auto launch = [&]() {
    const int rc = fa_fwd_sm100(&p, stream);
    if (rc != FA_OK) {
      std::fprintf(stderr, "fa_fwd_sm100: %s: %s\n", fa_status_string(rc), fa_last_error());
      std::exit(1);
    }
  };

  for (int i = 0; i < o.warmup; ++i) launch();
  CHECK_CUDA(cudaStreamSynchronize(stream));

  std::vector<cudaEvent_t> ev(2 * size_t(o.iters));
  for (auto& e : ev) CHECK_CUDA(cudaEventCreate(&e));
  for (int i = 0; i < o.iters; ++i) {
    if (o.flush) CHECK_CUDA(cudaMemsetAsync(flush_buf, i & 0xff, flush_bytes, stream));
    CHECK_CUDA(cudaEventRecord(ev[2 * i], stream));
    launch();
    CHECK_CUDA(cudaEventRecord(ev[2 * i + 1], stream));
  }
  CHECK_CUDA(cudaStreamSynchronize(stream));
  std::vector<float> ms(o.iters);
  for (int i = 0; i < o.iters; ++i) CHECK_CUDA(cudaEventElapsedTime(&ms[i], ev[2 * i], ev[2 * i + 1]));
  int status_word = 0;
  CHECK_CUDA(cudaMemcpy(&status_word, status, sizeof(int), cudaMemcpyDeviceToHost));

  std::vector<uint16_t> out(elems);
  std::vector<float> lse_host(rows);
  CHECK_CUDA(cudaMemcpy(out.data(), dev[3], elems * 2, cudaMemcpyDeviceToHost));
  CHECK_CUDA(cudaMemcpy(lse_host.data(), lse, rows * sizeof(float), cudaMemcpyDeviceToHost));
  size_t nonfinite = 0;
  for (size_t i = 0; i < elems; ++i) nonfinite += !std::isfinite(from_bits(out[i], w.dtype));
  for (size_t i = 0; i < rows; ++i) nonfinite += !std::isfinite(lse_host[i]);

  std::vector<float> sorted = ms;
  std::sort(sorted.begin(), sorted.end());
  const double median = sorted[sorted.size() / 2];
  double mean = 0;
  for (float x : ms) mean += x;
  mean /= ms.size();
  const double flops = 4.0 * w.b * w.h * double(w.n) * w.n * w.d * (w.causal ? 0.5 : 1.0);

  if (!o.dump.empty()) {
    bool ok = write_file(o.dump + "/q.bin", host[0].data(), elems * 2) &&
              write_file(o.dump + "/k.bin", host[1].data(), elems * 2) &&
              write_file(o.dump + "/v.bin", host[2].data(), elems * 2) &&
              write_file(o.dump + "/o.bin", out.data(), elems * 2) &&
              write_file(o.dump + "/lse.bin", lse_host.data(), rows * sizeof(float));
    char meta[256];
    std::snprintf(meta, sizeof(meta), "{\"shape\": [%d, %d, %d, %d], \"dtype\": \"%s\", \"causal\": %d, \"scale\": %.9g}\n",
                  w.b, w.h, w.n, w.d, dtype_name, w.causal, double(o.scale));
    ok = ok && write_file(o.dump + "/meta.json", meta, std::strlen(meta));
    if (!ok) {
      std::fprintf(stderr, "fa_driver: cannot write the dump to %s\n", o.dump.c_str());
      return 1;
    }
  }

  std::printf(
      "{\"workload\": \"%s\", \"shape\": [%d, %d, %d, %d], \"dtype\": \"%s\", \"causal\": %d, \"scale\": %.9g, "
      "\"seed\": %llu, \"mode\": \"%s\", \"warmup\": %d, \"iters\": %d, \"l2_flush\": %s, "
      "\"ms_median\": %.6f, \"ms_mean\": %.6f, \"ms_min\": %.6f, \"tflops\": %.2f, \"status\": %d, "
      "\"nonfinite\": %zu}\n",
      w.name, w.b, w.h, w.n, w.d, dtype_name, w.causal, double(o.scale), (unsigned long long)o.seed,
      o.ncu ? "ncu" : "benchmark", o.warmup, o.iters, o.flush ? "true" : "false", median, mean, double(sorted[0]),
      flops / (median * 1e-3) / 1e12, status_word, nonfinite);

  for (auto& e : ev) cudaEventDestroy(e);
  for (int t = 0; t < 4; ++t) cudaFree(dev[t]);
  cudaFree(lse);
  cudaFree(status);
  if (flush_buf) cudaFree(flush_buf);
  cudaStreamDestroy(stream);
  return (status_word == 0 && nonfinite == 0) ? 0 : 3;
}
