// TEST INFRASTRUCTURE ONLY - builds the reference's OWN CPU attention from the
// file where it lies (wenssir/flash-attention benchmark/cpp/correctness_v6.cu,
// function cpu_reference_attention at :23-72) into oracle/_ref/libref_attention.so.
// Nothing is copied: the reference translation unit is #included in place
// (include path set by oracle/Makefile) with its main() renamed so the result
// can be a shared library.  Used to pin the oracle restatement bit-for-bit and as
// the timed CPU baseline of the reference arm.
#define main fa_reference_correctness_v6_main
#include "correctness_v6.cu"
#undef main

#include <thread>
#include <vector>

extern "C" {

// Direct call of the reference function: fp32 [B, H, N, D] contiguous.
void ref_cpu_reference_attention(const float* q, const float* k, const float* v, float* o, int B, int H, int N,
                                 int D, float scale, int causal) {
  cpu_reference_attention(q, k, v, o, B, H, N, D, scale, causal != 0);
}

// The reference function applied per (b, h) slice (B = H = 1 on offset
// pointers, as its own loop does), slices [begin, end) spread over threads.
void ref_cpu_attention_slices(const float* q, const float* k, const float* v, float* o, int slice_begin,
                              int slice_end, int N, int D, float scale, int causal, int threads) {
  if (threads <= 0) threads = static_cast<int>(std::thread::hardware_concurrency());
  if (threads < 1) threads = 1;
  const int count = slice_end - slice_begin;
  if (count <= 0) return;
  if (threads > count) threads = count;
  const long long per = static_cast<long long>(N) * D;
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) {
    pool.emplace_back([=] {
      for (int s = slice_begin + t; s < slice_end; s += threads)
        cpu_reference_attention(q + s * per, k + s * per, v + s * per, o + s * per, 1, 1, N, D, scale,
                                causal != 0);
    });
  }
  for (auto& th : pool) th.join();
}

}  // extern "C"
