// TEST INFRASTRUCTURE ONLY - the parity oracle and the timed CPU baseline ("port").
// Nothing on the product path links or calls this file; only tests/, the smoke
// check of __graft_entry__.py and bench.py's CPU-baseline leg load it.
//
// CPU restatement of the reference's own attention oracle `cpu_reference_attention`
// (wenssir/flash-attention benchmark/cpp/correctness_v6.cu:23-72; identical copies
// at benchmark/cpp/correctness_v4.cu:15-64 and benchmark/cpp/correctness.cu:13-54):
// fp32 throughout, per query row i an online softmax over all keys j in order,
//   s = (sum_d q[i,d] * k[j,d]) * scale;  s = -inf if causal and j > i
//   m' = max(m, s); alpha = exp(m - m'); p = exp(s - m')
//   acc[d] = acc[d] * alpha + p * v[j,d];  l = l * alpha + p;  m = m'
//   o[i,d] = acc[d] * (1 / l)
// with the same operation order, so its output is bit-identical to the
// reference's when both are compiled without floating-point contraction.
// Added here (the reference has no logsumexp): lse[i] = m + log(l), natural log,
// scale included.  Slices (b, h) are independent and are spread over threads;
// this does not change any result bit.  With the causal mask, the keys j > i are
// skipped: for them the reference computes s = -inf, m' = m (key 0 already made
// m finite), alpha = exp(0) = 1 and p = exp(-inf) = 0, so acc = acc * 1 + 0 * v
// and l = l * 1 + 0 leave every value unchanged (at most the sign of a zero in
// acc), and the output equals the reference's, at half the cost.
#include <cmath>
#include <thread>
#include <vector>

namespace {

void attention_slice(const float* q, const float* k, const float* v, float* o, float* lse, int n, int d,
                     float scale, bool causal) {
  std::vector<float> acc(d);
  for (int i = 0; i < n; ++i) {
    float m = -INFINITY;
    float l = 0.0f;
    for (int c = 0; c < d; ++c) acc[c] = 0.0f;
    const int j_end = causal ? i + 1 : n;
    for (int j = 0; j < j_end; ++j) {
      float s = 0.0f;
      for (int c = 0; c < d; ++c) s += q[i * d + c] * k[j * d + c];
      s *= scale;
      const float m_new = fmaxf(m, s);
      const float alpha = expf(m - m_new);
      const float p = expf(s - m_new);
      for (int c = 0; c < d; ++c) acc[c] = acc[c] * alpha + p * v[j * d + c];
      l = l * alpha + p;
      m = m_new;
    }
    const float inv_l = 1.0f / l;
    for (int c = 0; c < d; ++c) o[i * d + c] = acc[c] * inv_l;
    if (lse) lse[i] = m + logf(l);
  }
}

}  // namespace

extern "C" {

// q, k, v, o: contiguous fp32 [B, H, N, D]; lse: fp32 [B, H, N] or NULL.
// Processes slices [slice_begin, slice_end) of the B*H slices with `threads`
// worker threads (<= 0: hardware concurrency).
void oracle_attention_slices(const float* q, const float* k, const float* v, float* o, float* lse, int slice_begin,
                             int slice_end, int n, int d, float scale, int causal, int threads) {
  if (threads <= 0) threads = static_cast<int>(std::thread::hardware_concurrency());
  if (threads < 1) threads = 1;
  const long long per = static_cast<long long>(n) * d;
  const int count = slice_end - slice_begin;
  if (count <= 0) return;
  if (threads > count) threads = count;
  std::vector<std::thread> pool;
  for (int t = 0; t < threads; ++t) {
    pool.emplace_back([=] {
      for (int s = slice_begin + t; s < slice_end; s += threads)
        attention_slice(q + s * per, k + s * per, v + s * per, o + s * per, lse ? lse + static_cast<long long>(s) * n : nullptr,
                        n, d, scale, causal != 0);
    });
  }
  for (auto& th : pool) th.join();
}

void oracle_attention(const float* q, const float* k, const float* v, float* o, float* lse, int B, int H, int N,
                      int D, float scale, int causal, int threads) {
  oracle_attention_slices(q, k, v, o, lse, 0, B * H, N, D, scale, causal, threads);
}

}  // extern "C"
