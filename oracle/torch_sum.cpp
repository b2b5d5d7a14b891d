// Test infrastructure (parity oracle). Restates the order in which torch's CPU reduction adds a
// contiguous fp32 vector (ATen's cascade sum for an inner reduction: vectorized_inner_sum ->
// row_sum -> multi_row_sum in aten/src/ATen/native/cpu/SumKernel.cpp, torch 2.x), the sum the
// reference's `priors.sum()` (python/mcts/core/wave_search.py:894-895) performs:
//   * the vector is read as 8-lane vectors (the fp32 vector width of the kernel's load policy);
//   * 4 interleaved vector accumulators ("ILP" rows of 4 vectors = 32 elements) add rows in order;
//     after every 2^p rows (p = max(4, ceil(log2(rows)) / 4)) each cascade level is added into the
//     next one and restarted, stopping at the first level whose block is not complete;
//   * full vectors after the last complete row go into accumulator 0; accumulators are then
//     combined as ((a0 + a1) + a2) + a3, lane by lane;
//   * a scalar starting at 0 adds the elements after the last full vector, then the 8 lanes in order;
//   * fewer than 8 elements: the same scheme with 4 scalar accumulators.
// tests/test_oracle_golden.py pins it bit for bit against torch.sum for lengths 1..5000.
#include "torch_sum.h"

#include <algorithm>

namespace {

int ceil_log2(long x) {
  if (x <= 2) return 1;
  int b = 0;
  unsigned long v = (unsigned long)(x - 1);
  while (v) { ++b; v >>= 1; }
  return b;
}

// multi_row_sum over `rows` items of `nrows` accumulators x `lanes` lanes; item i, accumulator k,
// lane l is x[i * nrows * lanes + k * lanes + l].
void multi_row(const float* x, long rows, int nrows, int lanes, float* out /* [nrows*lanes] */) {
  const int kLevels = 4;
  const int lp = std::max(4, ceil_log2(rows) / kLevels);
  const long step = 1L << lp, mask = step - 1;
  const int w = nrows * lanes;
  float acc[kLevels][32] = {};
  long i = 0;
  while (i + step <= rows) {
    for (long j = 0; j < step; ++j, ++i)
      for (int e = 0; e < w; ++e) acc[0][e] = acc[0][e] + x[i * w + e];
    for (int l = 1; l < kLevels; ++l) {
      for (int e = 0; e < w; ++e) {
        acc[l][e] = acc[l][e] + acc[l - 1][e];
        acc[l - 1][e] = 0.0f;
      }
      if (i & (mask << (l * lp))) break;
    }
  }
  for (; i < rows; ++i)
    for (int e = 0; e < w; ++e) acc[0][e] = acc[0][e] + x[i * w + e];
  for (int l = 1; l < kLevels; ++l)
    for (int e = 0; e < w; ++e) acc[0][e] = acc[0][e] + acc[l][e];
  for (int e = 0; e < w; ++e) out[e] = acc[0][e];
}

// row_sum: 4 interleaved accumulators of `lanes` lanes over `items` items, remainder into 0
void row_sum(const float* x, long items, int lanes, float* out /* [lanes] */) {
  const long rows = items / 4;
  float ps[32];
  multi_row(x, rows, 4, lanes, ps);
  for (long i = rows * 4; i < items; ++i)
    for (int l = 0; l < lanes; ++l) ps[l] = ps[l] + x[i * lanes + l];
  for (int k = 1; k < 4; ++k)
    for (int l = 0; l < lanes; ++l) ps[l] = ps[l] + ps[k * lanes + l];
  for (int l = 0; l < lanes; ++l) out[l] = ps[l];
}

}  // namespace

float torch_cpu_sum(const float* x, int n) {
  constexpr int V = 8;
  if (n < V) {
    float r;
    row_sum(x, n, 1, &r);
    return r;
  }
  const long vecs = n / V;
  float lanes[V];
  row_sum(x, vecs, V, lanes);
  float fin = 0.0f;
  for (long k = vecs * V; k < n; ++k) fin = fin + x[k];
  for (int l = 0; l < V; ++l) fin = fin + lanes[l];
  return fin;
}

extern "C" float oracle_torch_sum(const float* x, int n) { return torch_cpu_sum(x, n); }
