// Test infrastructure (parity oracle): the summation order of torch's CPU sum over a contiguous
// fp32 vector, which the reference's prior normalisation `priors / (priors.sum() + 1e-8)`
// (python/mcts/core/wave_search.py:894-895) runs on its CPU path.
#pragma once

float torch_cpu_sum(const float* x, int n);

extern "C" float oracle_torch_sum(const float* x, int n);
