// Device-side token sampling and log-probabilities (sampler.cu).
#pragma once

#include "common.cuh"

namespace tvb {

constexpr int kMaxLogprobsHost = 64;   // top entries per scored token

// Per row r of logits [n][ld] (V valid columns): out_lp[r] = the log-probability
// of token target[r]; with k > 0 the k largest log-probabilities (descending,
// equal values by smaller index) and their token ids.
tvb_status logprob_rows(const float* logits, int n, int V, int ld, const int* target, int k, float* out_lp,
                        int* out_ids, float* out_top, cudaStream_t st);

}  // namespace tvb
