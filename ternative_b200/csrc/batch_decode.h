// Kernels of the batched decode step (batch_decode.cu): B independent
// sequences advance one token each, every weight byte read once per step.
#pragma once

#include "gemv.cuh"

namespace tvb {

constexpr int kMaxBatch = 32;   // sequences per batched step (argmax key area)

// Attention of B sequences, one query row each (Model::forward_gpu's
// attention_d, model.cpp:1413-1417, per sequence): sequence b attends over KV
// rows [0, pos[b]] of its cache slot (kcache + b * slot_stride, layer rows
// [pos][nkv * hd]).  q [B][nh * hd] -> out [B][nh * hd].  `part` holds
// B * nh * nsplit * (hd + 4) floats of split partials.
tvb_status batch_attention(const float* q, const float* kcache, const float* vcache, size_t slot_stride,
                           const int* pos, int B, int nh, int nkv, int hd, int nsplit, float scale, float* part,
                           float* out, cudaStream_t st, bool pdl = false);

// Per-row greedy argmax of logits [B][ld] (n valid columns, global index =
// vocab0 + column): keys[b] = the packed (ordered value, ~index) maximum.
tvb_status batch_argmax(const float* logits, int B, int n, int ld, int vocab0, unsigned long long* keys,
                        cudaStream_t st, bool pdl = false);

// next[b] = index of the largest key over the sources (one per tensor-parallel
// rank, in rank order; a single source without tensor parallelism).
struct KeySources {
    const unsigned long long* p[kMaxTp];
    int n;
};
tvb_status batch_pick(const KeySources& src, int B, int* next, cudaStream_t st, bool pdl = false);

}  // namespace tvb
