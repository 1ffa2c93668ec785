// Tensor-parallel batched prefill: the exchanges between the tensor-core
// kernels of prefill.cu when each rank holds a shard of every layer
// (q/k/v and gate/up by rows, o_proj and down by columns).
//
// Every rank's exchange buffer (the IPC mapping the decode step uses) holds,
// after the decode area, two prefill regions; one region is `rows` partial
// output rows [rows][H] followed by `rows` per-row sums of squares.  A rank
// writes only its own regions; the others read them over NVLink after a flag
// sync.  Per layer:
//
//   attention -> sub-norm input scaled by its weight, row sums of squares out
//   -> o_proj partial rows (region 0) -> sync -> residual += inv_rms * sum of
//   the ranks' partial rows (rank order) -> ffn_norm -> gate/up -> the same
//   with down (region 1).
//
// The sub-norm's 1/rms needs the squares of the full row, which the ranks hold
// in parts; o_proj and down are linear, so each rank multiplies its shard
// un-normalised and the reduction applies the factor of the summed squares
// (as the decode step's fold does).  A region is rewritten one exchange after
// its sync: by then every rank has signalled the next sync, which it does only
// after its reads of the region, so two regions need no extra sync.
#include "tp_prefill.h"

#include <algorithm>

namespace tvb {

// One thread: order this rank's earlier writes (previous kernels of the
// stream) at system scope, signal every rank, wait (bounded) for all of them.
__global__ void tp_sync_kernel(const __grid_constant__ TpArgs t, StepState* st) {
    pdl_wait();   // launched after the kernel that writes this one's inputs
    pdl_launch_dependents();
    const unsigned e = st->tp_epoch + 1u;
    tp_signal(t, e);
    if (tp_wait(t, e, &st->abort, &st->status)) st->tp_epoch = e;
}

// Row s of x [S][H] += inv_s * (sum over ranks, in rank order, of their partial
// row s at float offset `off`), inv_s = 1/sqrt(sum_r ss_r[s] / norm_n + eps)
// (tensor.cpp:672-673) or 1 without a sub-norm (norm_n == 0).  Block (s, y)
// takes float4 y * blockDim.x + tid of row s.  The partials live in every
// rank's own buffer and are read over NVLink: a thread issues all ranks' loads
// (and thread 0 all ranks' sums of squares) before it uses any, so the kernel
// waits one remote round trip, where a loop of load-then-add waited one per
// rank and per float4.
__global__ void tp_reduce_rows_kernel(const __grid_constant__ TpArgs t, size_t off, int S, int H, int norm_n,
                                      float eps, float* __restrict__ x) {
    pdl_wait();   // launched after the kernel that writes this one's inputs
    pdl_launch_dependents();
    const int row = blockIdx.x, tid = threadIdx.x;
    const int k = blockIdx.y * blockDim.x + tid;
    const bool in = k < (H >> 2);
    const size_t base = off + (size_t)row * H;
    float4* x4 = reinterpret_cast<float4*>(x + (size_t)row * H);
    float4 p[kMaxTp];
    float ssr[kMaxTp];
#pragma unroll
    for (int r = 0; r < kMaxTp; ++r) {
        p[r] = (r < t.world && in) ? __ldcg(reinterpret_cast<const float4*>(t.peer[r] + base) + k)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
        ssr[r] = (tid == 0 && norm_n > 0 && r < t.world) ? __ldcg(t.peer[r] + off + (size_t)S * H + row) : 0.f;
    }
    float4 v = in ? x4[k] : make_float4(0.f, 0.f, 0.f, 0.f);
    __shared__ float s_inv;
    if (tid == 0) {
        float inv = 1.0f;
        if (norm_n > 0) {
            float ss = 0.f;
#pragma unroll
            for (int r = 0; r < kMaxTp; ++r)
                if (r < t.world) ss += ssr[r];
            inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)norm_n), eps)));
        }
        s_inv = inv;
    }
    __syncthreads();
    if (!in) return;
    const float inv = s_inv;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int r = 0; r < kMaxTp; ++r)
        if (r < t.world) acc = make_float4(acc.x + p[r].x, acc.y + p[r].y, acc.z + p[r].z, acc.w + p[r].w);
    v = make_float4(__fadd_rn(v.x, acc.x * inv), __fadd_rn(v.y, acc.y * inv), __fadd_rn(v.z, acc.z * inv),
                    __fadd_rn(v.w, acc.w * inv));
    x4[k] = v;
}

size_t tp_prefill_region_floats(int rows, int H) {
    return ((size_t)rows * H + (size_t)rows + 63) / 64 * 64;
}

tvb_status tp_sync(const TpArgs& t, StepState* st, cudaStream_t stream, bool pdl) {
    TVB_CUDA(launch_maybe_pdl(tp_sync_kernel, dim3(1), dim3(1), 0, stream, pdl, t, st));
    return check_launch("tp_sync_kernel");
}

tvb_status tp_reduce_rows(const TpArgs& t, size_t off, int S, int H, int norm_n, float eps, float* x,
                          cudaStream_t stream, bool pdl) {
    TVB_REQUIRE(S > 0 && H % 4 == 0 && off % 4 == 0, "tp_reduce_rows: bad arguments");
    const int n4 = H >> 2;
    TVB_CUDA(launch_maybe_pdl(tp_reduce_rows_kernel, dim3(S, (n4 + 255) / 256), dim3(256), 0, stream, pdl, t, off, S, H,
                              norm_n, eps, x));
    return check_launch("tp_reduce_rows_kernel");
}

}  // namespace tvb
