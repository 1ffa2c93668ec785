// Batched decode step kernels: attention of B sequences over their own KV
// cache slots, and the per-row greedy argmax.  The projections of the step are
// the tensor-core GEMM of prefill.cu with B activation rows (one per
// sequence), split over K so that the few rows still keep every SM streaming
// weights.
#include "batch_decode.h"

#include <algorithm>

#include "attn_split.cuh"

namespace tvb {

// CTA (kv head x split, sequence): the decode step's attention work item for
// sequence blockIdx.y (16 warps share the split's positions and all query
// heads of the KV head, then merge in shared memory).
__global__ void __launch_bounds__(kGemvThreads, 1)
batch_attn_kernel(const __grid_constant__ AttnArgs base, const int* __restrict__ pos, size_t slot_stride) {
    extern __shared__ __align__(128) unsigned char bd_smem[];
    pdl_wait();   // launched after the kernel that writes this one's inputs
    pdl_launch_dependents();
    const int b = blockIdx.y;
    AttnArgs a = base;
    a.q = base.q + (size_t)b * base.nh * base.hd;
    a.kcache = base.kcache + (size_t)b * slot_stride;
    a.vcache = base.vcache + (size_t)b * slot_stride;
    a.part = base.part + (size_t)b * base.nh * base.nsplit * (base.hd + 4);
    attn_item(a, blockIdx.x, bd_smem, __ldg(pos + b));
}

// Merge of the splits of (head blockIdx.x, sequence blockIdx.y), flash-decoding
// rescaling in split order (the decode step's o_proj prologue arithmetic);
// each lane owns 4 dimensions (hd == 128).
__global__ void batch_attn_merge_kernel(const float* __restrict__ part, int nh, int nsplit, int hd,
                                        float* __restrict__ out) {
    pdl_wait();   // launched after the kernel that writes this one's inputs
    pdl_launch_dependents();
    const int h = blockIdx.x, b = blockIdx.y, lane = threadIdx.x;
    const float* pb = part + ((size_t)b * nh + h) * nsplit * (hd + 4);
    float ms[kMaxAttnSplits], ls[kMaxAttnSplits];
    float4 pv[kMaxAttnSplits];
#pragma unroll
    for (int sp = 0; sp < kMaxAttnSplits; ++sp) {
        if (sp < nsplit) {
            const float* ps = pb + sp * (hd + 4);
            ms[sp] = ps[hd];
            ls[sp] = ps[hd + 1];
            pv[sp] = *reinterpret_cast<const float4*>(ps + lane * 4);
        } else {
            ms[sp] = -INFINITY;
            ls[sp] = 0.f;
            pv[sp] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    float M = -INFINITY;
#pragma unroll
    for (int sp = 0; sp < kMaxAttnSplits; ++sp) M = fmaxf(M, ms[sp]);
    float Ls = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int sp = 0; sp < kMaxAttnSplits; ++sp) {
        const float w = (ms[sp] == -INFINITY) ? 0.f : expf(ms[sp] - M);
        Ls = fmaf(ls[sp], w, Ls);
        o = make_float4(fmaf(pv[sp].x, w, o.x), fmaf(pv[sp].y, w, o.y), fmaf(pv[sp].z, w, o.z),
                        fmaf(pv[sp].w, w, o.w));
    }
    const float inv = 1.0f / Ls;
    *reinterpret_cast<float4*>(out + ((size_t)b * nh + h) * hd + lane * 4) =
        make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
}

constexpr int kArgThreads = 1024;

__device__ __forceinline__ unsigned long long key_max(unsigned long long a, unsigned long long b) {
    return a > b ? a : b;
}

__global__ void __launch_bounds__(kArgThreads)
batch_argmax_kernel(const float* __restrict__ logits, int n, int ld, int vocab0, unsigned long long* __restrict__ keys) {
    pdl_wait();   // launched after the kernel that writes this one's inputs
    pdl_launch_dependents();
    const int b = blockIdx.x, tid = threadIdx.x;
    const float* row = logits + (size_t)b * ld;
    unsigned long long k = 0ull;
    for (int j = tid; j < n; j += kArgThreads) {
        const float v = row[j];
        if (v == v) k = key_max(k, argmax_pack(v, vocab0 + j));   // NaN never wins
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) k = key_max(k, __shfl_xor_sync(0xffffffffu, k, o));
    __shared__ unsigned long long red[kArgThreads / 32];
    if ((tid & 31) == 0) red[tid >> 5] = k;
    __syncthreads();
    if (tid == 0) {
        unsigned long long t = 0ull;
        for (int w = 0; w < kArgThreads / 32; ++w) t = key_max(t, red[w]);
        keys[b] = t;
    }
}

__global__ void batch_pick_kernel(const KeySources src, int B, int* __restrict__ next) {
    pdl_wait();   // launched after the kernel that writes this one's inputs
    pdl_launch_dependents();
    const int b = threadIdx.x;
    if (b >= B) return;
    unsigned long long k = 0ull;
    for (int r = 0; r < src.n; ++r) k = key_max(k, __ldcg(src.p[r] + b));
    next[b] = k ? argmax_index(k) : 0;   // every logit NaN: token 0, never index -1
}

tvb_status batch_attention(const float* q, const float* kcache, const float* vcache, size_t slot_stride,
                           const int* pos, int B, int nh, int nkv, int hd, int nsplit, float scale, float* part,
                           float* out, cudaStream_t st, bool pdl) {
    TVB_REQUIRE(q && kcache && vcache && pos && part && out && B > 0, "batch attention: bad arguments");
    TVB_REQUIRE(hd == 128 && nh % nkv == 0 && nsplit >= 1 && nsplit <= kMaxAttnSplits,
                "batch attention: head_dim %d, heads %d/%d, splits %d", hd, nh, nkv, nsplit);
    static int smem_set = 0;
    const int smem = attn_item_smem(nh / nkv, hd);
    if (smem > smem_set) {
        TVB_CUDA(cudaFuncSetAttribute(batch_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
        smem_set = smem;
    }
    AttnArgs a = {};
    a.q = q;
    a.kcache = kcache;
    a.vcache = vcache;
    a.part = part;
    a.nh = nh;
    a.nkv = nkv;
    a.hd = hd;
    a.nsplit = nsplit;
    a.scale = scale;
    a.kv_len = -1;
    TVB_CUDA(launch_maybe_pdl(batch_attn_kernel, dim3((unsigned)(nkv * nsplit), (unsigned)B), dim3(kGemvThreads),
                              (size_t)smem, st, pdl, a, pos, slot_stride));
    TVB_TRY(check_launch("batch_attn_kernel"));
    TVB_CUDA(launch_maybe_pdl(batch_attn_merge_kernel, dim3((unsigned)nh, (unsigned)B), dim3(32), 0, st, pdl,
                              (const float*)part, nh, nsplit, hd, out));
    return check_launch("batch_attn_merge_kernel");
}

tvb_status batch_argmax(const float* logits, int B, int n, int ld, int vocab0, unsigned long long* keys,
                        cudaStream_t st, bool pdl) {
    TVB_REQUIRE(logits && keys && B > 0 && n > 0 && ld >= n, "batch argmax: bad arguments");
    TVB_CUDA(launch_maybe_pdl(batch_argmax_kernel, dim3(B), dim3(kArgThreads), 0, st, pdl, logits, n, ld, vocab0,
                              keys));
    return check_launch("batch_argmax_kernel");
}

tvb_status batch_pick(const KeySources& src, int B, int* next, cudaStream_t st, bool pdl) {
    TVB_REQUIRE(B > 0 && B <= kMaxBatch && src.n >= 1 && src.n <= kMaxTp && next, "batch pick: bad arguments");
    TVB_CUDA(launch_maybe_pdl(batch_pick_kernel, dim3(1), dim3(32), 0, st, pdl, src, B, next));
    return check_launch("batch_pick_kernel");
}

}  // namespace tvb
