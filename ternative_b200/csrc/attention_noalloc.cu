// tvb_attention_decode_noalloc: split-KV single-query attention whose scratch
// lives in this library's own static device memory, for callers that cannot
// allocate device memory when they call (a host whose device memory is owned
// by its own pool after start-up, or a thread that must not risk the device
// synchronisation cudaMalloc/cudaFree can imply).  Same inputs and outputs as
// tvb_attention_decode; the work is the decode step's attention phase
// (attn_item: positions split over CTAs and warps, online softmax) followed
// by the flash-decoding merge of the splits.
#include "attn_split.cuh"

#include <algorithm>
#include <mutex>

namespace tvb {

// Static scratch: per (head, split) one partial = hd accumulators + max + sum
// (padded to hd + 4 floats).  Limit: 64 heads x 8 splits x head_dim 128
// = 67,584 floats (264 KiB), held by every GPU that loads the library.
constexpr int kNoAllocMaxHeads = 64;
constexpr int kNoAllocMaxSplits = kMaxAttnSplits;   // 8
constexpr int kNoAllocHeadDim = 128;
constexpr size_t kNoAllocScratchFloats =
    (size_t)kNoAllocMaxHeads * kNoAllocMaxSplits * (kNoAllocHeadDim + 4);
static __device__ __align__(256) float g_attn_noalloc_scratch[kNoAllocScratchFloats];

// One CTA per (kv head, split): the decode step's attention work item.
__global__ void __launch_bounds__(kGemvThreads)
attn_split_noalloc_kernel(const __grid_constant__ AttnArgs a) {
    extern __shared__ __align__(128) unsigned char smem[];
    attn_item(a, blockIdx.x, smem, a.kv_len - 1);
}

// One warp per query head: merge the head's splits (lane owns 4 dims).
__global__ void attn_merge_noalloc_kernel(const float* __restrict__ part, int nsplit, int hd,
                                          float* __restrict__ out) {
    const int h = blockIdx.x, lane = threadIdx.x;
    const float* pb = part + (size_t)h * nsplit * (hd + 4);
    float ms[kNoAllocMaxSplits], ls[kNoAllocMaxSplits];
    float4 pv[kNoAllocMaxSplits];
#pragma unroll
    for (int s = 0; s < kNoAllocMaxSplits; ++s) {
        if (s < nsplit) {
            const float* ps = pb + s * (hd + 4);
            ms[s] = ps[hd];
            ls[s] = ps[hd + 1];
            pv[s] = *reinterpret_cast<const float4*>(ps + lane * 4);
        } else {
            ms[s] = -INFINITY;
            ls[s] = 0.f;
            pv[s] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
    }
    float M = -INFINITY;
#pragma unroll
    for (int s = 0; s < kNoAllocMaxSplits; ++s) M = fmaxf(M, ms[s]);
    float L = 0.f;
    float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int s = 0; s < kNoAllocMaxSplits; ++s) {
        const float w = (ms[s] == -INFINITY) ? 0.f : expf(ms[s] - M);
        L = fmaf(ls[s], w, L);
        o = make_float4(fmaf(pv[s].x, w, o.x), fmaf(pv[s].y, w, o.y), fmaf(pv[s].z, w, o.z),
                        fmaf(pv[s].w, w, o.w));
    }
    const float inv = 1.0f / L;
    *reinterpret_cast<float4*>(out + h * hd + lane * 4) =
        make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
}

// Device address of the static scratch, looked up once per device with that
// device current.  (In host code the array's name is only a host-side stand-in.)
static float* scratch_for_current_device(tvb_status* st) {
    constexpr int kMaxDevices = 64;
    static float* ptrs[kMaxDevices] = {};
    static std::mutex mu;
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        *st = cuda_error(e, "cudaGetDevice");
        return nullptr;
    }
    if (dev < 0 || dev >= kMaxDevices) {
        *st = set_error(TVB_ERR_UNSUPPORTED, "attention_decode_noalloc: device %d", dev);
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!ptrs[dev]) {
        float* p = nullptr;
        e = cudaGetSymbolAddress(reinterpret_cast<void**>(&p), g_attn_noalloc_scratch);
        if (e != cudaSuccess) {
            *st = cuda_error(e, "cudaGetSymbolAddress(attention scratch)");
            return nullptr;
        }
        // the largest attention item: 4 query heads per KV head
        e = cudaFuncSetAttribute(attn_split_noalloc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 attn_item_smem(4, kNoAllocHeadDim));
        if (e != cudaSuccess) {
            *st = cuda_error(e, "cudaFuncSetAttribute");
            return nullptr;
        }
        ptrs[dev] = p;
    }
    *st = TVB_OK;
    return ptrs[dev];
}

}  // namespace tvb

using namespace tvb;

extern "C" tvb_status tvb_attention_decode_noalloc(const float* q, const float* k_cache,
                                                   const float* v_cache, int kv_len, float* out,
                                                   int n_heads, int n_kv_heads, int head_dim,
                                                   float scale, void* stream) {
    TVB_REQUIRE(q && k_cache && v_cache && out, "attention_decode_noalloc: null pointer");
    TVB_REQUIRE(head_dim == kNoAllocHeadDim, "attention_decode_noalloc: head_dim %d (only %d)",
                head_dim, kNoAllocHeadDim);
    TVB_REQUIRE(n_heads > 0 && n_kv_heads > 0 && n_heads % n_kv_heads == 0,
                "attention_decode_noalloc: heads %d / kv heads %d", n_heads, n_kv_heads);
    const int group = n_heads / n_kv_heads;
    TVB_REQUIRE(group <= kGemvWarps && kGemvWarps % group == 0,
                "attention_decode_noalloc: %d query heads per kv head (must divide %d)", group,
                kGemvWarps);
    TVB_REQUIRE(kv_len > 0, "attention_decode_noalloc: kv_len %d", kv_len);
    TVB_REQUIRE(n_heads <= kNoAllocMaxHeads,
                "attention_decode_noalloc: %d heads exceed the static scratch limit of %d heads",
                n_heads, kNoAllocMaxHeads);
    const int nsplit = std::max(1, std::min(kNoAllocMaxSplits, (kv_len + 127) / 128));
    tvb_status s;
    float* scratch = scratch_for_current_device(&s);
    if (!scratch) return s;
    // Every (head, split) partial read by the merge is written by the split
    // kernel of the same call, so no part of the scratch must start at zero.
    AttnArgs a = {};
    a.q = q;
    a.kcache = k_cache;
    a.vcache = v_cache;
    a.part = scratch;
    a.nh = n_heads;
    a.nkv = n_kv_heads;
    a.hd = head_dim;
    a.nsplit = nsplit;
    a.scale = scale;
    a.kv_len = kv_len;
    const cudaStream_t st = as_stream(stream);
    attn_split_noalloc_kernel<<<n_kv_heads * nsplit, kGemvThreads,
                                attn_item_smem(group, head_dim), st>>>(a);
    TVB_CUDA(cudaGetLastError());
    attn_merge_noalloc_kernel<<<n_heads, 32, 0, st>>>(scratch, nsplit, head_dim, out);
    return check_launch("attn_merge_noalloc_kernel");
}
