// Single-query GQA attention over the F32 KV cache (decode), split along the
// sequence: CTA (kv_head, split) handles one slice of positions for all query
// heads of that KV head, keeping an online softmax; the last CTA of a KV head
// to finish merges the slices.  Same math as decode_attention_kernel
// (cuda/ops_cuda.cu:205-259) and the CPU attention (src/model.cpp:1071-1137):
// scores = q.k * (1/sqrt(hd)), max-subtracted softmax over kv_len = pos + 1
// (self-inclusive), out = P.V.
#pragma once

#include "gemv.cuh"

namespace tvb {

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;

struct AttnArgs {
    const float* q;        // [nh][hd]
    const float* kcache;   // [max_seq][nkv][hd]
    const float* vcache;
    float* out;            // [nh][hd]
    float* part;           // [nh][nsplit][hd + 4] workspace
    int nh, nkv, hd, nsplit;
    float scale;
    int kv_len;            // >= 0: fixed length; < 0: read pos + 1 from st
    StepState* st;         // completion counters (and pos when kv_len < 0)
    unsigned* status;
};

// hd == 128: each lane owns 4 consecutive dimensions.
static __global__ void __launch_bounds__(kAttnThreads)
attn_decode_kernel(const __grid_constant__ AttnArgs a) {
    pdl_launch_dependents();
    pdl_wait();
    const int kvh = blockIdx.x, split = blockIdx.y;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hd = a.hd, group = a.nh / a.nkv;
    const int kv_len = a.kv_len >= 0 ? a.kv_len : a.st->pos + 1;
    const int chunk = (kv_len + a.nsplit - 1) / a.nsplit;
    const int t0 = split * chunk;
    const int t1 = min(kv_len, t0 + chunk);
    const size_t row = (size_t)a.nkv * hd;

    for (int hh = warp; hh < group; hh += kAttnWarps) {
        const int h = kvh * group + hh;
        const float4 q4 = *reinterpret_cast<const float4*>(a.q + h * hd + lane * 4);
        float m = -INFINITY, l = 0.f;
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
        const float* kb = a.kcache + kvh * hd + lane * 4;
        const float* vb = a.vcache + kvh * hd + lane * 4;
        int t = t0;
        for (; t + 4 <= t1; t += 4) {
            float s[4];
            float4 vv[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float4 k4 = *reinterpret_cast<const float4*>(kb + (size_t)(t + u) * row);
                vv[u] = *reinterpret_cast<const float4*>(vb + (size_t)(t + u) * row);
                s[u] = q4.x * k4.x + q4.y * k4.y + q4.z * k4.z + q4.w * k4.w;
            }
#pragma unroll
            for (int u = 0; u < 4; ++u) s[u] = warp_sum(s[u]) * a.scale;
            float mn = fmaxf(fmaxf(fmaxf(m, s[0]), fmaxf(s[1], s[2])), s[3]);
            const float corr = expf(m - mn);
            l *= corr;
            acc.x *= corr; acc.y *= corr; acc.z *= corr; acc.w *= corr;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float p = expf(s[u] - mn);
                l += p;
                acc.x = fmaf(p, vv[u].x, acc.x);
                acc.y = fmaf(p, vv[u].y, acc.y);
                acc.z = fmaf(p, vv[u].z, acc.z);
                acc.w = fmaf(p, vv[u].w, acc.w);
            }
            m = mn;
        }
        for (; t < t1; ++t) {
            const float4 k4 = *reinterpret_cast<const float4*>(kb + (size_t)t * row);
            const float4 v4 = *reinterpret_cast<const float4*>(vb + (size_t)t * row);
            const float s = warp_sum(q4.x * k4.x + q4.y * k4.y + q4.z * k4.z + q4.w * k4.w) * a.scale;
            const float mn = fmaxf(m, s);
            const float corr = expf(m - mn), p = expf(s - mn);
            l = l * corr + p;
            acc.x = fmaf(p, v4.x, acc.x * corr);
            acc.y = fmaf(p, v4.y, acc.y * corr);
            acc.z = fmaf(p, v4.z, acc.z * corr);
            acc.w = fmaf(p, v4.w, acc.w * corr);
            m = mn;
        }
        if (a.nsplit == 1) {
            const float inv = 1.0f / l;
            *reinterpret_cast<float4*>(a.out + h * hd + lane * 4) =
                make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
            continue;
        }
        float* pp = a.part + ((size_t)h * a.nsplit + split) * (hd + 4);
        *reinterpret_cast<float4*>(pp + lane * 4) = acc;
        if (lane == 0) {
            pp[hd] = m;
            pp[hd + 1] = l;
        }
    }

    if (a.nsplit == 1) return;
    // Last CTA of this KV head merges the splits.
    __shared__ bool last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned done = atomicAdd(&a.st->attn_done[kvh], 1u);
        last = (done == (unsigned)a.nsplit - 1u);
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    // Merge: lane s owns split s (nsplit <= 32) for the running max and the
    // normaliser; the partial vectors are then summed with independent loads.
    for (int hh = warp; hh < group; hh += kAttnWarps) {
        const int h = kvh * group + hh;
        const float* pb = a.part + (size_t)h * a.nsplit * (hd + 4);
        const float ms = lane < a.nsplit ? __ldcg(pb + lane * (hd + 4) + hd) : -INFINITY;
        const float ls = lane < a.nsplit ? __ldcg(pb + lane * (hd + 4) + hd + 1) : 0.f;
        const float M = warp_max(ms);
        const float ws = (ms == -INFINITY) ? 0.f : expf(ms - M);
        const float L = warp_sum(ls * ws);
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
        for (int s2 = 0; s2 < a.nsplit; ++s2) {
            const float w = __shfl_sync(0xffffffffu, ws, s2);
            const float4 v = __ldcg(reinterpret_cast<const float4*>(pb + s2 * (hd + 4) + lane * 4));
            o.x = fmaf(v.x, w, o.x);
            o.y = fmaf(v.y, w, o.y);
            o.z = fmaf(v.z, w, o.z);
            o.w = fmaf(v.w, w, o.w);
        }
        const float inv = 1.0f / L;
        *reinterpret_cast<float4*>(a.out + h * hd + lane * 4) =
            make_float4(o.x * inv, o.y * inv, o.z * inv, o.w * inv);
    }
    if (threadIdx.x == 0) a.st->attn_done[kvh] = 0u;
}

}  // namespace tvb
