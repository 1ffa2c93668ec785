// Split-KV single-query attention work item shared by the decode-step kernel
// and the allocation-free stand-alone entry.
#pragma once

#include "attention.cuh"

namespace tvb {

// Grouped variant for G query heads per KV head (G = 1, 2 or 4): the split's
// positions are cut into 16 contiguous ranges, one per warp, and each warp
// serves all G heads of the group, so every K/V row is read once per CTA and
// each warp's sequential chain is 1/16 of the split.  Per head an online
// softmax; the 16 warps' partials of each head merge in shared memory into one
// partial (acc[hd], max, sum) per (head, split), the layout the o_proj phase
// merges.  Shared memory: 16 * G * (hd + 4) floats.
template <int G>
__device__ __forceinline__ void attn_item_grouped(const AttnArgs& a, int b, unsigned char* smem, int pos) {
    const int kvh = b / a.nsplit, split = b - kvh * a.nsplit;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hd = a.hd;
    const int kv_len = pos + 1;
    const int chunk = (kv_len + a.nsplit - 1) / a.nsplit;
    const int c0 = split * chunk, c1 = min(kv_len, c0 + chunk);
    const int sub_len = (max(c1 - c0, 0) + kGemvWarps - 1) / kGemvWarps;
    const int t0 = c0 + warp * sub_len, t1 = min(c1, t0 + sub_len);
    const size_t row = (size_t)a.nkv * hd;
    float* red = reinterpret_cast<float*>(smem);   // [warp][head][hd + 4]
    float m[G], l[G];
    float4 acc[G], q4[G];
#pragma unroll
    for (int h = 0; h < G; ++h) {
        m[h] = -INFINITY;
        l[h] = 0.f;
        acc[h] = make_float4(0.f, 0.f, 0.f, 0.f);
        q4[h] = __ldcg(reinterpret_cast<const float4*>(a.q + (kvh * G + h) * hd + lane * 4));
    }
    const float* kb = a.kcache + kvh * hd + lane * 4;
    const float* vb = a.vcache + kvh * hd + lane * 4;
    // pairs of positions; the next pair's K/V rows load while this one computes
    float4 kc[2], vc[2], kn[2], vn[2];
    auto load = [&](int t, float4* kk, float4* vv) {
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            if (t + u < t1) {
                kk[u] = __ldcg(reinterpret_cast<const float4*>(kb + (size_t)(t + u) * row));
                vv[u] = __ldcg(reinterpret_cast<const float4*>(vb + (size_t)(t + u) * row));
            } else {
                kk[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                vv[u] = kk[u];
            }
        }
    };
    load(t0, kc, vc);
    for (int t = t0; t < t1; t += 2) {
        load(t + 2, kn, vn);
#pragma unroll
        for (int h = 0; h < G; ++h) {
            float s[2];
#pragma unroll
            for (int u = 0; u < 2; ++u)
                s[u] = q4[h].x * kc[u].x + q4[h].y * kc[u].y + q4[h].z * kc[u].z + q4[h].w * kc[u].w;
#pragma unroll
            for (int u = 0; u < 2; ++u) s[u] = (t + u < t1) ? warp_sum(s[u]) * a.scale : -INFINITY;
            const float mn = fmaxf(m[h], fmaxf(s[0], s[1]));
            const float corr = expf(m[h] - mn);
            l[h] *= corr;
            acc[h] = make_float4(acc[h].x * corr, acc[h].y * corr, acc[h].z * corr, acc[h].w * corr);
#pragma unroll
            for (int u = 0; u < 2; ++u) {
                const float p = expf(s[u] - mn);
                l[h] += p;
                acc[h] = make_float4(fmaf(p, vc[u].x, acc[h].x), fmaf(p, vc[u].y, acc[h].y),
                                     fmaf(p, vc[u].z, acc[h].z), fmaf(p, vc[u].w, acc[h].w));
            }
            m[h] = mn;
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            kc[u] = kn[u];
            vc[u] = vn[u];
        }
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
        float* rw = red + (warp * G + h) * (hd + 4);
        *reinterpret_cast<float4*>(rw + lane * 4) = acc[h];
        if (lane == 0) {
            rw[hd] = m[h];
            rw[hd + 1] = l[h];
        }
    }
    __syncthreads();
    // warp h merges head h's 16 partials (warps with no positions carry max -inf)
    if (warp < G) {
        const int h = warp;
        float M = -INFINITY;
        for (int w = 0; w < kGemvWarps; ++w) M = fmaxf(M, red[(w * G + h) * (hd + 4) + hd]);
        float L = 0.f;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int w = 0; w < kGemvWarps; ++w) {
            const float* rw = red + (w * G + h) * (hd + 4);
            const float mw = rw[hd];
            const float sc = (mw == -INFINITY) ? 0.f : expf(mw - M);
            L = fmaf(rw[hd + 1], sc, L);
            const float4 v = *reinterpret_cast<const float4*>(rw + lane * 4);
            o = make_float4(fmaf(v.x, sc, o.x), fmaf(v.y, sc, o.y), fmaf(v.z, sc, o.z), fmaf(v.w, sc, o.w));
        }
        float* pp = a.part + ((size_t)(kvh * G + h) * a.nsplit + split) * (hd + 4);
        *reinterpret_cast<float4*>(pp + lane * 4) = o;
        if (lane == 0) {
            pp[hd] = M;
            pp[hd + 1] = L;
        }
    }
}

// Shared memory the attention work item needs for `group` heads per KV head.
__host__ __device__ inline int attn_item_smem(int group, int hd) {
    const bool grouped = group == 1 || group == 2 || group == 4;
    return (grouped ? kGemvWarps * group : kGemvWarps) * (hd + 4) * 4;
}

// Attention work item `b` = (kv head b / nsplit, split b % nsplit) for one CTA:
// the positions of the split are shared by the 16 warps (warps per head =
// 16 / group), each keeping an online softmax; the warps of a head merge in
// shared memory and write one partial (acc[hd], max, sum) per (head, split).
// The o_proj phase merges the splits while it loads its input.
__device__ __forceinline__ void attn_item(const AttnArgs& a, int b, unsigned char* smem, int pos) {
    switch (a.nh / a.nkv) {
        case 1: attn_item_grouped<1>(a, b, smem, pos); return;
        case 2: attn_item_grouped<2>(a, b, smem, pos); return;
        case 4: attn_item_grouped<4>(a, b, smem, pos); return;
        default: break;
    }
    const int kvh = b / a.nsplit, split = b - kvh * a.nsplit;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int hd = a.hd, group = a.nh / a.nkv;
    const int wph = kGemvWarps / group;                 // warps per head
    const int hh = warp / wph, sub = warp - hh * wph;
    const int kv_len = pos + 1;
    const int chunk = (kv_len + a.nsplit - 1) / a.nsplit;
    const int c0 = split * chunk, c1 = min(kv_len, c0 + chunk);
    const int sub_len = (max(c1 - c0, 0) + wph - 1) / wph;
    const int t0 = c0 + sub * sub_len, t1 = min(c1, t0 + sub_len);
    const size_t row = (size_t)a.nkv * hd;
    float* red = reinterpret_cast<float*>(smem);        // [warp][hd + 4]
    float m = -INFINITY, l = 0.f;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
    if (hh < group) {
        const int h = kvh * group + hh;
        const float4 q4 = __ldcg(reinterpret_cast<const float4*>(a.q + h * hd + lane * 4));
        const float* kb = a.kcache + kvh * hd + lane * 4;
        const float* vb = a.vcache + kvh * hd + lane * 4;
        // batches of 4 positions; the next batch's K/V rows load while this one computes
        float4 kc[4], vc[4], kn[4], vn[4];
        auto load = [&](int t, float4* kk, float4* vv) {
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                if (t + u < t1) {
                    kk[u] = __ldcg(reinterpret_cast<const float4*>(kb + (size_t)(t + u) * row));
                    vv[u] = __ldcg(reinterpret_cast<const float4*>(vb + (size_t)(t + u) * row));
                } else {
                    kk[u] = make_float4(0.f, 0.f, 0.f, 0.f);
                    vv[u] = kk[u];
                }
            }
        };
        load(t0, kc, vc);
        for (int t = t0; t < t1; t += 4) {
            load(t + 4, kn, vn);
            float s[4];
#pragma unroll
            for (int u = 0; u < 4; ++u) s[u] = q4.x * kc[u].x + q4.y * kc[u].y + q4.z * kc[u].z + q4.w * kc[u].w;
#pragma unroll
            for (int u = 0; u < 4; ++u) s[u] = (t + u < t1) ? warp_sum(s[u]) * a.scale : -INFINITY;
            const float mn = fmaxf(fmaxf(fmaxf(m, s[0]), fmaxf(s[1], s[2])), s[3]);
            const float corr = expf(m - mn);
            l *= corr;
            acc.x *= corr; acc.y *= corr; acc.z *= corr; acc.w *= corr;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                const float p = expf(s[u] - mn);
                l += p;
                acc.x = fmaf(p, vc[u].x, acc.x);
                acc.y = fmaf(p, vc[u].y, acc.y);
                acc.z = fmaf(p, vc[u].z, acc.z);
                acc.w = fmaf(p, vc[u].w, acc.w);
            }
            m = mn;
#pragma unroll
            for (int u = 0; u < 4; ++u) {
                kc[u] = kn[u];
                vc[u] = vn[u];
            }
        }
        float* rw = red + warp * (hd + 4);
        *reinterpret_cast<float4*>(rw + lane * 4) = acc;
        if (lane == 0) {
            rw[hd] = m;
            rw[hd + 1] = l;
        }
    }
    __syncthreads();
    // merge the wph sub-splits of each head (warp `sub == 0` of the head)
    if (hh < group && sub == 0) {
        const int h = kvh * group + hh;
        float M = -INFINITY;
        for (int w = 0; w < wph; ++w) M = fmaxf(M, red[(warp + w) * (hd + 4) + hd]);
        float L = 0.f;
        float4 o = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int w = 0; w < wph; ++w) {
            const float* rw = red + (warp + w) * (hd + 4);
            const float mw = rw[hd];
            const float s = (mw == -INFINITY) ? 0.f : expf(mw - M);
            L = fmaf(rw[hd + 1], s, L);
            const float4 v = *reinterpret_cast<const float4*>(rw + lane * 4);
            o = make_float4(fmaf(v.x, s, o.x), fmaf(v.y, s, o.y), fmaf(v.z, s, o.z), fmaf(v.w, s, o.w));
        }
        float* pp = a.part + ((size_t)h * a.nsplit + split) * (hd + 4);
        *reinterpret_cast<float4*>(pp + lane * 4) = o;
        if (lane == 0) {
            pp[hd] = M;
            pp[hd + 1] = L;
        }
    }
}

}  // namespace tvb
