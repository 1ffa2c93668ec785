// Causal GQA prefill attention on the tensor cores (compute_batched_attention,
// src/model.cpp:1071-1137: scores = q.k * scale, softmax over keys 0..pos,
// out = sum p * v).
//
// pf_attn_prep_*: q, K and V^T are split once per layer into F16 hi + lo planes
// (x = hi + lo to ~2^-22 of |x|), so tcgen05.mma on F16 operands reproduces
// the F32 products: scores from hi.hi + hi.lo + lo.hi, the output from the
// same three terms of P and V.
//
// pf_attn_tc_kernel: one CTA per (KV head, block of 128 / group positions);
// its 128 rows are the (position, query head) pairs of that KV head, loaded by
// one 3-D TMA box per plane and 64-column swizzle atom.  Pass 1 streams the
// 64-key K tiles (TMA), S = Q.K^T (M=128, N=64, F32 in TMEM) and keeps each
// row's running max and sum (one thread per TMEM lane).  Pass 2 recomputes S,
// writes the normalised probabilities p = exp(s - max) / sum as F16 hi + lo
// into shared memory and accumulates O += P.V (M=128, N=128 dims, K=64 keys)
// in TMEM, so the output needs no rescaling.  The next tile's TMA load is
// issued as soon as the MMA that read the buffer has committed.  Every
// mbarrier wait is bounded.
#include "prefill.h"

#include <algorithm>
#include <cstring>
#include <mutex>

#include "tcgen05.cuh"

namespace tvb {

constexpr int kAtRows = 128, kAtKeys = 64, kAtHd = 128, kAtThreads = 256;
constexpr int kAtQAtom = kAtRows * 128;   // 128 rows x 64 F16
constexpr int kAtKAtom = kAtKeys * 128;   // 64 keys x 64 F16
constexpr int kAtVt = kAtHd * 128;        // 128 dims x 64 keys
constexpr int kAtP = kAtRows * 128;       // 128 rows x 64 keys
constexpr int kAtOffQ = 0;                              // Qh[2 atoms], Ql[2 atoms]
constexpr int kAtOffK = kAtOffQ + 4 * kAtQAtom;          // Kh[2], Kl[2]
constexpr int kAtOffV = kAtOffK + 4 * kAtKAtom;          // Vth, Vtl
constexpr int kAtOffP = kAtOffV + 2 * kAtVt;             // Ph, Pl
constexpr int kAtOffBar = kAtOffP + 2 * kAtP;
constexpr int kAtSmem = kAtOffBar + 64 + 4 * 128 * 4 + 1024;   // + barriers + row exchange

struct AtMaps {
    CUtensorMap qh, ql, kh, kl, vth, vtl;
};

struct AtArgs {
    int S, pos0, nh, nkv, group, bq;
    float scale;
    float* out;   // [S][nh * 128]
    unsigned* status;
};

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int x, int y, int z, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
        : "memory");
}

__global__ void __launch_bounds__(kAtThreads, 1)
pf_attn_tc_kernel(const __grid_constant__ AtMaps mp, const __grid_constant__ AtArgs a) {
    extern __shared__ unsigned char at_smem_raw[];
    const uint32_t raw = smem_u32(at_smem_raw);
    const uint32_t base = (raw + 1023u) & ~1023u;
    unsigned char* smem = at_smem_raw + (base - raw);
    uint64_t* qbar = reinterpret_cast<uint64_t*>(smem + kAtOffBar);
    uint64_t* kbar = qbar + 1;
    uint64_t* vbar = qbar + 2;
    uint64_t* sbar = qbar + 3;
    uint64_t* obar = qbar + 4;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(qbar + 5);
    volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tid = threadIdx.x, warp = tid >> 5;
    const int kvh = blockIdx.x;
    const int qb = gridDim.y - 1 - blockIdx.y;   // longest blocks first
    const int qlo = qb * a.bq;
    const int last = a.pos0 + min(a.S, qlo + a.bq) - 1;   // largest position of the block
    const int ntiles = last / kAtKeys + 1;

    if (tid == 0) {
        for (int i = 0; i < 5; ++i) mbar_init(qbar + i, 1);
        *abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 0) tmem_alloc(tmem_slot, 256);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const uint32_t s_t = tmem, o_t = tmem + 64;

    const uint32_t q_s = base + kAtOffQ, k_s = base + kAtOffK, v_s = base + kAtOffV, p_s = base + kAtOffP;
    auto load_k = [&](int kt) {
        mbar_expect_tx(kbar, 4 * kAtKAtom);
        for (int at = 0; at < 2; ++at) {
            tma_load_2d(k_s + at * kAtKAtom, &mp.kh, kvh * kAtHd + at * 64, kt * kAtKeys, kbar);
            tma_load_2d(k_s + (2 + at) * kAtKAtom, &mp.kl, kvh * kAtHd + at * 64, kt * kAtKeys, kbar);
        }
    };
    auto load_v = [&](int kt) {
        mbar_expect_tx(vbar, 2 * kAtVt);
        tma_load_2d(v_s, &mp.vth, kt * kAtKeys, kvh * kAtHd, vbar);
        tma_load_2d(v_s + kAtVt, &mp.vtl, kt * kAtKeys, kvh * kAtHd, vbar);
    };
    auto fail = [&]() {
        *abort_flag = 1;
        if (a.status) atomicOr(a.status, kStatusTimeout);
    };
    if (tid == 0) {
        mbar_expect_tx(qbar, 4 * kAtQAtom);
        for (int at = 0; at < 2; ++at) {
            tma_load_3d(q_s + at * kAtQAtom, &mp.qh, at * 64, kvh * a.group, qlo, qbar);
            tma_load_3d(q_s + (2 + at) * kAtQAtom, &mp.ql, at * 64, kvh * a.group, qlo, qbar);
        }
        load_k(0);
    }

    // S = Q.K^T for the K tile in shared memory (thread 0), into TMEM columns [0, 64)
    constexpr uint32_t idesc_s = umma_idesc_f16(kAtRows, kAtKeys);
    constexpr uint32_t idesc_o = umma_idesc_f16(kAtRows, kAtHd);
    auto mma_s = [&]() {
#pragma unroll
        for (int kk = 0; kk < kAtHd / 16; ++kk) {
            const int at = kk >> 2, sub = (kk & 3) * 32;
            const uint64_t qh = sw128_desc(q_s + at * kAtQAtom + sub), ql = sw128_desc(q_s + (2 + at) * kAtQAtom + sub);
            const uint64_t kh = sw128_desc(k_s + at * kAtKAtom + sub), kl = sw128_desc(k_s + (2 + at) * kAtKAtom + sub);
            tc_mma(s_t, qh, kh, idesc_s, kk ? 1u : 0u);
            tc_mma(s_t, qh, kl, idesc_s, 1u);
            tc_mma(s_t, ql, kh, idesc_s, 1u);
        }
        tc_commit(sbar);
    };

    // Softmax: every thread takes 32 of a row's 64 keys (TMEM lane quarter
    // warp % 4, column half warp / 4); the two halves of a row combine their
    // max and sum through shared memory in a fixed order.  Scores are kept in
    // the log2 domain (scale * log2(e) folded in), exponentials are exp2f.
    const int r = 32 * (warp & 3) + (tid & 31);
    const int half = warp >> 2;
    const int rq = qlo + r / a.group;
    const int rpos = rq < a.S ? a.pos0 + rq : -1;
    const uint32_t s_part = s_t + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(32 * half);
    float* red = reinterpret_cast<float*>(smem + kAtOffBar + 64);   // [2 halves][128 rows]
    float* red2 = red + 2 * kAtRows;
    const float sc2 = a.scale * 1.4426950408889634f;   // log2(e)
    float m = -INFINITY, l = 0.f;
    uint32_t kpar = 0, spar = 0, vpar = 0, opar = 0;

    // ---- pass 1: row max and sum ---------------------------------------------------
    for (int kt = 0; kt < ntiles && !*abort_flag; ++kt) {
        if (tid == 0) {
            bool ok = (kt > 0 || mbar_wait_bounded(qbar, 0u)) && mbar_wait_bounded(kbar, kpar);
            if (ok) {
                tc_fence_after();
                mma_s();
            } else {
                fail();
            }
        }
        kpar ^= 1u;
        if (!mbar_wait_bounded(sbar, spar)) fail();
        spar ^= 1u;
        tc_fence_after();
        if (tid == 0) load_k(kt + 1 < ntiles ? kt + 1 : 0);   // the K buffer is free; pass 2 starts at tile 0
        uint32_t sv[32];
        tmem_ld32(s_part, sv);
        tmem_wait_ld();
        const int key0 = kt * kAtKeys + 32 * half;
        float tmax = -INFINITY;
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (key0 + j <= rpos) tmax = fmaxf(tmax, __uint_as_float(sv[j]) * sc2);
        red[half * kAtRows + r] = tmax;
        tc_fence_before();
        __syncthreads();
        const float mn = fmaxf(m, fmaxf(red[r], red[kAtRows + r]));
        float sum = 0.f;
        if (mn > -INFINITY) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (key0 + j <= rpos) sum += exp2f(__uint_as_float(sv[j]) * sc2 - mn);
        }
        red2[half * kAtRows + r] = sum;
        __syncthreads();
        if (mn > -INFINITY) {
            l = (m > -INFINITY ? l * exp2f(m - mn) : 0.f) + (red2[r] + red2[kAtRows + r]);
            m = mn;
        }
    }

    // ---- pass 2: normalised probabilities, O = P.V -----------------------------------
    const float inv_l = l > 0.f ? 1.0f / l : 0.f;
    if (tid == 0) load_v(0);
    for (int kt = 0; kt < ntiles && !*abort_flag; ++kt) {
        if (tid == 0) {
            if (mbar_wait_bounded(kbar, kpar)) {
                tc_fence_after();
                mma_s();
            } else {
                fail();
            }
        }
        kpar ^= 1u;
        if (!mbar_wait_bounded(sbar, spar)) fail();
        spar ^= 1u;
        tc_fence_after();
        if (tid == 0 && kt + 1 < ntiles) load_k(kt + 1);
        {
            uint32_t sv[32];
            tmem_ld32(s_part, sv);
            tmem_wait_ld();
            const int key0 = kt * kAtKeys + 32 * half;
            unsigned char* ph = smem + kAtOffP;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                __half hi[8], lo[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int j = c * 8 + i;
                    const float p = key0 + j <= rpos ? exp2f(__uint_as_float(sv[j]) * sc2 - m) * inv_l : 0.f;
                    hi[i] = __float2half_rn(p);
                    lo[i] = __float2half_rn(p - __half2float(hi[i]));
                }
                *reinterpret_cast<uint4*>(ph + sw128_offset(r, 4 * half + c)) = *reinterpret_cast<const uint4*>(hi);
                *reinterpret_cast<uint4*>(ph + kAtP + sw128_offset(r, 4 * half + c)) = *reinterpret_cast<const uint4*>(lo);
            }
            fence_proxy_async_smem_cta();
        }
        tc_fence_before();
        __syncthreads();
        tc_fence_after();
        if (tid == 0) {
            if (mbar_wait_bounded(vbar, vpar)) {
#pragma unroll
                for (int kk = 0; kk < kAtKeys / 16; ++kk) {
                    const uint64_t pdh = sw128_desc(p_s + kk * 32), pdl = sw128_desc(p_s + kAtP + kk * 32);
                    const uint64_t vdh = sw128_desc(v_s + kk * 32), vdl = sw128_desc(v_s + kAtVt + kk * 32);
                    tc_mma(o_t, pdh, vdh, idesc_o, (kt | kk) ? 1u : 0u);
                    tc_mma(o_t, pdh, vdl, idesc_o, 1u);
                    tc_mma(o_t, pdl, vdh, idesc_o, 1u);
                }
                tc_commit(obar);
            } else {
                fail();
                tc_commit(obar);
            }
        }
        vpar ^= 1u;
        if (!mbar_wait_bounded(obar, opar)) fail();
        opar ^= 1u;
        tc_fence_after();
        if (tid == 0 && kt + 1 < ntiles) load_v(kt + 1);
    }

    // ---- output rows: each thread stores 64 of its row's 128 dims ----------------
    if (!*abort_flag) {
        const uint32_t o_row = o_t + ((uint32_t)(32 * (warp & 3)) << 16) + (uint32_t)(64 * half);
        float* dst = rpos >= 0 ? a.out + (size_t)rq * a.nh * kAtHd + (size_t)(kvh * a.group + r % a.group) * kAtHd +
                                     64 * half
                               : nullptr;
        for (int c = 0; c < 2; ++c) {
            __syncwarp();
            uint32_t ov[32];
            tmem_ld32(o_row + c * 32, ov);
            tmem_wait_ld();
            if (dst) {
                float4* d4 = reinterpret_cast<float4*>(dst + c * 32);
#pragma unroll
                for (int v = 0; v < 8; ++v)
                    d4[v] = make_float4(__uint_as_float(ov[4 * v]), __uint_as_float(ov[4 * v + 1]),
                                        __uint_as_float(ov[4 * v + 2]), __uint_as_float(ov[4 * v + 3]));
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (tid == 0 && *abort_flag) {
        // no TMA write may still be landing in this CTA's shared memory
        mbar_wait_bounded(kbar, kpar);
        mbar_wait_bounded(vbar, vpar);
    }
    __syncthreads();
    if (warp == 0) {
        tc_fence_after();
        tmem_dealloc(tmem, 256);
    }
}

// ---- hi/lo planes ----------------------------------------------------------------
__device__ __forceinline__ void at_split(float v, __half& hi, __half& lo) {
    hi = __float2half_rn(v);
    lo = __float2half_rn(v - __half2float(hi));
}

// elementwise: rows [0, n) of a [n][w] F32 matrix -> hi/lo F16 planes of the same layout
__global__ void pf_attn_split_rows(const float* __restrict__ src, size_t n4, __half2* __restrict__ hi,
                                   __half2* __restrict__ lo) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n4; i += (size_t)gridDim.x * blockDim.x) {
        const float4 v = reinterpret_cast<const float4*>(src)[i];
        __half h[4], l[4];
        at_split(v.x, h[0], l[0]);
        at_split(v.y, h[1], l[1]);
        at_split(v.z, h[2], l[2]);
        at_split(v.w, h[3], l[3]);
        hi[2 * i] = __halves2half2(h[0], h[1]);
        hi[2 * i + 1] = __halves2half2(h[2], h[3]);
        lo[2 * i] = __halves2half2(l[0], l[1]);
        lo[2 * i + 1] = __halves2half2(l[2], l[3]);
    }
}

// V rows [0, T) of [T][Hk] -> V^T hi/lo planes [Hk][Tp]: thread (dim d, 8 keys)
__global__ void pf_attn_split_vt(const float* __restrict__ v, int T, int Hk, int Tp, __half* __restrict__ hi,
                                 __half* __restrict__ lo) {
    const int d = blockIdx.x * blockDim.x + threadIdx.x;
    const int t0 = blockIdx.y * 8;
    if (d >= Hk || t0 >= T) return;
    __half h[8], l[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const float x = (t0 + i < T) ? v[(size_t)(t0 + i) * Hk + d] : 0.f;
        at_split(x, h[i], l[i]);
    }
    *reinterpret_cast<uint4*>(hi + (size_t)d * Tp + t0) = *reinterpret_cast<const uint4*>(h);
    *reinterpret_cast<uint4*>(lo + (size_t)d * Tp + t0) = *reinterpret_cast<const uint4*>(l);
}

size_t pf_attn_planes_bytes(int max_rows, int max_keys, int nh, int nkv) {
    const size_t Hq = (size_t)nh * kAtHd, Hk = (size_t)nkv * kAtHd;
    const size_t Tp = ((size_t)max_keys + 63) / 64 * 64;
    return 2 * (size_t)max_rows * Hq * 2 + 2 * Tp * Hk * 2 + 2 * Hk * Tp * 2 + 4 * 256;
}

bool pf_attention_tc_supported(int nh, int nkv, int hd) {
    return hd == kAtHd && nkv > 0 && nh % nkv == 0 && kAtRows % (nh / nkv) == 0;
}

tvb_status pf_attention_tc(const float* q, const float* kcache, const float* vcache, int S, int pos0, int nh,
                           int nkv, int hd, float scale, float* out, void* planes, int max_rows, int max_keys,
                           unsigned* status, cudaStream_t st) {
    TVB_REQUIRE(q && kcache && vcache && out && planes && S > 0 && pos0 >= 0, "attention_tc: bad arguments");
    TVB_REQUIRE(pf_attention_tc_supported(nh, nkv, hd), "attention_tc: heads %d / %d, head_dim %d", nh, nkv, hd);
    const int T = pos0 + S;
    TVB_REQUIRE(S <= max_rows && T <= max_keys, "attention_tc: %d rows / %d keys exceed the planes", S, T);
    static std::once_flag once;
    static cudaError_t err = cudaSuccess;
    std::call_once(once, [] {
        err = cudaFuncSetAttribute(pf_attn_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kAtSmem);
    });
    if (err != cudaSuccess) return cuda_error(err, "cudaFuncSetAttribute(pf_attn_tc_kernel)");
    const size_t Hq = (size_t)nh * hd, Hk = (size_t)nkv * hd;
    const int Tp = (max_keys + 63) / 64 * 64;
    uint16_t* qh = static_cast<uint16_t*>(planes);
    uint16_t* ql = qh + (size_t)max_rows * Hq;
    uint16_t* kh = ql + (size_t)max_rows * Hq;
    uint16_t* kl = kh + (size_t)Tp * Hk;
    uint16_t* vth = kl + (size_t)Tp * Hk;
    uint16_t* vtl = vth + Hk * Tp;
    // planes of this call: q rows [0, S), K rows [0, T), V^T columns [0, T)
    const int blocks = num_sms() * 4;
    pf_attn_split_rows<<<blocks, 256, 0, st>>>(q, (size_t)S * Hq / 4, reinterpret_cast<__half2*>(qh),
                                              reinterpret_cast<__half2*>(ql));
    TVB_TRY(check_launch("pf_attn_split_rows(q)"));
    pf_attn_split_rows<<<blocks, 256, 0, st>>>(kcache, (size_t)T * Hk / 4, reinterpret_cast<__half2*>(kh),
                                              reinterpret_cast<__half2*>(kl));
    TVB_TRY(check_launch("pf_attn_split_rows(k)"));
    pf_attn_split_vt<<<dim3((unsigned)((Hk + 127) / 128), (unsigned)((T + 7) / 8)), 128, 0, st>>>(
        vcache, T, (int)Hk, Tp, reinterpret_cast<__half*>(vth), reinterpret_cast<__half*>(vtl));
    TVB_TRY(check_launch("pf_attn_split_vt"));

    AtMaps mp;
    std::memset(&mp, 0, sizeof(mp));
    const int group = nh / nkv, bq = kAtRows / group;
    {   // q planes [S][nh][128]: boxes of 64 dims x group heads x bq positions
        const uint64_t dims[3] = {(uint64_t)hd, (uint64_t)nh, (uint64_t)S};
        const uint64_t strides[2] = {(uint64_t)hd * 2, (uint64_t)Hq * 2};
        const uint32_t box[3] = {64u, (uint32_t)group, (uint32_t)bq};
        TVB_TRY(encode_f16_tiled(&mp.qh, qh, 3, dims, strides, box));
        TVB_TRY(encode_f16_tiled(&mp.ql, ql, 3, dims, strides, box));
    }
    {   // K planes [T][Hk]: boxes of 64 dims x 64 keys
        const uint64_t dims[2] = {(uint64_t)Hk, (uint64_t)T};
        const uint64_t strides[1] = {(uint64_t)Hk * 2};
        const uint32_t box[2] = {64u, (uint32_t)kAtKeys};
        TVB_TRY(encode_f16_tiled(&mp.kh, kh, 2, dims, strides, box));
        TVB_TRY(encode_f16_tiled(&mp.kl, kl, 2, dims, strides, box));
    }
    {   // V^T planes [Hk][Tp]: boxes of 64 keys x 128 dims
        const uint64_t dims[2] = {(uint64_t)T, (uint64_t)Hk};
        const uint64_t strides[1] = {(uint64_t)Tp * 2};
        const uint32_t box[2] = {(uint32_t)kAtKeys, (uint32_t)kAtHd};
        TVB_TRY(encode_f16_tiled(&mp.vth, vth, 2, dims, strides, box));
        TVB_TRY(encode_f16_tiled(&mp.vtl, vtl, 2, dims, strides, box));
    }
    AtArgs a;
    a.S = S;
    a.pos0 = pos0;
    a.nh = nh;
    a.nkv = nkv;
    a.group = group;
    a.bq = bq;
    a.scale = scale;
    a.out = out;
    a.status = status;
    const dim3 grid((unsigned)nkv, (unsigned)((S + bq - 1) / bq));
    pf_attn_tc_kernel<<<grid, kAtThreads, kAtSmem, st>>>(mp, a);
    return check_launch("pf_attn_tc_kernel");
}

}  // namespace tvb
