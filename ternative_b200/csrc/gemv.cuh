// Batch-1 GEMV for the decode path: y[n] = sum_k W[n][k] * x[k] with F16 or
// INT8 weights and F32 activations/accumulation, fused with the prologue and
// epilogue the reference runs as separate kernels around each GEMV
// (src/model.cpp:1399-1451, cuda/ops_cuda.cu:46-158):
//
//   GM_PLAIN   y = W.x (scaled for INT8)                        gemv_d2d(_int8)
//   GM_QKV     rms_norm(x) -> q,k,v rows -> RoPE -> KV append     :1403-1413
//   GM_RESID   rms_norm_sub(in) -> x += W.in                      :1422-1430, :1442-1450
//   GM_GATEUP  rms_norm(x) -> relu(gate)^2 * up                   :1433-1439
//   GM_LMHEAD  rms_norm(x) -> logits + greedy argmax              :1571-1580
//
// B200 mapping.  A persistent grid (one CTA per SM) splits the output rows
// into groups of R rows; each CTA streams its groups' rows from HBM into a
// ring of shared-memory slots with 1-D bulk copies (cp.async.bulk, one per
// contiguous weight row) completed on mbarriers.  The CTA issues the first
// slots' copies before griddepcontrol.wait, so under programmatic dependent
// launch the weight stream of kernel i+1 starts while kernel i drains.  The
// activation vector is normalised once per CTA into shared memory; the 8 warps
// split each group's 256-column chunks and reduce across warps in a fixed order.
#pragma once

#include "stream.cuh"

namespace tvb {

enum GemvMode { GM_PLAIN = 0, GM_QKV = 1, GM_RESID = 2, GM_GATEUP = 3, GM_LMHEAD = 4 };
enum WType { WT_F16 = 0, WT_I8 = 1 };

constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kMaxKvHeads = 64;

// Device-resident per-context step state (read/written by the fused kernels).
struct StepState {
    int pos;                        // position of the token being decoded
    int token;                      // token being decoded
    unsigned long long argmax_key;  // packed (ordered logit, ~index) running max
    unsigned lm_done;               // lm_head CTAs finished this step
    unsigned status;                // kStatus* bits, sticky
    int next_token;                 // argmax of this step's logits
    float max_logit;
    unsigned attn_done[kMaxKvHeads];
};

struct GemvArgs {
    const void* w[3];
    const float* row_scale[3];  // TVB_I8_ROW scales or nullptr
    float tscale[3];            // per-tensor scale (1 for F16)
    int N;                      // rows per matrix (PLAIN/RESID/LMHEAD/GATEUP)
    int K;
    const float* x;             // input vector (unused when gathering the embedding)
    const uint16_t* embd;       // GM_QKV layer 0: gather x = f32(embd[token])
    float* x_out;               // GM_QKV layer 0: residual stream initialised from the gather
    const float* norm_w;        // prologue RMSNorm weight, nullptr = no norm
    float eps;
    float* y;                   // PLAIN: y; RESID: residual (in/out); GATEUP: h; LMHEAD: logits
    int nh, nkv, hd;            // GM_QKV geometry
    float* q_out;
    float* kcache;              // this layer's K rows [max_seq][Hk]
    float* vcache;
    const float* rope_cos;      // [max_seq][hd/2]
    const float* rope_sin;
    StepState* st;
    unsigned* status;
    int gather_token;           // GM_QKV: 1 on layer 0
};

__device__ __forceinline__ unsigned long long argmax_pack(float v, int idx) {
    uint32_t b = __float_as_uint(v);
    uint32_t ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)ord << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)idx);
}
__device__ __forceinline__ int argmax_index(unsigned long long key) {
    return (int)(0xFFFFFFFFu - (uint32_t)(key & 0xFFFFFFFFull));
}
__device__ __forceinline__ float argmax_value(unsigned long long key) {
    uint32_t ord = (uint32_t)(key >> 32);
    uint32_t b = (ord & 0x80000000u) ? (ord & 0x7FFFFFFFu) : ~ord;
    return __uint_as_float(b);
}

// Row i of group g -> (matrix, row within matrix, valid).
template <int MODE, int R>
__device__ __forceinline__ bool group_row(const GemvArgs& a, int g, int i, int& m, int& row) {
    if (MODE == GM_QKV) {
        const int half = a.hd >> 1;
        int p = g;
        const int nq = a.nh * half, nk = a.nkv * half;
        if (p < nq) m = 0;
        else if (p < nq + nk) { m = 1; p -= nq; }
        else { m = 2; p -= nq + nk; }
        row = (p / half) * a.hd + (p % half) + i * half;
        return true;
    } else if (MODE == GM_GATEUP) {
        m = i;
        row = g;
        return row < a.N;
    } else {
        m = 0;
        row = g * R + i;
        return row < a.N;
    }
}

template <int MODE>
__host__ __device__ inline int gemv_groups(const GemvArgs& a, int R) {
    if (MODE == GM_QKV) return (a.nh + 2 * a.nkv) * (a.hd >> 1);
    if (MODE == GM_GATEUP) return a.N;
    return (a.N + R - 1) / R;
}

template <int WT>
__device__ __forceinline__ float dot8(const unsigned char* wp, const float4& xlo, const float4& xhi) {
    float w[8];
    if (WT == WT_F16) {
        uint4 u = *reinterpret_cast<const uint4*>(wp);
        h8_to_f8(u, w);
    } else {
        uint2 u = *reinterpret_cast<const uint2*>(wp);
        i8x4_to_f4(u.x, w);
        i8x4_to_f4(u.y, w + 4);
    }
    float s = w[0] * xlo.x;
    s = fmaf(w[1], xlo.y, s);
    s = fmaf(w[2], xlo.z, s);
    s = fmaf(w[3], xlo.w, s);
    s = fmaf(w[4], xhi.x, s);
    s = fmaf(w[5], xhi.y, s);
    s = fmaf(w[6], xhi.z, s);
    s = fmaf(w[7], xhi.w, s);
    return s;
}

// Shared memory layout (bytes):
//   [0, 64*8)                   mbarriers (up to 64 slots)
//   [512, 512 + 2*8*R*4)        cross-warp partial sums, double buffered
//   [.., + K*4)                 activation vector (16-byte aligned)
//   [.., + S*stage)             weight slots (128-byte aligned)
struct GemvSmem {
    int part_off, x_off, stage_off, total;
};
__host__ __device__ inline GemvSmem gemv_smem_layout(int R, int K, int stages, int stage_bytes) {
    GemvSmem s;
    s.part_off = 512;
    s.x_off = s.part_off + ((2 * kGemvWarps * R * 4 + 127) / 128) * 128;
    s.stage_off = s.x_off + ((K * 4 + 127) / 128) * 128;
    s.total = s.stage_off + stages * stage_bytes;
    return s;
}

template <int MODE, int WT, int R>
__global__ void __launch_bounds__(kGemvThreads)
stream_gemv_kernel(const __grid_constant__ GemvArgs a, int stages) {
    extern __shared__ __align__(128) unsigned char smem[];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int K = a.K;
    const int esz = (WT == WT_F16) ? 2 : 1;
    const int row_bytes = K * esz;
    const int stage_bytes = R * row_bytes;
    const GemvSmem L = gemv_smem_layout(R, K, stages, stage_bytes);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
    float* part = reinterpret_cast<float*>(smem + L.part_off);
    float* xs = reinterpret_cast<float*>(smem + L.x_off);
    unsigned char* slots = smem + L.stage_off;

    const int n_groups = gemv_groups<MODE>(a, R);
    const int G = gridDim.x, b = blockIdx.x;
    const int g0 = (int)((long long)n_groups * b / G);
    const int g1 = (int)((long long)n_groups * (b + 1) / G);
    const int my = g1 - g0;

    auto issue = [&](int g, int slot) {
        uint32_t bytes = 0;
        int ms[R], rows[R];
        bool ok[R];
#pragma unroll
        for (int i = 0; i < R; ++i) {
            ok[i] = group_row<MODE, R>(a, g, i, ms[i], rows[i]);
            if (ok[i]) bytes += row_bytes;
        }
        mbar_expect_tx(&bar[slot], bytes);
#pragma unroll
        for (int i = 0; i < R; ++i) {
            if (!ok[i]) continue;
            const unsigned char* src =
                static_cast<const unsigned char*>(a.w[ms[i]]) + (size_t)rows[i] * row_bytes;
            bulk_g2s(slots + slot * stage_bytes + i * row_bytes, src, row_bytes, &bar[slot]);
        }
    };

    if (tid == 0) {
        for (int s = 0; s < stages; ++s) mbar_init(&bar[s], 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (tid == 0) {
        const int pre = my < stages ? my : stages;
        for (int s = 0; s < pre; ++s) issue(g0 + s, s);
    }
    pdl_launch_dependents();
    pdl_wait();

    // ---- prologue: activation vector into shared memory ------------------------
    {
        const float* src = a.x;
        const uint16_t* esrc = nullptr;
        if (MODE == GM_QKV && a.gather_token) esrc = a.embd + (size_t)a.st->token * K;
        float ss = 0.f;
        for (int k = tid * 4; k < K; k += kGemvThreads * 4) {
            float4 v;
            if (esrc) {
                uint2 h = *reinterpret_cast<const uint2*>(esrc + k);
                float2 l0 = __half22float2(*reinterpret_cast<const __half2*>(&h.x));
                float2 l1 = __half22float2(*reinterpret_cast<const __half2*>(&h.y));
                v = make_float4(l0.x, l0.y, l1.x, l1.y);
                if (b == 0) *reinterpret_cast<float4*>(a.x_out + k) = v;
            } else {
                v = *reinterpret_cast<const float4*>(src + k);
            }
            *reinterpret_cast<float4*>(xs + k) = v;
            ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
        }
        if (a.norm_w) {
            __shared__ float red[kGemvWarps];
            __shared__ float inv_s;
            ss = warp_sum(ss);
            if (lane == 0) red[warp] = ss;
            __syncthreads();
            if (tid == 0) {
                float t = 0.f;
                for (int w = 0; w < kGemvWarps; ++w) t += red[w];
                // tensor.cpp:675-676: rms = sqrt(ss/n + eps); inv = 1/rms
                float rms = __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)K), a.eps));
                inv_s = __fdiv_rn(1.0f, rms);
            }
            __syncthreads();
            const float inv = inv_s;
            for (int k = tid; k < K; k += kGemvThreads)
                xs[k] = __fmul_rn(xs[k], __fmul_rn(inv, a.norm_w[k]));   // x * (inv * w)
        }
    }
    __syncthreads();

    const int nch = (K + 255) >> 8;
    const int hsel = (lane >> 2) & 1;   // bank-conflict-free order for the x loads
    float best_v = -INFINITY;
    int best_i = 0;

    for (int it = 0; it < my; ++it) {
        const int slot = it % stages;
        const uint32_t parity = (uint32_t)((it / stages) & 1);
        if (!mbar_wait_bounded(&bar[slot], parity)) {
            atomicOr(a.status, kStatusTimeout);
            return;
        }
        const unsigned char* stg = slots + slot * stage_bytes;
        float acc[R];
#pragma unroll
        for (int i = 0; i < R; ++i) acc[i] = 0.f;
        for (int c = warp; c < nch; c += kGemvWarps) {
            const int k = c * 256 + lane * 8;
            if (k < K) {
                const float* xp = xs + k;
                float4 p0 = *reinterpret_cast<const float4*>(xp + 4 * hsel);
                float4 p1 = *reinterpret_cast<const float4*>(xp + 4 * (1 - hsel));
                float4 xlo = hsel ? p1 : p0;
                float4 xhi = hsel ? p0 : p1;
#pragma unroll
                for (int i = 0; i < R; ++i)
                    acc[i] += dot8<WT>(stg + i * row_bytes + k * esz, xlo, xhi);
            }
        }
        float* pb = part + (it & 1) * kGemvWarps * R;
#pragma unroll
        for (int i = 0; i < R; ++i) {
            float v = warp_sum(acc[i]);
            if (lane == 0) pb[warp * R + i] = v;
        }
        __syncthreads();
        if (tid == 0 && it + stages < my) issue(g0 + it + stages, slot);

        // ---- epilogue ---------------------------------------------------------
        const int g = g0 + it;
        if (MODE == GM_QKV || MODE == GM_GATEUP) {
            if (tid == 0) {
                float y[R];
                int ms[R], rows[R];
#pragma unroll
                for (int i = 0; i < R; ++i) {
                    group_row<MODE, R>(a, g, i, ms[i], rows[i]);
                    float t = 0.f;
                    for (int w = 0; w < kGemvWarps; ++w) t += pb[w * R + i];
                    const float sc = a.row_scale[ms[i]] ? a.row_scale[ms[i]][rows[i]] : a.tscale[ms[i]];
                    y[i] = (WT == WT_F16 && !a.row_scale[ms[i]]) ? t : t * sc;
                }
                if (MODE == GM_GATEUP) {
                    // relu2_d then mul_d (ops_cuda.cu:123-130, 116-121)
                    const float gr = fmaxf(y[0], 0.0f);
                    a.y[rows[0]] = __fmul_rn(__fmul_rn(gr, gr), y[1]);
                } else {
                    const int half = a.hd >> 1;
                    const int pos = a.st->pos;
                    const int d = rows[0] % a.hd;            // < half
                    const int head = rows[0] / a.hd;
                    float y0 = y[0], y1 = y[1];
                    if (ms[0] < 2) {
                        // NeoX pair (d, d + hd/2), tensor.cpp:918-925
                        const float c = a.rope_cos[(size_t)pos * half + d];
                        const float s = a.rope_sin[(size_t)pos * half + d];
                        const float r0 = __fsub_rn(__fmul_rn(y0, c), __fmul_rn(y1, s));
                        const float r1 = __fadd_rn(__fmul_rn(y0, s), __fmul_rn(y1, c));
                        y0 = r0;
                        y1 = r1;
                    }
                    if (ms[0] == 0) {
                        a.q_out[head * a.hd + d] = y0;
                        a.q_out[head * a.hd + d + half] = y1;
                    } else {
                        float* dst = (ms[0] == 1 ? a.kcache : a.vcache) +
                                     (size_t)pos * a.nkv * a.hd + head * a.hd + d;
                        dst[0] = y0;
                        dst[half] = y1;
                    }
                }
            }
        } else if (tid < R) {
            int m, row;
            if (group_row<MODE, R>(a, g, tid, m, row)) {
                float t = 0.f;
                for (int w = 0; w < kGemvWarps; ++w) t += pb[w * R + tid];
                float y;
                if (WT == WT_F16 && !a.row_scale[0]) y = (a.tscale[0] == 1.0f) ? t : t * a.tscale[0];
                else y = t * (a.row_scale[0] ? a.row_scale[0][row] : a.tscale[0]);
                if (MODE == GM_PLAIN) a.y[row] = y;
                else if (MODE == GM_RESID) a.y[row] = __fadd_rn(a.y[row], y);
                else {
                    a.y[row] = y;
                    if (y > best_v) { best_v = y; best_i = row; }
                }
            }
        }
    }

    if (MODE == GM_LMHEAD) {
        __shared__ unsigned long long kbest[R];
        __syncthreads();
        if (tid < R) kbest[tid] = (best_v == -INFINITY) ? 0ull : argmax_pack(best_v, best_i);
        __syncthreads();
        if (tid == 0) {
            unsigned long long k = 0;
            for (int i = 0; i < R; ++i) k = kbest[i] > k ? kbest[i] : k;
            if (k) atomicMax(&a.st->argmax_key, k);
            __threadfence();
            const unsigned done = atomicAdd(&a.st->lm_done, 1u);
            if (done == gridDim.x - 1) {
                // Last CTA: publish this step's argmax and advance the step state.
                __threadfence();
                const unsigned long long fin = atomicAdd(&a.st->argmax_key, 0ull);
                a.st->next_token = argmax_index(fin);
                a.st->max_logit = argmax_value(fin);
                a.st->token = argmax_index(fin);
                a.st->pos = a.st->pos + 1;
                a.st->argmax_key = 0ull;
                a.st->lm_done = 0u;
            }
        }
    }
}

}  // namespace tvb
