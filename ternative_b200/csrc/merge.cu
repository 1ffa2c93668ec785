// Part 1: load-time I2_S unpack + LoRA merge + F16 / per-row INT8 cast, fused.
//
// Semantics follow the reference's CPU merge exactly (src/model.cpp:180-247):
//   delta[n][k] = sum_{j<r} A[j][k]*B[n][j]   (j ascending, each product and
//                                              each sum rounded separately)
//   merged      = scale*map(code) + delta*(alpha/r)
//   F16         = truncating cast (tensor.cpp:33-57)
//   INT8 row    = the quantizer of model.cpp:381-401 applied per output row
// so F32, F16 and INT8 outputs are bit-identical to the reference.
//
// B200 mapping: the rank-r delta is FP32 CUDA-core work with a fixed
// summation order and IEEE-rounded, never-contracted multiplies and adds
// (__fmul_rn/__fadd_rn).  Packed mul/add.rn.f32x2 would halve the issue count,
// but ptxas contracts those pairs into fused multiply-adds, which changes the
// low bit of the delta.  Each CTA owns ROWS output rows of one tensor;
// its 8 warps stride across the 128-column I2_S blocks of those rows.  One
// launch covers many tensors through a by-value descriptor table.
#include "common.cuh"

#include <algorithm>
#include <vector>

namespace tvb {

constexpr int kMergeThreads = 256;
constexpr int kMergeWarps = kMergeThreads / 32;
constexpr int kMaxDescs = 192;
constexpr int kMaxRank = 256;

enum MergeMode { kOutF32 = 0, kOutF16 = 1, kOutI8Row = 2 };

struct MergeDescDev {
    const uint8_t* i2s;
    const float* A;
    const float* B;
    void* dst;
    float* row_scales;
    float scale;
    float sf;       // alpha / r, rounded once as the reference does (model.cpp:226)
    int K, N, r;
    int k0, ld;     // columns [k0, k0 + K) of source rows of ld columns
};

struct MergeBatch {
    MergeDescDev d[kMaxDescs];
    int cta_start[kMaxDescs + 1];
    int n;
};

__device__ __forceinline__ float code_value(uint32_t word, int byte, int shift, float scale) {
    // map2bit = {-1, 0, +1, 0} (tensor.cpp:1020); value = scale * map[c].
    uint32_t c = (word >> (8 * byte + shift)) & 3u;
    float m = (c == 0u) ? -1.0f : (c == 2u ? 1.0f : 0.0f);
    return __fmul_rn(scale, m);
}

template <int ROWS, int MODE>
__global__ void __launch_bounds__(kMergeThreads)
merge_kernel(const __grid_constant__ MergeBatch batch) {
    extern __shared__ __align__(16) unsigned char smem[];
    const int cta = blockIdx.x;
    // Locate this CTA's tensor (cta_start is ascending).
    int lo = 0, hi = batch.n - 1;
    while (lo < hi) {
        int mid = (lo + hi + 1) >> 1;
        if (batch.cta_start[mid] <= cta) lo = mid; else hi = mid - 1;
    }
    const MergeDescDev& D = batch.d[lo];
    const int K = D.K, N = D.N, r = D.r;
    const int row0 = (cta - batch.cta_start[lo]) * ROWS;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    // B rows of this CTA, transposed: Bs[j][i] = B[row0+i][j].
    float* Bs = reinterpret_cast<float*>(smem);
    for (int idx = tid; idx < ROWS * r; idx += kMergeThreads) {
        int i = idx / r, j = idx - i * r;
        Bs[j * ROWS + i] = (row0 + i < N) ? D.B[(int64_t)(row0 + i) * r + j] : 0.0f;
    }
    uint16_t* stage = reinterpret_cast<uint16_t*>(smem + sizeof(float) * ROWS * kMaxRank);
    __shared__ float wmax[kMergeWarps][ROWS];
    float rmax[ROWS];
#pragma unroll
    for (int i = 0; i < ROWS; ++i) rmax[i] = 0.0f;
    __syncthreads();

    const int nchunks = K >> 7;
    const int src_blocks = D.ld >> 7, blk0 = D.k0 >> 7;   // I2_S blocks per source row, first block
    const int byte_off = (lane & 7) * 4;
    const int shift = 6 - 2 * (lane >> 3);
    for (int c = warp; c < nchunks; c += kMergeWarps) {
        const int col = c * 128 + lane * 4;
        float2 acc[ROWS][2];
#pragma unroll
        for (int i = 0; i < ROWS; ++i) acc[i][0] = acc[i][1] = make_float2(0.f, 0.f);
        const float* Ap = D.A + D.k0 + col;
#pragma unroll 4
        for (int j = 0; j < r; ++j) {
            float4 a = __ldg(reinterpret_cast<const float4*>(Ap + (int64_t)j * D.ld));
            float2 a01 = make_float2(a.x, a.y), a23 = make_float2(a.z, a.w);
            float bj[ROWS];
#pragma unroll
            for (int i4 = 0; i4 < ROWS; i4 += 4) {
                float4 t = *reinterpret_cast<const float4*>(Bs + j * ROWS + i4);
                bj[i4] = t.x; bj[i4 + 1] = t.y; bj[i4 + 2] = t.z; bj[i4 + 3] = t.w;
            }
#pragma unroll
            for (int i = 0; i < ROWS; ++i) {
                // __fmul_rn/__fadd_rn are never contracted into an FMA.
                acc[i][0].x = __fadd_rn(acc[i][0].x, __fmul_rn(a01.x, bj[i]));
                acc[i][0].y = __fadd_rn(acc[i][0].y, __fmul_rn(a01.y, bj[i]));
                acc[i][1].x = __fadd_rn(acc[i][1].x, __fmul_rn(a23.x, bj[i]));
                acc[i][1].y = __fadd_rn(acc[i][1].y, __fmul_rn(a23.y, bj[i]));
            }
        }
        const float2 sf2 = make_float2(D.sf, D.sf);
#pragma unroll
        for (int i = 0; i < ROWS; ++i) {
            const int row = row0 + i;
            if (row >= N) break;
            const int64_t blk = (int64_t)row * src_blocks + blk0 + c;
            uint32_t word = *reinterpret_cast<const uint32_t*>(D.i2s + blk * 32 + byte_off);
            float2 d01 = make_float2(__fmul_rn(acc[i][0].x, sf2.x), __fmul_rn(acc[i][0].y, sf2.y));
            float2 d23 = make_float2(__fmul_rn(acc[i][1].x, sf2.x), __fmul_rn(acc[i][1].y, sf2.y));
            float2 b01 = make_float2(code_value(word, 0, shift, D.scale),
                                     code_value(word, 1, shift, D.scale));
            float2 b23 = make_float2(code_value(word, 2, shift, D.scale),
                                     code_value(word, 3, shift, D.scale));
            float2 v01 = make_float2(__fadd_rn(b01.x, d01.x), __fadd_rn(b01.y, d01.y));
            float2 v23 = make_float2(__fadd_rn(b23.x, d23.x), __fadd_rn(b23.y, d23.y));
            const int64_t off = (int64_t)row * K + col;
            if (MODE == kOutF32) {
                *reinterpret_cast<float4*>(static_cast<float*>(D.dst) + off) =
                    make_float4(v01.x, v01.y, v23.x, v23.y);
            } else {
                uint32_t h0 = f32_to_f16_trunc_fast(v01.x) | ((uint32_t)f32_to_f16_trunc_fast(v01.y) << 16);
                uint32_t h1 = f32_to_f16_trunc_fast(v23.x) | ((uint32_t)f32_to_f16_trunc_fast(v23.y) << 16);
                if (MODE == kOutF16) {
                    *reinterpret_cast<uint2*>(static_cast<uint16_t*>(D.dst) + off) = make_uint2(h0, h1);
                } else {
                    *reinterpret_cast<uint2*>(stage + i * K + col) = make_uint2(h0, h1);
                    // |F16 value| compares like its magnitude bits.
                    uint32_t m = max(max(h0 & 0x7FFFu, (h0 >> 16) & 0x7FFFu),
                                     max(h1 & 0x7FFFu, (h1 >> 16) & 0x7FFFu));
                    rmax[i] = fmaxf(rmax[i], __half2float(__ushort_as_half((uint16_t)m)));
                }
            }
        }
    }

    if (MODE == kOutI8Row) {
#pragma unroll
        for (int i = 0; i < ROWS; ++i) {
            float m = warp_max(rmax[i]);
            if (lane == 0) wmax[warp][i] = m;
        }
        __syncthreads();
        __shared__ float sscale[ROWS];
        if (tid < ROWS) {
            float m = 0.0f;
            for (int w = 0; w < kMergeWarps; ++w) m = fmaxf(m, wmax[w][tid]);
            if (m == 0.0f) m = 1.0f;
            float s = __fdiv_rn(m, 127.0f);
            sscale[tid] = s;
            if (row0 + tid < N) D.row_scales[row0 + tid] = s;
        }
        __syncthreads();
        const int nrows = min(ROWS, N - row0);
        int8_t* out = static_cast<int8_t*>(D.dst) + (int64_t)row0 * K;
        // 16 codes per thread per step, coalesced 16-byte stores.
        for (int e = tid * 16; e < nrows * K; e += kMergeThreads * 16) {
            const int i = e / K;
            const float s = sscale[i];
            const uint4 hv = *reinterpret_cast<const uint4*>(stage + e);
            const uint4 hw = *reinterpret_cast<const uint4*>(stage + e + 8);
            const uint32_t hs[8] = {hv.x, hv.y, hv.z, hv.w, hw.x, hw.y, hw.z, hw.w};
            uint32_t words[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                uint32_t acc = 0;
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                    uint32_t h2 = hs[2 * q + t];
                    float lo_v = __half2float(__ushort_as_half((uint16_t)(h2 & 0xFFFFu)));
                    float hi_v = __half2float(__ushort_as_half((uint16_t)(h2 >> 16)));
                    acc |= ((uint32_t)(uint8_t)int8_code(lo_v, s)) << (16 * t);
                    acc |= ((uint32_t)(uint8_t)int8_code(hi_v, s)) << (16 * t + 8);
                }
                words[q] = acc;
            }
            *reinterpret_cast<uint4*>(out + e) = make_uint4(words[0], words[1], words[2], words[3]);
        }
    }
}

// I2_S -> F32 (tensor.cpp:1006-1050): one thread per code byte.
__global__ void i2s_unpack_kernel(const uint8_t* __restrict__ i2s, int64_t nbytes, float scale,
                                  float* __restrict__ out) {
    int64_t t = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= nbytes) return;
    uint32_t b = i2s[t];
    int64_t base = (t >> 5) * 128 + (t & 31);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint32_t c = (b >> (6 - 2 * q)) & 3u;
        float m = (c == 0u) ? -1.0f : (c == 2u ? 1.0f : 0.0f);
        out[base + 32 * q] = __fmul_rn(scale, m);
    }
}

// Per-row INT8 from F16 weights: one warp per row, two passes over the row.
__global__ void quant_rows_kernel(const uint16_t* __restrict__ w, int N, int K,
                                  int8_t* __restrict__ q, float* __restrict__ scales) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= N) return;
    const uint16_t* wr = w + (int64_t)row * K;
    uint32_t m = 0;
    for (int k = lane; k < K; k += 32) m = max(m, (uint32_t)(wr[k] & 0x7FFFu));
    float mx = warp_max(__half2float(__ushort_as_half((uint16_t)m)));
    if (mx == 0.0f) mx = 1.0f;
    const float s = __fdiv_rn(mx, 127.0f);
    if (lane == 0) scales[row] = s;
    int8_t* qr = q + (int64_t)row * K;
    for (int k = lane; k < K; k += 32) qr[k] = int8_code(__half2float(__ushort_as_half(wr[k])), s);
}

// Per-tensor INT8 (model.cpp:381-401): max |w| over the tensor, then codes.
__global__ void tensor_absmax_kernel(const uint16_t* __restrict__ w, int64_t n,
                                     unsigned int* __restrict__ maxbits) {
    uint32_t m = 0;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        m = max(m, (uint32_t)(w[i] & 0x7FFFu));
    float f = warp_max(__half2float(__ushort_as_half((uint16_t)m)));
    if ((threadIdx.x & 31) == 0) atomicMax(maxbits, __float_as_uint(f));  // f >= 0
}

__global__ void tensor_quant_kernel(const uint16_t* __restrict__ w, int64_t n,
                                    const unsigned int* __restrict__ maxbits,
                                    int8_t* __restrict__ q) {
    float mx = __uint_as_float(*maxbits);
    if (mx == 0.0f) mx = 1.0f;
    const float s = __fdiv_rn(mx, 127.0f);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n;
         i += (int64_t)gridDim.x * blockDim.x)
        q[i] = int8_code(__half2float(__ushort_as_half(w[i])), s);
}

__global__ void tensor_scale_kernel(float* scales) {
    float mx = scales[0];   // holds the max bits written by tensor_absmax_kernel
    if (mx == 0.0f) mx = 1.0f;
    scales[0] = __fdiv_rn(mx, 127.0f);
}

// ---------------------------------------------------------------------------
static bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

static size_t merge_smem(int rows, int mode, int K) {
    size_t s = sizeof(float) * rows * kMaxRank;
    if (mode == kOutI8Row) s += (size_t)rows * K * sizeof(uint16_t);
    return s;
}

template <int ROWS, int MODE>
static tvb_status launch_merge(MergeBatch& b, int total_ctas, int maxK, cudaStream_t st) {
    size_t smem = merge_smem(ROWS, MODE, maxK);
    auto kern = merge_kernel<ROWS, MODE>;
    TVB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    kern<<<total_ctas, kMergeThreads, smem, st>>>(b);
    return check_launch("merge_kernel");
}

static tvb_status validate(const tvb_merge_desc& d, tvb_dtype out) {
    TVB_REQUIRE(d.i2s && d.dst, "merge: null i2s/dst");
    TVB_REQUIRE(d.K > 0 && d.N > 0 && d.K % 128 == 0, "merge: K=%d must be a positive multiple of 128", d.K);
    TVB_REQUIRE(d.r >= 0 && d.r <= kMaxRank, "merge: rank %d outside [0, %d]", d.r, kMaxRank);
    TVB_REQUIRE(d.r == 0 || (d.A && d.B), "merge: rank %d needs A and B", d.r);
    TVB_REQUIRE(aligned(d.i2s, 4), "merge: i2s must be 4-byte aligned");
    TVB_REQUIRE(aligned(d.dst, 16), "merge: dst must be 16-byte aligned");
    TVB_REQUIRE(!d.A || aligned(d.A, 16), "merge: A must be 16-byte aligned");
    TVB_REQUIRE(out != TVB_I8_ROW || d.row_scales, "merge: TVB_I8_ROW needs row_scales");
    const int ld = d.ld ? d.ld : d.K;
    TVB_REQUIRE(d.k0 >= 0 && d.k0 % 128 == 0 && ld % 128 == 0 && d.k0 + d.K <= ld,
                "merge: column slice [%d, %d) of %d columns (multiples of 128)", d.k0, d.k0 + d.K, ld);
    return TVB_OK;
}

static tvb_status merge_run(const tvb_merge_desc* descs, int n, tvb_dtype out, cudaStream_t st) {
    if (n <= 0) return TVB_OK;
    TVB_REQUIRE(descs, "merge: descs is NULL");
    if (out == TVB_I8_TENSOR)
        return set_error(TVB_ERR_UNSUPPORTED,
                         "merge: per-tensor INT8 needs a whole-tensor max; merge to TVB_F16 "
                         "and call tvb_quantize_int8(per_row=0)");
    TVB_REQUIRE(out == TVB_F32 || out == TVB_F16 || out == TVB_I8_ROW, "merge: bad dtype %d", (int)out);
    for (int i = 0; i < n; ++i) {
        tvb_status s = validate(descs[i], out);
        if (s != TVB_OK) return s;
    }
    // I8 rows stage ROWS*K F16 values in shared memory: 8 rows up to K=13312.
    int maxK = 0;
    for (int i = 0; i < n; ++i) maxK = std::max(maxK, descs[i].K);
    const bool narrow = (out == TVB_I8_ROW) && merge_smem(8, kOutI8Row, maxK) > 220 * 1024;
    if (narrow && merge_smem(4, kOutI8Row, maxK) > 220 * 1024)
        return set_error(TVB_ERR_UNSUPPORTED, "merge: K=%d too large for per-row INT8", maxK);
    const int rows = narrow ? 4 : 8;

    static thread_local MergeBatch b;
    for (int base = 0; base < n; base += kMaxDescs) {
        const int cnt = std::min(kMaxDescs, n - base);
        int ctas = 0;
        for (int i = 0; i < cnt; ++i) {
            const tvb_merge_desc& s = descs[base + i];
            MergeDescDev& d = b.d[i];
            d.i2s = s.i2s;
            d.A = s.r ? s.A : nullptr;
            d.B = s.r ? s.B : nullptr;
            d.dst = s.dst;
            d.row_scales = s.row_scales;
            d.scale = s.scale;
            d.r = s.r;
            d.sf = s.r ? s.alpha / (float)s.r : 0.0f;
            d.K = s.K;
            d.N = s.N;
            d.k0 = s.k0;
            d.ld = s.ld ? s.ld : s.K;
            b.cta_start[i] = ctas;
            ctas += (s.N + rows - 1) / rows;
        }
        b.cta_start[cnt] = ctas;
        b.n = cnt;
        tvb_status st_ = TVB_OK;
        if (out == TVB_F32) st_ = launch_merge<8, kOutF32>(b, ctas, maxK, st);
        else if (out == TVB_F16) st_ = launch_merge<8, kOutF16>(b, ctas, maxK, st);
        else if (!narrow) st_ = launch_merge<8, kOutI8Row>(b, ctas, maxK, st);
        else st_ = launch_merge<4, kOutI8Row>(b, ctas, maxK, st);
        if (st_ != TVB_OK) return st_;
    }
    return TVB_OK;
}

tvb_status merge_exact(const tvb_merge_desc* descs, int n, tvb_dtype out, cudaStream_t st) {
    return merge_run(descs, n, out, st);
}

}  // namespace tvb

using namespace tvb;

extern "C" {

tvb_status tvb_merge_i2s_lora(const uint8_t* i2s, float scale, int K, int N, const float* A,
                              const float* B, int r, float alpha, tvb_dtype out, void* dst,
                              float* row_scales, void* stream) {
    tvb_merge_desc d{i2s, scale, K, N, A, B, A ? r : 0, alpha, dst, row_scales};
    return merge_run(&d, 1, out, as_stream(stream));
}

tvb_status tvb_merge_batch(const tvb_merge_desc* descs, int n, tvb_dtype out, void* stream) {
    return merge_run(descs, n, out, as_stream(stream));
}

tvb_status tvb_i2s_unpack(const uint8_t* i2s, int64_t n, float scale, float* out, void* stream) {
    TVB_REQUIRE(i2s && out, "i2s_unpack: null pointer");
    TVB_REQUIRE(n >= 0 && n % 128 == 0, "i2s_unpack: n=%lld must be a multiple of 128", (long long)n);
    if (!n) return TVB_OK;
    int64_t nbytes = n / 4;
    i2s_unpack_kernel<<<(unsigned)((nbytes + 255) / 256), 256, 0, as_stream(stream)>>>(i2s, nbytes, scale, out);
    return check_launch("i2s_unpack_kernel");
}

tvb_status tvb_quantize_int8(const uint16_t* w, int N, int K, int per_row, int8_t* q,
                             float* scales, void* stream) {
    TVB_REQUIRE(w && q && scales, "quantize_int8: null pointer");
    TVB_REQUIRE(N > 0 && K > 0, "quantize_int8: bad shape %dx%d", N, K);
    cudaStream_t st = as_stream(stream);
    if (per_row) {
        quant_rows_kernel<<<(N + 7) / 8, 256, 0, st>>>(w, N, K, q, scales);
        return check_launch("quant_rows_kernel");
    }
    const int64_t n = (int64_t)N * K;
    TVB_CUDA(cudaMemsetAsync(scales, 0, sizeof(float), st));
    const int grid = num_sms() * 4;
    tensor_absmax_kernel<<<grid, 256, 0, st>>>(w, n, reinterpret_cast<unsigned int*>(scales));
    tvb_status s = check_launch("tensor_absmax_kernel");
    if (s != TVB_OK) return s;
    tensor_quant_kernel<<<grid, 256, 0, st>>>(w, n, reinterpret_cast<const unsigned int*>(scales), q);
    s = check_launch("tensor_quant_kernel");
    if (s != TVB_OK) return s;
    tensor_scale_kernel<<<1, 1, 0, st>>>(scales);
    return check_launch("tensor_scale_kernel");
}

}  // extern "C"
