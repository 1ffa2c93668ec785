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
// low bit of the delta.  Each CTA owns a 64-row x 128-column tile of one
// tensor (the 128 columns are one I2_S block of each row) and stages A and B
// through shared memory 32 rank-columns at a time; each thread accumulates a
// 4-row x 8-column register tile over j in order.  A CTA of whole rows re-read
// all of A per 8 rows (32 bytes of L2 traffic per output at rank 64); the tile
// reads 6.  One launch covers many tensors through a by-value descriptor table.
// Per-row INT8 needs each row's largest magnitude before any code: the tiles
// write the exact F16 values into a workspace and fold their rows' maxima into
// per-row words, and a second kernel writes the codes and scales.
#include "common.cuh"

#include <algorithm>
#include <vector>

namespace tvb {

constexpr int kMergeThreads = 256;
constexpr int kMaxDescs = 192;
constexpr int kMaxRank = 256;
constexpr int kTileRows = 64, kTileCols = 128, kJChunk = 32;
constexpr int kBsLd = kTileRows + 4;   // Bs row stride: 16-byte rows, 4-way store conflicts at most

enum MergeMode { kOutF32 = 0, kOutF16 = 1, kOutF16Stage = 2 };

struct MergeDescDev {
    const uint8_t* i2s;
    const float* A;
    const float* B;
    void* dst;           // output; kOutF16Stage: the F16 workspace of this tensor
    unsigned* rowmax;    // kOutF16Stage: per-row largest |F16| (as float bits)
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

__device__ __forceinline__ int find_desc(const MergeBatch& b, int cta) {
    int lo = 0, hi = b.n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (b.cta_start[mid] <= cta) lo = mid; else hi = mid - 1;
    }
    return lo;
}

template <int MODE>
__global__ void __launch_bounds__(kMergeThreads)
merge_tile_kernel(const __grid_constant__ MergeBatch batch) {
    __shared__ __align__(16) float As[kJChunk][kTileCols];   // As[jj][c] = A[j0 + jj][col0 + c]
    __shared__ __align__(16) float Bs[kJChunk][kBsLd];       // Bs[jj][i] = B[row0 + i][j0 + jj]
    const int di = find_desc(batch, blockIdx.x);
    const MergeDescDev& D = batch.d[di];
    const int K = D.K, N = D.N, r = D.r;
    const int ctiles = K / kTileCols;
    const int t = blockIdx.x - batch.cta_start[di];
    const int rt = t / ctiles, ct = t - rt * ctiles;
    const int row0 = rt * kTileRows, col0 = ct * kTileCols;
    const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;

    float acc[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int q = 0; q < 8; ++q) acc[i][q] = 0.f;

    for (int j0 = 0; j0 < r; j0 += kJChunk) {
        const int jn = min(kJChunk, r - j0);
        __syncthreads();   // the previous chunk is consumed
        for (int idx = tid; idx < kJChunk * (kTileCols / 4); idx += kMergeThreads) {
            const int jj = idx >> 5, c4 = idx & 31;
            float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
            if (jj < jn)
                v = __ldg(reinterpret_cast<const float4*>(D.A + (int64_t)(j0 + jj) * D.ld + D.k0 + col0) + c4);
            *reinterpret_cast<float4*>(&As[jj][c4 * 4]) = v;
        }
        for (int idx = tid; idx < kTileRows * kJChunk; idx += kMergeThreads) {
            const int i = idx >> 5, jj = idx & 31;
            Bs[jj][i] = (jj < jn && row0 + i < N) ? __ldg(D.B + (int64_t)(row0 + i) * r + j0 + jj) : 0.f;
        }
        __syncthreads();
#pragma unroll 2
        for (int jj = 0; jj < jn; ++jj) {
            const float4 a0 = *reinterpret_cast<const float4*>(&As[jj][tx * 8]);
            const float4 a1 = *reinterpret_cast<const float4*>(&As[jj][tx * 8 + 4]);
            const float4 bv = *reinterpret_cast<const float4*>(&Bs[jj][ty * 4]);
            const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
            const float b[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int q = 0; q < 8; ++q) acc[i][q] = __fadd_rn(acc[i][q], __fmul_rn(a[q], b[i]));
        }
    }

    // epilogue: the I2_S codes of this thread's 8 columns sit in bytes
    // (8 tx) % 32 .. + 7 of the row's 128-column block, at one bit position
    const int src_blocks = D.ld >> 7, blk0 = D.k0 >> 7;
    const int cb = (tx * 8) & 31, shift = 6 - 2 * ((tx * 8) >> 5);
    __shared__ unsigned smax[kTileRows];
    if (MODE == kOutF16Stage) {
        for (int i = tid; i < kTileRows; i += kMergeThreads) smax[i] = 0u;
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int row = row0 + ty * 4 + i;
        if (row >= N) continue;
        const uint8_t* blk = D.i2s + ((int64_t)row * src_blocks + blk0 + ct) * 32 + cb;
        const uint32_t words[2] = {*reinterpret_cast<const uint32_t*>(blk),
                                   *reinterpret_cast<const uint32_t*>(blk + 4)};
        float v[8];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
            // map2bit = {-1, 0, +1, 0} (tensor.cpp:1020); value = scale * map[c]
            const uint32_t c = (words[q >> 2] >> (8 * (q & 3) + shift)) & 3u;
            const float m = (c == 0u) ? -1.0f : (c == 2u ? 1.0f : 0.0f);
            v[q] = __fadd_rn(__fmul_rn(D.scale, m), __fmul_rn(acc[i][q], D.sf));
        }
        const int64_t off = (int64_t)row * K + col0 + tx * 8;
        if (MODE == kOutF32) {
            float4* o = reinterpret_cast<float4*>(static_cast<float*>(D.dst) + off);
            o[0] = make_float4(v[0], v[1], v[2], v[3]);
            o[1] = make_float4(v[4], v[5], v[6], v[7]);
        } else {
            uint32_t h[4];
            uint32_t mbits = 0;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t lo = f32_to_f16_trunc_fast(v[2 * q]), hi = f32_to_f16_trunc_fast(v[2 * q + 1]);
                h[q] = lo | (hi << 16);
                mbits = max(mbits, max(lo & 0x7FFFu, hi & 0x7FFFu));   // |F16| compares like its bits
            }
            *reinterpret_cast<uint4*>(static_cast<uint16_t*>(D.dst) + off) = make_uint4(h[0], h[1], h[2], h[3]);
            if (MODE == kOutF16Stage)
                atomicMax(&smax[ty * 4 + i],
                          __float_as_uint(__half2float(__ushort_as_half((uint16_t)mbits))));   // >= 0
        }
    }
    if (MODE == kOutF16Stage) {
        __syncthreads();
        for (int i = tid; i < kTileRows; i += kMergeThreads)
            if (row0 + i < N && smax[i]) atomicMax(D.rowmax + row0 + i, smax[i]);
    }
}

// Per-row INT8, second pass: one warp per row reads the row's exact F16
// values and writes the codes and the row's scale (model.cpp:381-401 per row).
struct CodeDescDev {
    const uint16_t* f16;
    const unsigned* rowmax;
    int8_t* q;
    float* row_scales;
    int K;
};
struct CodeBatch {
    CodeDescDev d[kMaxDescs];
    int row_start[kMaxDescs + 1];
    int n;
};

__global__ void __launch_bounds__(256) merge_codes_kernel(const __grid_constant__ CodeBatch batch, int total_rows) {
    const int grow = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (grow >= total_rows) return;
    int lo = 0, hi = batch.n - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (batch.row_start[mid] <= grow) lo = mid; else hi = mid - 1;
    }
    const CodeDescDev& D = batch.d[lo];
    const int row = grow - batch.row_start[lo];
    float mx = __uint_as_float(D.rowmax[row]);
    if (mx == 0.0f) mx = 1.0f;
    const float s = __fdiv_rn(mx, 127.0f);
    if (lane == 0) D.row_scales[row] = s;
    const uint16_t* src = D.f16 + (int64_t)row * D.K;
    int8_t* out = D.q + (int64_t)row * D.K;
    for (int e = lane * 16; e < D.K; e += 32 * 16) {   // K % 128 == 0: whole 16-element groups
        const uint4 hv = *reinterpret_cast<const uint4*>(src + e);
        const uint4 hw = *reinterpret_cast<const uint4*>(src + e + 8);
        const uint32_t hs[8] = {hv.x, hv.y, hv.z, hv.w, hw.x, hw.y, hw.z, hw.w};
        uint32_t words[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            uint32_t acc = 0;
#pragma unroll
            for (int t = 0; t < 2; ++t) {
                const uint32_t h2 = hs[2 * q + t];
                const float lo_v = __half2float(__ushort_as_half((uint16_t)(h2 & 0xFFFFu)));
                const float hi_v = __half2float(__ushort_as_half((uint16_t)(h2 >> 16)));
                acc |= ((uint32_t)(uint8_t)int8_code(lo_v, s)) << (16 * t);
                acc |= ((uint32_t)(uint8_t)int8_code(hi_v, s)) << (16 * t + 8);
            }
            words[q] = acc;
        }
        *reinterpret_cast<uint4*>(out + e) = make_uint4(words[0], words[1], words[2], words[3]);
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

// Per-row INT8 goes through an F16 workspace in groups of tensors of at most
// this many bytes.
constexpr size_t kI8WorkspaceBytes = 512ull << 20;

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
    static thread_local MergeBatch b;
    static thread_local CodeBatch cb;
    auto fill = [&](MergeDescDev& d, const tvb_merge_desc& s) {
        d.i2s = s.i2s;
        d.A = s.r ? s.A : nullptr;
        d.B = s.r ? s.B : nullptr;
        d.dst = s.dst;
        d.rowmax = nullptr;
        d.scale = s.scale;
        d.r = s.r;
        d.sf = s.r ? s.alpha / (float)s.r : 0.0f;
        d.K = s.K;
        d.N = s.N;
        d.k0 = s.k0;
        d.ld = s.ld ? s.ld : s.K;
    };
    auto tiles = [](const tvb_merge_desc& s) { return ((s.N + kTileRows - 1) / kTileRows) * (s.K / kTileCols); };
    if (out != TVB_I8_ROW) {
        for (int base = 0; base < n; base += kMaxDescs) {
            const int cnt = std::min(kMaxDescs, n - base);
            int ctas = 0;
            for (int i = 0; i < cnt; ++i) {
                fill(b.d[i], descs[base + i]);
                b.cta_start[i] = ctas;
                ctas += tiles(descs[base + i]);
            }
            b.cta_start[cnt] = ctas;
            b.n = cnt;
            if (out == TVB_F32) merge_tile_kernel<kOutF32><<<ctas, kMergeThreads, 0, st>>>(b);
            else merge_tile_kernel<kOutF16><<<ctas, kMergeThreads, 0, st>>>(b);
            TVB_TRY(check_launch("merge_tile_kernel"));
        }
        return TVB_OK;
    }
    // Per-row INT8: groups of tensors whose F16 images and row maxima fit the workspace.
    size_t need = 0;
    for (int i = 0; i < n; ++i)
        need = std::max(need, (size_t)descs[i].N * descs[i].K * 2 + (size_t)descs[i].N * 4 + 256);
    const size_t ws_bytes = std::max(need, std::min(kI8WorkspaceBytes, [&] {
        size_t t = 0;
        for (int i = 0; i < n; ++i) t += (size_t)descs[i].N * descs[i].K * 2 + (size_t)descs[i].N * 4 + 256;
        return t;
    }()));
    void* ws = nullptr;
    TVB_CUDA(cudaMallocAsync(&ws, ws_bytes, st));
    tvb_status result = TVB_OK;
    int i = 0;
    while (i < n && result == TVB_OK) {
        size_t used = 0;
        int cnt = 0, ctas = 0, rows = 0;
        unsigned char* p = static_cast<unsigned char*>(ws);
        while (i + cnt < n && cnt < kMaxDescs) {
            const tvb_merge_desc& s = descs[i + cnt];
            const size_t f16 = ((size_t)s.N * s.K * 2 + 255) / 256 * 256, mx = ((size_t)s.N * 4 + 255) / 256 * 256;
            if (cnt > 0 && used + f16 + mx > ws_bytes) break;
            MergeDescDev& d = b.d[cnt];
            fill(d, s);
            d.dst = p + used;
            d.rowmax = reinterpret_cast<unsigned*>(p + used + f16);
            cb.d[cnt] = CodeDescDev{static_cast<const uint16_t*>(d.dst), d.rowmax, static_cast<int8_t*>(s.dst),
                                    s.row_scales, s.K};
            b.cta_start[cnt] = ctas;
            cb.row_start[cnt] = rows;
            ctas += tiles(s);
            rows += s.N;
            used += f16 + mx;
            ++cnt;
        }
        b.cta_start[cnt] = ctas;
        cb.row_start[cnt] = rows;
        b.n = cb.n = cnt;
        cudaError_t e = cudaMemsetAsync(ws, 0, used, st);   // row maxima start at 0 (workspace images too)
        if (e != cudaSuccess) { result = cuda_error(e, "cudaMemsetAsync"); break; }
        merge_tile_kernel<kOutF16Stage><<<ctas, kMergeThreads, 0, st>>>(b);
        result = check_launch("merge_tile_kernel");
        if (result != TVB_OK) break;
        merge_codes_kernel<<<(rows + 7) / 8, 256, 0, st>>>(cb, rows);
        result = check_launch("merge_codes_kernel");
        i += cnt;
    }
    cudaError_t e = cudaFreeAsync(ws, st);
    if (result == TVB_OK && e != cudaSuccess) result = cuda_error(e, "cudaFreeAsync");
    return result;
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
