// The CUDABackend per-op device API (include/ternative/ops.h:102-142,
// cuda/ops_cuda.cu:109-201, 714-789) as stand-alone kernels.  The fused decode
// step does not use these; they keep the reference's call-by-call interface
// available to a host that drives the layer loop itself.
#include "common.cuh"
#include "prefill.h"

namespace tvb {

// tvb_matmul takes the tensor-core GEMM from this many activation rows on
// (below it, one streaming GEMV per row reads the weights fewer times).
constexpr int kMatmulTensorRows = 8;

tvb_status standalone_gemv(float* y, const float* x, const void* W, int wt, const float* row_scales,
                           float tscale, int K, int N, cudaStream_t st);
tvb_status standalone_attention(const float* q, const float* kc, const float* vc, int kv_len, float* out,
                                int nh, int nkv, int hd, float scale, cudaStream_t st);

__global__ void add_kernel(float* __restrict__ o, const float* __restrict__ a,
                           const float* __restrict__ b, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) o[i] = __fadd_rn(a[i], b[i]);
}

__global__ void mul_kernel(float* __restrict__ o, const float* __restrict__ a,
                           const float* __restrict__ b, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) o[i] = __fmul_rn(a[i], b[i]);
}

__global__ void relu2_kernel(float* __restrict__ o, const float* __restrict__ x, int n) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) {
        float v = fmaxf(x[i], 0.0f);
        o[i] = __fmul_rn(v, v);
    }
}

// One CTA: sum of squares, rms = sqrt(ss/N + eps), out = x * (inv * w)
// (tensor.cpp:661-686).  Safe in place (out == x).
__global__ void rms_norm_kernel(float* out, const float* x, const float* __restrict__ w, float eps,
                                int n) {
    __shared__ float red[32];
    __shared__ float inv_s;
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
        float t = 0.f;
        for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
        inv_s = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(t, (float)n), eps)));
    }
    __syncthreads();
    const float inv = inv_s;
    for (int i = threadIdx.x; i < n; i += blockDim.x) out[i] = __fmul_rn(x[i], __fmul_rn(inv, w[i]));
}

// NeoX RoPE for one position (tensor.cpp:840-888 formulas, IEEE cos/sin of the
// F32 angle): CTA per head, thread per pair.
__global__ void rope_kernel(float* q, float* k, int pos, float theta, int nh, int nkv, int hd) {
    const int head = blockIdx.x, ic = threadIdx.x, half = hd >> 1;
    if (head >= nh + nkv || ic >= half) return;
    float* v = head < nh ? q + head * hd : k + (head - nh) * hd;
    const float freq = 1.0f / powf(theta, (float)(2 * ic) / (float)hd);
    const float ang = (float)pos * freq;
    float s, c;
    sincosf(ang, &s, &c);
    const float x0 = v[ic], x1 = v[ic + half];
    v[ic] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    v[ic + half] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
}

__global__ void kv_write_kernel(const float* __restrict__ k, const float* __restrict__ v,
                                float* __restrict__ kc, float* __restrict__ vc, int pos, int hk) {
    int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < hk) {
        kc[(size_t)pos * hk + i] = k[i];
        vc[(size_t)pos * hk + i] = v[i];
    }
}

}  // namespace tvb

using namespace tvb;

extern "C" {

tvb_status tvb_gemv_f16(float* y, const float* x, const void* W, int K, int N, void* stream) {
    return standalone_gemv(y, x, W, 0, nullptr, 1.0f, K, N, as_stream(stream));
}

tvb_status tvb_gemv_int8(float* y, const float* x, const void* W, float scale, int K, int N,
                         void* stream) {
    return standalone_gemv(y, x, W, 1, nullptr, scale, K, N, as_stream(stream));
}

tvb_status tvb_gemv_int8_rows(float* y, const float* x, const void* W, const float* row_scales, int K,
                              int N, void* stream) {
    TVB_REQUIRE(row_scales, "gemv_int8_rows: row_scales is NULL");
    return standalone_gemv(y, x, W, 1, row_scales, 1.0f, K, N, as_stream(stream));
}

tvb_status tvb_rms_norm(float* out, const float* x, const float* w, float eps, int N, void* stream) {
    TVB_REQUIRE(out && x && w && N > 0, "rms_norm: bad argument");
    rms_norm_kernel<<<1, 1024, 0, as_stream(stream)>>>(out, x, w, eps, N);
    return check_launch("rms_norm_kernel");
}

tvb_status tvb_add(float* out, const float* a, const float* b, int N, void* stream) {
    TVB_REQUIRE(out && a && b && N >= 0, "add: bad argument");
    if (!N) return TVB_OK;
    add_kernel<<<(N + 255) / 256, 256, 0, as_stream(stream)>>>(out, a, b, N);
    return check_launch("add_kernel");
}

tvb_status tvb_mul(float* out, const float* a, const float* b, int N, void* stream) {
    TVB_REQUIRE(out && a && b && N >= 0, "mul: bad argument");
    if (!N) return TVB_OK;
    mul_kernel<<<(N + 255) / 256, 256, 0, as_stream(stream)>>>(out, a, b, N);
    return check_launch("mul_kernel");
}

tvb_status tvb_relu2(float* out, const float* x, int N, void* stream) {
    TVB_REQUIRE(out && x && N >= 0, "relu2: bad argument");
    if (!N) return TVB_OK;
    relu2_kernel<<<(N + 255) / 256, 256, 0, as_stream(stream)>>>(out, x, N);
    return check_launch("relu2_kernel");
}

tvb_status tvb_rope_inplace(float* q, float* k, int pos, float theta, int nh, int nkv, int hd,
                            void* stream) {
    TVB_REQUIRE(q && k && nh > 0 && nkv >= 0 && hd > 0 && hd % 2 == 0 && hd <= 2048 && pos >= 0,
                "rope_inplace: bad argument");
    rope_kernel<<<nh + nkv, hd / 2, 0, as_stream(stream)>>>(q, k, pos, theta, nh, nkv, hd);
    return check_launch("rope_kernel");
}

tvb_status tvb_kv_write(const float* k, const float* v, float* kc, float* vc, int pos, int Hk,
                        void* stream) {
    TVB_REQUIRE(k && v && kc && vc && pos >= 0 && Hk > 0, "kv_write: bad argument");
    kv_write_kernel<<<(Hk + 255) / 256, 256, 0, as_stream(stream)>>>(k, v, kc, vc, pos, Hk);
    return check_launch("kv_write_kernel");
}

tvb_status tvb_matmul(float* y, const float* x, int M, int K, const tvb_weight* w, int N,
                      void* stream) {
    TVB_REQUIRE(y && x && w && w->w, "matmul: null pointer");
    TVB_REQUIRE(M >= 0 && K > 0 && N > 0, "matmul: bad shape %dx%dx%d", M, K, N);
    int wt;
    if (w->dtype == TVB_F16) wt = 0;
    else if (w->dtype == TVB_I8_ROW || w->dtype == TVB_I8_TENSOR) wt = 1;
    else return set_error(TVB_ERR_UNSUPPORTED, "matmul: weight dtype %d", (int)w->dtype);
    const float* rs = w->dtype == TVB_I8_ROW ? w->row_scales : nullptr;
    const float ts = w->dtype == TVB_I8_TENSOR ? w->tensor_scale : 1.0f;
    const cudaStream_t st = as_stream(stream);
    if (M >= kMatmulTensorRows && K % 64 == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
        (reinterpret_cast<uintptr_t>(w->w) & 15) == 0) {
        // Batched rows: one tensor-core GEMM.  x is split into F16 hi/lo planes
        // (with a power-of-two row scale) in stream-ordered scratch; INT8
        // weights are widened to F16 there too.
        const size_t plane = (size_t)M * K;
        const size_t wide = wt ? (size_t)N * K : 0;
        unsigned char* buf = nullptr;
        // then the split-K / stream-K workspace: SMs x 128 x 256 partial sums
        // and SMs x 4 zeroed piece flags
        const size_t part_floats = (size_t)num_sms() * 128 * 256;
        const size_t head = ((2 * plane + wide) * 2 + (size_t)M * 4 + 255) & ~(size_t)255;
        const size_t bytes = head + part_floats * 4 + (size_t)num_sms() * 16;
        TVB_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&buf), bytes, st));
        uint16_t* xh = reinterpret_cast<uint16_t*>(buf);
        uint16_t* xl = xh + plane;
        uint16_t* w16 = xl + plane;
        int* ex = reinterpret_cast<int*>(w16 + wide);
        float* part = reinterpret_cast<float*>(buf + head);
        unsigned* flags = reinterpret_cast<unsigned*>(part + part_floats);
        tvb_status s = TVB_OK;
        const cudaError_t me = cudaMemsetAsync(flags, 0, (size_t)num_sms() * 16, st);
        if (me != cudaSuccess) s = cuda_error(me, "cudaMemsetAsync");
        if (s == TVB_OK) s = pf_norm_split(x, nullptr, M, K, 0.f, xh, xl, ex, st);
        if (s == TVB_OK && wt) s = pf_i8_to_f16(static_cast<const int8_t*>(w->w), wide, w16, st);
        if (s == TVB_OK) {
            PfGemm g;
            g.mode = PF_STORE;
            g.S = M;
            g.K = K;
            g.xh = xh;
            g.xl = xl;
            g.row_exp = ex;
            g.m[0].w = wt ? w16 : static_cast<const uint16_t*>(w->w);
            g.m[0].rows = N;
            g.m[0].row_scales = rs;
            g.m[0].scale = ts;
            g.y = y;
            g.ldy = N;
            g.part = part;
            g.part_floats = part_floats;
            g.flags = flags;
            s = pf_gemm(g, st);
        }
        cudaFreeAsync(buf, st);
        return s;
    }
    // One streaming GEMV per activation row.
    for (int m = 0; m < M; ++m) {
        tvb_status s = standalone_gemv(y + (size_t)m * N, x + (size_t)m * K, w->w, wt, rs, ts, K, N,
                                       as_stream(stream));
        if (s != TVB_OK) return s;
    }
    return TVB_OK;
}

tvb_status tvb_attention_decode(const float* q, const float* kc, const float* vc, int kv_len, float* out,
                                int nh, int nkv, int hd, float scale, void* stream) {
    return standalone_attention(q, kc, vc, kv_len, out, nh, nkv, hd, scale, as_stream(stream));
}

}  // extern "C"
