// Shared device/host helpers for the tvb200 kernels (sm_100a only).
#pragma once

#include <utility>

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "tvb200.h"

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "tvb200 is written for sm_100a only"
#endif

namespace tvb {

// ---- host-side error plumbing (status.cpp) --------------------------------
tvb_status set_error(tvb_status s, const char* fmt, ...);
tvb_status cuda_error(cudaError_t e, const char* what);
// Reports a failed launch (cudaGetLastError) as TVB_ERR_CUDA.
tvb_status check_launch(const char* what);

#define TVB_CUDA(call)                                                   \
    do {                                                                 \
        cudaError_t _e = (call);                                         \
        if (_e != cudaSuccess) return ::tvb::cuda_error(_e, #call);      \
    } while (0)

#define TVB_REQUIRE(cond, ...)                                                        \
    do {                                                                              \
        if (!(cond)) return ::tvb::set_error(TVB_ERR_INVALID, __VA_ARGS__);           \
    } while (0)

#define TVB_TRY(x)                   \
    do {                             \
        tvb_status _s = (x);         \
        if (_s != TVB_OK) return _s; \
    } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

// ---- numerics shared with the reference --------------------------------------

// F32 -> F16 by truncation, the reference's f16_t(float) (tensor.cpp:33-57):
// mantissa shifted right without rounding, subnormals truncated, exponent
// overflow -> signed infinity, NaN/inf keep the top payload bits.
__host__ __device__ __forceinline__ uint16_t f32_to_f16_trunc(float f) {
#ifdef __CUDA_ARCH__
    uint32_t x = __float_as_uint(f);
#else
    uint32_t x;
    __builtin_memcpy(&x, &f, 4);
#endif
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t e = (x >> 23) & 0xFFu;
    uint32_t m = x & 0x7FFFFFu;
    if (e == 0xFFu) return (uint16_t)(sign | 0x7C00u | (m >> 13));
    int32_t ne = (int32_t)e - 112;
    if (ne >= 31) return (uint16_t)(sign | 0x7C00u);
    if (ne <= 0) {
        if (ne < -10) return (uint16_t)sign;
        m = (m | 0x800000u) >> (1 - ne);
        return (uint16_t)(sign | (m >> 13));
    }
    return (uint16_t)(sign | ((uint32_t)ne << 10) | (m >> 13));
}

// The same truncation with the hardware round-toward-zero conversion where the
// two agree: finite |f| < 65536 (RTZ keeps the top 10 mantissa bits, subnormals
// included, like the bit routine).  Larger magnitudes (the reference gives
// infinity where RTZ saturates at 65504) and NaN take the bit routine.
__device__ __forceinline__ uint16_t f32_to_f16_trunc_fast(float f) {
    if (fabsf(f) < 65536.0f) return __half_as_ushort(__float2half_rz(f));
    return f32_to_f16_trunc(f);
}

// Round half away from zero (std::round) for |x| < 2^23, built from truncation.
__device__ __forceinline__ float round_half_away(float x) {
    float t = truncf(x);
    float d = fabsf(x - t);   // exact for |x| < 2^23
    return d >= 0.5f ? t + copysignf(1.0f, x) : t;
}

// Reference per-span INT8 code (model.cpp:395-399) given the F32 value of the
// F16 weight and the span's scale: IEEE division, clip, round half away.
__device__ __forceinline__ int8_t int8_code(float v, float s) {
    float q = __fdiv_rn(v, s);
    q = fminf(fmaxf(q, -127.f), 127.f);
    return (int8_t)(int)round_half_away(q);
}

// ---- small PTX wrappers ---------------------------------------------------------

// 16-byte streaming load that bypasses L1 (weights are read exactly once).
__device__ __forceinline__ uint4 ld_stream16(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

// Programmatic dependent launch controls (sm_90+): a kernel launched with the
// programmatic-serialization attribute may start before its predecessor ends;
// it must wait here before touching anything the predecessor writes.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// Launch with or without programmatic dependent launch (the kernel must call
// pdl_wait before touching what earlier kernels of the stream write).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_maybe_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                                    bool pdl, Args&&... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// 8 F16 (one uint4) -> 8 F32.
__device__ __forceinline__ void h8_to_f8(const uint4& u, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        float2 t = __half22float2(h[i]);
        f[2 * i] = t.x;
        f[2 * i + 1] = t.y;
    }
}

// 4 packed int8 -> 4 F32 exactly: the biased byte b+128 is placed in the low
// mantissa bits of 2^23 and the bias is subtracted (all steps exact).
__device__ __forceinline__ void i8x4_to_f4(uint32_t w, float* f) {
    uint32_t u = w ^ 0x80808080u;
    f[0] = __uint_as_float(0x4B000000u | (u & 0xFFu)) - 8388736.0f;
    f[1] = __uint_as_float(0x4B000000u | ((u >> 8) & 0xFFu)) - 8388736.0f;
    f[2] = __uint_as_float(0x4B000000u | ((u >> 16) & 0xFFu)) - 8388736.0f;
    f[3] = __uint_as_float(0x4B000000u | (u >> 24)) - 8388736.0f;
}

}  // namespace tvb
