// Error plumbing for the C ABI: status codes and a per-thread message.
#include <cstdarg>
#include <cstdio>
#include <cuda_runtime.h>

#include "tvb200.h"

namespace tvb {

static thread_local char g_msg[512] = "";

tvb_status set_error(tvb_status s, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(g_msg, sizeof(g_msg), fmt, ap);
    va_end(ap);
    return s;
}

tvb_status cuda_error(cudaError_t e, const char* what) {
    tvb_status s = (e == cudaErrorMemoryAllocation) ? TVB_ERR_OOM : TVB_ERR_CUDA;
    return set_error(s, "%s: %s (%d)", what, cudaGetErrorString(e), (int)e);
}

tvb_status check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_error(e, what);
    return TVB_OK;
}

}  // namespace tvb

extern "C" {

int tvb_version(void) { return 1; }

const char* tvb_status_string(tvb_status s) {
    switch (s) {
        case TVB_OK: return "ok";
        case TVB_ERR_INVALID: return "invalid argument";
        case TVB_ERR_CUDA: return "CUDA error";
        case TVB_ERR_OOM: return "out of memory";
        case TVB_ERR_UNSUPPORTED: return "unsupported";
        case TVB_ERR_TIMEOUT: return "device wait timed out";
        case TVB_ERR_COMM: return "communicator error";
        case TVB_ERR_STATE: return "call out of order";
    }
    return "unknown status";
}

const char* tvb_last_error(void) { return tvb::g_msg; }

tvb_status tvb_free_vram_bytes(size_t* free_bytes) {
    if (!free_bytes) return tvb::set_error(TVB_ERR_INVALID, "free_bytes is NULL");
    size_t f = 0, t = 0;
    cudaError_t e = cudaMemGetInfo(&f, &t);
    if (e != cudaSuccess) return tvb::cuda_error(e, "cudaMemGetInfo");
    *free_bytes = f;
    return TVB_OK;
}

tvb_status tvb_alloc(size_t bytes, void** dptr) {
    if (!dptr) return tvb::set_error(TVB_ERR_INVALID, "dptr is NULL");
    *dptr = nullptr;
    cudaError_t e = cudaMalloc(dptr, bytes ? bytes : 1);
    if (e != cudaSuccess) return tvb::cuda_error(e, "cudaMalloc");
    return TVB_OK;
}

tvb_status tvb_upload(void* dst, const void* src, size_t bytes) {
    if (!bytes) return TVB_OK;
    if (!dst || !src) return tvb::set_error(TVB_ERR_INVALID, "null pointer");
    cudaError_t e = cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return tvb::cuda_error(e, "cudaMemcpy H2D");
    return TVB_OK;
}

tvb_status tvb_download(void* dst, const void* src, size_t bytes) {
    if (!bytes) return TVB_OK;
    if (!dst || !src) return tvb::set_error(TVB_ERR_INVALID, "null pointer");
    cudaError_t e = cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) return tvb::cuda_error(e, "cudaMemcpy D2H");
    return TVB_OK;
}

tvb_status tvb_release(void* dptr) {
    if (!dptr) return TVB_OK;
    cudaError_t e = cudaFree(dptr);
    if (e != cudaSuccess) return tvb::cuda_error(e, "cudaFree");
    return TVB_OK;
}

}  // extern "C"
