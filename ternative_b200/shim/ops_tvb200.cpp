// Drop-in replacement for the reference's cuda/ops_cuda.cu: the
// ternative::CUDABackend class (include/ternative/ops.h:47-168) implemented on
// libtvb200's C ABI.  Compile this file instead of ops_cuda.cu, with
// -DTERNATIVE_USE_CUDA and the reference's include/ on the include path, and
// link libtvb200.so; src/model.cpp and the rest of the host are unchanged.
//
// Behaviour kept from the reference:
//   * every tvb_status other than TVB_OK becomes std::runtime_error, as
//     CUDA_CHECK throws (ops_cuda.cu:30-37);
//   * host-tensor ops (rms_norm, rope, softmax, relu2, add, mul and matmul on
//     weights that are not GPU-resident) stay on the host's CPUBackend, exactly
//     as ops_cuda.cu:628-669 delegates them;
//   * matmul with GPU-resident F16 or INT8 weights stages the host activations
//     through device buffers (ops_cuda.cu:600-631).
// Changed on purpose:
//   * all device work runs on one non-blocking stream owned by the context;
//     upload_pinned / download_pinned / sync_d synchronise that stream;
//   * the device KV cache holds cfg.max_seq_len positions instead of 1024
//     (ops_cuda.cu:376), so forward_gpu no longer drops to the CPU path past
//     1024 tokens.
#include "ternative/model.h"
#include "ternative/ops.h"
#include "tvb200.h"

#include <algorithm>
#include <stdexcept>
#include <string>

namespace ternative {

namespace {

void tvb_check(tvb_status s, const char* what) {
    if (s != TVB_OK)
        throw std::runtime_error(std::string("[tvb200] ") + what + ": " + tvb_status_string(s) +
                                 ": " + tvb_last_error());
}

}  // namespace

class CUDABackend::Impl {
public:
    tvb_context* ctx = nullptr;
    tvb_buffers bufs{};
    int Hk = 0;   // KV row length (n_kv_heads * head_dim)
    float* d_in = nullptr;
    float* d_out = nullptr;
    size_t in_cap = 0, out_cap = 0;

    void* stream() const { return ctx ? tvb_context_stream(ctx) : nullptr; }

    void sync() const {
        if (ctx) tvb_check(tvb_context_sync(ctx), "sync");
    }

    void reserve(float** p, size_t* cap, size_t n) {
        if (n <= *cap) return;
        if (*p) tvb_release(*p);
        *p = nullptr;
        *cap = 0;
        void* q = nullptr;
        tvb_check(tvb_alloc(n * sizeof(float), &q), "alloc staging");
        *p = static_cast<float*>(q);
        *cap = n;
    }

    ~Impl() {
        if (ctx) tvb_context_destroy(ctx);
        if (d_in) tvb_release(d_in);
        if (d_out) tvb_release(d_out);
    }
};

CUDABackend::CUDABackend() : impl_(std::make_unique<Impl>()) {}
CUDABackend::~CUDABackend() = default;

void CUDABackend::matmul(const Tensor& a, const Tensor& b, Tensor& out) {
    const bool gpu_w = b.on_gpu() && a.type == ggml_type::F32 && out.type == ggml_type::F32 &&
                       (b.gpu_is_int8 || b.type == ggml_type::F16);
    if (!gpu_w) {
        cpu_.matmul(a, b, out);
        return;
    }
    const int M = (int)a.shape[0], K = (int)a.shape[1], N = (int)b.shape[1];
    impl_->reserve(&impl_->d_in, &impl_->in_cap, (size_t)M * K);
    impl_->reserve(&impl_->d_out, &impl_->out_cap, (size_t)M * N);
    impl_->sync();
    tvb_check(tvb_upload(impl_->d_in, a.data.data(), (size_t)M * K * sizeof(float)), "matmul upload");
    tvb_weight w{b.gpu_ptr, b.gpu_is_int8 ? TVB_I8_TENSOR : TVB_F16, nullptr, b.scale};
    tvb_check(tvb_matmul(impl_->d_out, impl_->d_in, M, K, &w, N, impl_->stream()), "matmul");
    impl_->sync();
    tvb_check(tvb_download(out.data.data(), impl_->d_out, (size_t)M * N * sizeof(float)),
              "matmul download");
}

void CUDABackend::matmul_batch(const Tensor& a, const std::vector<const Tensor*>& bs,
                               std::vector<Tensor*>& outs) {
    for (size_t i = 0; i < bs.size(); ++i) matmul(a, *bs[i], *outs[i]);
}

void CUDABackend::rms_norm(const Tensor& x, const Tensor& w, float eps, Tensor& out) {
    cpu_.rms_norm(x, w, eps, out);
}
void CUDABackend::rope(Tensor& q, Tensor& k, int pos, float theta) { cpu_.rope(q, k, pos, theta); }
void CUDABackend::softmax(const Tensor& x, Tensor& out) { cpu_.softmax(x, out); }
void CUDABackend::relu2(const Tensor& x, Tensor& out) { cpu_.relu2(x, out); }
void CUDABackend::add(const Tensor& a, const Tensor& b, Tensor& out) { cpu_.add(a, b, out); }
void CUDABackend::mul(const Tensor& a, const Tensor& b, Tensor& out) { cpu_.mul(a, b, out); }

size_t CUDABackend::free_vram_bytes() {
    size_t f = 0;
    return tvb_free_vram_bytes(&f) == TVB_OK ? f : 0;
}

void* CUDABackend::alloc_gpu_mem(size_t bytes) {
    void* p = nullptr;
    tvb_check(tvb_alloc(bytes, &p), "alloc_gpu_mem");
    return p;
}

void CUDABackend::upload(void* dst, const void* src, size_t bytes) {
    impl_->sync();
    tvb_check(tvb_upload(dst, src, bytes), "upload");
}

void CUDABackend::release_gpu_mem(void* ptr) {
    if (ptr) tvb_release(ptr);
}

void CUDABackend::init_gpu_activations(const ModelConfig& cfg) {
    if (impl_->ctx) return;
    tvb_model_config c{};
    c.vocab_size = cfg.vocab_size;
    c.hidden_size = cfg.hidden_size;
    c.num_layers = cfg.num_layers;
    c.num_heads = cfg.num_heads;
    c.num_kv_heads = cfg.num_kv_heads;
    c.head_dim = cfg.head_dim;
    c.intermediate_size = cfg.intermediate_size;
    c.max_seq_len = cfg.max_seq_len;
    c.rope_theta = cfg.rope_theta;
    c.rms_norm_eps = cfg.rms_norm_eps;
    c.max_prefill = 0;
    tvb_check(tvb_context_create(&c, &impl_->ctx), "init_gpu_activations");
    tvb_check(tvb_context_buffers(impl_->ctx, &impl_->bufs), "context buffers");
    impl_->Hk = cfg.num_kv_heads * cfg.head_dim;
}

bool CUDABackend::has_gpu_activations() const { return impl_->ctx != nullptr; }

float* CUDABackend::d_x() { return impl_->bufs.d_x; }
float* CUDABackend::d_norm() { return impl_->bufs.d_norm; }
float* CUDABackend::d_q() { return impl_->bufs.d_q; }
float* CUDABackend::d_k() { return impl_->bufs.d_k; }
float* CUDABackend::d_v() { return impl_->bufs.d_v; }
float* CUDABackend::d_gate() { return impl_->bufs.d_gate; }
float* CUDABackend::d_up() { return impl_->bufs.d_up; }
float* CUDABackend::h_qkv() { return impl_->bufs.h_qkv; }
float* CUDABackend::h_attn() { return impl_->bufs.h_attn; }
float* CUDABackend::h_logit() { return impl_->bufs.h_logit; }

void CUDABackend::add_d(float* o, const float* a, const float* b, int n) {
    tvb_check(tvb_add(o, a, b, n, impl_->stream()), "add_d");
}
void CUDABackend::mul_d(float* o, const float* a, const float* b, int n) {
    tvb_check(tvb_mul(o, a, b, n, impl_->stream()), "mul_d");
}
void CUDABackend::relu2_d(float* o, const float* x, int n) {
    tvb_check(tvb_relu2(o, x, n, impl_->stream()), "relu2_d");
}
void CUDABackend::rms_norm_d(float* o, const float* x, const float* w, float eps, int n) {
    tvb_check(tvb_rms_norm(o, x, w, eps, n, impl_->stream()), "rms_norm_d");
}
void CUDABackend::gemv_d2d(float* o, const float* in, const void* w, int K, int N) {
    tvb_check(tvb_gemv_f16(o, in, w, K, N, impl_->stream()), "gemv_d2d");
}
void CUDABackend::gemv_d2d_int8(float* o, const float* in, const void* w, float scale, int K, int N) {
    tvb_check(tvb_gemv_int8(o, in, w, scale, K, N, impl_->stream()), "gemv_d2d_int8");
}
void CUDABackend::upload_pinned(float* d_dst, const float* h_src, size_t n) {
    impl_->sync();
    tvb_check(tvb_upload(d_dst, h_src, n * sizeof(float)), "upload_pinned");
}
void CUDABackend::download_pinned(float* h_dst, const float* d_src, size_t n) {
    impl_->sync();
    tvb_check(tvb_download(h_dst, d_src, n * sizeof(float)), "download_pinned");
}
void CUDABackend::sync_d() { impl_->sync(); }

void CUDABackend::rope_inplace_d(float* q, float* k, int pos, float theta, int nh, int nkv, int hd) {
    tvb_check(tvb_rope_inplace(q, k, pos, theta, nh, nkv, hd, impl_->stream()), "rope_inplace_d");
}

void CUDABackend::kv_write_d(const float* k, const float* v, int layer, int pos) {
    float *kc = nullptr, *vc = nullptr;
    tvb_check(tvb_kv_layer_ptrs(impl_->ctx, layer, &kc, &vc), "kv_write_d");
    tvb_check(tvb_kv_write(k, v, kc, vc, pos, impl_->Hk, impl_->stream()), "kv_write_d");
}

void CUDABackend::attention_d(const float* q, int layer, int kv_len, float* out, int nh, int nkv,
                              int hd, float scale) {
    float *kc = nullptr, *vc = nullptr;
    tvb_check(tvb_kv_layer_ptrs(impl_->ctx, layer, &kc, &vc), "attention_d");
    tvb_check(tvb_attention_decode(q, kc, vc, kv_len, out, nh, nkv, hd, scale, impl_->stream()),
              "attention_d");
}

void CUDABackend::clear_kv_d() {
    if (impl_->ctx) tvb_check(tvb_kv_clear(impl_->ctx), "clear_kv_d");
}

bool CUDABackend::has_gpu_kv(int min_seq) const {
    return impl_->ctx != nullptr && tvb_kv_capacity(impl_->ctx) >= min_seq;
}

int CUDABackend::gpu_kv_max_seq() const { return impl_->ctx ? tvb_kv_capacity(impl_->ctx) : 0; }

void CUDABackend::upload_kv_layer_d(int layer, int n_positions, const float* h_k, const float* h_v) {
    if (!impl_->ctx || n_positions <= 0) return;
    impl_->sync();
    tvb_check(tvb_kv_upload_layer(impl_->ctx, layer, n_positions, h_k, h_v), "upload_kv_layer_d");
}

void CUDABackend::download_kv_slot_d(int layer, int pos, int n_floats, float* h_dst) {
    if (!impl_->ctx) return;
    impl_->sync();
    tvb_check(tvb_kv_download_slot(impl_->ctx, layer, pos, n_floats, h_dst), "download_kv_slot_d");
}

}  // namespace ternative
