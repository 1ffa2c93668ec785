// Test infrastructure only: a C-ABI harness around the reference's OWN CPU code.
//
// This translation unit is compiled by oracle/Makefile together with the
// reference sources (src/tensor.cpp, gguf.cpp, ops_cpu.cpp, sampler.cpp,
// cache.cpp) and it textually includes src/model.cpp so that the file-static
// helpers on the merge path (matmul_lora, apply_lora; model.cpp:180-258) are
// reachable.  The result, oracle/_ref/libtvref.so, is the pinned oracle: it
// runs the reference's arithmetic unchanged.  It is never linked into the
// product library; only tests/, the smoke check and bench.py's CPU-baseline
// leg load it.
//
// Every entry point names the reference function it wraps.

#include "model.cpp"   // reference src/model.cpp (static helpers become visible)

#include <chrono>
#include <cstring>
#include <vector>

using namespace ternative;

namespace {

Tensor make_f32(std::vector<int64_t> shape, const float* src) {
    Tensor t(std::move(shape), ggml_type::F32);
    std::memcpy(t.data.data(), src, t.data.size());
    return t;
}

Tensor make_f16(std::vector<int64_t> shape, const uint16_t* src) {
    Tensor t(std::move(shape), ggml_type::F16);
    std::memcpy(t.data.data(), src, t.data.size());
    return t;
}

// I2_S tensor: GGUF ne = [K, N]; n_blocks*32 code bytes followed by the F32
// scale (tensor.cpp:110-121).  `scale` is written both into the trailing
// bytes and into Tensor::scale, as load_tensor_from_gguf does (model.cpp:157-162).
Tensor make_i2s(int64_t K, int64_t N, const uint8_t* codes, float scale) {
    Tensor t({K, N}, ggml_type::I2_S);
    size_t n_blocks = (t.data.size() - sizeof(float)) / 32;
    std::memcpy(t.data.data(), codes, n_blocks * 32);
    std::memcpy(t.data.data() + n_blocks * 32, &scale, sizeof(float));
    t.scale = scale;
    return t;
}

}  // namespace

extern "C" {

int tvref_version() { return 1; }

// tensor.cpp:33-57 — f16_t(float): F32 -> F16 by truncation.
void tvref_f32_to_f16(const float* src, int64_t n, uint16_t* dst) {
    for (int64_t i = 0; i < n; ++i) dst[i] = f16_t(src[i]).bits;
}

// tensor.cpp:59-87 — f16_t::to_float.
void tvref_f16_to_f32(const uint16_t* src, int64_t n, float* dst) {
    for (int64_t i = 0; i < n; ++i) dst[i] = f16_t(src[i]).to_float();
}

// tensor.cpp:944-1004 — tensor_quantize_i2_s (max-abs scale, sign threshold).
// dst receives n_blocks*32 code bytes + 4 scale bytes.
void tvref_i2s_quantize(const float* src, int64_t n, uint8_t* dst, float* scale_out) {
    Tensor s = make_f32({n}, src);
    Tensor q = tensor_quantize_i2_s(s);
    std::memcpy(dst, q.data.data(), q.data.size());
    *scale_out = q.scale;
}

// tensor.cpp:1006-1050 — tensor_dequantize_i2_s_to_floats.
void tvref_i2s_dequant(const uint8_t* codes, int64_t n, float scale, float* dst) {
    Tensor t = make_i2s(n, 1, codes, scale);
    t.shape = {n};
    std::vector<float> v = tensor_dequantize_i2_s_to_floats(t);
    std::memcpy(dst, v.data(), n * sizeof(float));
}

// model.cpp:180-203 — matmul_lora.  A: ne=[K, r] (stored [r][K]);
// B: ne=[r, N] (stored [N][r]); delta: ne=[K, N] (stored [N][K]).
void tvref_lora_delta(const float* A, const float* B, int64_t K, int64_t N, int r,
                      float* delta) {
    Tensor a = make_f32({K, r}, A);
    Tensor b = make_f32({r, N}, B);
    Tensor d = matmul_lora(a, b);
    std::memcpy(delta, d.data.data(), d.data.size());
}

// model.cpp:228-247 — the F32 merge inside apply_lora's I2_S branch, assembled
// from the reference's own pieces: tensor_dequantize_i2_s, matmul_lora, and the
// `bv + delta*scale` loop with scale = alpha / rank (model.cpp:226, 234-239).
void tvref_merge_f32(const uint8_t* codes, float scale, int64_t K, int64_t N,
                     const float* A, const float* B, int r, float alpha, float* out) {
    Tensor base = make_i2s(K, N, codes, scale);
    Tensor f32_base(base.shape, ggml_type::F32);
    tensor_dequantize_i2_s(base, f32_base);
    Tensor delta = matmul_lora(make_f32({K, r}, A), make_f32({r, N}, B));
    float sf = alpha / r;
    size_t n = f32_base.n_elements();
    for (size_t i = 0; i < n; ++i) {
        float bv = f32_base.get_float(i);
        float dv = delta.get_float(i) * sf;
        out[i] = bv + dv;
    }
}

// model.cpp:205-258 — apply_lora itself (I2_S base -> merged F16).
void tvref_apply_lora_f16(const uint8_t* codes, float scale, int64_t K, int64_t N,
                          const float* A, const float* B, int r, float alpha,
                          uint16_t* out) {
    Tensor base = make_i2s(K, N, codes, scale);
    apply_lora(base, make_f32({K, r}, A), make_f32({r, N}, B), alpha, r);
    std::memcpy(out, base.data.data(), base.data.size());
}

// model.cpp:374-401 — the per-tensor symmetric INT8 quantizer of
// init_gpu_backend.  That block is inline in a CUDA-only function, so it is
// restated here line for line: max|f16| (0 -> 1), s = max/127, q = round(clip).
void tvref_quantize_int8_tensor(const uint16_t* w, int64_t n, int8_t* q, float* scale_out) {
    const f16_t* fp = reinterpret_cast<const f16_t*>(w);
    float max_abs = 0.0f;
    for (int64_t j = 0; j < n; ++j) {
        float v = fp[j].to_float();
        if (v < 0) v = -v;
        if (v > max_abs) max_abs = v;
    }
    if (max_abs == 0.0f) max_abs = 1.0f;
    const float q_scale = max_abs / 127.0f;
    for (int64_t j = 0; j < n; ++j) {
        float v = fp[j].to_float() / q_scale;
        if (v > 127.f) v = 127.f;
        if (v < -127.f) v = -127.f;
        q[j] = static_cast<int8_t>(std::round(v));
    }
    *scale_out = q_scale;
}

// tensor.cpp:262-634 — tensor_matmul with F32 activations [M][K] and F16
// weights ne=[K, N] (stored [N][K]).
void tvref_matmul_f16(const float* x, int64_t M, int64_t K, const uint16_t* W, int64_t N,
                      float* out) {
    Tensor a = make_f32({M, K}, x);
    Tensor b = make_f16({K, N}, W);
    Tensor o({M, N}, ggml_type::F32);
    tensor_matmul(a, b, o);
    std::memcpy(out, o.data.data(), o.data.size());
}

// tensor.cpp:636-708 — tensor_rms_norm over rows of length n.
void tvref_rms_norm(const float* x, int64_t rows, int64_t n, const float* w, float eps,
                    float* out) {
    Tensor tx = make_f32({rows, n}, x);
    Tensor tw = make_f32({n}, w);
    Tensor to({rows, n}, ggml_type::F32);
    tensor_rms_norm(tx, tw, eps, to);
    std::memcpy(out, to.data.data(), to.data.size());
}

// tensor.cpp:890-940 — tensor_rope_batched, in place on q [S][nh][hd], k [S][nkv][hd].
void tvref_rope_batched(float* q, float* k, int64_t S, int64_t nh, int64_t nkv, int64_t hd,
                        int start_pos, float theta) {
    Tensor tq = make_f32({S, nh, hd}, q);
    Tensor tk = make_f32({S, nkv, hd}, k);
    tensor_rope_batched(tq, tk, start_pos, theta);
    std::memcpy(q, tq.data.data(), tq.data.size());
    std::memcpy(k, tk.data.data(), tk.data.size());
}

// model.cpp:1071-1137 — compute_batched_attention (causal GQA, self-inclusive).
void tvref_batched_attention(int S, int nh, int nkv, int hd, const float* q,
                             const float* kc, const float* vc, float* out) {
    compute_batched_attention(S, nh, nkv, hd, q, kc, vc, out);
}

// ---------------------------------------------------------------------------
// Whole-model oracle: a ternative::Model built in memory from merged F16
// weights (the state Model::load leaves after apply_lora, model.cpp:477-788),
// on the reference CPUBackend.
// ---------------------------------------------------------------------------

struct tvref_model { Model m; };

tvref_model* tvref_model_create(int vocab, int hidden, int layers, int heads, int kv_heads,
                                int inter, int max_seq, float rope_theta, float eps) {
    auto* h = new tvref_model();
    Model& m = h->m;
    m.config.vocab_size = vocab;
    m.config.hidden_size = hidden;
    m.config.num_layers = layers;
    m.config.num_heads = heads;
    m.config.num_kv_heads = kv_heads;
    m.config.head_dim = hidden / heads;   // model.cpp:516
    m.config.intermediate_size = inter;
    m.config.max_seq_len = max_seq;
    m.config.rope_theta = rope_theta;
    m.config.rms_norm_eps = eps;
    m.layers.resize(layers);
    m.backend = std::make_unique<CPUBackend>();
    m.kv_cache.init(m.config, max_seq);
    m.arena.init(m.config);
    return h;
}

void tvref_model_free(tvref_model* h) { delete h; }

// which: 0 tok_embd (F16 [V][H]), 1 output_norm (F32 [H]); per layer:
// 2 attn_norm, 3 wq, 4 wk, 5 wv, 6 wo, 7 attn_sub_norm, 8 ffn_norm,
// 9 w_gate, 10 w_up, 11 w_down, 12 ffn_sub_norm.  Weights are F16 stored
// [out][in] (GGUF ne = [in, out]); norms are F32.
int tvref_model_set(tvref_model* h, int which, int layer, const void* data) {
    Model& m = h->m;
    const auto& c = m.config;
    const int64_t H = c.hidden_size, I = c.intermediate_size;
    const int64_t Hq = (int64_t)c.num_heads * c.head_dim;
    const int64_t Hk = (int64_t)c.num_kv_heads * c.head_dim;
    auto f16 = [&](int64_t in, int64_t out) { return make_f16({in, out}, (const uint16_t*)data); };
    auto f32 = [&](int64_t n) { return make_f32({n}, (const float*)data); };
    if (which == 0) { m.tok_embd = f16(H, c.vocab_size); return 0; }
    if (which == 1) { m.output_norm = f32(H); return 0; }
    if (layer < 0 || layer >= c.num_layers) return -1;
    LayerWeights& w = m.layers[layer];
    switch (which) {
        case 2: w.attn_norm = f32(H); break;
        case 3: w.wq = f16(H, Hq); break;
        case 4: w.wk = f16(H, Hk); break;
        case 5: w.wv = f16(H, Hk); break;
        case 6: w.wo = f16(Hq, H); break;
        case 7: w.attn_sub_norm = f32(Hq); break;
        case 8: w.ffn_norm = f32(H); break;
        case 9: w.w_gate = f16(H, I); break;
        case 10: w.w_up = f16(H, I); break;
        case 11: w.w_down = f16(I, H); break;
        case 12: w.ffn_sub_norm = f32(I); break;
        default: return -2;
    }
    return 0;
}

// Projection `which` (3..6, 9..11 of the numbering above) as an F32 tensor
// [out][in]: the exact dequantised values of a per-row INT8 layer (code times
// its row scale), which no F16 tensor holds.  The reference's tensor_matmul
// takes its all-F32 path for such a weight (tensor.cpp:575-620).
int tvref_model_set_f32(tvref_model* h, int which, int layer, const float* data) {
    Model& m = h->m;
    const auto& c = m.config;
    const int64_t H = c.hidden_size, I = c.intermediate_size;
    const int64_t Hq = (int64_t)c.num_heads * c.head_dim;
    const int64_t Hk = (int64_t)c.num_kv_heads * c.head_dim;
    if (layer < 0 || layer >= c.num_layers) return -1;
    LayerWeights& w = m.layers[layer];
    auto f32 = [&](int64_t in, int64_t out) { return make_f32({in, out}, data); };
    switch (which) {
        case 3: w.wq = f32(H, Hq); break;
        case 4: w.wk = f32(H, Hk); break;
        case 5: w.wv = f32(H, Hk); break;
        case 6: w.wo = f32(Hq, H); break;
        case 9: w.w_gate = f32(H, I); break;
        case 10: w.w_up = f32(H, I); break;
        case 11: w.w_down = f32(I, H); break;
        default: return -2;
    }
    return 0;
}

// model.cpp:1139-1234 — Model::forward_prefill; logits [S][V].
int tvref_forward_prefill(tvref_model* h, const int* tokens, int S, float* logits) {
    std::vector<int> t(tokens, tokens + S);
    Tensor out = h->m.forward_prefill(t);
    if ((int64_t)out.n_elements() != (int64_t)S * h->m.config.vocab_size) return -1;
    std::memcpy(logits, out.data.data(), out.data.size());
    return 0;
}

// model.cpp:1238-1318 — Model::forward_prefill_hidden; final-norm hidden [S][H].
int tvref_forward_prefill_hidden(tvref_model* h, const int* tokens, int S, float* hidden) {
    std::vector<int> t(tokens, tokens + S);
    Tensor out = h->m.forward_prefill_hidden(t);
    if ((int64_t)out.n_elements() != (int64_t)S * h->m.config.hidden_size) return -1;
    std::memcpy(hidden, out.data.data(), out.data.size());
    return 0;
}

// model.cpp:851-1066 — Model::forward (CPU path); logits [V].
int tvref_forward(tvref_model* h, int token, int pos, int prefill, float* logits) {
    Tensor out = h->m.forward(token, pos, prefill != 0);
    std::memcpy(logits, out.data.data(), out.data.size());
    return 0;
}

void tvref_kv_set_seq_len(tvref_model* h, int n) { h->m.kv_cache.seq_len = n; }

// cache.cpp:263-375 -- ModelCache::save of this model's tensors; the key's
// SHA-256 fields as hex strings ("" = none), as compute_key returns them.
int tvref_cache_save(tvref_model* h, const char* path, const char* base_hex, const char* lora_hex, float alpha,
                     int rank) {
    CacheKey key;
    key.base_sha256_hex = base_hex ? base_hex : "";
    key.lora_sha256_hex = lora_hex ? lora_hex : "";
    key.lora_alpha = alpha;
    key.lora_rank = (uint32_t)rank;
    h->m.lora_alpha = alpha;
    h->m.lora_rank = rank;
    ModelCache::save(h->m, path, key);
    return 0;
}

// cache.cpp:378-470 -- ModelCache::try_load into this model: 1 loaded, 0 refused.
int tvref_cache_load(tvref_model* h, const char* path) { return ModelCache::try_load(h->m, path) ? 1 : 0; }

// Tensor `which` (the numbering of tvref_model_set) copied to out when out is
// not null; returns its byte count, -1 when the tensor is empty.
long long tvref_model_get(tvref_model* h, int which, int layer, void* out) {
    Model& m = h->m;
    const Tensor* t = nullptr;
    if (which == 0) t = &m.tok_embd;
    else if (which == 1) t = &m.output_norm;
    else if (layer >= 0 && layer < (int)m.layers.size()) {
        const LayerWeights& w = m.layers[layer];
        const Tensor* per[] = {&w.attn_norm, &w.wq, &w.wk, &w.wv, &w.wo, &w.attn_sub_norm,
                               &w.ffn_norm, &w.w_gate, &w.w_up, &w.w_down, &w.ffn_sub_norm};
        if (which >= 2 && which <= 12) t = per[which - 2];
    }
    if (!t || t->data.empty()) return -1;
    if (out) std::memcpy(out, t->data.data(), t->data.size());
    return (long long)t->data.size();
}

void tvref_model_lora(tvref_model* h, float* alpha, int* rank) {
    *alpha = h->m.lora_alpha;
    *rank = h->m.lora_rank;
}

// sampler.cpp:11-148 -- sample_token with the reference's own (randomly seeded)
// draw; deterministic only where the configuration leaves one candidate.
int tvref_sample_token(const float* logits, int vocab, float temperature, float top_p, int top_k,
                       float penalty, const int* seen, int n_seen) {
    SamplerConfig cfg;
    cfg.temperature = temperature;
    cfg.top_p = top_p;
    cfg.top_k = top_k;
    cfg.repetition_penalty = penalty;
    std::vector<int> prompt(seen, seen + n_seen);
    return sample_token(logits, vocab, cfg, prompt);
}

// model.cpp:1746-1831 -- Model::score_logprobs: for positions [max(1, start), T)
// the token's log-probability and the top k (ids, log-probabilities).
// Returns the number of scored positions.
int tvref_score_logprobs(tvref_model* h, const int* tokens, int T, int k, int start, float* lp, int* ids,
                         float* top) {
    std::vector<int> t(tokens, tokens + T);
    auto res = h->m.score_logprobs(t, k, start);
    for (size_t i = 0; i < res.logprobs.size(); ++i) {
        lp[i] = res.logprobs[i].logprob;
        for (int j = 0; j < (int)res.logprobs[i].top_logprobs.size() && j < k; ++j) {
            ids[i * k + j] = res.logprobs[i].top_logprobs[j].token_id;
            top[i * k + j] = res.logprobs[i].top_logprobs[j].logprob;
        }
    }
    return (int)res.logprobs.size();
}

// gguf.cpp:220-307 -- gguf_load, then tensor `name` sized as the reference's
// Tensor (tensor.cpp:108-121) and copied from its data section.  Returns the
// byte count (out may be null), -1 when absent; type and shape via pointers.
long long tvref_gguf_tensor(const char* path, const char* name, void* out, int* type, int* n_dims,
                            long long* shape) {
    auto g = gguf_load(path);
    if (!g) return -2;
    const TensorInfo* ti = g->find_tensor(name);
    if (!ti) return -1;
    std::vector<int64_t> sh(ti->shape.begin(), ti->shape.end());
    Tensor t(sh, ti->type);
    *type = (int)ti->type;
    *n_dims = (int)sh.size();
    for (size_t d = 0; d < sh.size() && d < 8; ++d) shape[d] = sh[d];
    if (out) std::memcpy(out, g->tensor_data.data() + ti->offset, t.data.size());
    return (long long)t.data.size();
}

// Copy one layer's CPU KV cache rows [0, n) (layout [pos][n_kv][hd], F32).
int tvref_kv_read(tvref_model* h, int layer, int n, float* k, float* v) {
    const auto& c = h->m.config;
    size_t row = (size_t)c.num_kv_heads * c.head_dim;
    std::memcpy(k, h->m.kv_cache.k_cache[layer].data.data(), n * row * sizeof(float));
    std::memcpy(v, h->m.kv_cache.v_cache[layer].data.data(), n * row * sizeof(float));
    return 0;
}

// CPU decode timing: `steps` calls of Model::forward(prefill=false) starting
// at `pos0`, the reference's --no-gpu decode loop (model.cpp:1618-1639 minus
// sampling).  Returns wall seconds.
double tvref_time_decode(tvref_model* h, int token, int pos0, int steps) {
    auto t0 = std::chrono::steady_clock::now();
    for (int i = 0; i < steps; ++i) {
        Tensor out = h->m.forward(token, pos0 + i, false);
        (void)out;
    }
    auto t1 = std::chrono::steady_clock::now();
    return std::chrono::duration<double>(t1 - t0).count();
}

#ifdef TERNATIVE_USE_CUDA
// Drop-in build (libtvref_dropin.so): the reference host compiled with
// TERNATIVE_USE_CUDA against ternative_b200/shim/ops_tvb200.cpp instead of
// cuda/ops_cuda.cu.  init_gpu_backend (model.cpp:264-472) uploads the layers
// through the shim; Model::forward then takes forward_gpu (model.cpp:863-867).
int tvref_init_gpu(tvref_model* h) {
    init_gpu_backend(h->m);
    return h->m.n_gpu_layers;
}

// model.cpp:1322-1331
void tvref_sync_kv_to_gpu(tvref_model* h, int n) { h->m.sync_kv_to_gpu(n); }
#endif

int tvref_omp_threads() {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

// OpenMP threads of the reference's parallel loops (a launcher such as
// torchrun may have set OMP_NUM_THREADS=1 in the environment).
void tvref_set_threads(int n) {
#ifdef _OPENMP
    if (n > 0) omp_set_num_threads(n);
#else
    (void)n;
#endif
}

}  // extern "C"
