// Batched prefill over S tokens (Model::forward_prefill, src/model.cpp:1139-1234)
// on sm_100a: dense projections on the 5th-generation tensor cores (tcgen05.mma
// with TMEM accumulators, operands staged by TMA), the RMSNorms that feed them,
// and causal GQA attention.  Host-side launchers; kernels live in prefill.cu.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace tvb {

// Epilogue of one projection GEMM.  Every mode computes
//   acc[s][n] = sum_k x[s][k] * W[n][k]    (x given as F16 hi + lo planes, x = hi + lo)
// and then, per output row n of W (scaled by the row's INT8 scale, if any):
enum PfMode {
    PF_STORE = 0,   // y[s][n] = acc                         (CUDABackend::matmul, M > 1)
    PF_RESID = 1,   // y[s][n] += acc                        (o_proj / down + residual add)
    PF_QKV = 2,     // q/k/v rows, NeoX RoPE on q and k at position pos0 + s, q -> q_out,
                    // k/v -> the layer's KV cache rows           (model.cpp:1165-1177)
    PF_GATEUP = 3,  // y[s][n] = relu(gate)^2 * up               (model.cpp:1203-1209)
};

// One operand matrix [rows][K] of F16 (INT8 weights are widened to F16 first;
// their scales apply in the epilogue).
struct PfMatrix {
    const uint16_t* w = nullptr;
    int rows = 0;
    const float* row_scales = nullptr;   // per-row scale (INT8 per row), or nullptr
    float scale = 1.0f;                  // per-tensor scale (INT8 per tensor), else 1
    bool widened = false;                // w was written by an earlier kernel of the stream
};

struct PfGemm {
    int mode = PF_STORE;
    int S = 0, K = 0;
    const uint16_t* xh = nullptr;   // [S][K] F16, hi part of the activations
    const uint16_t* xl = nullptr;   // [S][K] F16, lo part (x - hi), or nullptr for F16 x
    const int* row_exp = nullptr;   // [S]: x = (hi + lo) * 2^row_exp[s] (pf_norm_split), or nullptr
    PfMatrix m[3];                  // STORE/RESID: m[0]; GATEUP: gate, up; QKV: q, k, v
    float* y = nullptr;             // STORE/RESID/GATEUP output [S][ldy]
    int ldy = 0;
    // PF_QKV
    int nh = 0, nkv = 0, hd = 128, pos0 = 0;
    float* q_out = nullptr;         // [S][nh * hd]
    float* kcache = nullptr;        // this layer's rows [max_seq][nkv * hd]
    float* vcache = nullptr;
    const float* rope_cos = nullptr;   // [max_seq][hd / 2]
    const float* rope_sin = nullptr;
    // rows that are different sequences (batched decode): row s is at position
    // row_pos[s] and writes its K/V rows kv_slot_stride floats further per row
    const int* row_pos = nullptr;
    size_t kv_slot_stride = 0;
    unsigned* status = nullptr;     // device word; kStatusTimeout on a pipeline stall
    // split-K workspace: with few activation rows the weight tiles alone do not
    // keep the SMs busy, so the K range is cut over CTAs that store raw partial
    // sums here and a second kernel adds them (in split order) and applies the
    // epilogue; nullptr or too small: no split
    float* part = nullptr;
    size_t part_floats = 0;
    // With many output tiles the persistent stream-K kernel runs instead: it
    // needs one flag word per epilogue warp of every CTA (SMs x 4, zeroed once
    // at allocation) besides the workspace (SMs x 128 x 256 floats)
    unsigned* flags = nullptr;
    bool pdl = false;   // programmatic dependent launch after the kernel that writes x
};


tvb_status pf_gemm(const PfGemm& g, cudaStream_t st);

// x[s] = f32(embd[tokens[s]])  (extract_embeddings_batched)
tvb_status pf_embed(const uint16_t* embd, const int* tokens, int S, int H, float* x, cudaStream_t st,
                    bool pdl = false);

// RMSNorm of each row of x [S][K] (tensor.cpp:636-708, x * (inv_rms * w)),
// written as F16 hi + lo planes for the tensor cores with a power-of-two row
// scale: v = (hi + lo) * 2^row_exp, |v / 2^row_exp| < 2^15.  w == nullptr: no
// norm (the plain split, for CUDABackend::matmul).
// ss_out (optional, with w): defer the normalisation -- the rows are scaled by
// w only and each row's sum of squares is written to ss_out[s] (a sub-norm
// whose rows span the tensor-parallel ranks).
tvb_status pf_norm_split(const float* x, const float* w, int S, int K, float eps, uint16_t* xh,
                         uint16_t* xl, int* row_exp, cudaStream_t st, float* ss_out = nullptr,
                         bool pdl = false);

// Causal GQA attention of S query rows at positions pos0 .. pos0 + S - 1 over
// KV rows [0, pos0 + s] (compute_batched_attention, model.cpp:1071-1137).
// q [S][nh * hd], caches [pos][nkv * hd], out [S][nh * hd].
tvb_status pf_attention(const float* q, const float* kcache, const float* vcache, int S, int pos0,
                        int nh, int nkv, int hd, float scale, float* out, cudaStream_t st);

// The same attention on the tensor cores (prefill_attn.cu): q, K and V^T are
// split into F16 hi/lo planes in `planes` (pf_attn_planes_bytes for up to
// max_rows query rows and max_keys KV rows), then a two-pass tcgen05 kernel.
// |q|, |k|, |v| must stay below the F16 range (65504).
bool pf_attention_tc_supported(int nh, int nkv, int hd);
size_t pf_attn_planes_bytes(int max_rows, int max_keys, int nh, int nkv);
tvb_status pf_attention_tc(const float* q, const float* kcache, const float* vcache, int S, int pos0, int nh,
                           int nkv, int hd, float scale, float* out, void* planes, int max_rows, int max_keys,
                           unsigned* status, cudaStream_t st);

// Tiled TMA descriptor of an F16 tensor (128-byte swizzle unless given, zero
// fill outside).
tvb_status encode_f16_tiled(CUtensorMap* m, const void* p, int rank, const uint64_t* dims, const uint64_t* strides,
                            const uint32_t* box, CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B);

// INT8 -> F16 (exact: |q| <= 127).
tvb_status pf_i8_to_f16(const int8_t* q, size_t n, uint16_t* out, cudaStream_t st, bool pdl = false);

}  // namespace tvb
