/* Test infrastructure only: plain-C restatement of the reference's CPU
 * arithmetic on the quantized-weight path.  Used by tests/, the smoke check
 * and bench.py's CPU-baseline leg as the checker; never by the product.
 * Each function cites the reference file:line it restates. */
#ifndef TVORACLE_H
#define TVORACLE_H
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

uint16_t tvo_f32_to_f16(float f);                 /* tensor.cpp:33-57  */
float    tvo_f16_to_f32(uint16_t h);              /* tensor.cpp:59-87  */
void     tvo_f32_to_f16_n(const float* src, int64_t n, uint16_t* dst);
void     tvo_f16_to_f32_n(const uint16_t* src, int64_t n, float* dst);

/* tensor.cpp:1006-1050; codes = n_blocks*32 bytes (scale passed separately). */
void tvo_i2s_unpack(const uint8_t* codes, int64_t n, float scale, float* out);
/* tensor.cpp:944-1004 packing of already-ternary codes {0,1,2} (one per byte). */
void tvo_i2s_pack(const uint8_t* code_per_elem, int64_t n, uint8_t* packed);

/* model.cpp:180-247: merged F32 of one I2_S tensor, W[N][K] (GGUF ne=[K,N]),
 * A stored [r][K], B stored [N][r], scale factor alpha/r. Any output may be NULL. */
void tvo_merge(const uint8_t* codes, float scale, int64_t K, int64_t N,
               const float* A, const float* B, int r, float alpha,
               float* out_f32, uint16_t* out_f16);

/* model.cpp:374-401 per-tensor INT8, and the same formula applied per row. */
void tvo_quantize_int8_tensor(const uint16_t* w, int64_t n, int8_t* q, float* scale);
void tvo_quantize_int8_rows(const uint16_t* w, int64_t N, int64_t K, int8_t* q, float* scales);

/* ops_cuda.cu:46-103 semantics, accumulated in double: y[n] = sum_k W[n][k] x[k]. */
void tvo_gemv_f16(const float* x, const uint16_t* W, int64_t K, int64_t N, float* y);
void tvo_gemv_int8(const float* x, const int8_t* W, const float* row_scales, float tensor_scale,
                   int64_t K, int64_t N, float* y);

/* tensor.cpp:636-708 (one row). */
void tvo_rms_norm(const float* x, int64_t n, const float* w, float eps, float* out);

/* tensor.cpp:830-888 NeoX RoPE for one position: q [nh][hd], k [nkv][hd]. */
void tvo_rope(float* q, float* k, int nh, int nkv, int hd, int pos, float theta);
/* cos/sin table [n_pos][hd/2] with the CPU formulas of tensor.cpp:830-838. */
void tvo_rope_table(int n_pos, int hd, float theta, float* cos_t, float* sin_t);

/* model.cpp:1071-1137 / ops_cuda.cu:205-259: one query row against kv_len cached
 * rows (layout [t][nkv][hd]), self-inclusive when kv_len = pos + 1. */
void tvo_attention_decode(const float* q, const float* kc, const float* vc, int kv_len,
                          int nh, int nkv, int hd, float* out);

#ifdef __cplusplus
}
#endif
#endif
