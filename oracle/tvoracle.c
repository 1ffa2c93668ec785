/* Test infrastructure only (see tvoracle.h): the checker for the CUDA path.
 * Compiled with -ffp-contract=off so every `a*b + c` below is two roundings,
 * as in the reference's stock x86-64 build. */
#include "tvoracle.h"

#include <math.h>
#include <string.h>
#include <stdlib.h>

/* tensor.cpp:33-57: truncating F32 -> F16 (round toward zero, subnormals
 * truncated, overflow -> inf, NaN payload shifted). */
uint16_t tvo_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = x >> 31, e = (x >> 23) & 0xFFu, m = x & 0x7FFFFFu;
    if (e == 0xFFu) return (uint16_t)((sign << 15) | 0x7C00u | (m >> 13));
    int32_t ne = (int32_t)e - 112;
    if (ne >= 31) return (uint16_t)((sign << 15) | 0x7C00u);
    if (ne <= 0) {
        if (ne < -10) return (uint16_t)(sign << 15);
        m = (m | 0x800000u) >> (1 - ne);
        return (uint16_t)((sign << 15) | (m >> 13));
    }
    return (uint16_t)((sign << 15) | ((uint32_t)ne << 10) | (m >> 13));
}

/* tensor.cpp:59-87: exact F16 -> F32. */
float tvo_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h >> 15), e = (h >> 10) & 0x1Fu, m = h & 0x3FFu, r;
    if (e == 0x1Fu) {
        r = (sign << 31) | 0x7F800000u | (m << 13);
    } else if (e == 0) {
        if (m == 0) {
            r = sign << 31;
        } else {
            int ex = -14;
            while (!(m & 0x400u)) { m <<= 1; ex--; }
            r = (sign << 31) | ((uint32_t)(ex + 127) << 23) | ((m & 0x3FFu) << 13);
        }
    } else {
        r = (sign << 31) | ((e + 112u) << 23) | (m << 13);
    }
    float f;
    memcpy(&f, &r, 4);
    return f;
}

void tvo_f32_to_f16_n(const float* src, int64_t n, uint16_t* dst) {
    for (int64_t i = 0; i < n; ++i) dst[i] = tvo_f32_to_f16(src[i]);
}

void tvo_f16_to_f32_n(const uint16_t* src, int64_t n, float* dst) {
    for (int64_t i = 0; i < n; ++i) dst[i] = tvo_f16_to_f32(src[i]);
}

/* tensor.cpp:1006-1050: 128-element blocks of 32 bytes; byte gp of a block
 * holds elements gp, gp+32, gp+64, gp+96 in bits [7:6],[5:4],[3:2],[1:0];
 * codes 0,1,2,3 -> -1,0,+1,0; value = scale * map[code]. */
static const float k_map2bit[4] = {-1.0f, 0.0f, 1.0f, 0.0f};

void tvo_i2s_unpack(const uint8_t* codes, int64_t n, float scale, float* out) {
    for (int64_t i = 0; i < n; ++i) {
        int64_t blk = i / 128, o = i % 128;
        uint8_t b = codes[blk * 32 + (o % 32)];
        int sh = 6 - 2 * (int)(o / 32);
        out[i] = scale * k_map2bit[(b >> sh) & 3];
    }
}

/* tensor.cpp:984-1000 bit placement, for already-ternary codes. */
void tvo_i2s_pack(const uint8_t* q8, int64_t n, uint8_t* packed) {
    int64_t nb = (n + 127) / 128;
    memset(packed, 0, (size_t)nb * 32);
    for (int64_t i = 0; i < n; ++i) {
        int64_t blk = i / 128, o = i % 128;
        packed[blk * 32 + (o % 32)] |= (uint8_t)((q8[i] & 3) << (6 - 2 * (o / 32)));
    }
}

/* model.cpp:192-201 (delta, sequential k, unfused), :226 (alpha/rank),
 * :234-239 (bv + dv), :242-246 (F16 by truncation). */
void tvo_merge(const uint8_t* codes, float scale, int64_t K, int64_t N,
               const float* A, const float* B, int r, float alpha,
               float* out_f32, uint16_t* out_f16) {
    const float sf = alpha / (float)r;
    float* row = (float*)malloc((size_t)K * sizeof(float));
    for (int64_t n = 0; n < N; ++n) {
        tvo_i2s_unpack(codes + (n * K / 128) * 32, K, scale, row);
        for (int64_t m = 0; m < K; ++m) {
            float sum = 0.0f;
            for (int k = 0; k < r; ++k) sum += A[(int64_t)k * K + m] * B[n * r + k];
            float dv = sum * sf;
            float v = row[m] + dv;
            if (out_f32) out_f32[n * K + m] = v;
            if (out_f16) out_f16[n * K + m] = tvo_f32_to_f16(v);
        }
    }
    free(row);
}

/* model.cpp:381-401, applied to n values. */
static void quant_span(const uint16_t* w, int64_t n, int8_t* q, float* scale) {
    float max_abs = 0.0f;
    for (int64_t j = 0; j < n; ++j) {
        float v = tvo_f16_to_f32(w[j]);
        if (v < 0) v = -v;
        if (v > max_abs) max_abs = v;
    }
    if (max_abs == 0.0f) max_abs = 1.0f;
    const float s = max_abs / 127.0f;
    for (int64_t j = 0; j < n; ++j) {
        float v = tvo_f16_to_f32(w[j]) / s;
        if (v > 127.f) v = 127.f;
        if (v < -127.f) v = -127.f;
        q[j] = (int8_t)roundf(v);   /* std::round: half away from zero */
    }
    *scale = s;
}

void tvo_quantize_int8_tensor(const uint16_t* w, int64_t n, int8_t* q, float* scale) {
    quant_span(w, n, q, scale);
}

void tvo_quantize_int8_rows(const uint16_t* w, int64_t N, int64_t K, int8_t* q, float* scales) {
    for (int64_t n = 0; n < N; ++n) quant_span(w + n * K, K, q + n * K, scales + n);
}

void tvo_gemv_f16(const float* x, const uint16_t* W, int64_t K, int64_t N, float* y) {
    for (int64_t n = 0; n < N; ++n) {
        double s = 0.0;
        for (int64_t k = 0; k < K; ++k) s += (double)tvo_f16_to_f32(W[n * K + k]) * (double)x[k];
        y[n] = (float)s;
    }
}

void tvo_gemv_int8(const float* x, const int8_t* W, const float* row_scales, float tensor_scale,
                   int64_t K, int64_t N, float* y) {
    for (int64_t n = 0; n < N; ++n) {
        double s = 0.0;
        for (int64_t k = 0; k < K; ++k) s += (double)W[n * K + k] * (double)x[k];
        float sc = row_scales ? row_scales[n] : tensor_scale;
        y[n] = (float)s * sc;
    }
}

/* tensor.cpp:655-685 scalar path: ss, rms = sqrt(ss/n + eps), inv = 1/rms. */
void tvo_rms_norm(const float* x, int64_t n, const float* w, float eps, float* out) {
    float ss = 0.0f;
    for (int64_t i = 0; i < n; ++i) ss += x[i] * x[i];
    float rms = sqrtf(ss / (float)n + eps);
    float inv = 1.0f / rms;
    for (int64_t i = 0; i < n; ++i) out[i] = x[i] * inv * w[i];
}

/* tensor.cpp:830-838: freq = 1/pow(theta, i/hd) with i the even index. */
void tvo_rope_table(int n_pos, int hd, float theta, float* cos_t, float* sin_t) {
    int half = hd / 2;
    for (int p = 0; p < n_pos; ++p) {
        for (int ic = 0; ic < half; ++ic) {
            float freq = 1.0f / powf(theta, (float)(2 * ic) / (float)hd);
            cos_t[p * half + ic] = cosf((float)p * freq);
            sin_t[p * half + ic] = sinf((float)p * freq);
        }
    }
}

/* tensor.cpp:840-888 NeoX pairs (ic, ic + hd/2). */
void tvo_rope(float* q, float* k, int nh, int nkv, int hd, int pos, float theta) {
    int half = hd / 2;
    for (int h = 0; h < nh + nkv; ++h) {
        float* v = h < nh ? q + h * hd : k + (h - nh) * hd;
        for (int ic = 0; ic < half; ++ic) {
            float freq = 1.0f / powf(theta, (float)(2 * ic) / (float)hd);
            float c = cosf((float)pos * freq), s = sinf((float)pos * freq);
            float x0 = v[ic], x1 = v[ic + half];
            v[ic] = x0 * c - x1 * s;
            v[ic + half] = x0 * s + x1 * c;
        }
    }
}

/* model.cpp:1071-1137: scores * 1/sqrt(hd), max-subtracted softmax, P.V. */
void tvo_attention_decode(const float* q, const float* kc, const float* vc, int kv_len,
                          int nh, int nkv, int hd, float* out) {
    float scale = 1.0f / sqrtf((float)hd);
    int group = nh / nkv;
    double* sc = (double*)malloc((size_t)(kv_len > 0 ? kv_len : 1) * sizeof(double));
    for (int h = 0; h < nh; ++h) {
        int kvh = h / group;
        double mx = -1e300;
        for (int t = 0; t < kv_len; ++t) {
            double d = 0.0;
            const float* kr = kc + ((int64_t)t * nkv + kvh) * hd;
            for (int i = 0; i < hd; ++i) d += (double)q[h * hd + i] * kr[i];
            sc[t] = d * scale;
            if (sc[t] > mx) mx = sc[t];
        }
        double sum = 0.0;
        for (int t = 0; t < kv_len; ++t) { sc[t] = exp(sc[t] - mx); sum += sc[t]; }
        for (int i = 0; i < hd; ++i) {
            double acc = 0.0;
            for (int t = 0; t < kv_len; ++t) acc += sc[t] * vc[((int64_t)t * nkv + kvh) * hd + i];
            out[h * hd + i] = (float)(acc / sum);
        }
    }
    free(sc);
}
