/* reef_oracle.c -- CPU restatement of reef's W8A8 / int8 arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY (see reef_oracle.h): the checker for the sm_100a
 * kernels, never the thing measured or shipped.
 *
 * Citations are to files under inference-engine/reference/cpp/include/
 * inference_engine/ of LonghornSilicon/reef unless stated otherwise.
 * Build with -ffp-contract=off: each float step below is one IEEE operation.
 */
#include "reef_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

/* ------------------------------------------------------------------------ */
/* Seeded inputs                                                             */
/* ------------------------------------------------------------------------ */

uint32_t ro_lcg_next(uint32_t* state) {
    /* weights.hpp:237-247, gen_golden.cpp:80-83 */
    *state = (*state * 1664525u) + 1013904223u;
    return *state;
}

void ro_fill_uniform(uint32_t seed, size_t n, float low, float high,
                     float* out) {
    /* gen_golden.cpp:52-56 */
    const float unit = 1.0f / 16777216.0f;
    uint32_t s = seed;
    for (size_t i = 0; i < n; ++i) {
        const float fraction = (float)(ro_lcg_next(&s) >> 8u) * unit;
        out[i] = low + ((high - low) * fraction);
    }
}

void ro_fill_int8(uint32_t seed, size_t n, int32_t low, int32_t high,
                  int8_t* out) {
    /* gen_golden.cpp:59-68 */
    const uint32_t span = (uint32_t)(high - low) + 1u;
    uint32_t s = seed;
    for (size_t i = 0; i < n; ++i) {
        out[i] = (int8_t)(low + (int32_t)((ro_lcg_next(&s) >> 8u) % span));
    }
}

void ro_fill_int32(uint32_t seed, size_t n, int32_t low, int32_t high,
                   int32_t* out) {
    const uint32_t span = (uint32_t)(high - low) + 1u;
    uint32_t s = seed;
    for (size_t i = 0; i < n; ++i) {
        out[i] = low + (int32_t)((ro_lcg_next(&s) >> 8u) % span);
    }
}

void ro_fill_normal(uint32_t seed, size_t n, float mean, float std_dev,
                    float* out) {
    const double unit = 1.0 / 16777216.0;
    const double two_pi = 6.283185307179586476925286766559;
    uint32_t s = seed;
    for (size_t i = 0; i < n; i += 2) {
        const double u1 = ((double)(ro_lcg_next(&s) >> 8u) + 1.0) * unit;
        const double u2 = (double)(ro_lcg_next(&s) >> 8u) * unit;
        const double r = sqrt(-2.0 * log(u1));
        out[i] = (float)((double)mean + (double)std_dev * r * cos(two_pi * u2));
        if (i + 1 < n) {
            out[i + 1] =
                (float)((double)mean + (double)std_dev * r * sin(two_pi * u2));
        }
    }
}

/* ------------------------------------------------------------------------ */
/* Quantization, quant.hpp                                                   */
/* ------------------------------------------------------------------------ */

float ro_int8_scale(float max_magnitude) {
    /* quant.hpp:51-57 */
    return max_magnitude > 0.0f ? max_magnitude / 127.0f : 1.0f;
}

int8_t ro_quantize_int8(float value, float scale, int* bad) {
    /* quant.hpp:68-81 */
    if (!isfinite(value) || !isfinite(scale)) {
        if (bad) *bad = 1;
        return 0;
    }
    float rounded = nearbyintf(value / scale); /* ties to even */
    if (rounded < -127.0f) rounded = -127.0f;
    if (rounded > 127.0f) rounded = 127.0f;
    return (int8_t)rounded;
}

int ro_quantize_rows(size_t rows, size_t cols, const float* x, int8_t* q,
                     size_t ldq, float* scales) {
    /* quant.hpp:90-98 (row_max_magnitude), :112-133 (quantize_rows) */
    int bad = 0;
    for (size_t r = 0; r < rows; ++r) {
        const float* xr = x + r * cols;
        float largest = 0.0f;
        for (size_t c = 0; c < cols; ++c) {
            const float m = fabsf(xr[c]);
            /* std::max(largest, m): keeps largest unless largest < m */
            if (largest < m) largest = m;
        }
        const float scale = ro_int8_scale(largest);
        scales[r] = scale;
        for (size_t c = 0; c < cols; ++c) {
            q[r * ldq + c] = ro_quantize_int8(xr[c], scale, &bad);
        }
    }
    return bad ? -1 : 0;
}

/* ------------------------------------------------------------------------ */
/* Exact int8 x int8 -> int32 GEMM (tensor.hpp:178-246)                      */
/* ------------------------------------------------------------------------ */

typedef struct {
    size_t m0, m1, n, k;
    const int8_t* a;
    size_t lda;
    const int8_t* b;
    size_t ldb;
    int32_t* c;
    size_t ldc;
} gemm_job;

static void* gemm_worker(void* arg) {
    const gemm_job* j = (const gemm_job*)arg;
    const size_t nb = 64; /* a block of B rows stays in cache */
    for (size_t n0 = 0; n0 < j->n; n0 += nb) {
        const size_t n1 = n0 + nb < j->n ? n0 + nb : j->n;
        for (size_t m = j->m0; m < j->m1; ++m) {
            const int8_t* ar = j->a + m * j->lda;
            for (size_t n = n0; n < n1; ++n) {
                const int8_t* br = j->b + n * j->ldb;
                int32_t s = 0;
                for (size_t kk = 0; kk < j->k; ++kk) {
                    s += (int32_t)ar[kk] * (int32_t)br[kk];
                }
                j->c[m * j->ldc + n] = s;
            }
        }
    }
    return NULL;
}

static int host_threads(int threads) {
    if (threads > 0) return threads;
    long n = sysconf(_SC_NPROCESSORS_ONLN);
    return n > 0 ? (int)n : 1;
}

void ro_gemm_i8_i32(size_t m, size_t n, size_t k, const int8_t* a,
                    size_t lda, const int8_t* b, size_t ldb, int32_t* c,
                    size_t ldc, int threads) {
    int t = host_threads(threads);
    if ((size_t)t > m) t = (int)(m ? m : 1);
    if (t > 256) t = 256;
    gemm_job jobs[256];
    pthread_t tids[256];
    const size_t per = (m + (size_t)t - 1) / (size_t)t;
    int launched = 0;
    for (int i = 0; i < t; ++i) {
        const size_t m0 = (size_t)i * per;
        if (m0 >= m) break;
        const size_t m1 = m0 + per < m ? m0 + per : m;
        jobs[i] = (gemm_job){m0, m1, n, k, a, lda, b, ldb, c, ldc};
        if (t == 1) {
            gemm_worker(&jobs[i]);
        } else {
            pthread_create(&tids[i], NULL, gemm_worker, &jobs[i]);
            ++launched;
        }
    }
    for (int i = 0; i < launched; ++i) pthread_join(tids[i], NULL);
}

/* ------------------------------------------------------------------------ */
/* Linear layers                                                             */
/* ------------------------------------------------------------------------ */

void ro_w8a8_epilogue(size_t rows, size_t out, const int32_t* acc,
                      const float* x_scale, const float* w_scale,
                      const float* bias, float* y) {
    /* linear.hpp:122-130: safe_multiply(float(sum),
     *   safe_multiply(row_scale, w_scale[c])), then add_bias (:44-49). */
    for (size_t r = 0; r < rows; ++r) {
        for (size_t c = 0; c < out; ++c) {
            const float combined = x_scale[r] * w_scale[c];
            float v = (float)acc[r * out + c] * combined;
            if (bias) v = v + bias[c];
            y[r * out + c] = v;
        }
    }
}

int ro_linear_w8a8(size_t rows, size_t in, size_t out, const float* x,
                   const int8_t* w, size_t ldw, const float* w_scale,
                   const float* bias, float* y, int threads) {
    /* linear.hpp:106-134 */
    int8_t* xq = (int8_t*)malloc(rows * in ? rows * in : 1);
    float* xs = (float*)malloc((rows ? rows : 1) * sizeof(float));
    int32_t* acc = (int32_t*)malloc((rows * out ? rows * out : 1) *
                                    sizeof(int32_t));
    int rc = ro_quantize_rows(rows, in, x, xq, in, xs);
    if (rc == 0) {
        ro_gemm_i8_i32(rows, out, in, xq, in, w, ldw, acc, out, threads);
        ro_w8a8_epilogue(rows, out, acc, xs, w_scale, bias, y);
    }
    free(xq);
    free(xs);
    free(acc);
    return rc;
}

int32_t ro_rounding_shift(int32_t value, unsigned shift) {
    /* int8.hpp:43-49: floor(value / 2^shift + 1/2) */
    if (shift == 0) return value;
    return (value >> shift) + ((value >> (shift - 1)) & 1);
}

int8_t ro_saturate_int8(int32_t value) {
    /* int8.hpp:56-60 */
    if (value < -128) return -128;
    if (value > 127) return 127;
    return (int8_t)value;
}

void ro_linear_int8(size_t rows, size_t in, size_t out, const int8_t* x,
                    size_t ldx, const int8_t* w, size_t ldw, unsigned shift,
                    const int32_t* bias, int8_t* y, int threads) {
    /* int8.hpp:74-101 */
    int32_t* acc = (int32_t*)malloc((rows * out ? rows * out : 1) *
                                    sizeof(int32_t));
    ro_gemm_i8_i32(rows, out, in, x, ldx, w, ldw, acc, out, threads);
    for (size_t r = 0; r < rows; ++r) {
        for (size_t c = 0; c < out; ++c) {
            int32_t s = acc[r * out + c];
            if (bias) s += bias[c];
            y[r * out + c] = ro_saturate_int8(ro_rounding_shift(s, shift));
        }
    }
    free(acc);
}

/* ------------------------------------------------------------------------ */
/* Reproducible math, math.hpp                                               */
/* ------------------------------------------------------------------------ */

float ro_exp_nonpositive(float x) {
    /* math.hpp:34-71: x = k ln2 + r, Cephes expf polynomial in r, then
     * scale by 2^k built from the exponent field.  Every step is a single
     * IEEE operation in the order the engine writes them. */
    if (x < -87.0f) return 0.0f;
    const float log2e = 1.44269504088896341f;
    const float round_to_int = 12582912.0f; /* 1.5 * 2^23 */
    const float ln2_hi = 0.693359375f;
    const float ln2_lo = -2.12194440e-4f;
    const float kf = ((x * log2e) + round_to_int) - round_to_int;
    const float r = (x - (kf * ln2_hi)) - (kf * ln2_lo);
    const float r2 = r * r;
    float p = 1.9875691500E-4f;
    p = (p * r) + 1.3981999507E-3f;
    p = (p * r) + 8.3334519073E-3f;
    p = (p * r) + 4.1665795894E-2f;
    p = (p * r) + 1.6666665459E-1f;
    p = (p * r) + 5.0000001201E-1f;
    p = ((p * r2) + r) + 1.0f;
    const uint32_t bits = (uint32_t)((int32_t)kf + 127) << 23u;
    float scale;
    memcpy(&scale, &bits, sizeof scale);
    return p * scale;
}

float ro_tanh_float(float x) {
    /* math.hpp:77-81 */
    const float e = ro_exp_nonpositive(-2.0f * fabsf(x));
    const float magnitude = (1.0f - e) / (1.0f + e);
    return copysignf(magnitude, x);
}

/* ------------------------------------------------------------------------ */
/* Integer softmax and attention, int8.hpp                                   */
/* ------------------------------------------------------------------------ */

void ro_exp_table(float step, uint16_t table[256]) {
    /* int8.hpp:156-164 */
    for (int d = 0; d < 256; ++d) {
        table[d] = (uint16_t)lroundf(
            32768.0f * ro_exp_nonpositive(-(float)d * step));
    }
}

void ro_softmax_int8_row(size_t n, const int32_t* scores, unsigned shift,
                         const uint16_t* table, uint8_t* probs) {
    /* int8.hpp:198-231 with every key of the row visible */
    int32_t largest = scores[0];
    for (size_t k = 1; k < n; ++k) {
        if (largest < scores[k]) largest = scores[k];
    }
    uint32_t sum = 0;
    for (size_t k = 0; k < n; ++k) {
        uint32_t d = (uint32_t)((largest - scores[k]) >> (int32_t)shift);
        sum += table[d < 255u ? d : 255u];
    }
    const uint32_t reciprocal = (255u << 16u) / sum;
    for (size_t k = 0; k < n; ++k) {
        uint32_t d = (uint32_t)((largest - scores[k]) >> (int32_t)shift);
        const uint32_t scaled = (uint32_t)table[d < 255u ? d : 255u] *
                                reciprocal;
        uint32_t rounded = (scaled >> 16u) + ((scaled >> 15u) & 1u);
        probs[k] = (uint8_t)(rounded < 255u ? rounded : 255u);
    }
}

int ro_visible_range(size_t query_start, size_t i, size_t key_len,
                     size_t window, size_t* first, size_t* end) {
    /* causal_visibility, attention.hpp:82-100 */
    const size_t position = query_start + i;
    const size_t e = position + 1 < key_len ? position + 1 : key_len;
    const size_t f =
        (window > 0 && position + 1 > window) ? position + 1 - window : 0;
    *first = f;
    *end = e;
    return f < e;
}

int ro_attention_head_int8(size_t query_len, size_t key_len, size_t head_dim,
                           size_t query_start, size_t window, const int8_t* q,
                           size_t q_stride, const int8_t* k, const int8_t* v,
                           unsigned score_shift, const uint16_t* table,
                           unsigned out_shift, int8_t* out,
                           size_t out_stride) {
    /* int8.hpp:250-279 */
    int32_t* scores = (int32_t*)malloc((key_len ? key_len : 1) * 4);
    uint8_t* probs = (uint8_t*)malloc(key_len ? key_len : 1);
    int rc = 0;
    for (size_t i = 0; i < query_len; ++i) {
        size_t first, end;
        if (!ro_visible_range(query_start, i, key_len, window, &first, &end)) {
            rc = -1;
            break;
        }
        const int8_t* qi = q + i * q_stride;
        for (size_t j = first; j < end; ++j) {
            int32_t s = 0;
            for (size_t d = 0; d < head_dim; ++d) {
                s += (int32_t)qi[d] * (int32_t)k[j * head_dim + d];
            }
            scores[j] = s;
        }
        ro_softmax_int8_row(end - first, scores + first, score_shift, table,
                            probs + first);
        for (size_t c = 0; c < head_dim; ++c) {
            int32_t s = 0;
            for (size_t j = first; j < end; ++j) {
                s += (int32_t)probs[j] * (int32_t)v[j * head_dim + c];
            }
            out[i * out_stride + c] =
                ro_saturate_int8(ro_rounding_shift(s, out_shift));
        }
    }
    free(scores);
    free(probs);
    return rc;
}

/* ------------------------------------------------------------------------ */
/* Float operators                                                           */
/* ------------------------------------------------------------------------ */

int ro_attention_head_f32(size_t query_len, size_t key_len, size_t head_dim,
                          size_t query_start, size_t window, const float* q,
                          size_t q_stride, const float* k, const float* v,
                          size_t kv_stride, float* out, size_t out_stride) {
    /* attention.hpp:117-123: scores = matmul(q, k^T) (tensor.hpp:178-192,
     * sums from 0 in order), masked_softmax (activation.hpp:188-229), then
     * matmul(probs, v).  Masked keys have probability exactly 0, and adding
     * a zero product never changes a sum that started at +0, so visiting
     * only the visible keys in order reproduces the engine's bits. */
    float* p = (float*)malloc((key_len ? key_len : 1) * sizeof(float));
    int rc = 0;
    for (size_t i = 0; i < query_len; ++i) {
        size_t first, end;
        if (!ro_visible_range(query_start, i, key_len, window, &first, &end)) {
            rc = -1;
            break;
        }
        const float* qi = q + i * q_stride;
        for (size_t j = first; j < end; ++j) {
            float s = 0.0f;
            for (size_t d = 0; d < head_dim; ++d) {
                s = s + qi[d] * k[j * kv_stride + d];
            }
            p[j] = s;
        }
        float m = p[first];
        for (size_t j = first + 1; j < end; ++j) {
            m = (m < p[j]) ? p[j] : m; /* std::max */
        }
        float sum = 0.0f;
        for (size_t j = first; j < end; ++j) {
            p[j] = ro_exp_nonpositive(p[j] - m);
            sum = sum + p[j];
        }
        for (size_t j = first; j < end; ++j) p[j] = p[j] / sum;
        for (size_t c = 0; c < head_dim; ++c) {
            float s = 0.0f;
            for (size_t j = first; j < end; ++j) {
                s = s + p[j] * v[j * kv_stride + c];
            }
            out[i * out_stride + c] = s;
        }
    }
    free(p);
    return rc;
}

void ro_layernorm_f32(size_t rows, size_t width, const float* x,
                      const float* gain, const float* shift, float eps,
                      float* y) {
    /* layernorm.hpp:62-80 */
    for (size_t r = 0; r < rows; ++r) {
        const float* xr = x + r * width;
        float mean = 0.0f;
        for (size_t k = 0; k < width; ++k) mean = mean + xr[k];
        mean = mean / (float)width;
        float var = 0.0f;
        for (size_t k = 0; k < width; ++k) {
            const float c = xr[k] - mean;
            var = var + c * c;
        }
        var = var / (float)width;
        const float inv_std = 1.0f / sqrtf(var + eps);
        for (size_t k = 0; k < width; ++k) {
            float v = ((xr[k] - mean) * inv_std) * gain[k];
            if (shift) v = v + shift[k];
            y[r * width + k] = v;
        }
    }
}

void ro_gelu_f32(size_t n, const float* x, float* y) {
    /* activation.hpp:78-90, evaluated left to right as written */
    const float coefficient = (float)0.7978845608028654;
    const float cubic = (float)0.044715;
    for (size_t i = 0; i < n; ++i) {
        const float v = x[i];
        const float inner = coefficient * (v + (((cubic * v) * v) * v));
        y[i] = (0.5f * v) * (1.0f + ro_tanh_float(inner));
    }
}

void ro_add_f32(size_t n, const float* a, const float* b, float* y) {
    for (size_t i = 0; i < n; ++i) y[i] = a[i] + b[i];
}

/* ------------------------------------------------------------------------ */
/* lm_head and greedy choice: model.hpp:86-112, 32-42                        */
/* ------------------------------------------------------------------------ */

int ro_matvec_rows_f32(size_t out, size_t in, const float* w, const float* x, float* y) {
    /* linear(row, w) for one row: operator/linear.hpp:75-84 through
       tensor.hpp:179-192 -- the sum starts at 0 and adds each product in k
       order; util.hpp:81-131 reject a non-finite product or sum (1 here) */
    int bad = 0;
    for (size_t c = 0; c < out; ++c) {
        const float* wr = w + c * in;
        float sum = 0.0f;
        for (size_t k = 0; k < in; ++k) {
            const float p = x[k] * wr[k];
            if (!isfinite(p)) bad = 1;
            sum = sum + p;
            if (!isfinite(sum)) bad = 1;
        }
        y[c] = sum;
    }
    return bad;
}

size_t ro_argmax_f32(size_t n, const float* x) {
    /* model.hpp:32-42: the best index moves only on a strictly greater value */
    size_t best = 0;
    for (size_t i = 1; i < n; ++i)
        if (x[i] > x[best]) best = i;
    return best;
}

/* ------------------------------------------------------------------------ */
/* GPT-Neo W8A8 block, operator/block.hpp:97-108                             */
/* ------------------------------------------------------------------------ */

int ro_gptneo_block_w8a8(size_t seq, size_t d, size_t heads, size_t ffn,
                         size_t window, float eps, const float* x,
                         const float* ln1_g, const float* ln1_b,
                         const int8_t* wq, const float* sq, const int8_t* wk,
                         const float* sk, const int8_t* wv, const float* sv,
                         const int8_t* wo, const float* so, const float* bo,
                         const float* ln2_g, const float* ln2_b,
                         const int8_t* wfc, const float* sfc,
                         const float* bfc, const int8_t* wproj,
                         const float* sproj, const float* bproj, float* y,
                         int threads) {
    const size_t hd = d / heads;
    float* h = (float*)malloc(seq * d * sizeof(float));
    float* q = (float*)malloc(seq * d * sizeof(float));
    float* k = (float*)malloc(seq * d * sizeof(float));
    float* v = (float*)malloc(seq * d * sizeof(float));
    float* ctx = (float*)malloc(seq * d * sizeof(float));
    float* a = (float*)malloc(seq * d * sizeof(float));
    float* f = (float*)malloc(seq * ffn * sizeof(float));
    int rc = 0;
    /* attention.hpp:354-372: ln1, q/k/v projections (no bias) */
    ro_layernorm_f32(seq, d, x, ln1_g, ln1_b, eps, h);
    rc |= ro_linear_w8a8(seq, d, d, h, wq, d, sq, NULL, q, threads);
    rc |= ro_linear_w8a8(seq, d, d, h, wk, d, sk, NULL, k, threads);
    rc |= ro_linear_w8a8(seq, d, d, h, wv, d, sv, NULL, v, threads);
    /* context, attention.hpp:374-432: every head over the whole sequence,
     * queries are the last seq keys (query_start 0 for an empty cache) */
    for (size_t hh = 0; hh < heads && rc == 0; ++hh) {
        rc |= ro_attention_head_f32(seq, seq, hd, 0, window, q + hh * hd, d,
                                    k + hh * hd, v + hh * hd, d, ctx + hh * hd,
                                    d);
    }
    rc |= ro_linear_w8a8(seq, d, d, ctx, wo, d, so, bo, h, threads);
    ro_add_f32(seq * d, x, h, a); /* residual_add(input, attention) */
    ro_layernorm_f32(seq, d, a, ln2_g, ln2_b, eps, h);
    /* mlp.hpp:108-133: c_proj(gelu(c_fc(x))) */
    rc |= ro_linear_w8a8(seq, d, ffn, h, wfc, d, sfc, bfc, f, threads);
    ro_gelu_f32(seq * ffn, f, f);
    rc |= ro_linear_w8a8(seq, ffn, d, f, wproj, ffn, sproj, bproj, h,
                         threads);
    ro_add_f32(seq * d, a, h, y);
    free(h);
    free(q);
    free(k);
    free(v);
    free(ctx);
    free(a);
    free(f);
    return rc ? -1 : 0;
}
