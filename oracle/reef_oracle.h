/* reef_oracle.h -- CPU restatement of reef's W8A8 / int8 arithmetic.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the parity checker for the
 * sm_100a kernels in reef_b200/csrc: only tests/, __graft_entry__.smoke()
 * and bench.py's CPU-baseline / reference arm may load it.  The product
 * path never calls into it.
 *
 * Every function restates one function of reef's header-only engine
 * (inference-engine/reference/cpp/include/inference_engine/) and cites the
 * file:line it follows.  The restatement is pinned against the golden
 * vectors that reef's own generator (inference-engine/coral/host/
 * gen_golden.cpp) writes, committed under tests/golden/, and against the
 * engine itself compiled in place (oracle/_ref, built by oracle/Makefile).
 *
 * Build: gcc -O2 -ffp-contract=off (the engine is built with
 * -ffp-contract=off, inference-engine/CMakeLists.txt:10-13; every float step
 * here must be one correctly rounded IEEE operation, never a fused
 * multiply-add).
 *
 * Layouts: row-major; linear weights are [out][in] (the engine's
 * QuantizedWeight layout, quant.hpp:38-43) with an explicit row stride.
 */
#ifndef REEF_ORACLE_H
#define REEF_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- seeded inputs ---------------------------------------------------- */

/* The 32-bit LCG of weights.hpp:237-247 and gen_golden.cpp:48-86:
 * state = state * 1664525 + 1013904223; values use the top 24 bits. */
uint32_t ro_lcg_next(uint32_t* state);
/* gen_golden Rng::uniform (gen_golden.cpp:52-56): low + (high-low)*u,
 * u = (next >> 8) * 2^-24. */
void ro_fill_uniform(uint32_t seed, size_t n, float low, float high,
                     float* out);
/* gen_golden Rng::integers (gen_golden.cpp:59-68): low + (next>>8) % span. */
void ro_fill_int8(uint32_t seed, size_t n, int32_t low, int32_t high,
                  int8_t* out);
void ro_fill_int32(uint32_t seed, size_t n, int32_t low, int32_t high,
                   int32_t* out);
/* N(mean, std) by the Box-Muller transform over the same LCG (the reference
 * has uniform generators only; this transform is this build's own
 * definition, documented beside it).  u1 = ((next>>8)+1) * 2^-24 in (0,1],
 * u2 = (next>>8) * 2^-24; z0 = r cos(2 pi u2), z1 = r sin(2 pi u2),
 * r = sqrt(-2 ln u1), evaluated in double and rounded to float. */
void ro_fill_normal(uint32_t seed, size_t n, float mean, float std_dev,
                    float* out);

/* ---- quantization (quant.hpp) ----------------------------------------- */

/* int8_scale, quant.hpp:51-57. */
float ro_int8_scale(float max_magnitude);
/* quantize_int8, quant.hpp:68-81 (nearbyint ties-to-even, clamp +-127).
 * Returns 0 and sets *bad when value or scale is not finite (the engine
 * throws std::invalid_argument there). */
int8_t ro_quantize_int8(float value, float scale, int* bad);
/* quantize_rows, quant.hpp:90-133: per-row max |x|, scale, codes.
 * q has row stride ldq.  Returns 0, or -1 when a value is not finite. */
int ro_quantize_rows(size_t rows, size_t cols, const float* x, int8_t* q,
                     size_t ldq, float* scales);

/* ---- integer GEMM (tensor.hpp:178-246) -------------------------------- */

/* c[m][n] = sum_k a[m][k] * b[n][k] in int32 (matmul<int8,int32> of a and
 * transpose(b)).  Integer sums are order-free, so any order gives the
 * engine's bits.  Runs on `threads` host threads (0 = all cores). */
void ro_gemm_i8_i32(size_t m, size_t n, size_t k, const int8_t* a,
                    size_t lda, const int8_t* b, size_t ldb, int32_t* c,
                    size_t ldc, int threads);

/* ---- linear layers ---------------------------------------------------- */

/* W8A8 linear, operator/linear.hpp:106-134: quantize_rows(x), int32 sums,
 * y = float(sum) * (row_scale * w_scale[c]), then + bias[c] (add_bias,
 * linear.hpp:30-50).  bias may be NULL.  w is [out][ldw].
 * Returns 0, or -1 on a non-finite input. */
int ro_linear_w8a8(size_t rows, size_t in, size_t out, const float* x,
                   const int8_t* w, size_t ldw, const float* w_scale,
                   const float* bias, float* y, int threads);
/* The epilogue alone: y = float(acc) * (x_scale[r] * w_scale[c]) (+bias). */
void ro_w8a8_epilogue(size_t rows, size_t out, const int32_t* acc,
                      const float* x_scale, const float* w_scale,
                      const float* bias, float* y);

/* rounding_shift / saturate_int8, int8.hpp:43-60. */
int32_t ro_rounding_shift(int32_t value, unsigned shift);
int8_t ro_saturate_int8(int32_t value);
/* linear_int8, int8.hpp:74-101: sat8(rshift(sum + bias32[c], shift)). */
void ro_linear_int8(size_t rows, size_t in, size_t out, const int8_t* x,
                    size_t ldx, const int8_t* w, size_t ldw, unsigned shift,
                    const int32_t* bias, int8_t* y, int threads);

/* ---- reproducible math (math.hpp) ------------------------------------- */

/* exp_nonpositive, math.hpp:34-71 (Cephes expf polynomial, no FMA). */
float ro_exp_nonpositive(float x);
/* tanh_float, math.hpp:77-81. */
float ro_tanh_float(float x);

/* ---- integer softmax / attention (int8.hpp) --------------------------- */

/* exp_table, int8.hpp:156-164: round(32768 * exp_nonpositive(-d*step)). */
void ro_exp_table(float step, uint16_t table[256]);
/* masked_softmax_int8 for one row over the contiguous visible keys
 * [0, n) (int8.hpp:180-232; the Coral softmax_int8 entry point). */
void ro_softmax_int8_row(size_t n, const int32_t* scores, unsigned shift,
                         const uint16_t* table, uint8_t* probs);
/* Visible keys of query row i: [first, end), causal_visibility
 * (attention.hpp:82-100).  Returns 0 when the row sees no key. */
int ro_visible_range(size_t query_start, size_t i, size_t key_len,
                     size_t window, size_t* first, size_t* end);
/* attend_head_int8, int8.hpp:250-279, with the Coral argument list
 * (kernels.hpp:122-129).  Returns -1 when a row sees no key. */
int ro_attention_head_int8(size_t query_len, size_t key_len, size_t head_dim,
                           size_t query_start, size_t window, const int8_t* q,
                           size_t q_stride, const int8_t* k, const int8_t* v,
                           unsigned score_shift, const uint16_t* table,
                           unsigned out_shift, int8_t* out,
                           size_t out_stride);

/* ---- float operators -------------------------------------------------- */

/* attend_head + masked_softmax (attention.hpp:117-123,
 * activation.hpp:166-231) with the Coral argument list (kernels.hpp:75-79):
 * in-order dot products, exp_nonpositive, in-order sum, divide, in-order
 * P.V.  k, v have row stride kv_stride.  Returns -1 when a row sees no key. */
int ro_attention_head_f32(size_t query_len, size_t key_len, size_t head_dim,
                          size_t query_start, size_t window, const float* q,
                          size_t q_stride, const float* k, const float* v,
                          size_t kv_stride, float* out, size_t out_stride);
/* layernorm, operator/layernorm.hpp:36-82 (sequential mean and variance). */
void ro_layernorm_f32(size_t rows, size_t width, const float* x,
                      const float* gain, const float* shift, float eps,
                      float* y);
/* gelu (tanh form), operator/activation.hpp:69-92. */
void ro_gelu_f32(size_t n, const float* x, float* y);
/* residual_add, operator/block.hpp:27-39. */
void ro_add_f32(size_t n, const float* a, const float* b, float* y);
/* GPT-Neo's lm_head row (linear with w [out][in]) and argmax */
int ro_matvec_rows_f32(size_t out, size_t in, const float* w, const float* x, float* y);
size_t ro_argmax_f32(size_t n, const float* x);

/* ---- GPT-Neo W8A8 block (operator/block.hpp:97-108) ------------------- */

/* One pre-norm GPT-Neo block over `seq` new positions of an empty cache,
 * W8A8 projections:  x + attn(ln1(x)), then + mlp(ln2(.)).
 * wq/wk/wv/wo are [d][d] int8 with [d] scales, wfc [ffn][d], wproj [d][ffn].
 * bo [d], bfc [ffn], bproj [d]; window 0 = global attention.
 * Returns 0, or -1 on a non-finite value. */
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
                         int threads);

#ifdef __cplusplus
}
#endif

#endif /* REEF_ORACLE_H */
