// ref_shim.cpp -- C entry points over reef's own header-only engine.
//
// TEST INFRASTRUCTURE ONLY.  oracle/Makefile compiles this file against the
// unmodified engine headers where they lie in the reference checkout
// (inference-engine/reference/cpp/include), with the engine's own flags
// (-std=c++17 -ffp-contract=off, inference-engine/CMakeLists.txt:9-13), into
// oracle/_ref/libreef_ref.so.  No reference source is copied into this
// repository: the headers are only #included at build time.
//
// Uses: (1) a second, independent checker for the C restatement in
// reef_oracle.c; (2) the CPU baseline that bench.py times ("kind":
// "reference").  Every wrapper catches the engine's exceptions and returns
// -1 (std::invalid_argument / length_error) or -2 (std::overflow_error).
#include "inference_engine/int8.hpp"
#include "inference_engine/model.hpp"
#include "inference_engine/operator/attention.hpp"
#include "inference_engine/operator/block.hpp"
#include "inference_engine/operator/linear.hpp"
#include "inference_engine/quant.hpp"
#include "inference_engine/tensor.hpp"
#include "inference_engine/weights.hpp"
#include "pack_model.hpp"

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <functional>
#include <optional>
#include <stdexcept>
#include <vector>

namespace ie = inference_engine;

namespace {

template <typename T>
ie::Tensor<T> matrix(std::size_t rows, std::size_t cols, const T* data) {
    return ie::Tensor<T>{{rows, cols}, std::vector<T>(data, data + rows * cols)};
}

template <typename T>
ie::Tensor<T> vector1(std::size_t n, const T* data) {
    return ie::Tensor<T>{{n}, std::vector<T>(data, data + n)};
}

template <typename F> int guarded(F&& body) {
    try {
        body();
        return 0;
    } catch (const std::overflow_error&) {
        return -2;
    } catch (const std::exception&) {
        return -1;
    }
}

std::optional<std::size_t> window_of(std::size_t window) {
    return window > 0 ? std::optional<std::size_t>(window) : std::nullopt;
}

} // namespace

extern "C" {

// quantize_rows (quant.hpp:112-133).
int ref_quantize_rows(std::size_t rows, std::size_t cols, const float* x,
                      std::int8_t* q, float* scales) {
    return guarded([&] {
        const ie::QuantizedWeight<float> r =
            ie::quantize_rows(matrix(rows, cols, x));
        std::memcpy(q, r.values.values.data(), rows * cols);
        std::memcpy(scales, r.scales.data(), rows * sizeof(float));
    });
}

// W8A8 linear (operator/linear.hpp:106-134); w is [out][in] int8 with one
// scale per output row, bias may be NULL.
int ref_linear_w8a8(std::size_t rows, std::size_t in, std::size_t out,
                    const float* x, const std::int8_t* w,
                    const float* w_scale, const float* bias, float* y) {
    return guarded([&] {
        const ie::QuantizedWeight<float> qw{
            matrix(out, in, w), std::vector<float>(w_scale, w_scale + out)};
        const ie::Tensor<float> xs = matrix(rows, in, x);
        ie::Tensor<float> result;
        if (bias != nullptr) {
            const ie::Tensor<float> b = vector1(out, bias);
            result = ie::linear<float>(xs, qw, std::cref(b));
        } else {
            result = ie::linear<float>(xs, qw);
        }
        std::memcpy(y, result.values.data(), rows * out * sizeof(float));
    });
}

// A W8A8 weight built once as the engine's QuantizedWeight (quant.hpp:38-43),
// for repeated linear() calls on it: each call still does the engine's own
// per-call work (linear.hpp:106-134 transposes W inside), but the weight is
// not copied into a new Tensor per call.  NULL on failure.
void* ref_weight_new(std::size_t out, std::size_t in, const std::int8_t* w,
                     const float* w_scale) {
    try {
        return new ie::QuantizedWeight<float>{
            matrix(out, in, w), std::vector<float>(w_scale, w_scale + out)};
    } catch (const std::exception&) {
        return nullptr;
    }
}

void ref_weight_free(void* weight) {
    delete static_cast<ie::QuantizedWeight<float>*>(weight);
}

// W8A8 linear (operator/linear.hpp:106-134) of x [rows][in] by a weight from
// ref_weight_new: y [rows][out].
int ref_linear_w8a8_weight(const void* weight, std::size_t rows, std::size_t in,
                           const float* x, float* y) {
    return guarded([&] {
        const auto& qw = *static_cast<const ie::QuantizedWeight<float>*>(weight);
        const ie::Tensor<float> result = ie::linear<float>(matrix(rows, in, x), qw);
        std::memcpy(y, result.values.data(), result.values.size() * sizeof(float));
    });
}

// linear_int8 (int8.hpp:74-101); bias may be NULL.
int ref_linear_int8(std::size_t rows, std::size_t in, std::size_t out,
                    const std::int8_t* x, const std::int8_t* w,
                    unsigned shift, const std::int32_t* bias,
                    std::int8_t* y) {
    return guarded([&] {
        const ie::Tensor<std::int8_t> xs = matrix(rows, in, x);
        const ie::Tensor<std::int8_t> ws = matrix(out, in, w);
        ie::Tensor<std::int8_t> result;
        if (bias != nullptr) {
            const ie::Tensor<std::int32_t> b = vector1(out, bias);
            result = ie::linear_int8(xs, ws, shift, std::cref(b));
        } else {
            result = ie::linear_int8(xs, ws, shift);
        }
        std::memcpy(y, result.values.data(), rows * out);
    });
}

// matmul<int8, int32>(a, transpose(b)) (tensor.hpp:209-246).
int ref_matmul_i8(std::size_t m, std::size_t n, std::size_t k,
                  const std::int8_t* a, const std::int8_t* b,
                  std::int32_t* c) {
    return guarded([&] {
        const ie::Tensor<std::int32_t> r =
            ie::matmul<std::int8_t, std::int32_t>(
                matrix(m, k, a), ie::transpose(matrix(n, k, b), 0, 1));
        std::memcpy(c, r.values.data(), m * n * sizeof(std::int32_t));
    });
}

// exp_table (int8.hpp:156-164).
int ref_exp_table(float step, std::uint16_t* table) {
    return guarded([&] {
        const ie::ExpTable t = ie::exp_table(step);
        std::memcpy(table, t.data(), sizeof(std::uint16_t) * 256);
    });
}

// exp_nonpositive (math.hpp:34-71), elementwise.
int ref_exp_nonpositive(std::size_t n, const float* x, float* y) {
    for (std::size_t i = 0; i < n; ++i) y[i] = ie::exp_nonpositive(x[i]);
    return 0;
}

// masked_softmax_int8 (int8.hpp:180-232) over [rows, n] with every key
// visible, as the Coral softmax_int8 entry point runs it row by row.
int ref_softmax_int8(std::size_t rows, std::size_t n,
                     const std::int32_t* scores, unsigned shift,
                     std::uint8_t* probs) {
    return guarded([&] {
        const ie::Tensor<bool> all{{rows, n}, std::vector<bool>(rows * n, true)};
        const ie::Tensor<std::uint8_t> p = ie::masked_softmax_int8(
            matrix(rows, n, scores), all, shift, ie::exp_table());
        std::memcpy(probs, p.values.data(), rows * n);
    });
}

// attend_head_int8 (int8.hpp:250-279) with causal_visibility
// (attention.hpp:82-100) and the default exp_table(); q, k, v contiguous.
int ref_attend_head_int8(std::size_t query_len, std::size_t key_len,
                         std::size_t head_dim, std::size_t query_start,
                         std::size_t window, const std::int8_t* q,
                         const std::int8_t* k, const std::int8_t* v,
                         unsigned score_shift, unsigned out_shift,
                         std::int8_t* out) {
    return guarded([&] {
        const ie::Tensor<std::int8_t> r = ie::attend_head_int8(
            matrix(query_len, head_dim, q), matrix(key_len, head_dim, k),
            matrix(key_len, head_dim, v),
            ie::causal_visibility(query_len, key_len, query_start,
                                  window_of(window)),
            score_shift, ie::exp_table(), out_shift);
        std::memcpy(out, r.values.data(), query_len * head_dim);
    });
}

// attend_head (attention.hpp:117-123), float.
int ref_attend_head_f32(std::size_t query_len, std::size_t key_len,
                        std::size_t head_dim, std::size_t query_start,
                        std::size_t window, const float* q, const float* k,
                        const float* v, float* out) {
    return guarded([&] {
        const ie::Tensor<float> r = ie::attend_head(
            matrix(query_len, head_dim, q), matrix(key_len, head_dim, k),
            matrix(key_len, head_dim, v),
            ie::causal_visibility(query_len, key_len, query_start,
                                  window_of(window)));
        std::memcpy(out, r.values.data(), query_len * head_dim * sizeof(float));
    });
}

// Block<float>::forward (operator/block.hpp:97-108) on `seq` positions of a
// fresh cache, with the projections quantized by quantize_rows as
// quantize_w8a8 does (weights.hpp:460-472).  Float weights in the engine's
// [out][in] layout; layer 0 (global attention) unless `local` is set.
int ref_block_w8a8(std::size_t seq, std::size_t d, std::size_t heads,
                   std::size_t ffn, std::size_t window, int local, float eps,
                   const float* x, const float* ln1_g, const float* ln1_b,
                   const float* wq, const float* wk, const float* wv,
                   const float* wo, const float* bo, const float* ln2_g,
                   const float* ln2_b, const float* wfc, const float* bfc,
                   const float* wproj, const float* bproj, float* y) {
    return guarded([&] {
        ie::GptNeoConfig config;
        config.vocab_size = 1;
        config.max_positions = seq;
        config.hidden_size = d;
        config.num_layers = 2;
        config.num_heads = heads;
        config.inner_size = ffn;
        config.window_size = window > 0 ? window : seq;
        config.layer_norm_eps = eps;

        ie::LayerWeights<float> lw{};
        lw.ln_1_weight = vector1(d, ln1_g);
        lw.ln_1_bias = vector1(d, ln1_b);
        lw.attention.num_heads = heads;
        lw.attention.query_weights = matrix(d, d, wq);
        lw.attention.key_weights = matrix(d, d, wk);
        lw.attention.value_weights = matrix(d, d, wv);
        lw.attention.output_weights = matrix(d, d, wo);
        lw.attention.output_bias = vector1(d, bo);
        lw.ln_2_weight = vector1(d, ln2_g);
        lw.ln_2_bias = vector1(d, ln2_b);
        lw.mlp.input_size = d;
        lw.mlp.inner_size = ffn;
        lw.mlp.c_fc_weight = matrix(ffn, d, wfc);
        lw.mlp.c_fc_bias = vector1(ffn, bfc);
        lw.mlp.c_proj_weight = matrix(d, ffn, wproj);
        lw.mlp.c_proj_bias = vector1(d, bproj);
        // quantize_w8a8 for one layer (weights.hpp:460-472).
        lw.attention.quantized = std::array<ie::QuantizedWeight<float>, 4>{
            ie::quantize_rows(lw.attention.query_weights),
            ie::quantize_rows(lw.attention.key_weights),
            ie::quantize_rows(lw.attention.value_weights),
            ie::quantize_rows(lw.attention.output_weights)};
        lw.mlp.quantized = std::array<ie::QuantizedWeight<float>, 2>{
            ie::quantize_rows(lw.mlp.c_fc_weight),
            ie::quantize_rows(lw.mlp.c_proj_weight)};

        ie::Block<float> block(lw, config, local ? 1 : 0);
        const ie::Tensor<float> r = block.forward(matrix(seq, d, x));
        std::memcpy(y, r.values.data(), seq * d * sizeof(float));
    });
}

// GPT-Neo's lm_head for one row: linear<float>(row, wte) (model.hpp:107-110).
int ref_matvec_rows_f32(std::size_t out, std::size_t in, const float* w, const float* x,
                        float* y) {
    return guarded([&] {
        const ie::Tensor<float> r = ie::linear<float>(matrix(1, in, x), matrix(out, in, w));
        std::memcpy(y, r.values.data(), out * sizeof(float));
    });
}

// A random GPT-Neo (weights.hpp:407), quantize_w8a8 (weights.hpp:460), then
// reef's packer for the firmware, W8A8 (coral/host/pack_model.hpp:88-160):
// the "REEF" v1 blob.  *size gets its length; cap bytes at out are filled.
int ref_pack_random_gpt_neo(std::size_t vocab, std::size_t positions, std::size_t hidden,
                            std::size_t layers, std::size_t heads, std::size_t inner,
                            std::size_t window, std::uint32_t seed, std::uint8_t* out,
                            std::size_t cap, std::size_t* size) {
    return guarded([&] {
        ie::GptNeoConfig config;
        config.vocab_size = vocab;
        config.max_positions = positions;
        config.hidden_size = hidden;
        config.num_layers = layers;
        config.num_heads = heads;
        config.inner_size = inner;
        config.window_size = window;
        ie::ModelWeights<float> weights = ie::random_gpt_neo(config, seed);
        ie::quantize_w8a8(weights);
        const std::vector<std::uint8_t> blob =
            coral_host::pack_gpt_neo(weights, reef_kernels::Precision::kW8A8);
        *size = blob.size();
        if (blob.size() <= cap) std::memcpy(out, blob.data(), blob.size());
    });
}

// argmax (model.hpp:32-42).
int ref_argmax_f32(std::size_t n, const float* x, std::size_t* index) {
    return guarded([&] { *index = ie::argmax(vector1(n, x)); });
}

// The float linear of Coral's linear_f32 / linear_bias_f32: the engine's
// linear<float> (operator/linear.hpp:75-84) on the weight wt [in][out]
// transposed back to the engine's [out][in]; bias may be null.
int ref_linear_f32(std::size_t rows, std::size_t in, std::size_t out, const float* x,
                   const float* wt, const float* bias, float* y) {
    return guarded([&] {
        ie::Tensor<float> w{{out, in}, std::vector<float>(out * in)};
        for (std::size_t k = 0; k < in; ++k)
            for (std::size_t c = 0; c < out; ++c) w.values[c * in + k] = wt[k * out + c];
        const ie::Tensor<float> x_t = matrix(rows, in, x);
        ie::Tensor<float> r;
        if (bias != nullptr) {
            const ie::Tensor<float> b = vector1(out, bias);
            r = ie::linear<float>(x_t, w, std::cref(b));
        } else {
            r = ie::linear<float>(x_t, w);
        }
        std::memcpy(y, r.values.data(), rows * out * sizeof(float));
    });
}

// layernorm_int8 (int8.hpp:332-374).
int ref_layernorm_int8(std::size_t rows, std::size_t width, const std::int8_t* x,
                       const std::int8_t* gain, const std::int8_t* shift, std::int8_t* y) {
    return guarded([&] {
        const ie::Tensor<std::int8_t> r = ie::layernorm_int8(
            matrix(rows, width, x), vector1(width, gain), vector1(width, shift));
        std::memcpy(y, r.values.data(), rows * width);
    });
}

// add_int8 (int8.hpp:382-397).
int ref_add_int8(std::size_t n, const std::int8_t* a, const std::int8_t* b, std::int8_t* y) {
    return guarded([&] {
        const ie::Tensor<std::int8_t> r = ie::add_int8(vector1(n, a), vector1(n, b));
        std::memcpy(y, r.values.data(), n);
    });
}

// gelu_table then gelu_int8 (int8.hpp:112-147): the table for the given
// scales into table[256], and x looked up through it into y.
int ref_gelu_int8(std::size_t n, const std::int8_t* x, float in_scale, float out_scale,
                  std::int8_t* table, std::int8_t* y) {
    return guarded([&] {
        const ie::Int8Table t = ie::gelu_table(in_scale, out_scale);
        std::memcpy(table, t.data(), t.size());
        const ie::Tensor<std::int8_t> r = ie::gelu_int8(vector1(n, x), t);
        std::memcpy(y, r.values.data(), n);
    });
}

} // extern "C"
