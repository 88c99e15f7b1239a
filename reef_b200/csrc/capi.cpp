// capi.cpp -- the extern "C" surface declared in include/reef_b200.h.
// Validates arguments (returning the status codes the header documents) and
// forwards to the launchers in ops.h.
#include "../../include/reef_b200.h"

#include "ops.h"

#include <cuda_fp16.h>

using namespace reef;

namespace {

inline cudaStream_t S(reef_b200_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }

constexpr size_t kMaxDim = (1u << 31) - 1;

bool dims_ok(size_t rows, size_t in, size_t out) {
  return in > 0 && out > 0 && rows <= kMaxDim && in <= kMaxDim && out <= kMaxDim;
}

int gemm(size_t rows, size_t in, size_t out, const int8_t* a, const int8_t* b, int epi,
         GemmArgs args, void* y, cudaStream_t stream) {
  if (int rc = check_device()) return rc;
  GemmProblem p{};
  p.M = static_cast<int>(rows);
  p.N = static_cast<int>(out);
  p.K = static_cast<int>(in);
  p.a = a;
  p.lda = static_cast<long long>(kpad(in));
  p.b = b;
  p.ldb = static_cast<long long>(kpad(in));
  args.y = y;
  args.ldy = static_cast<long long>(out);
  p.args = args;
  return gemm_i8(p, epi, stream);
}

}  // namespace

extern "C" {

const char* reef_b200_status_string(int status) {
  switch (status) {
    case REEF_B200_OK: return "ok";
    case REEF_B200_ERR_INVALID: return "invalid argument";
    case REEF_B200_ERR_ALIGNMENT: return "pointer or stride not 16-byte aligned";
    case REEF_B200_ERR_CUDA: return "CUDA error";
    case REEF_B200_ERR_UNSUPPORTED: return "device is not sm_100 (B200)";
    case REEF_B200_ERR_NCCL: return "NCCL error";
    case REEF_B200_ERR_TIMEOUT: return "a bounded device wait gave up";
    case REEF_B200_ERR_TOO_LARGE: return "size exceeds the documented maximum";
    default: return "unknown status";
  }
}

int reef_b200_version(void) { return 200; }

size_t reef_b200_kpad(size_t in) { return kpad(in); }

int reef_b200_check_device(void) { return check_device(); }

int reef_b200_device_error(int* code) {
  if (code == nullptr) return REEF_B200_ERR_INVALID;
  if (cudaDeviceSynchronize() != cudaSuccess) return REEF_B200_ERR_CUDA;
  return read_device_error(code);
}

int reef_b200_matvec_rows_f32(size_t out, size_t in, const float* w, const float* x, float* y,
                              reef_b200_stream_t stream) {
  if (out == 0 || in == 0 || !w || !x || !y) return REEF_B200_ERR_INVALID;
  if (out > (1ull << 40) || in > (1ull << 40) || out > (1ull << 62) / in)
    return REEF_B200_ERR_TOO_LARGE;
  if (int rc = check_device()) return rc;
  return matvec_rows_f32(static_cast<long long>(out), static_cast<long long>(in), w, x, y,
                         S(stream));
}

int reef_b200_argmax_f32(size_t n, const float* x, uint32_t* index, reef_b200_stream_t stream) {
  if (n == 0 || !x || !index) return REEF_B200_ERR_INVALID;
  if (n > 0xffffffffull) return REEF_B200_ERR_TOO_LARGE;
  if (int rc = check_device()) return rc;
  return argmax_f32(static_cast<long long>(n), x, index, S(stream));
}

int reef_b200_embedding_f32(size_t width, size_t count, const uint32_t* ids,
                            size_t first_position, size_t vocab, size_t max_positions,
                            const float* wte, const float* wpe, float* y,
                            reef_b200_stream_t stream) {
  if (count == 0) return REEF_B200_OK;
  if (width == 0 || width > kMaxDim || count > kMaxDim || vocab == 0 || max_positions == 0 ||
      first_position > max_positions || count > max_positions - first_position || !ids ||
      !wte || !wpe || !y)
    return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  return embedding_f32(static_cast<int>(width), static_cast<long long>(count), ids,
                       static_cast<long long>(first_position), static_cast<long long>(vocab),
                       static_cast<long long>(max_positions), wte, wpe, y, S(stream));
}

int reef_b200_linear_bias_f32(size_t rows, size_t in, size_t out, const float* x,
                              const float* wt, const float* bias, float* y,
                              reef_b200_stream_t stream) {
  if (rows == 0) return REEF_B200_OK;
  if (!dims_ok(rows, in, out) || !x || !wt || !y) return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  return linear_f32(static_cast<long long>(rows), static_cast<int>(in), static_cast<int>(out), x,
                    wt, bias, y, S(stream));
}

int reef_b200_linear_f32(size_t rows, size_t in, size_t out, const float* x, const float* wt,
                         float* y, reef_b200_stream_t stream) {
  return reef_b200_linear_bias_f32(rows, in, out, x, wt, nullptr, y, stream);
}

int reef_b200_layernorm_f32(size_t rows, size_t width, const float* x, const float* gain,
                            const float* shift, float eps, float* y, reef_b200_stream_t stream) {
  if (rows == 0) return REEF_B200_OK;
  if (width == 0 || width > kMaxDim || rows > kMaxDim || !x || !gain || !y)
    return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  return layernorm_exact(static_cast<long long>(rows), static_cast<int>(width), eps, x, gain,
                         shift, y, S(stream));
}

static int unary(int op, size_t n, const float* x, float* y, reef_b200_stream_t stream) {
  if (n == 0) return REEF_B200_OK;
  if (!x || !y) return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  return unary_exact(op, static_cast<long long>(n), x, y, S(stream));
}

int reef_b200_exp_nonpositive_f32(size_t n, const float* x, float* y,
                                  reef_b200_stream_t stream) {
  return unary(kUnaryExp, n, x, y, stream);
}

int reef_b200_tanh_f32(size_t n, const float* x, float* y, reef_b200_stream_t stream) {
  return unary(kUnaryTanh, n, x, y, stream);
}

int reef_b200_gelu_f32(size_t n, const float* x, float* y, reef_b200_stream_t stream) {
  return unary(kUnaryGelu, n, x, y, stream);
}

int reef_b200_add_f32(size_t n, const float* a, const float* b, float* y,
                      reef_b200_stream_t stream) {
  if (n == 0) return REEF_B200_OK;
  if (!a || !b || !y) return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  return add_f32(static_cast<long long>(n), a, b, y, S(stream));
}

int reef_b200_gelu_int8(size_t n, const int8_t* x, const int8_t* table, int8_t* y,
                        reef_b200_stream_t stream) {
  if (n == 0) return REEF_B200_OK;
  if (!x || !table || !y) return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  return gelu_int8(static_cast<long long>(n), x, table, y, S(stream));
}

int reef_b200_layernorm_int8(size_t rows, size_t width, const int8_t* x, const int8_t* gain,
                             const int8_t* shift, int8_t* y, reef_b200_stream_t stream) {
  if (rows == 0) return REEF_B200_OK;
  if (width == 0 || width > 32767 || rows > kMaxDim || !x || !gain || !shift || !y)
    return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  return layernorm_int8(static_cast<long long>(rows), static_cast<int>(width), x, gain, shift, y,
                        S(stream));
}

int reef_b200_add_int8(size_t n, const int8_t* a, const int8_t* b, int8_t* y,
                       reef_b200_stream_t stream) {
  if (n == 0) return REEF_B200_OK;
  if (!a || !b || !y) return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  return add_int8(static_cast<long long>(n), a, b, y, S(stream));
}

int reef_b200_embedding_int8(size_t width, size_t count, const uint32_t* ids,
                             size_t first_position, size_t vocab, size_t max_positions,
                             const int8_t* wte, const int8_t* wpe, int8_t* y,
                             reef_b200_stream_t stream) {
  if (count == 0) return REEF_B200_OK;
  if (width == 0 || width > kMaxDim || count > kMaxDim || vocab == 0 || max_positions == 0 ||
      first_position > max_positions || count > max_positions - first_position || !ids ||
      !wte || !wpe || !y)
    return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  return embedding_int8(static_cast<int>(width), static_cast<long long>(count), ids,
                        static_cast<long long>(first_position), static_cast<long long>(vocab),
                        static_cast<long long>(max_positions), wte, wpe, y, S(stream));
}

int reef_b200_quantize_rows(size_t rows, size_t in, const float* x, int8_t* x_q,
                            float* x_scale, reef_b200_stream_t stream) {
  if (rows == 0) return REEF_B200_OK;
  if (!dims_ok(rows, in, 1) || !x || !x_q || !x_scale) return REEF_B200_ERR_INVALID;
  return quantize_rows(rows, in, x, x_q, kpad(in), x_scale, nullptr, S(stream));
}

int reef_b200_pack_weight_i8(size_t in, size_t out, const int8_t* wt, int8_t* w,
                             reef_b200_stream_t stream) {
  if (!dims_ok(0, in, out) || !wt || !w) return REEF_B200_ERR_INVALID;
  return pack_weight_i8(in, out, wt, w, kpad(in), S(stream));
}

int reef_b200_pad_rows_i8(size_t rows, size_t in, const int8_t* x, int8_t* x_pad,
                          reef_b200_stream_t stream) {
  if (rows == 0) return REEF_B200_OK;
  if (!dims_ok(rows, in, 1) || !x || !x_pad) return REEF_B200_ERR_INVALID;
  return pad_rows_i8(rows, in, x, in, x_pad, kpad(in), S(stream));
}

int reef_b200_gemm_w8a8(size_t rows, size_t in, size_t out, const int8_t* x_q,
                        const float* x_scale, const int8_t* w, const float* w_scale,
                        const float* bias, float* y, reef_b200_stream_t stream) {
  if (rows == 0) return REEF_B200_OK;
  if (!dims_ok(rows, in, out) || !x_q || !x_scale || !w || !w_scale || !y)
    return REEF_B200_ERR_INVALID;
  GemmArgs a{};
  a.x_scale = x_scale;
  a.w_scale = w_scale;
  a.bias_f = bias;
  return gemm(rows, in, out, x_q, w, kEpiF32W8A8, a, y, S(stream));
}

int reef_b200_linear_w8a8_bias(size_t rows, size_t in, size_t out, const float* x,
                               const int8_t* w, const float* w_scale, const float* bias,
                               int8_t* x_q, float* x_scale, float* y,
                               reef_b200_stream_t stream) {
  if (rows == 0) return REEF_B200_OK;
  if (!dims_ok(rows, in, out) || !x || !w || !w_scale || !x_q || !x_scale || !y)
    return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  if (int rc = quantize_rows(rows, in, x, x_q, kpad(in), x_scale, nullptr, S(stream)))
    return rc;
  return reef_b200_gemm_w8a8(rows, in, out, x_q, x_scale, w, w_scale, bias, y, stream);
}

int reef_b200_rmsnorm_quant(size_t rows, size_t width, float eps, const float* x,
                            const float* gain, int8_t* x_q, float* x_scale,
                            reef_b200_stream_t stream) {
  if (rows == 0) return REEF_B200_OK;
  if (width == 0 || width > 16384 || rows > kMaxDim || !x || !gain || !x_q || !x_scale)
    return REEF_B200_ERR_INVALID;
  if (width % 32 != 0) return REEF_B200_ERR_ALIGNMENT;
  if (int rc = check_device()) return rc;
  return rmsnorm_quant(static_cast<long long>(rows), static_cast<int>(width), eps, x, gain, x_q,
                       x_scale, S(stream));
}

int reef_b200_linear_w8a8_swiglu(size_t rows, size_t in, size_t ffn, const int8_t* x_q,
                                 const float* x_scale, const int8_t* w_gu,
                                 const float* w_scale, float* h, float* row_max,
                                 reef_b200_stream_t stream) {
  if (rows == 0) return REEF_B200_OK;
  if (!dims_ok(rows, in, 2 * ffn) || !x_q || !x_scale || !w_gu || !w_scale || !h || !row_max)
    return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  return linear_w8a8_swiglu(static_cast<long long>(rows), static_cast<int>(in),
                            static_cast<int>(ffn), x_q, x_scale, w_gu, w_scale, h, row_max,
                            S(stream));
}

int reef_b200_linear_w8a8(size_t rows, size_t in, size_t out, const float* x,
                          const int8_t* w, const float* w_scale, int8_t* x_q,
                          float* x_scale, float* y, reef_b200_stream_t stream) {
  return reef_b200_linear_w8a8_bias(rows, in, out, x, w, w_scale, nullptr, x_q, x_scale, y,
                                    stream);
}

int reef_b200_linear_bias_int8(size_t rows, size_t in, size_t out, const int8_t* x,
                               const int8_t* w, const int32_t* bias, unsigned shift,
                               int8_t* y, reef_b200_stream_t stream) {
  if (rows == 0) return REEF_B200_OK;
  if (!dims_ok(rows, in, out) || !x || !w || !y || shift > 31) return REEF_B200_ERR_INVALID;
  GemmArgs a{};
  a.bias_i = bias;
  a.shift = shift;
  return gemm(rows, in, out, x, w, kEpiI8Shift, a, y, S(stream));
}

int reef_b200_linear_int8(size_t rows, size_t in, size_t out, const int8_t* x,
                          const int8_t* w, unsigned shift, int8_t* y,
                          reef_b200_stream_t stream) {
  return reef_b200_linear_bias_int8(rows, in, out, x, w, nullptr, shift, y, stream);
}

int reef_b200_gemm_i8_i32(size_t m, size_t n, size_t k, const int8_t* a, const int8_t* b,
                          int32_t* c, reef_b200_stream_t stream) {
  if (m == 0) return REEF_B200_OK;
  if (!dims_ok(m, k, n) || !a || !b || !c) return REEF_B200_ERR_INVALID;
  GemmArgs args{};
  return gemm(m, k, n, a, b, kEpiI32, args, c, S(stream));
}

int reef_b200_softmax_int8(size_t rows, size_t n, const int32_t* scores, unsigned shift,
                           const uint16_t* table, uint8_t* probs, reef_b200_stream_t stream) {
  if (rows == 0) return REEF_B200_OK;
  if (!dims_ok(rows, n, 1) || !scores || !table || !probs || shift > 31)
    return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  return softmax_int8_rows(rows, static_cast<int>(n), scores, shift, table, probs, S(stream));
}

namespace {

// Every query row must see at least one key (the engine throws otherwise,
// attention.hpp:82-100 + activation.hpp:204-207 / int8.hpp:211-214).
int attn_args(size_t heads, size_t query_len, size_t key_len, size_t head_dim,
              size_t query_start, size_t window, AttnHeadArgs* a) {
  if (heads == 0 || query_len == 0) return REEF_B200_OK;
  if (key_len == 0 || head_dim == 0 || head_dim > kMaxDim || query_len > kMaxDim ||
      heads > 65535 || window > kMaxDim)
    return REEF_B200_ERR_INVALID;
  if (key_len > static_cast<size_t>(kMaxKeysExact)) return REEF_B200_ERR_TOO_LARGE;
  const size_t last = query_start + query_len;  // position of the last row + 1
  if (window > 0 && last > window && last - window >= key_len) return REEF_B200_ERR_INVALID;
  a->heads = static_cast<int>(heads);
  a->query_len = static_cast<int>(query_len);
  a->key_len = static_cast<int>(key_len);
  a->head_dim = static_cast<int>(head_dim);
  a->window = static_cast<int>(window);
  a->query_start = static_cast<long long>(query_start);
  return -1;  // valid, non-empty
}

}  // namespace

int reef_b200_attention_heads_int8(size_t heads, size_t query_len, size_t key_len,
                                   size_t head_dim, size_t query_start, size_t window,
                                   const int8_t* q, size_t q_stride, size_t q_head,
                                   const int8_t* k, const int8_t* v, size_t kv_stride,
                                   size_t kv_head, unsigned score_shift,
                                   const uint16_t* table, unsigned out_shift, int8_t* out,
                                   size_t out_stride, size_t out_head,
                                   reef_b200_stream_t stream) {
  AttnHeadArgs a{};
  const int v0 = attn_args(heads, query_len, key_len, head_dim, query_start, window, &a);
  if (v0 >= 0) return v0;
  if (!q || !k || !v || !table || !out || score_shift > 31 || out_shift > 31)
    return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  a.q_stride = static_cast<long long>(q_stride);
  a.q_head = static_cast<long long>(q_head);
  a.kv_stride = static_cast<long long>(kv_stride);
  a.kv_head = static_cast<long long>(kv_head);
  a.out_stride = static_cast<long long>(out_stride);
  a.out_head = static_cast<long long>(out_head);
  return attention_head_int8(a, q, k, v, score_shift, table, out_shift, out, S(stream));
}

int reef_b200_attention_head_int8(size_t query_len, size_t key_len, size_t head_dim,
                                  size_t query_start, size_t window, const int8_t* q,
                                  size_t q_stride, const int8_t* k, const int8_t* v,
                                  unsigned score_shift, const uint16_t* table,
                                  unsigned out_shift, int32_t* /*scores*/,
                                  uint8_t* /*probs*/, int8_t* out, size_t out_stride,
                                  reef_b200_stream_t stream) {
  return reef_b200_attention_heads_int8(1, query_len, key_len, head_dim, query_start, window,
                                        q, q_stride, 0, k, v, head_dim, 0, score_shift, table,
                                        out_shift, out, out_stride, 0, stream);
}

int reef_b200_attention_heads_f32(size_t heads, size_t query_len, size_t key_len,
                                  size_t head_dim, size_t query_start, size_t window,
                                  const float* q, size_t q_stride, size_t q_head,
                                  const float* k, const float* v, size_t kv_stride,
                                  size_t kv_head, float* out, size_t out_stride,
                                  size_t out_head, reef_b200_stream_t stream) {
  AttnHeadArgs a{};
  const int v0 = attn_args(heads, query_len, key_len, head_dim, query_start, window, &a);
  if (v0 >= 0) return v0;
  if (!q || !k || !v || !out) return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  a.q_stride = static_cast<long long>(q_stride);
  a.q_head = static_cast<long long>(q_head);
  a.kv_stride = static_cast<long long>(kv_stride);
  a.kv_head = static_cast<long long>(kv_head);
  a.out_stride = static_cast<long long>(out_stride);
  a.out_head = static_cast<long long>(out_head);
  return attention_head_f32(a, q, k, v, out, S(stream));
}

int reef_b200_attention_head_f32(size_t query_len, size_t key_len, size_t head_dim,
                                 size_t query_start, size_t window, const float* q,
                                 size_t q_stride, const float* k, const float* v,
                                 float* /*scores*/, float* out, size_t out_stride,
                                 reef_b200_stream_t stream) {
  return reef_b200_attention_heads_f32(1, query_len, key_len, head_dim, query_start, window, q,
                                       q_stride, 0, k, v, head_dim, 0, out, out_stride, 0,
                                       stream);
}

}  // extern "C"

extern "C" {

int reef_b200_rope_qkv_quant(size_t batch, size_t seq, size_t heads_q, size_t heads_kv,
                             float rope_base, const float* qkv, int8_t* q8, int8_t* k8,
                             int8_t* v8, float* q_scale, float* k_scale, float* v_scale,
                             void* vt, reef_b200_stream_t stream) {
  if (batch == 0 || seq == 0) return REEF_B200_OK;
  if (heads_q == 0 || heads_kv == 0 || heads_q % heads_kv != 0 || batch * seq > kMaxDim ||
      !qkv || !q8 || !k8 || !v8 || !q_scale || !k_scale || !v_scale || !vt)
    return REEF_B200_ERR_INVALID;
  if (seq % 2 != 0) return REEF_B200_ERR_ALIGNMENT;
  if (int rc = check_device()) return rc;
  return rope_qkv_quant(static_cast<int>(batch), static_cast<int>(seq),
                        static_cast<int>(heads_q), static_cast<int>(heads_kv), rope_base, qkv,
                        q8, k8, v8, q_scale, k_scale, v_scale, vt, nullptr,
                        S(stream));
}

int reef_b200_selftest_wait_timeout(unsigned limit_us, int* done, reef_b200_stream_t stream) {
  if (done == nullptr || limit_us == 0 || limit_us > 2000000u) return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  return selftest_wait_timeout(1000ull * limit_us, done, S(stream));
}

size_t reef_b200_weight_tiles_bytes(size_t rows, size_t in) {
  if (rows == 0 || in == 0 || rows > (1u << 31) - 1 || in > (1u << 31) - 1) return 0;
  return weight_tiles_bytes(static_cast<long long>(rows), static_cast<long long>(in));
}

int reef_b200_pack_weight_tiles(size_t rows, size_t in, const int8_t* w, int8_t* tiles,
                                reef_b200_stream_t stream) {
  if (rows == 0) return REEF_B200_OK;
  if (in == 0 || rows > (1u << 31) - 1 || in > (1u << 31) - 1 || !w || !tiles)
    return REEF_B200_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(tiles) % 1024 != 0) return REEF_B200_ERR_ALIGNMENT;
  if (int rc = check_device()) return rc;
  return pack_weight_tiles(static_cast<long long>(rows), static_cast<long long>(in), w,
                           static_cast<long long>(kpad(in)), tiles, S(stream));
}

int reef_b200_selftest_peer_wait_timeout(unsigned limit_us, const unsigned* counter,
                                         unsigned target, reef_b200_stream_t stream) {
  if (counter == nullptr || limit_us == 0 || limit_us > 2000000u) return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  CounterWaits w;
  w.n = 1;
  w.p[0] = counter;
  w.target[0] = target;
  return signal_and_wait(PeerFlags{}, w, 1000ull * limit_us, S(stream));
}

int reef_b200_linear_w8a8_qkv_rope(size_t batch, size_t seq, size_t in, size_t heads_q,
                                   size_t heads_kv, float rope_base, const int8_t* x_q,
                                   const float* x_scale, const int8_t* w_qkv,
                                   const float* w_scale, int8_t* q8, int8_t* k8, int8_t* v8,
                                   float* q_scale, float* k_scale, float* v_scale, void* vt,
                                   void* rope_table, reef_b200_stream_t stream) {
  if (batch == 0 || seq == 0) return REEF_B200_OK;
  if (heads_q == 0 || heads_kv == 0 || heads_q > 4096 || heads_kv > 4096 ||
      batch * seq > kMaxDim || in == 0 || in > kMaxDim || !x_q || !x_scale || !w_qkv ||
      !w_scale || !q8 || !k8 || !q_scale || !k_scale || !vt || !rope_table)
    return REEF_B200_ERR_INVALID;
  if (seq % 2 != 0) return REEF_B200_ERR_ALIGNMENT;
  if (int rc = check_device()) return rc;
  QkvOut o{};
  o.rope = static_cast<const float2*>(rope_table);
  o.seq = static_cast<int>(seq);
  o.heads_q = static_cast<int>(heads_q);
  o.heads_kv = static_cast<int>(heads_kv);
  o.q8 = q8;
  o.k8 = k8;
  o.v8 = v8;
  o.qs = q_scale;
  o.ks = k_scale;
  o.vs = v_scale;
  o.vt = vt;
  return linear_w8a8_qkv_rope(static_cast<long long>(batch * seq), static_cast<int>(in), x_q,
                              x_scale, w_qkv, w_scale, rope_base, o, S(stream));
}

int reef_b200_flash_attn_i8(size_t batch, size_t seq, size_t heads_q, size_t heads_kv,
                            size_t head_dim, int causal, float sm_scale, const int8_t* q8,
                            const float* q_scale, const int8_t* k8, const float* k_scale,
                            const void* vt, float* out, reef_b200_stream_t stream) {
  if (batch == 0 || seq == 0) return REEF_B200_OK;
  if (head_dim != 128 || heads_q == 0 || heads_kv == 0 || heads_q % heads_kv != 0 ||
      batch * seq > kMaxDim || heads_q > 4096 || !q8 || !q_scale || !k8 || !k_scale || !vt ||
      !out)
    return REEF_B200_ERR_INVALID;
  if (seq % 8 != 0) return REEF_B200_ERR_ALIGNMENT;
  if (int rc = check_device()) return rc;
  FlashProblem p{};
  p.batch = static_cast<int>(batch);
  p.heads_q = static_cast<int>(heads_q);
  p.heads_kv = static_cast<int>(heads_kv);
  p.seq = static_cast<int>(seq);
  p.head_dim = 128;
  p.causal = causal != 0;
  p.sm_scale = sm_scale;
  p.q8 = q8;
  p.k8 = k8;
  p.vt = vt;
  p.q_scale = q_scale;
  p.k_scale = k_scale;
  p.out = out;
  p.out_ld = static_cast<long long>(heads_q) * 128;
  return flash_prefill_i8(p, S(stream));
}

}  // extern "C"

extern "C" {

size_t reef_b200_decode_attn_workspace_bytes(size_t batch, size_t heads_q, size_t max_len) {
  if (batch == 0 || heads_q == 0 || max_len == 0 || batch > (1u << 20) || heads_q > 4096 ||
      max_len > (1u << 24))
    return 0;
  return decode_attn_partial_floats(static_cast<int>(batch), static_cast<int>(heads_q),
                                    static_cast<int>(max_len)) *
         sizeof(float);
}

int reef_b200_decode_attn_i8(size_t batch, size_t heads_q, size_t heads_kv, size_t head_dim,
                             size_t max_len, const int32_t* lens, size_t len, float sm_scale,
                             const int8_t* q8, const float* q_scale, const int8_t* k_cache,
                             const float* k_scale, const int8_t* v_cache, const float* v_scale,
                             void* workspace, size_t workspace_bytes, float* out,
                             reef_b200_stream_t stream) {
  if (batch == 0) return REEF_B200_OK;
  const size_t need = reef_b200_decode_attn_workspace_bytes(batch, heads_q, max_len);
  if (need == 0 || head_dim != 128 || heads_kv == 0 || heads_q % heads_kv != 0 ||
      batch * heads_kv > 65535 || !q8 || !q_scale || !k_cache || !k_scale || !v_cache ||
      !v_scale || !workspace || !out || workspace_bytes < need)
    return REEF_B200_ERR_INVALID;
  const size_t g = heads_q / heads_kv;
  if (g != 1 && g != 2 && g != 4 && g != 8 && g != 16) return REEF_B200_ERR_INVALID;
  if (lens == nullptr && (len == 0 || len > max_len)) return REEF_B200_ERR_INVALID;
  if ((reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(q8) % 4 != 0)
    return REEF_B200_ERR_ALIGNMENT;
  if (int rc = check_device()) return rc;
  DecodeProblem p{};
  p.batch = static_cast<int>(batch);
  p.heads_q = static_cast<int>(heads_q);
  p.heads_kv = static_cast<int>(heads_kv);
  p.max_len = static_cast<int>(max_len);
  p.sm_scale = sm_scale;
  p.q8 = q8;
  p.q_scale = q_scale;
  p.k_cache = k_cache;
  p.k_scale = k_scale;
  p.v_cache = v_cache;
  p.v_scale = v_scale;
  p.lens = lens;
  p.len = static_cast<int>(len);
  p.partial = static_cast<float*>(workspace);
  p.out = out;
  // a programmatic dependent of the kernel before it: the launch and set-up
  // overlap that kernel, and nothing is read before it has finished
  PdlScope pdl;
  return decode_attn_i8(p, S(stream));
}

}  // extern "C"

extern "C" {

size_t reef_b200_gemm_skinny_workspace_bytes(size_t rows, size_t in, size_t out) {
  if (rows == 0 || rows > 128 || in == 0 || out == 0 || in > kMaxDim || out > kMaxDim) return 0;
  if (check_device() != kOk) return 0;
  return skinny_partial_bytes(static_cast<int>(rows), static_cast<int>(out), static_cast<int>(in));
}

int reef_b200_gemm_w8a8_skinny(size_t rows, size_t in, size_t out, const int8_t* x_q,
                               const float* x_scale, const int8_t* w, const float* w_scale,
                               const float* bias, void* workspace, size_t workspace_bytes,
                               float* y, reef_b200_stream_t stream) {
  if (rows == 0) return REEF_B200_OK;
  if (rows > 128 || !dims_ok(rows, in, out) || !x_q || !x_scale || !w || !w_scale || !y ||
      !workspace)
    return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  if (workspace_bytes < skinny_partial_bytes(static_cast<int>(rows), static_cast<int>(out),
                                             static_cast<int>(in)))
    return REEF_B200_ERR_INVALID;
  return gemm_i8_skinny(static_cast<int>(rows), static_cast<int>(out), static_cast<int>(in), x_q,
                        w, kEpiF32W8A8, x_scale, w_scale, bias, nullptr, y, workspace, S(stream));
}

}  // extern "C"
