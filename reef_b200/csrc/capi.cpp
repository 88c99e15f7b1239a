// capi.cpp -- the extern "C" surface declared in include/reef_b200.h.
// Validates arguments (returning the status codes the header documents) and
// forwards to the launchers in ops.h.
#include "../../include/reef_b200.h"

#include "ops.h"

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

int reef_b200_version(void) { return 100; }

size_t reef_b200_kpad(size_t in) { return kpad(in); }

int reef_b200_check_device(void) { return check_device(); }

int reef_b200_device_error(int* code) {
  if (code == nullptr) return REEF_B200_ERR_INVALID;
  if (cudaDeviceSynchronize() != cudaSuccess) return REEF_B200_ERR_CUDA;
  return read_device_error(code);
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

}  // extern "C"
