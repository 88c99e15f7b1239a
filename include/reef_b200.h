/* reef_b200.h -- C ABI of libreef_b200, reef's W8A8 / int8 hot path on B200.
 *
 * These entry points replace the Coral NPU kernels of reef's operator API,
 * namespace reef_kernels in inference-engine/coral/include/reef_kernels/
 * kernels.hpp (cited per function below), and compute exactly what reef's
 * header-only engine computes (inference-engine/reference/cpp/include/
 * inference_engine/).  Integer and W8A8 outputs are bit-identical to the
 * engine's; see each function.
 *
 * Conventions (differences from reef_kernels are deliberate and listed):
 *  - Every pointer is a DEVICE pointer unless stated.  Every call is
 *    asynchronous on `stream` (a cudaStream_t; NULL = the legacy default
 *    stream) and returns a status code, REEF_B200_OK on success.  reef's
 *    kernels have no error reporting; the engine throws
 *    std::invalid_argument where these return REEF_B200_ERR_INVALID.
 *  - rows == 0 is a no-op (as the Coral loops are); in == 0 or out == 0 is
 *    REEF_B200_ERR_INVALID (the engine rejects empty matrices,
 *    tensor.hpp:42-62).
 *  - Linear weights are [out][ldk] int8, K-major: the engine's
 *    QuantizedWeight layout (quant.hpp:38-43), not Coral's transposed
 *    [in][out] (kernels.hpp:15-16).  reef_b200_pack_weight_i8 converts a
 *    Coral weight once, at load time, as the firmware's blob loader would.
 *  - Every int8 matrix the tensor cores read (weights, x_q, int8 x) has a
 *    row stride of ldk = reef_b200_kpad(in) bytes: in rounded up to 16
 *    (the TMA alignment rule).  For every model width ldk == in.
 *  - Scratch is caller-owned, as in reef_kernels; the library allocates no
 *    device memory in any entry point.
 *  - Non-finite inputs to the quantiser give unspecified codes (the engine
 *    throws there, quant.hpp:72-74; the Coral kernels do not check).
 */
#ifndef REEF_B200_H
#define REEF_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct CUstream_st* reef_b200_stream_t; /* == cudaStream_t */

enum reef_b200_status {
  REEF_B200_OK = 0,
  REEF_B200_ERR_INVALID = 1,     /* bad shape, null pointer or argument */
  REEF_B200_ERR_ALIGNMENT = 2,   /* pointer / stride breaks the 16-byte rule */
  REEF_B200_ERR_CUDA = 3,        /* a CUDA call failed */
  REEF_B200_ERR_UNSUPPORTED = 4, /* current device is not sm_100 */
  REEF_B200_ERR_NCCL = 5,        /* a NCCL call failed */
  REEF_B200_ERR_TIMEOUT = 6,     /* a bounded device wait gave up */
  REEF_B200_ERR_TOO_LARGE = 7    /* a size exceeds a documented maximum */
};

/* ---- library ------------------------------------------------------------ */

/* Human-readable name of a status code. */
const char* reef_b200_status_string(int status);
/* ABI version: major * 10000 + minor * 100 + patch. */
int reef_b200_version(void);
/* Row stride in bytes of an int8 matrix with `in` columns: in rounded up to a
 * multiple of 16. */
size_t reef_b200_kpad(size_t in);
/* REEF_B200_OK when the current device is a B200 (sm_100). */
int reef_b200_check_device(void);
/* Synchronizes the current device, stores its device error word in *code
 * (0 = none; otherwise the bounded wait that gave up) and clears it. */
int reef_b200_device_error(int* code);

/* ---- quantization (quant.hpp) ------------------------------------------- */

/* quantize_rows (quant.hpp:112-133) of x [rows][in] fp32: per row
 * scale = max|x|/127 (1 for an all-zero row), x_q = clamp(rne(x/scale)).
 * x_q is [rows][kpad(in)] (padding zeroed), x_scale [rows].
 * Replaces the per-row quantize step of linear_w8a8 (kernels.hpp:34-40,
 * coral/kernels/linear.cc:60-86). */
int reef_b200_quantize_rows(size_t rows, size_t in, const float* x, int8_t* x_q,
                            float* x_scale, reef_b200_stream_t stream);

/* Coral weight layout [in][out] (kernels.hpp:15-16) -> [out][kpad(in)]. */
int reef_b200_pack_weight_i8(size_t in, size_t out, const int8_t* wt, int8_t* w,
                             reef_b200_stream_t stream);

/* Contiguous [rows][in] int8 -> [rows][kpad(in)], padding zeroed. */
int reef_b200_pad_rows_i8(size_t rows, size_t in, const int8_t* x, int8_t* x_pad,
                          reef_b200_stream_t stream);

/* ---- W8A8 linear (operator/linear.hpp:106-134) --------------------------- */

/* reef_kernels::linear_w8a8 (kernels.hpp:38-40), batched over rows:
 *   y[r][c] = float(sum_k x_q[r][k] * w[c][k]) * (x_scale[r] * w_scale[c])
 * with x quantized per row first.  x [rows][in] fp32, w [out][kpad(in)]
 * int8, w_scale [out], y [rows][out].  Scratch: x_q [rows][kpad(in)] int8
 * (Coral's x_q holds one row) and x_scale [rows] fp32. Bit-identical to the
 * engine. */
int reef_b200_linear_w8a8(size_t rows, size_t in, size_t out, const float* x,
                          const int8_t* w, const float* w_scale, int8_t* x_q,
                          float* x_scale, float* y, reef_b200_stream_t stream);

/* reef_kernels::linear_w8a8_bias (kernels.hpp:43-46): as above, then
 * y[r][c] + bias[c]. */
int reef_b200_linear_w8a8_bias(size_t rows, size_t in, size_t out, const float* x,
                               const int8_t* w, const float* w_scale,
                               const float* bias, int8_t* x_q, float* x_scale,
                               float* y, reef_b200_stream_t stream);

/* The GEMM + dequant epilogue of linear_w8a8 on an already quantized input
 * (x_q [rows][kpad(in)], x_scale [rows]); bias may be NULL. */
int reef_b200_gemm_w8a8(size_t rows, size_t in, size_t out, const int8_t* x_q,
                        const float* x_scale, const int8_t* w, const float* w_scale,
                        const float* bias, float* y, reef_b200_stream_t stream);

/* ---- integer-only linear (int8.hpp:74-101) ------------------------------ */

/* reef_kernels::linear_int8 (kernels.hpp:101-103):
 *   y[r][c] = saturate_int8(rounding_shift(sum_k x[r][k] * w[c][k], shift))
 * x [rows][kpad(in)] int8, w [out][kpad(in)], y [rows][out] int8.
 * shift <= 31. */
int reef_b200_linear_int8(size_t rows, size_t in, size_t out, const int8_t* x,
                          const int8_t* w, unsigned shift, int8_t* y,
                          reef_b200_stream_t stream);

/* reef_kernels::linear_bias_int8 (kernels.hpp:106-108): int32 bias[c] added
 * to the sum before the shift. */
int reef_b200_linear_bias_int8(size_t rows, size_t in, size_t out, const int8_t* x,
                               const int8_t* w, const int32_t* bias, unsigned shift,
                               int8_t* y, reef_b200_stream_t stream);

/* matmul<int8, int32> (tensor.hpp:209-246) of a and transpose(b):
 * c[m][n] = sum_k a[m][k] * b[n][k].  a [m][kpad(k)], b [n][kpad(k)],
 * c [m][n] int32.  The partial sums of a row-parallel shard. */
int reef_b200_gemm_i8_i32(size_t m, size_t n, size_t k, const int8_t* a,
                          const int8_t* b, int32_t* c, reef_b200_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* REEF_B200_H */
