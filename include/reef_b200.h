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
  REEF_B200_ERR_UNSUPPORTED = 4, /* current device is not sm_100, or a mode the call does not run */
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
/* Synchronizes the current device, stores its device error word in *code and
 * clears it.  0 = none; otherwise the first error any kernel recorded since
 * the last call:
 *   0x101..0x106  a bounded wait gave up (TMA stage full / empty,
 *                 accumulator full / empty, the MMA drain, a peer's flag);
 *   0x201         a decode or embedding position outside the cache / table;
 *   0x202         a token id outside the vocabulary;
 *   0x301         a float product or sum that is not finite (the engine
 *                 throws std::overflow_error there). */
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

/* Llama pre-norm then int8 (no counterpart in reef, whose GPT-Neo block uses
 * LayerNorm): y = x * gain * r, r = 1 / sqrt(sum(x^2) / width + eps), then
 * reef's quantiser per row (quant.hpp:112-133 on y).  The sum of squares has
 * a fixed order that a tensor-parallel shard reproduces: 8 chunks of width/8
 * columns; in chunk c, 128 partial sums p_i (i < 128) over the float4s
 * i, i + 128, ... of the chunk, each float4 adding ((x0^2 + x1^2) + x2^2) +
 * x3^2; the partials of i in [32w, 32w + 32) reduced by an xor butterfly
 * (offsets 16, 8, 4, 2, 1) to w_w; chunk = ((w_0 + w_1) + w_2) + w_3; total =
 * ((c0 + c1) + (c2 + c3)) + ((c4 + c5) + (c6 + c7)).  max |y| is taken as
 * max |x * gain| * r.  x [rows][width] fp32 (width a multiple of 32),
 * gain [width]; x_q [rows][width] int8, x_scale [rows]. */
int reef_b200_rmsnorm_quant(size_t rows, size_t width, float eps, const float* x,
                            const float* gain, int8_t* x_q, float* x_scale,
                            reef_b200_stream_t stream);

/* Gate/up projection of a SwiGLU MLP with the activation in the GEMM
 * epilogue (no counterpart in reef, whose GPT-Neo MLP is GELU; the Llama
 * layer's MLP uses it):
 *   g = gemm_w8a8(x_q, w_gu rows [0, ffn)),  u = ... rows [ffn, 2 ffn)
 *   h[r][c] = silu(g[r][c]) * u[r][c] = g / (1 + e^-g) * u
 *   row_max[r] = max_c |h[r][c]|   (the scale of the int8 h that follows)
 * x_q [rows][kpad(in)] int8 + x_scale [rows]; w_gu [2*ffn][kpad(in)] int8
 * (gate rows, then up rows) + w_scale [2*ffn]; h [rows][ffn] fp32.  g and u
 * are bit-identical to reef_b200_gemm_w8a8 on the same operands. */
int reef_b200_linear_w8a8_swiglu(size_t rows, size_t in, size_t ffn, const int8_t* x_q,
                                 const float* x_scale, const int8_t* w_gu,
                                 const float* w_scale, float* h, float* row_max,
                                 reef_b200_stream_t stream);

/* reef_b200_linear_w8a8_bias for callers that cannot allocate device memory
 * at all (a host that owns every byte through its own arena, a port of
 * reef's never-allocating Coral firmware, or a latency-critical path that
 * cannot take cudaMalloc's synchronisation).  No counterpart in the
 * reference: reef's kernels take their scratch from the caller.  Same
 * arguments and bit-identical result as reef_b200_linear_w8a8_bias (bias may
 * be NULL), but no scratch arguments: the int8 rows and row scales live in a
 * fixed array of REEF_B200_NOALLOC_SCRATCH_BYTES inside the library, held by
 * every GPU that loads it until the process exits.  Limit:
 *   round_up(rows * reef_b200_kpad(in), 256) + 4 * rows
 *     <= REEF_B200_NOALLOC_SCRATCH_BYTES,
 * else REEF_B200_ERR_TOO_LARGE: at in = 4096, 4092 rows fit and 4093 are
 * refused; at in = 65536, 255 rows fit.  The first call in a CUDA context
 * (normally the device's primary context) looks up the array's device
 * address in that context and caches it under the context's id; make that
 * first call on each device before any stream capture.  Every call shares the array and it keeps the last call's
 * contents, so calls that overlap on the GPU (other streams or host threads
 * on the same device) race: serialise them.  No device memory is allocated. */
#define REEF_B200_NOALLOC_SCRATCH_BYTES (16u << 20)
int reef_b200_linear_w8a8_noalloc(size_t rows, size_t in, size_t out, const float* x,
                                  const int8_t* w, const float* w_scale, const float* bias,
                                  float* y, reef_b200_stream_t stream);

/* The decode layout of a K-major int8 weight w [rows][kpad(in)] (no
 * counterpart in reef): 16 KiB tiles of 128 rows x 128 bytes of K, each stored
 * exactly as the tensor cores read it from shared memory (128-byte swizzle:
 * 16-byte chunk c of tile row r at r * 128 + ((c ^ (r % 8)) * 16)), the tiles
 * of one 128-row block consecutive along K: tile (row block rb, k-block kb)
 * at byte (rb * ceil(in / 128) + kb) * 16384.  Bytes past the matrix are
 * zero.  A decode GEMM (few tokens, the weight on the tensor cores' 128-row
 * side) then reads each of its stages as one contiguous 16 KiB block instead
 * of 128 row pieces of 128 bytes, each kpad(in) bytes apart, which keeps HBM
 * streaming.  tiles: reef_b200_weight_tiles_bytes(rows, in) bytes, 1024-byte
 * aligned. */
size_t reef_b200_weight_tiles_bytes(size_t rows, size_t in);
int reef_b200_pack_weight_tiles(size_t rows, size_t in, const int8_t* w, int8_t* tiles,
                                reef_b200_stream_t stream);

/* The W8A8 GEMM for few rows (decode: one token per sequence, rows <= 128):
 * same result as reef_b200_gemm_w8a8 (bias may be NULL), computed with the
 * weights as the tensor cores' 128-row operand and K split across SMs, so a
 * 64-row GEMM streams its weights on every SM.  The int32 partial sums need
 * reef_b200_gemm_skinny_workspace_bytes(rows, in, out) of scratch. */
size_t reef_b200_gemm_skinny_workspace_bytes(size_t rows, size_t in, size_t out);
int reef_b200_gemm_w8a8_skinny(size_t rows, size_t in, size_t out, const int8_t* x_q,
                               const float* x_scale, const int8_t* w, const float* w_scale,
                               const float* bias, void* workspace, size_t workspace_bytes,
                               float* y, reef_b200_stream_t stream);

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

/* ---- integer softmax and attention (int8.hpp:156-279) ------------------- */

/* reef_kernels::softmax_int8 (kernels.hpp:114-117), batched: each of `rows`
 * rows of n int32 scores -> uint8 probabilities summing to about 255, through
 * a 256-entry exp_table (int8.hpp:156-164; a device pointer). */
int reef_b200_softmax_int8(size_t rows, size_t n, const int32_t* scores, unsigned shift,
                           const uint16_t* table, uint8_t* probs,
                           reef_b200_stream_t stream);

/* reef_kernels::attention_head_int8 (kernels.hpp:122-129) = attend_head_int8
 * (int8.hpp:250-279) with causal_visibility (attention.hpp:82-100):
 * query row i sits at position query_start + i; window 0 = global.
 * q rows are q_stride apart, k/v [key_len][head_dim] contiguous, out rows
 * out_stride apart.  scores/probs are Coral's per-row scratch; the GPU
 * kernel keeps them in shared memory, so they may be NULL.  key_len <= 32768
 * (REEF_B200_ERR_TOO_LARGE beyond).  Every query row must see a key
 * (REEF_B200_ERR_INVALID otherwise, as the engine throws). Bit-identical. */
int reef_b200_attention_head_int8(size_t query_len, size_t key_len, size_t head_dim,
                                  size_t query_start, size_t window, const int8_t* q,
                                  size_t q_stride, const int8_t* k, const int8_t* v,
                                  unsigned score_shift, const uint16_t* table,
                                  unsigned out_shift, int32_t* scores, uint8_t* probs,
                                  int8_t* out, size_t out_stride,
                                  reef_b200_stream_t stream);

/* reef_kernels::attention_head_f32 (kernels.hpp:75-79) = attend_head
 * (attention.hpp:117-123): unscaled float scores, masked softmax with
 * exp_nonpositive and in-order sums, in-order P.V.  Same argument meaning as
 * the int8 head; bit-identical to the engine. */
int reef_b200_attention_head_f32(size_t query_len, size_t key_len, size_t head_dim,
                                 size_t query_start, size_t window, const float* q,
                                 size_t q_stride, const float* k, const float* v,
                                 float* scores, float* out, size_t out_stride,
                                 reef_b200_stream_t stream);

/* Attention::context (attention.hpp:374-432) over `heads` heads in one
 * launch: head h reads q + h*q_head, k + h*kv_head, v + h*kv_head and writes
 * out + h*out_head (strides in elements; key/value rows kv_stride apart).
 * For a [len][d_model] projection split into heads, q_stride = kv_stride =
 * out_stride = d_model and the head strides are head_dim. */
int reef_b200_attention_heads_f32(size_t heads, size_t query_len, size_t key_len,
                                  size_t head_dim, size_t query_start, size_t window,
                                  const float* q, size_t q_stride, size_t q_head,
                                  const float* k, const float* v, size_t kv_stride,
                                  size_t kv_head, float* out, size_t out_stride,
                                  size_t out_head, reef_b200_stream_t stream);

/* The int8 head (reef_b200_attention_head_int8) over `heads` heads in one
 * launch, with the strides of reef_b200_attention_heads_f32. */
int reef_b200_attention_heads_int8(size_t heads, size_t query_len, size_t key_len,
                                   size_t head_dim, size_t query_start, size_t window,
                                   const int8_t* q, size_t q_stride, size_t q_head,
                                   const int8_t* k, const int8_t* v, size_t kv_stride,
                                   size_t kv_head, unsigned score_shift,
                                   const uint16_t* table, unsigned out_shift, int8_t* out,
                                   size_t out_stride, size_t out_head,
                                   reef_b200_stream_t stream);

/* ---- output projection and greedy choice (model.hpp:86-112, 32-42) ------ */

/* matvec_rows_f32 (kernels.hpp:48-52): y[c] = sum over k, in order, of
 * x[k] * w[c][k], for w [out][in] fp32 in its natural layout (GPT-Neo's
 * lm_head reuses the token embedding table this way); reef's float linear
 * (operator/linear.hpp:75-84, tensor.hpp:179-192): each sum starts at 0 and
 * every product and sum is rounded on its own, so y is bit-identical.  A
 * product or sum that is infinite or NaN (the engine throws
 * std::overflow_error, util.hpp:81-131) records 0x301 in the device error
 * word (reef_b200_device_error).  x [in], y [out] fp32. */
int reef_b200_matvec_rows_f32(size_t out, size_t in, const float* w, const float* x, float* y,
                              reef_b200_stream_t stream);
/* argmax_f32 (kernels.hpp:89-90; the engine's argmax, model.hpp:32-42): the
 * index of the first largest of x [n] fp32, written to *index (device
 * uint32).  Ties give the lowest index; a NaN never wins unless it is x[0]
 * (the engine's scan then keeps 0).  n in [1, 2^32 - 1]. */
int reef_b200_argmax_f32(size_t n, const float* x, uint32_t* index, reef_b200_stream_t stream);
/* embedding_f32 (kernels.hpp:81-84; the engine's lookup_token_embeddings +
 * add_position_embeddings, embedding.hpp:31-66) for `count` tokens:
 * y[t][c] = wte[ids[t]][c] + wpe[first_position + t][c], one rounded float
 * add.  ids [count] uint32 on the DEVICE (so a decode loop can feed the
 * previous argmax back without a host round trip); wte [vocab][width], wpe
 * [max_positions][width], y [count][width] fp32.  first_position + count
 * must not pass max_positions (REEF_B200_ERR_INVALID).  An id >= vocab
 * records 0x202 in the device error word and writes that row as zeros; a
 * non-finite sum records 0x301. */
int reef_b200_embedding_f32(size_t width, size_t count, const uint32_t* ids,
                            size_t first_position, size_t vocab, size_t max_positions,
                            const float* wte, const float* wpe, float* y,
                            reef_b200_stream_t stream);

/* ---- the rest of reef's Coral operator set (kernels.hpp:26-146) ---------- */

/* linear_f32 / linear_bias_f32 (kernels.hpp:26-33; the engine's float
 * linear, operator/linear.hpp:75-84): y[r][c] = sum over k, in order from 0,
 * of x[r][k] * wt[k][c], each product and sum rounded on its own, then
 * + bias[c] (bias may be NULL).  wt is the float weight transposed, [in][out]
 * (Coral's layout); x [rows][in], y [rows][out] fp32; rows <= 65535.  A
 * non-finite product or sum records 0x301 in the device error word (the
 * engine throws).  Bit-identical; written for exactness (the float GPT-Neo
 * path), not speed. */
int reef_b200_linear_f32(size_t rows, size_t in, size_t out, const float* x, const float* wt,
                         float* y, reef_b200_stream_t stream);
int reef_b200_linear_bias_f32(size_t rows, size_t in, size_t out, const float* x,
                              const float* wt, const float* bias, float* y,
                              reef_b200_stream_t stream);
/* layernorm_f32 (kernels.hpp:55-56; operator/layernorm.hpp:62-80): per row,
 * in-order mean and variance, y = ((x - mean) * inv_std) * gain + shift
 * (shift may be NULL).  x, y [rows][width] fp32.  Bit-identical. */
int reef_b200_layernorm_f32(size_t rows, size_t width, const float* x, const float* gain,
                            const float* shift, float eps, float* y, reef_b200_stream_t stream);
/* gelu_f32, exp_nonpositive_f32, tanh_f32 (kernels.hpp:59-64; activation.hpp:
 * 78-90, math.hpp:34-81), elementwise over n floats.  Bit-identical. */
int reef_b200_gelu_f32(size_t n, const float* x, float* y, reef_b200_stream_t stream);
int reef_b200_exp_nonpositive_f32(size_t n, const float* x, float* y,
                                  reef_b200_stream_t stream);
int reef_b200_tanh_f32(size_t n, const float* x, float* y, reef_b200_stream_t stream);
/* add_f32 (kernels.hpp:86-87): y = a + b, one rounded add per element; a
 * non-finite sum records 0x301. */
int reef_b200_add_f32(size_t n, const float* a, const float* b, float* y,
                      reef_b200_stream_t stream);
/* gelu_int8 (kernels.hpp:111-112; int8.hpp:135-147): y[i] = table[x[i] + 128]
 * for a 256-entry int8 table (gelu_table) in device memory. */
int reef_b200_gelu_int8(size_t n, const int8_t* x, const int8_t* table, int8_t* y,
                        reef_b200_stream_t stream);
/* layernorm_int8 (kernels.hpp:132-134; int8.hpp:319-374): per row mean =
 * floor(sum / width), std = isqrt(sum((x - mean)^2) / width), inv = 2^20 /
 * max(std, 1), y = sat8(rshift_rnu(((x - mean) * inv >> 16) * gain +
 * shift * 32, 5)).  width <= 32767 (the engine's int32 sum of squares).
 * Bit-identical. */
int reef_b200_layernorm_int8(size_t rows, size_t width, const int8_t* x, const int8_t* gain,
                             const int8_t* shift, int8_t* y, reef_b200_stream_t stream);
/* add_int8 (kernels.hpp:137-138; int8.hpp:382-397): y = sat8(a + b). */
int reef_b200_add_int8(size_t n, const int8_t* a, const int8_t* b, int8_t* y,
                       reef_b200_stream_t stream);
/* embedding_int8 (kernels.hpp:142-145) for `count` tokens: y[t][c] =
 * sat8(wte[ids[t]][c] + wpe[first_position + t][c]); ids on the device, the
 * same checks and error words as reef_b200_embedding_f32. */
int reef_b200_embedding_int8(size_t width, size_t count, const uint32_t* ids,
                             size_t first_position, size_t vocab, size_t max_positions,
                             const int8_t* wte, const int8_t* wpe, int8_t* y,
                             reef_b200_stream_t stream);

/* ---- int8 flash attention (the fast head) ------------------------------- */

/* Packs one QKV projection output for the flash head.  qkv [batch*seq]
 * [(heads_q + 2*heads_kv) * 128] fp32 rows (q heads, then k, then v).  q and
 * k get Llama rotate-half RoPE (theta_i = pos * rope_base^(-2i/128), pos =
 * token index within its sequence); then every (token, head) row of 128 is
 * quantised with reef's rule (quant.hpp:51-81: scale = max|x|/127, rne,
 * clamp +-127).  Outputs: q8 [tokens][heads_q*128], k8 and v8
 * [tokens][heads_kv*128] (the int8 KV-cache rows), scales [batch][heads][seq],
 * and vt [batch][heads_kv][128][seq] f16 holding the dequantised values
 * f16(v8 code * v_scale) transposed (the operand layout of the P.V
 * tensor-core product).  head_dim is 128 and seq even.  RoPE and this scale
 * granularity are not in reef (parity unpinned there). */
int reef_b200_rope_qkv_quant(size_t batch, size_t seq, size_t heads_q, size_t heads_kv,
                             float rope_base, const float* qkv, int8_t* q8, int8_t* k8,
                             int8_t* v8, float* q_scale, float* k_scale, float* v_scale,
                             void* vt, reef_b200_stream_t stream);

/* The QKV projection and reef_b200_rope_qkv_quant in one pass: the W8A8
 * GEMM (as reef_b200_gemm_w8a8, no bias) of x_q [batch*seq][kpad(in)] +
 * x_scale by w_qkv [(heads_q + 2*heads_kv)*128][kpad(in)] + w_scale, and in
 * its epilogue, per (token, head), the RoPE and int8 packing of
 * reef_b200_rope_qkv_quant: bit-identical outputs, without the fp32
 * projection ever reaching memory.  v8 and v_scale may be NULL (the flash
 * head reads only vt).  rope_table: [64][seq] float2 scratch (seq * 512
 * bytes).  seq must be even. */
int reef_b200_linear_w8a8_qkv_rope(size_t batch, size_t seq, size_t in, size_t heads_q,
                                   size_t heads_kv, float rope_base, const int8_t* x_q,
                                   const float* x_scale, const int8_t* w_qkv,
                                   const float* w_scale, int8_t* q8, int8_t* k8, int8_t* v8,
                                   float* q_scale, float* k_scale, float* v_scale, void* vt,
                                   void* rope_table, reef_b200_stream_t stream);

/* Failure-detection self-test (no counterpart in reef): launches one thread
 * that waits, with the library's bounded mbarrier wait but a limit of
 * limit_us microseconds (1 .. 2e6), on a barrier nothing completes.  The wait
 * gives up, records its timeout code (0x101) in the device error word that
 * reef_b200_device_error returns, and the kernel exits normally; *done
 * (device int) becomes 2 (1 would mean the wait was satisfied).  The device
 * stays usable. */
int reef_b200_selftest_wait_timeout(unsigned limit_us, int* done, reef_b200_stream_t stream);

/* Failure-detection self-test of the cross-rank wait (no counterpart in
 * reef): runs the wait the pipelined tensor-parallel forward puts before a
 * step, on one device counter (a device unsigned int the caller owns), with
 * a limit of limit_us microseconds (1 .. 2e6): the wait ends when *counter
 * reaches target (wrap-around >=, as the forward's counters only grow), or
 * after the limit, when it records 0x106 (a peer never signalled) in the
 * device error word and returns.  While the error word holds 0x106 (until
 * reef_b200_device_error reads it), a wait returns at once: a rank that lost
 * a peer pays one limit, not one per step.  A counter nothing increments is
 * how a dead peer looks to this rank; the device stays usable. */
int reef_b200_selftest_peer_wait_timeout(unsigned limit_us, const unsigned* counter,
                                         unsigned target, reef_b200_stream_t stream);

/* Flash attention over int8 q / k and f16 v (attend_head,
 * attention.hpp:117-123, on the dequantised values, with score scale
 * sm_scale and GQA: query head h reads kv head h / (heads_q / heads_kv)).
 * q8 / k8 with their per-(token, head) scales as reef_b200_rope_qkv_quant
 * writes them; vt [batch][heads_kv][128][seq] f16 is the dequantised v,
 * transposed (reef_b200_rope_qkv_quant's vt).  causal != 0 applies
 * causal_visibility with query_start 0.  out [batch*seq][heads_q*128] fp32.
 * head_dim must be 128, seq a multiple of 8 and k_scale 16-byte aligned.
 * Matches reef's float head on the dequantised inputs within 1e-2 (fp32
 * online softmax, f16 P). */
int reef_b200_flash_attn_i8(size_t batch, size_t seq, size_t heads_q, size_t heads_kv,
                            size_t head_dim, int causal, float sm_scale, const int8_t* q8,
                            const float* q_scale, const int8_t* k8, const float* k_scale,
                            const void* vt, float* out, reef_b200_stream_t stream);

/* Decode: one new query per sequence against an int8 KV cache (BASELINE
 * config 4).  attend_head (attention.hpp:117-123) for the query at the last
 * cached position (it sees every cached key), on the dequantised int8
 * q / k / v, score scale sm_scale, GQA (query head h reads kv head
 * h / (heads_q / heads_kv); heads_q / heads_kv in {1, 2, 4, 8, 16}).
 * q8 [batch][heads_q][128] + q_scale [batch][heads_q]; k_cache / v_cache
 * [batch][heads_kv][max_len][128] int8 (16-byte aligned) + k_scale / v_scale
 * [batch][heads_kv][max_len] fp32; lens [batch] int32 on the device (each in
 * [1, max_len]) or NULL for `len` keys in every sequence.  max_len must be
 * a multiple of 4 and the caches and scales 16-byte aligned (they are read
 * by bulk copies).  Split across CTAs along the keys (flash-decoding); the
 * partial results need
 * reef_b200_decode_attn_workspace_bytes() of scratch.  out
 * [batch][heads_q][128] fp32.  Within 1e-2 of the float head. */
size_t reef_b200_decode_attn_workspace_bytes(size_t batch, size_t heads_q, size_t max_len);
int reef_b200_decode_attn_i8(size_t batch, size_t heads_q, size_t heads_kv, size_t head_dim,
                             size_t max_len, const int32_t* lens, size_t len, float sm_scale,
                             const int8_t* q8, const float* q_scale, const int8_t* k_cache,
                             const float* k_scale, const int8_t* v_cache, const float* v_scale,
                             void* workspace, size_t workspace_bytes, float* out,
                             reef_b200_stream_t stream);

/* ---- tensor parallelism (new: reef runs on one core) -------------------- */

/* One communicator per rank (one process or host thread per GPU, over NCCL
 * on NVLink).  Rank 0 makes an id (reef_b200_comm_unique_id_bytes() bytes),
 * the host shares it with the other ranks, every rank calls
 * reef_b200_comm_init with the current device set.  Init is non-blocking
 * internally: when a rank never joins, it returns REEF_B200_ERR_TIMEOUT
 * after timeout_s seconds (<= 0: 60 s) instead of hanging. */
typedef struct reef_b200_comm reef_b200_comm;
size_t reef_b200_comm_unique_id_bytes(void);
int reef_b200_comm_unique_id(void* id, size_t bytes);
int reef_b200_comm_init(int rank, int world, const void* id, double timeout_s,
                        reef_b200_comm** comm);
/* Finalizes and frees; collective (every rank calls it).  When a pipelined
 * forward has made the peer-mapped arena, the ranks first drop their
 * mappings and meet at a barrier, so no rank frees memory a peer still maps.
 * REEF_B200_ERR_TIMEOUT (and an abort) when peers stall past the timeout. */
int reef_b200_comm_destroy(reef_b200_comm* comm);
/* Frees without waiting for peers (after a peer failed). */
int reef_b200_comm_abort(reef_b200_comm* comm);

/* Megatron row-parallel W8A8 linear: linear() (operator/linear.hpp:106-134)
 * with x split by columns (K) and W by input features across the ranks of
 * `comm`.  x_local [rows][in_local] (this rank's K-slice), w_shard
 * [out][kpad(in_local)], w_scale [out], bias [out] or NULL (added once).
 * Each rank quantises its slice with the FULL row's scale (all-reduce MAX of
 * row maxima), multiplies in int32, all-reduces the int32 partial sums (SUM,
 * exact) and dequantises: y [rows][out], identical on every rank and
 * bit-identical to reef_b200_linear_w8a8_bias on the unsplit x and W.
 * Scratch: x_q [rows][kpad(in_local)], x_scale [rows], row_max [rows], acc
 * [rows][out] int32 (row_max / acc may be NULL when comm is NULL).  The
 * column-parallel form needs no collective: it is reef_b200_linear_w8a8 on
 * the rank's rows of W. */
int reef_b200_linear_w8a8_rowpar(reef_b200_comm* comm, size_t rows, size_t in_local,
                                 size_t out, const float* x_local, const int8_t* w_shard,
                                 const float* w_scale, const float* bias, int8_t* x_q,
                                 float* x_scale, float* row_max, int32_t* acc, float* y,
                                 reef_b200_stream_t stream);

/* ---- decoder layers ------------------------------------------------------- */

/* One Llama-shape W8A8 decoder layer (BASELINE configs 3 and 4 shapes) on
 * this rank's shard: pre-RMSNorm, column-parallel QKV, rotate-half RoPE,
 * causal int8 flash attention, row-parallel o_proj + residual, pre-RMSNorm,
 * column-parallel gate/up, SwiGLU, row-parallel down + residual.  Every
 * projection is reef's W8A8 linear (per-token activation scale, per-channel
 * weight scale, int32 accumulation).  RMSNorm, RoPE and SwiGLU are not in
 * reef (parity unpinned; see the GPT-Neo block below for the pinned one).
 * Weights are this rank's shards, K-major; scales fp32.  Sizes are local
 * (heads_q, heads_kv, ffn = totals / TP degree); hidden is the full width. */
typedef struct reef_b200_llama_layer {
  size_t batch, seq;         /* tokens = batch * seq <= 2^30; seq % 8 == 0 */
  size_t hidden;             /* model width, multiple of 16, <= 2^20 */
  size_t heads_q, heads_kv;  /* this rank's heads, <= 4096 each */
  size_t head_dim;           /* 128 */
  size_t ffn;                /* this rank's FFN width, multiple of 16, <= 2^22 */
  float rms_eps, rope_base;
  const float* attn_norm;                       /* [hidden] */
  const int8_t* w_qkv; const float* s_qkv;      /* [(heads_q+2 heads_kv)*128][hidden] */
  const int8_t* w_o; const float* s_o;          /* [hidden][heads_q*128] */
  const float* mlp_norm;                        /* [hidden] */
  const int8_t* w_gu; const float* s_gu;        /* [2 ffn][hidden]: gate, then up */
  const int8_t* w_down; const float* s_down;    /* [hidden][ffn] */
  reef_b200_comm* comm;                         /* NULL: TP = 1 */
  int tp_mode;  /* with comm: REEF_B200_TP_ALLREDUCE or REEF_B200_TP_ALLGATHER */
  /* Optional, for the decode step (NULL: the K-major weights above are read):
   * w_qkv, w_o, w_gu and w_down again in the layout reef_b200_pack_weight_tiles
   * writes (1024-byte aligned), which the decode step's GEMMs stream as
   * contiguous 16 KiB blocks. */
  const int8_t* t_qkv;
  const int8_t* t_o;
  const int8_t* t_gu;
  const int8_t* t_down;
} reef_b200_llama_layer;

/* Two tensor-parallel plans for the Llama layer (both bit-identical to TP=1):
 *  REEF_B200_TP_ALLREDUCE  Megatron: x and y replicated; q/k/v and gate/up
 *    column-parallel; o-proj and down row-parallel (w_o [hidden][heads_q*128],
 *    w_down [hidden][ffn] = this rank's input features), their int32 partial
 *    sums all-reduced.
 *  REEF_B200_TP_ALLGATHER  every projection column-parallel on all-gathered
 *    int8 activations (quantised with the full row's scale first): x and y are
 *    this rank's hidden/world columns [tokens][hidden/world]; w_o
 *    [hidden/world][hidden_q] and w_down [hidden/world][ffn_total] are this
 *    rank's OUTPUT rows over the full K.  Moves int8 activations instead of
 *    int32 partial sums (about a third of the bytes) and shards every
 *    element-wise step.  world must divide 8.  When the batch splits into 2
 *    groups of whole sequences, the forward pipelines over them on the
 *    communicator's compute streams, one group a step behind the other; the
 *    kernels that produce exchanged data write it into every rank's memory
 *    over NVLink, and counters in a symmetric arena say when it has arrived
 *    and been consumed; each wait on them is a spin on the device with the
 *    communicator's timeout (same result; `stream` still orders everything
 *    before the call's last kernel). */
#define REEF_B200_TP_ALLREDUCE 0
#define REEF_B200_TP_ALLGATHER 1

/* Bytes of device workspace reef_b200_llama_layer_forward needs (0 when the
 * description is invalid). */
size_t reef_b200_llama_layer_workspace_bytes(const reef_b200_llama_layer* layer);
/* y [tokens][hidden] = layer(x [tokens][hidden]); fp32; y may not alias x.
 * workspace: 256-byte aligned device memory of at least the queried size. */
int reef_b200_llama_layer_forward(const reef_b200_llama_layer* layer, const float* x,
                                  float* y, void* workspace, size_t workspace_bytes,
                                  reef_b200_stream_t stream);

/* Kernels one reef_b200_llama_layer_forward launches (for launch accounting). */
size_t reef_b200_llama_layer_kernel_launches(const reef_b200_llama_layer* layer);
/* reef_b200_llama_layer_forward that also records 10 caller-created CUDA
 * events (cudaEvent_t, timing enabled) on `stream`: begin/end of the QKV
 * GEMM, the flash kernel, the o-proj GEMM, the gate/up GEMM and the down
 * GEMM, in that order (for per-kernel timing in a live run).  The steps run
 * in sequence on `stream` (the all-gather plan is not pipelined here). */
int reef_b200_llama_layer_forward_events(const reef_b200_llama_layer* layer, const float* x,
                                         float* y, void* workspace, size_t workspace_bytes,
                                         void* const* events, reef_b200_stream_t stream);

/* One decode step of the same layer: `batch` sequences
 * (layer->batch, <= 128; layer->seq is ignored) each add one token.  x / y
 * [batch][hidden] fp32.  positions [batch] int32 (device): the new token's
 * position in its sequence; its rotated k and its v are quantised per head
 * and appended to the int8 cache at that row, then the query attends over
 * rows [0, position].  Caches: k_cache / v_cache [batch][heads_kv][max_len]
 * [128] int8 (16-byte aligned), k_scale / v_scale [batch][heads_kv][max_len]
 * fp32 (one scale per token and head).  Every projection uses the skinny
 * W8A8 GEMM; the row-parallel ones all-reduce exactly as in the prefill
 * layer, so every rank's y is bit-identical to TP=1. */
size_t reef_b200_llama_decode_workspace_bytes(const reef_b200_llama_layer* layer,
                                              size_t max_len);
int reef_b200_llama_decode_forward(const reef_b200_llama_layer* layer, const float* x, float* y,
                                   const int32_t* positions, int8_t* k_cache, float* k_scale,
                                   int8_t* v_cache, float* v_scale, size_t max_len,
                                   void* workspace, size_t workspace_bytes,
                                   reef_b200_stream_t stream);

/* reef's GPT-Neo W8A8 block, Block<float>::forward (operator/block.hpp:97-108)
 * on `seq` positions of an empty cache (BASELINE configs 1 and 2): LayerNorm,
 * q/k/v W8A8 projections (no bias), reef's float head per head (unscaled,
 * causal, window 0 = global), o_proj + bias + residual, LayerNorm, c_fc +
 * bias, tanh GELU, c_proj + bias + residual.  Bit-identical to the engine at
 * every TP degree.  heads / ffn are this rank's (column-parallel q/k/v by
 * heads and c_fc by columns; row-parallel o_proj and c_proj). */
typedef struct reef_b200_gptneo_block {
  size_t seq, hidden, heads, head_dim, ffn, window;  /* hidden <= 2^20, heads and
                                                       head_dim <= 4096, ffn <= 2^22 */
  float eps;
  const float* ln1_g; const float* ln1_b;       /* [hidden] */
  const int8_t* wq; const float* sq;            /* [heads*head_dim][hidden] */
  const int8_t* wk; const float* sk;
  const int8_t* wv; const float* sv;
  const int8_t* wo; const float* so; const float* bo;            /* [hidden][heads*head_dim] */
  const float* ln2_g; const float* ln2_b;
  const int8_t* wfc; const float* sfc; const float* bfc;         /* [ffn][hidden] */
  const int8_t* wproj; const float* sproj; const float* bproj;   /* [hidden][ffn] */
  reef_b200_comm* comm;                                          /* NULL: TP = 1 */
} reef_b200_gptneo_block;

size_t reef_b200_gptneo_block_workspace_bytes(const reef_b200_gptneo_block* block);
int reef_b200_gptneo_block_forward(const reef_b200_gptneo_block* block, const float* x,
                                   float* y, void* workspace, size_t workspace_bytes,
                                   reef_b200_stream_t stream);
/* The same block on `seq` new positions [position, position + seq) of a
 * cache that holds the earlier ones (Attention::forward with a KV cache,
 * attention.hpp:290-372; the firmware's per-layer step, gpt_neo.cc:136-176):
 * the projected keys and values are written into k_cache / v_cache rows
 * [position, position + seq) and every query attends over cache rows
 * [0, position + its offset] (window as the block's).  The caches are this
 * layer's [max_tokens][heads*head_dim] fp32, token-major (a projection's
 * output rows land in place).  position + seq <= max_tokens.  Prefill and
 * decode give the same bits (a prompt run at once or one token at a time).
 * Workspace: reef_b200_gptneo_block_workspace_bytes. */
int reef_b200_gptneo_block_forward_cached(const reef_b200_gptneo_block* block, const float* x,
                                          float* y, size_t position, float* k_cache,
                                          float* v_cache, size_t max_tokens, void* workspace,
                                          size_t workspace_bytes, reef_b200_stream_t stream);

/* ---- GPT-Neo decode loop (the firmware's GptNeo::step) ------------------ */

/* A float GPT-Neo block (the firmware's kFloat32 layers, gpt_neo.cc:100-121
 * through linear_f32 / linear_bias_f32): weights in Coral's [in][out]
 * layout, fp32; TP = 1.  Run by reef_b200_gptneo_step (every operator the
 * engine's float Block<float>::forward uses, bit for bit). */
typedef struct reef_b200_gptneo_block_f32 {
  size_t seq, hidden, heads, head_dim, ffn, window;
  float eps;
  const float* ln1_g; const float* ln1_b;       /* [hidden] */
  const float* wq; const float* wk; const float* wv;   /* [hidden][heads*head_dim] */
  const float* wo; const float* bo;             /* [heads*head_dim][hidden], [hidden] */
  const float* ln2_g; const float* ln2_b;
  const float* wfc; const float* bfc;           /* [hidden][ffn], [ffn] */
  const float* wproj; const float* bproj;       /* [ffn][hidden], [hidden] */
} reef_b200_gptneo_block_f32;

/* A whole GPT-Neo model: the token and position tables, the final LayerNorm
 * and `layers` blocks -- W8A8 (`blocks`) or float (`blocks_f32`, the other
 * NULL), a HOST array whose seq fields are ignored.  wte doubles as the tied
 * lm_head. */
typedef struct reef_b200_gptneo_model {
  size_t vocab, max_positions, hidden, layers;
  float eps;
  const float* wte;      /* [vocab][hidden] */
  const float* wpe;      /* [max_positions][hidden] */
  const float* ln_f_g;   /* [hidden] */
  const float* ln_f_b;
  const reef_b200_gptneo_block* blocks;
  const reef_b200_gptneo_block_f32* blocks_f32;
} reef_b200_gptneo_model;

/* Workspace for reef_b200_gptneo_step on up to `count` tokens at once. */
size_t reef_b200_gptneo_step_workspace_bytes(const reef_b200_gptneo_model* model, size_t count);
/* GptNeo::step (coral/firmware/gpt_neo.cc:123-188), W8A8 or float, for
 * `count` tokens at once: ids [count] (device uint32) at positions
 * [position, position +
 * count) go through the embedding and every block, appending their keys and
 * values to the caches; then, for the last token, ln_f, the tied lm_head
 * (logits [vocab], when not NULL) and the greedy choice (*next_id, device
 * uint32, when not NULL).  With both NULL only the caches advance (the
 * firmware's want_logits = false).  k_cache and v_cache are [layers]
 * [max_tokens][heads*head_dim] fp32; position + count <= max_tokens <=
 * max_positions.  A prompt may go in at once (count = its length) or a
 * token at a time: the logits are the same bits, and equal the engine's
 * GPTNeo<float> forward at that precision.  Feeding next_id back as the next call's ids
 * makes a generation loop with no host round trip (capturable in a CUDA
 * graph for a fixed position). */
int reef_b200_gptneo_step(const reef_b200_gptneo_model* model, const uint32_t* ids,
                          size_t count, size_t position, float* k_cache, float* v_cache,
                          size_t max_tokens, float* logits, uint32_t* next_id, void* workspace,
                          size_t workspace_bytes, reef_b200_stream_t stream);

/* ---- reef's packed model ("REEF" blob v1, model_blob.hpp:18-66) --------- */

/* The header of a blob written by reef's packer (coral/host/pack_model.hpp:
 * 88-160).  precision: 0 float, 1 W8A8 (model_blob.hpp:23-26); wte, wpe,
 * ln_f_weight, ln_f_bias: byte offsets of those float arrays in the blob
 * ([vocab][hidden], [max_positions][hidden], [hidden], [hidden]); the token
 * embedding rows are also the tied lm_head (reef_b200_matvec_rows_f32). */
typedef struct reef_b200_blob_info {
  uint32_t precision;
  size_t vocab, max_positions, hidden, layers, heads, inner, window;
  float eps;
  size_t wte, wpe, ln_f_weight, ln_f_bias;
} reef_b200_blob_info;
/* Validates a blob in HOST memory (magic "REEF", version 1, every array
 * inside total_bytes <= bytes and 16-byte aligned) and reads its header.
 * Needs no GPU.  REEF_B200_ERR_INVALID for a malformed blob. */
int reef_b200_blob_read_info(const void* blob, size_t bytes, reef_b200_blob_info* info);
/* Device bytes one layer takes in reef_b200_blob_load_layer's arena. */
size_t reef_b200_blob_layer_bytes(const reef_b200_blob_info* info);
/* Copies layer `layer` of a W8A8 blob (host memory) into `arena` (device,
 * 256-byte aligned, >= reef_b200_blob_layer_bytes), repacking every [in][out]
 * int8 weight into the K-major [out][kpad(in)] layout, and fills the
 * block's weights and shape (heads, head_dim, ffn, window: the blob's window
 * for a local layer, 0 for a global one; eps); seq and comm are the
 * caller's.  A float blob is REEF_B200_ERR_UNSUPPORTED (these kernels run
 * W8A8 blocks).  Asynchronous on `stream`: a blob in page-locked memory must
 * stay unchanged until the stream has passed this call (pageable memory is
 * staged before the call returns). */
int reef_b200_blob_load_layer(const void* blob, size_t bytes, size_t layer, void* arena,
                              size_t arena_bytes, reef_b200_gptneo_block* block,
                              reef_b200_stream_t stream);
/* Device bytes a whole model (either precision) takes in
 * reef_b200_blob_load_model's arena. */
size_t reef_b200_blob_model_bytes(const reef_b200_blob_info* info);
/* Loads a whole blob (the firmware's GptNeo constructor, gpt_neo.cc:61-97,
 * which reads the blob in place): the tables, ln_f and every layer into
 * `arena` (device, 256-byte aligned, >= reef_b200_blob_model_bytes), and
 * fills `model`.  A W8A8 blob fills `blocks` (a host array of info.layers;
 * weights repacked K-major), a float blob `blocks_f32` (weights kept
 * [in][out]); the array of the other precision may be NULL.  Errors and
 * asynchrony as reef_b200_blob_load_layer. */
int reef_b200_blob_load_model(const void* blob, size_t bytes, void* arena, size_t arena_bytes,
                              reef_b200_gptneo_model* model, reef_b200_gptneo_block* blocks,
                              reef_b200_gptneo_block_f32* blocks_f32,
                              reef_b200_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* REEF_B200_H */
