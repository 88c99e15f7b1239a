// attention_exact.cu -- reef's two attention heads, bit for bit.
//
//  * attention_head_int8: attend_head_int8 (int8.hpp:250-279) with
//    masked_softmax_int8 (int8.hpp:180-232).  Integer only: int32 q.k scores,
//    uint16 table weights, uint8 probabilities, int32 p.v, then
//    saturate_int8(rounding_shift(., out_shift)).  Integer sums are
//    order-free, so any reduction order reproduces the engine.
//  * attention_head_f32: attend_head (attention.hpp:117-123) with
//    masked_softmax (activation.hpp:166-231).  Float sums are NOT order-free,
//    so every sum here runs in the engine's order on one thread: a score is
//    one thread's in-order dot product, the softmax denominator is one
//    thread's in-order sum over the visible keys, each output column is one
//    thread's in-order sum over keys; exp is exp_nonpositive (math.hpp:34-71)
//    in single IEEE steps.  This is the parity kernel for the float head;
//    the fast head is the flash kernel.
//
// Visibility is causal_visibility (attention.hpp:82-100): query row i at
// position query_start + i sees keys [first, end) with
// end = min(pos + 1, key_len), first = pos + 1 - window when window > 0 and
// pos + 1 > window, else 0.  Masked keys have probability 0 and contribute
// nothing, so only [first, end) is visited (as the Coral kernels do,
// coral/kernels/attention.cc:1-6).
//
// One CTA per (query row, head).  Scores live in shared memory (no scratch),
// which bounds key_len at kMaxKeysExact.
#include "common.cuh"
#include "ops.h"

namespace reef {

namespace {

constexpr int kHeadThreads = 256;

__device__ __forceinline__ void visible(long long query_start, int i, int key_len,
                                        int window, int& first, int& end) {
  const long long pos = query_start + i;
  end = static_cast<int>(pos + 1 < key_len ? pos + 1 : key_len);
  first = (window > 0 && pos + 1 > window) ? static_cast<int>(pos + 1 - window) : 0;
}

template <typename T>
__device__ __forceinline__ T block_reduce(T v, T* red, bool is_max) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const T w = __shfl_xor_sync(0xffffffffu, v, o);
    v = is_max ? (w > v ? w : v) : v + w;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    v = lane < nw ? red[lane] : red[0];
    if (!is_max && lane >= nw) v = 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const T w = __shfl_xor_sync(0xffffffffu, v, o);
      v = is_max ? (w > v ? w : v) : v + w;
    }
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  const T r = red[0];
  __syncthreads();
  return r;
}

// blockIdx.x = query row, blockIdx.y = head (tensors offset by head strides)
__global__ void __launch_bounds__(kHeadThreads)
    head_int8_kernel(int key_len, int head_dim, long long query_start, int window,
                     const int8_t* __restrict__ q, long long q_stride, long long q_head,
                     const int8_t* __restrict__ k, const int8_t* __restrict__ v,
                     long long kv_stride, long long kv_head, uint32_t score_shift,
                     const uint16_t* __restrict__ table_g, uint32_t out_shift,
                     int8_t* __restrict__ out, long long out_stride, long long out_head) {
  extern __shared__ uint8_t sm[];
  __shared__ uint16_t table[256];
  __shared__ int32_t red_i[32];
  __shared__ uint32_t red_u[32];
  __shared__ int32_t part[kHeadThreads];
  int32_t* scores = reinterpret_cast<int32_t*>(sm);
  uint8_t* probs = sm + static_cast<size_t>(key_len) * 4;

  const int i = blockIdx.x;
  const int h = blockIdx.y;
  q += h * q_head + static_cast<long long>(i) * q_stride;
  k += h * kv_head;
  v += h * kv_head;
  out += h * out_head + static_cast<long long>(i) * out_stride;
  for (int t = threadIdx.x; t < 256; t += blockDim.x) table[t] = table_g[t];
  int first, end;
  visible(query_start, i, key_len, window, first, end);

  // scores[j] = q . k[j] (int32)
  int32_t mx = INT32_MIN;
  for (int j = first + threadIdx.x; j < end; j += blockDim.x) {
    const int8_t* kj = k + static_cast<long long>(j) * kv_stride;
    int32_t s = 0;
    for (int d = 0; d < head_dim; ++d) s += static_cast<int32_t>(q[d]) * kj[d];
    scores[j] = s;
    mx = s > mx ? s : mx;
  }
  mx = block_reduce<int32_t>(mx, red_i, true);

  // weights = table[min((max - s) >> shift, 255)], sum (uint32)
  uint32_t sum = 0;
  for (int j = first + threadIdx.x; j < end; j += blockDim.x) {
    uint32_t d = static_cast<uint32_t>((mx - scores[j]) >> static_cast<int32_t>(score_shift));
    sum += table[d < 255u ? d : 255u];
  }
  sum = block_reduce<uint32_t>(sum, red_u, false);
  const uint32_t reciprocal = (255u << 16) / sum;  // the max's weight is 32768
  for (int j = first + threadIdx.x; j < end; j += blockDim.x) {
    uint32_t d = static_cast<uint32_t>((mx - scores[j]) >> static_cast<int32_t>(score_shift));
    const uint32_t scaled = static_cast<uint32_t>(table[d < 255u ? d : 255u]) * reciprocal;
    const uint32_t rounded = (scaled >> 16) + ((scaled >> 15) & 1u);
    probs[j] = static_cast<uint8_t>(rounded < 255u ? rounded : 255u);
  }
  __syncthreads();

  // out[c] = sat8(rshift(sum_j p[j] * v[j][c], out_shift)); warps split keys,
  // lanes split columns; int32 partials reduced through shared memory.
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nw = blockDim.x >> 5;
  for (int c0 = 0; c0 < head_dim; c0 += 32) {
    const int c = c0 + lane;
    int32_t acc = 0;
    if (c < head_dim) {
      for (int j = first + warp; j < end; j += nw)
        acc += static_cast<int32_t>(probs[j]) * v[static_cast<long long>(j) * kv_stride + c];
    }
    part[warp * 32 + lane] = acc;
    __syncthreads();
    if (warp == 0 && c < head_dim) {
      int32_t s = 0;
      for (int w = 0; w < nw; ++w) s += part[w * 32 + lane];
      out[c] = requant_rnu_sat8(s, out_shift);
    }
    __syncthreads();
  }
}

// exp_nonpositive (math.hpp:34-71), each step one IEEE operation.
__device__ __forceinline__ float exp_nonpositive(float x) {
  if (x < -87.0f) return 0.0f;
  const float kf = __fsub_rn(__fadd_rn(__fmul_rn(x, 1.44269504088896341f), 12582912.0f),
                             12582912.0f);
  const float r = __fsub_rn(__fsub_rn(x, __fmul_rn(kf, 0.693359375f)),
                            __fmul_rn(kf, -2.12194440e-4f));
  const float r2 = __fmul_rn(r, r);
  float p = 1.9875691500E-4f;
  p = __fadd_rn(__fmul_rn(p, r), 1.3981999507E-3f);
  p = __fadd_rn(__fmul_rn(p, r), 8.3334519073E-3f);
  p = __fadd_rn(__fmul_rn(p, r), 4.1665795894E-2f);
  p = __fadd_rn(__fmul_rn(p, r), 1.6666665459E-1f);
  p = __fadd_rn(__fmul_rn(p, r), 5.0000001201E-1f);
  p = __fadd_rn(__fadd_rn(__fmul_rn(p, r2), r), 1.0f);
  const float scale = __int_as_float((static_cast<int>(kf) + 127) << 23);
  return __fmul_rn(p, scale);
}

__global__ void __launch_bounds__(kHeadThreads)
    head_f32_kernel(int key_len, int head_dim, long long query_start, int window,
                    const float* __restrict__ q, long long q_stride, long long q_head,
                    const float* __restrict__ k, const float* __restrict__ v,
                    long long kv_stride, long long kv_head, float* __restrict__ out,
                    long long out_stride, long long out_head) {
  extern __shared__ uint8_t sm[];
  __shared__ float red[32];
  __shared__ float total;
  float* p = reinterpret_cast<float*>(sm);
  const int i = blockIdx.x;
  const int h = blockIdx.y;
  q += h * q_head + static_cast<long long>(i) * q_stride;
  k += h * kv_head;
  v += h * kv_head;
  out += h * out_head + static_cast<long long>(i) * out_stride;
  int first, end;
  visible(query_start, i, key_len, window, first, end);

  // in-order dot products (matrix_dot_product, tensor.hpp:178-192)
  float mx = -INFINITY;
  for (int j = first + threadIdx.x; j < end; j += blockDim.x) {
    const float* kj = k + static_cast<long long>(j) * kv_stride;
    float s = 0.0f;
    for (int d = 0; d < head_dim; ++d) s = __fadd_rn(s, __fmul_rn(q[d], kj[d]));
    p[j] = s;
    mx = fmaxf(mx, s);
  }
  mx = block_reduce<float>(mx, red, true);
  for (int j = first + threadIdx.x; j < end; j += blockDim.x)
    p[j] = exp_nonpositive(__fsub_rn(p[j], mx));
  __syncthreads();
  if (threadIdx.x == 0) {  // the engine's in-order sum (activation.hpp:210-221)
    float s = 0.0f;
    for (int j = first; j < end; ++j) s = __fadd_rn(s, p[j]);
    total = s;
  }
  __syncthreads();
  const float sum = total;
  for (int j = first + threadIdx.x; j < end; j += blockDim.x) p[j] = __fdiv_rn(p[j], sum);
  __syncthreads();
  for (int c = threadIdx.x; c < head_dim; c += blockDim.x) {
    float s = 0.0f;
    for (int j = first; j < end; ++j)
      s = __fadd_rn(s, __fmul_rn(p[j], v[static_cast<long long>(j) * kv_stride + c]));
    out[c] = s;
  }
}

// masked_softmax_int8 (int8.hpp:180-232) of one row with every key visible:
// the Coral softmax_int8 entry point (kernels.hpp:114-117), one CTA per row.
__global__ void __launch_bounds__(kHeadThreads)
    softmax_int8_kernel(int n, const int32_t* __restrict__ scores, uint32_t shift,
                        const uint16_t* __restrict__ table_g, uint8_t* __restrict__ probs) {
  __shared__ uint16_t table[256];
  __shared__ int32_t red_i[32];
  __shared__ uint32_t red_u[32];
  const long long row = blockIdx.x;
  scores += row * n;
  probs += row * n;
  for (int t = threadIdx.x; t < 256; t += blockDim.x) table[t] = table_g[t];
  int32_t mx = INT32_MIN;
  for (int j = threadIdx.x; j < n; j += blockDim.x) mx = scores[j] > mx ? scores[j] : mx;
  mx = block_reduce<int32_t>(mx, red_i, true);  // also orders the table load
  uint32_t sum = 0;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const uint32_t d = static_cast<uint32_t>((mx - scores[j]) >> static_cast<int32_t>(shift));
    sum += table[d < 255u ? d : 255u];
  }
  sum = block_reduce<uint32_t>(sum, red_u, false);
  const uint32_t reciprocal = (255u << 16) / sum;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    const uint32_t d = static_cast<uint32_t>((mx - scores[j]) >> static_cast<int32_t>(shift));
    const uint32_t scaled = static_cast<uint32_t>(table[d < 255u ? d : 255u]) * reciprocal;
    const uint32_t rounded = (scaled >> 16) + ((scaled >> 15) & 1u);
    probs[j] = static_cast<uint8_t>(rounded < 255u ? rounded : 255u);
  }
}

}  // namespace

int softmax_int8_rows(long long rows, int n, const int32_t* scores, uint32_t shift,
                      const uint16_t* table, uint8_t* probs, cudaStream_t stream) {
  if (rows == 0) return kOk;
  if (n <= 0 || shift > 31 || !scores || !table || !probs) return kErrInvalid;
  softmax_int8_kernel<<<static_cast<unsigned>(rows), kHeadThreads, 0, stream>>>(
      n, scores, shift, table, probs);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int attention_head_int8(const AttnHeadArgs& a, const int8_t* q, const int8_t* k,
                        const int8_t* v, uint32_t score_shift, const uint16_t* table,
                        uint32_t out_shift, int8_t* out, cudaStream_t stream) {
  if (a.query_len == 0 || a.heads == 0) return kOk;
  if (a.key_len <= 0 || a.head_dim <= 0 || score_shift > 31 || out_shift > 31)
    return kErrInvalid;
  if (a.key_len > kMaxKeysExact) return kErrTooLarge;
  const size_t smem = static_cast<size_t>(a.key_len) * 5;
  auto kern = head_int8_kernel;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return kErrCuda;
  dim3 grid(static_cast<unsigned>(a.query_len), static_cast<unsigned>(a.heads));
  kern<<<grid, kHeadThreads, smem, stream>>>(a.key_len, a.head_dim, a.query_start, a.window, q,
                                             a.q_stride, a.q_head, k, v, a.kv_stride,
                                             a.kv_head, score_shift, table, out_shift, out,
                                             a.out_stride, a.out_head);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int attention_head_f32(const AttnHeadArgs& a, const float* q, const float* k, const float* v,
                       float* out, cudaStream_t stream) {
  if (a.query_len == 0 || a.heads == 0) return kOk;
  if (a.key_len <= 0 || a.head_dim <= 0) return kErrInvalid;
  if (a.key_len > kMaxKeysExact) return kErrTooLarge;
  const size_t smem = static_cast<size_t>(a.key_len) * 4;
  auto kern = head_f32_kernel;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           static_cast<int>(smem)) != cudaSuccess)
    return kErrCuda;
  dim3 grid(static_cast<unsigned>(a.query_len), static_cast<unsigned>(a.heads));
  kern<<<grid, kHeadThreads, smem, stream>>>(a.key_len, a.head_dim, a.query_start, a.window, q,
                                             a.q_stride, a.q_head, k, v, a.kv_stride,
                                             a.kv_head, out, a.out_stride, a.out_head);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace reef
