// elementwise.cu -- the rest of reef's Coral operator set (kernels.hpp:26-146)
// on the GPU, bit for bit: the float linear, layernorm, gelu, exp / tanh and
// residual add of the float GPT-Neo path, and the integer-only operators of
// the int8 path (int8.hpp).
//
//   linear_f32        operator/linear.hpp:75-84 through tensor.hpp:179-192:
//                     y[r][c] = sum over k, in order from 0, of x[r][k] *
//                     wt[k][c] (wt = the weight transposed, [in][out]), every
//                     product and sum rounded on its own, then + bias[c].
//                     One thread owns one output and adds in order; a warp's
//                     32 threads read 32 consecutive columns of wt.
//   layernorm_f32     layernorm_exact (gptneo.cu), one row per CTA.
//   gelu / exp / tanh exact_math.cuh, elementwise.
//   add_f32           one rounded add (the engine's residual_add).
//   gelu_int8         y = table[x + 128] (int8.hpp:135-147).
//   layernorm_int8    int8.hpp:332-374: mean = floor(sum / width), std =
//                     isqrt(sum((x - mean)^2) / width), inv = 2^20 /
//                     max(std, 1), y = sat8(rshift_rnu(((x - mean) * inv >>
//                     16) * gain + shift * 32, 5)).  Integer sums are exact
//                     in any order, so the CTA reduces them in parallel.
//   add_int8          sat8(a + b) (int8.hpp:382-397).
//   embedding_int8    sat8(wte[id][c] + wpe[position][c]) (kernels.hpp:142-145).
//
// The engine throws std::overflow_error when a float product or sum is not
// finite (util.hpp:81-131); the float linear records kDevNonFinite in the
// device error word instead.  An embedding id past the vocabulary records
// kDevBadToken and writes zeros, as the float embedding does.
#include "common.cuh"
#include "exact_math.cuh"
#include "ops.h"

#include <cstdint>

namespace reef {

namespace {

constexpr int kLinTile = 32;  // columns per warp; rows of x staged per CTA

__global__ void __launch_bounds__(128)
    linear_f32_kernel(long long rows, int in, int out, const float* __restrict__ x,
                      const float* __restrict__ wt, const float* __restrict__ bias,
                      float* __restrict__ y, int* err) {
  // blockIdx.x: 128 consecutive output columns; blockIdx.y: one row
  const long long r = blockIdx.y;
  const long long c = static_cast<long long>(blockIdx.x) * 128 + threadIdx.x;
  __shared__ float xs[kLinTile];
  const float* xr = x + r * in;
  float sum = 0.0f;
  bool finite = true;
  for (int k0 = 0; k0 < in; k0 += kLinTile) {
    const int kc = in - k0 < kLinTile ? in - k0 : kLinTile;
    __syncthreads();
    if (threadIdx.x < kc) xs[threadIdx.x] = xr[k0 + threadIdx.x];
    __syncthreads();
    if (c < out) {
      for (int kk = 0; kk < kc; ++kk) {
        const float p = __fmul_rn(xs[kk], wt[static_cast<long long>(k0 + kk) * out + c]);
        sum = __fadd_rn(sum, p);
        finite = finite && isfinite(p) && isfinite(sum);
      }
    }
  }
  if (c >= out) return;
  if (bias != nullptr) {
    sum = __fadd_rn(sum, bias[c]);
    finite = finite && isfinite(sum);
  }
  y[r * out + c] = sum;
  if (!finite) record_error(err, kDevNonFinite);
}

template <int OP>
__global__ void unary_exact_kernel(long long n, const float* __restrict__ x,
                                   float* __restrict__ y) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float v = x[i];
    y[i] = OP == kUnaryExp    ? exp_nonpositive_dev(v)
           : OP == kUnaryTanh ? tanh_float_dev(v)
                              : gelu_dev(v);
  }
}

__global__ void add_f32_kernel(long long n, const float* __restrict__ a,
                               const float* __restrict__ b, float* __restrict__ y, int* err) {
  bool finite = true;
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const float v = __fadd_rn(a[i], b[i]);
    finite = finite && isfinite(v);
    y[i] = v;
  }
  if (!finite) record_error(err, kDevNonFinite);
}

__device__ __forceinline__ int8_t sat8(int v) {
  return static_cast<int8_t>(v < -128 ? -128 : (v > 127 ? 127 : v));
}

__global__ void gelu_int8_kernel(long long n, const int8_t* __restrict__ x,
                                 const int8_t* __restrict__ table, int8_t* __restrict__ y) {
  __shared__ int8_t t[256];
  t[threadIdx.x] = table[threadIdx.x];  // blockDim.x == 256
  __syncthreads();
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    y[i] = t[static_cast<int>(x[i]) + 128];
}

__global__ void add_int8_kernel(long long n, const int8_t* __restrict__ a,
                                const int8_t* __restrict__ b, int8_t* __restrict__ y) {
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    y[i] = sat8(static_cast<int>(a[i]) + static_cast<int>(b[i]));
}

__global__ void embedding_int8_kernel(int width, const uint32_t* __restrict__ ids,
                                      long long first_position, long long vocab,
                                      long long positions, const int8_t* __restrict__ wte,
                                      const int8_t* __restrict__ wpe, int8_t* __restrict__ y,
                                      int* err) {
  const long long t = blockIdx.x;
  const uint32_t id = ids[t];
  const long long pos = first_position + t;
  int8_t* yr = y + t * width;
  if (id >= vocab || pos >= positions) {
    if (threadIdx.x == 0) record_error(err, id >= vocab ? kDevBadToken : kDevBadPosition);
    for (int c = threadIdx.x; c < width; c += blockDim.x) yr[c] = 0;
    return;
  }
  const int8_t* a = wte + static_cast<long long>(id) * width;
  const int8_t* b = wpe + pos * width;
  for (int c = threadIdx.x; c < width; c += blockDim.x)
    yr[c] = sat8(static_cast<int>(a[c]) + static_cast<int>(b[c]));
}

// reef's isqrt (int8.hpp:291-303): the largest r with r * r <= value
__device__ __forceinline__ uint32_t isqrt_dev(uint32_t value) {
  uint32_t root = 0;
  for (uint32_t bit = 1u << 30; bit != 0; bit >>= 2) {
    if (value >= root + bit) {
      value -= root + bit;
      root = (root >> 1) + bit;
    } else {
      root >>= 1;
    }
  }
  return root;
}

__device__ __forceinline__ int block_sum(int v, int* scratch) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  __syncthreads();
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  int total = 0;
  for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) total += scratch[w];
  return total;
}

__global__ void __launch_bounds__(256)
    layernorm_int8_kernel(int width, const int8_t* __restrict__ x,
                          const int8_t* __restrict__ gain, const int8_t* __restrict__ shift,
                          int8_t* __restrict__ y) {
  __shared__ int scratch[8];
  const long long row = blockIdx.x;
  const int8_t* xr = x + row * width;
  int s = 0;
  for (int k = threadIdx.x; k < width; k += blockDim.x) s += xr[k];
  const int sum = block_sum(s, scratch);
  // floor_div (int8.hpp:311-316)
  const int q = sum / width;
  const int mean = (sum % width != 0 && sum < 0) ? q - 1 : q;
  int sq = 0;
  for (int k = threadIdx.x; k < width; k += blockDim.x) {
    const int cd = xr[k] - mean;
    sq += cd * cd;
  }
  const int squares = block_sum(sq, scratch);
  const uint32_t dev = isqrt_dev(static_cast<uint32_t>(squares / width));
  const int inv = (1 << 20) / static_cast<int>(dev > 1u ? dev : 1u);
  for (int k = threadIdx.x; k < width; k += blockDim.x) {
    const int normed = ((xr[k] - mean) * inv) >> 16;
    const int scaled = normed * gain[k] + static_cast<int>(shift[k]) * 32;
    y[row * width + k] = requant_rnu_sat8(scaled, 5);
  }
}

unsigned grid_for(long long n, int threads) {
  const long long want = (n + threads - 1) / threads;
  const long long cap = static_cast<long long>(num_sms()) * 16;
  return static_cast<unsigned>(want < cap ? (want > 0 ? want : 1) : cap);
}

int launched() { return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda; }

}  // namespace

int linear_f32(long long rows, int in, int out, const float* x, const float* wt,
               const float* bias, float* y, cudaStream_t stream) {
  if (rows <= 0 || in <= 0 || out <= 0 || !x || !wt || !y) return kErrInvalid;
  if (rows > 65535) return kErrTooLarge;
  const dim3 grid(static_cast<unsigned>((out + 127) / 128), static_cast<unsigned>(rows));
  linear_f32_kernel<<<grid, 128, 0, stream>>>(rows, in, out, x, wt, bias, y, device_error_ptr());
  return launched();
}

int unary_exact(int op, long long n, const float* x, float* y, cudaStream_t stream) {
  if (n <= 0 || !x || !y) return kErrInvalid;
  const unsigned g = grid_for(n, 256);
  if (op == kUnaryExp)
    unary_exact_kernel<kUnaryExp><<<g, 256, 0, stream>>>(n, x, y);
  else if (op == kUnaryTanh)
    unary_exact_kernel<kUnaryTanh><<<g, 256, 0, stream>>>(n, x, y);
  else if (op == kUnaryGelu)
    unary_exact_kernel<kUnaryGelu><<<g, 256, 0, stream>>>(n, x, y);
  else
    return kErrInvalid;
  return launched();
}

int add_f32(long long n, const float* a, const float* b, float* y, cudaStream_t stream) {
  if (n <= 0 || !a || !b || !y) return kErrInvalid;
  add_f32_kernel<<<grid_for(n, 256), 256, 0, stream>>>(n, a, b, y, device_error_ptr());
  return launched();
}

int gelu_int8(long long n, const int8_t* x, const int8_t* table, int8_t* y,
              cudaStream_t stream) {
  if (n <= 0 || !x || !table || !y) return kErrInvalid;
  gelu_int8_kernel<<<grid_for(n, 256), 256, 0, stream>>>(n, x, table, y);
  return launched();
}

int add_int8(long long n, const int8_t* a, const int8_t* b, int8_t* y, cudaStream_t stream) {
  if (n <= 0 || !a || !b || !y) return kErrInvalid;
  add_int8_kernel<<<grid_for(n, 256), 256, 0, stream>>>(n, a, b, y);
  return launched();
}

int embedding_int8(int width, long long count, const uint32_t* ids, long long first_position,
                   long long vocab, long long positions, const int8_t* wte, const int8_t* wpe,
                   int8_t* y, cudaStream_t stream) {
  if (width <= 0 || count <= 0 || vocab <= 0 || positions <= 0 || first_position < 0 || !ids ||
      !wte || !wpe || !y)
    return kErrInvalid;
  if (count > 0x7fffffffLL) return kErrTooLarge;
  embedding_int8_kernel<<<static_cast<unsigned>(count), 128, 0, stream>>>(
      width, ids, first_position, vocab, positions, wte, wpe, y, device_error_ptr());
  return launched();
}

int layernorm_int8(long long rows, int width, const int8_t* x, const int8_t* gain,
                   const int8_t* shift, int8_t* y, cudaStream_t stream) {
  // the engine's int32 sum of squares holds up to 32767 columns of 255^2
  if (rows <= 0 || width <= 0 || width > 32767 || !x || !gain || !shift || !y)
    return kErrInvalid;
  if (rows > 0x7fffffffLL) return kErrTooLarge;
  layernorm_int8_kernel<<<static_cast<unsigned>(rows), 256, 0, stream>>>(width, x, gain, shift, y);
  return launched();
}

}  // namespace reef
