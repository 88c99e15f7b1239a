// gptneo.cu -- the float element-wise operators of reef's GPT-Neo block,
// bit for bit, so a whole W8A8 block (operator/block.hpp:97-108) on the GPU
// reproduces Block<float>::forward exactly.
//
//   layernorm  operator/layernorm.hpp:62-80: mean and variance are in-order
//              sums over the row (one thread), inv_std = 1 / sqrt(var + eps),
//              y = ((x - mean) * inv_std) * gain + shift.
//   gelu       operator/activation.hpp:78-90: the tanh form evaluated left to
//              right, tanh_float from exp_nonpositive (math.hpp:34-81).
// Every float step is one IEEE operation (__f*_rn, and the library is built
// with -fmad=false).  These are tiny next to the GEMMs; they are written for
// exactness, not speed.
#include "common.cuh"
#include "ops.h"

namespace reef {

namespace {

__device__ __forceinline__ float exp_nonpositive_dev(float x) {
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
  return __fmul_rn(p, __int_as_float((static_cast<int>(kf) + 127) << 23));
}

__device__ __forceinline__ float tanh_float_dev(float x) {
  const float e = exp_nonpositive_dev(__fmul_rn(-2.0f, fabsf(x)));
  const float mag = __fdiv_rn(__fsub_rn(1.0f, e), __fadd_rn(1.0f, e));
  return copysignf(mag, x);
}

// One CTA per row: thread 0 forms the in-order sums, then all threads write.
__global__ void layernorm_exact_kernel(int width, float eps, const float* __restrict__ x,
                                       const float* __restrict__ gain,
                                       const float* __restrict__ shift, float* __restrict__ y) {
  __shared__ float stats[2];
  const long long row = blockIdx.x;
  const float* xr = x + row * width;
  if (threadIdx.x == 0) {
    float mean = 0.0f;
    for (int k = 0; k < width; ++k) mean = __fadd_rn(mean, xr[k]);
    mean = __fdiv_rn(mean, static_cast<float>(width));
    float var = 0.0f;
    for (int k = 0; k < width; ++k) {
      const float c = __fsub_rn(xr[k], mean);
      var = __fadd_rn(var, __fmul_rn(c, c));
    }
    var = __fdiv_rn(var, static_cast<float>(width));
    stats[0] = mean;
    stats[1] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
  }
  __syncthreads();
  const float mean = stats[0], inv = stats[1];
  for (int k = threadIdx.x; k < width; k += blockDim.x) {
    float v = __fmul_rn(__fmul_rn(__fsub_rn(xr[k], mean), inv), gain[k]);
    if (shift != nullptr) v = __fadd_rn(v, shift[k]);
    y[row * width + k] = v;
  }
}

__global__ void gelu_exact_kernel(long long n, const float* __restrict__ x, float* __restrict__ y) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = x[i];
  const float cubic = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v);
  const float inner = __fmul_rn(0.7978845608028654f, __fadd_rn(v, cubic));
  y[i] = __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanh_float_dev(inner)));
}

}  // namespace

int layernorm_exact(long long rows, int width, float eps, const float* x, const float* gain,
                    const float* shift, float* y, cudaStream_t stream) {
  if (rows == 0) return kOk;
  if (width <= 0 || !x || !gain || !y) return kErrInvalid;
  layernorm_exact_kernel<<<static_cast<unsigned>(rows), 128, 0, stream>>>(width, eps, x, gain,
                                                                          shift, y);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int gelu_exact(long long n, const float* x, float* y, cudaStream_t stream) {
  if (n == 0) return kOk;
  if (!x || !y) return kErrInvalid;
  gelu_exact_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(n, x, y);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace reef
