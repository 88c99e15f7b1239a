// gptneo.cu -- reef's float layernorm, bit for bit, so a whole W8A8 GPT-Neo
// block (operator/block.hpp:97-108) on the GPU reproduces
// Block<float>::forward exactly (its gelu runs in the c_fc GEMM's epilogue,
// exact_math.cuh); in the block it also quantises its rows for the next
// projection, so the normalised fp32 row never reaches memory.
//
//   layernorm  operator/layernorm.hpp:62-80: mean and variance are in-order
//              sums over the row (one thread), inv_std = 1 / sqrt(var + eps),
//              y = ((x - mean) * inv_std) * gain + shift.
// Every float step is one IEEE operation (__f*_rn, and the library is built
// with -fmad=false).  It is tiny next to the GEMMs; it is written for
// exactness, not speed.
#include "common.cuh"
#include "ops.h"

namespace reef {

namespace {

// One CTA per row: thread 0 forms the in-order sums, then all threads write.
// y (optional) gets the normalised row.  xq (optional) gets it quantised as
// quantize_rows does (quant.hpp:112-133): scale = max|y| / 127 (1 for a zero
// row) into xs, codes rint(y / scale) clamped to +-127 with the correctly
// rounded quotient, the stride padding [width, ldq) zeroed -- the same bits
// as layernorm then quantize_rows, without the fp32 row in between.
__global__ void layernorm_exact_kernel(int width, float eps, const float* __restrict__ x,
                                       const float* __restrict__ gain,
                                       const float* __restrict__ shift, float* __restrict__ y,
                                       int8_t* __restrict__ xq, long long ldq,
                                       float* __restrict__ xs) {
  __shared__ float stats[2];
  __shared__ float red[32];
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
  auto value = [&](int k) {
    float v = __fmul_rn(__fmul_rn(__fsub_rn(xr[k], mean), inv), gain[k]);
    if (shift != nullptr) v = __fadd_rn(v, shift[k]);
    return v;
  };
  float m = 0.0f;
  for (int k = threadIdx.x; k < width; k += blockDim.x) {
    const float v = value(k);
    if (y != nullptr) y[row * width + k] = v;
    m = fmaxf(m, fabsf(v));
  }
  if (xq == nullptr) return;
  // the row's max |y| (a max: any order gives the same value)
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = red[0];
    for (int w = 1; w < static_cast<int>(blockDim.x >> 5); ++w) mm = fmaxf(mm, red[w]);
    stats[0] = mm > 0.0f ? __fdiv_rn(mm, 127.0f) : 1.0f;
    xs[row] = stats[0];
  }
  __syncthreads();
  const float scale = stats[0];
  for (long long k = threadIdx.x; k < ldq; k += blockDim.x) {
    int c = 0;
    if (k < width) {
      c = __float2int_rn(__fdiv_rn(value(static_cast<int>(k)), scale));
      c = c < -127 ? -127 : (c > 127 ? 127 : c);
    }
    xq[row * ldq + k] = static_cast<int8_t>(c);
  }
}

}  // namespace

int layernorm_exact(long long rows, int width, float eps, const float* x, const float* gain,
                    const float* shift, float* y, cudaStream_t stream) {
  if (rows == 0) return kOk;
  if (width <= 0 || !x || !gain || !y) return kErrInvalid;
  layernorm_exact_kernel<<<static_cast<unsigned>(rows), 128, 0, stream>>>(
      width, eps, x, gain, shift, y, nullptr, 0, nullptr);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int layernorm_exact_quant(long long rows, int width, float eps, const float* x, const float* gain,
                          const float* shift, int8_t* x_q, long long ldq, float* x_scale,
                          cudaStream_t stream) {
  if (rows == 0) return kOk;
  if (width <= 0 || ldq < width || !x || !gain || !x_q || !x_scale) return kErrInvalid;
  layernorm_exact_kernel<<<static_cast<unsigned>(rows), 128, 0, stream>>>(
      width, eps, x, gain, shift, nullptr, x_q, ldq, x_scale);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace reef
