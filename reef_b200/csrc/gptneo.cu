// gptneo.cu -- reef's float layernorm, bit for bit, so a whole W8A8 GPT-Neo
// block (operator/block.hpp:97-108) on the GPU reproduces
// Block<float>::forward exactly (its gelu runs in the c_fc GEMM's epilogue,
// exact_math.cuh).
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

}  // namespace

int layernorm_exact(long long rows, int width, float eps, const float* x, const float* gain,
                    const float* shift, float* y, cudaStream_t stream) {
  if (rows == 0) return kOk;
  if (width <= 0 || !x || !gain || !y) return kErrInvalid;
  layernorm_exact_kernel<<<static_cast<unsigned>(rows), 128, 0, stream>>>(width, eps, x, gain,
                                                                          shift, y);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace reef
