// exact_math.cuh -- reef's float transcendentals as device code, bit for bit.
//
// exp_nonpositive and tanh_float (math.hpp:34-81) and the tanh-form gelu
// (operator/activation.hpp:78-90), each float operation rounded on its own
// (__f*_rn: no fused multiply-add), in the engine's order, so every result
// equals the engine's.  Shared by the element-wise kernels (elementwise.cu)
// and the GEMM epilogue that fuses gelu into c_fc.
#pragma once

#include <cuda_runtime.h>

namespace reef {

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

// gelu (activation.hpp:78-90): 0.5 v (1 + tanh(sqrt(2/pi) (v + 0.044715 v^3))),
// evaluated left to right as written
__device__ __forceinline__ float gelu_dev(float v) {
  const float cubic = __fmul_rn(__fmul_rn(__fmul_rn(0.044715f, v), v), v);
  const float inner = __fmul_rn(0.7978845608028654f, __fadd_rn(v, cubic));
  return __fmul_rn(__fmul_rn(0.5f, v), __fadd_rn(1.0f, tanh_float_dev(inner)));
}

}  // namespace reef
