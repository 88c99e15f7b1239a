// llama.cu -- the element-wise steps of a Llama-shape W8A8 decoder layer,
// each fused with the per-token quantisation the next int8 GEMM needs.
//
// reef has no Llama operators (its model is GPT-Neo): RMSNorm and SwiGLU are
// this build's own definitions (parity unpinned by the reference); the
// quantisation they feed is reef's (quant.hpp:51-81: scale = max|x|/127, 1
// for an all-zero row; codes = clamp(rne(x / scale), -127, 127)), so the int8
// GEMM inputs follow reef's rule exactly.
//
//   rmsnorm_quant   y = x * (1 / sqrt(mean(x^2) + eps)) * gain  -> int8 + scale
//   swiglu_quant    y = silu(gate) * up = gate / (1 + e^-gate) * up -> int8 + scale
//   swiglu_absmax   max |silu(gate) * up| per row (the tensor-parallel shard's
//                   partial maximum, all-reduced before swiglu_quant)
// One CTA per row; the row stays in registers between the reduction and the
// quantisation, so each input is read from HBM once.
#include "common.cuh"
#include "ops.h"

namespace reef {

namespace {

constexpr int kThreads = 256;

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (blockDim.x >> 5) ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  const float r = red[0];
  __syncthreads();
  return r;
}

__device__ __forceinline__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < (blockDim.x >> 5) ? red[lane] : 0.0f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[0] = v;
  }
  __syncthreads();
  const float r = red[0];
  __syncthreads();
  return r;
}

__device__ __forceinline__ char4 q8x4(float4 v, float scale) {
  auto q = [scale](float x) {
    int c = __float2int_rn(__fdiv_rn(x, scale));
    c = c < -127 ? -127 : (c > 127 ? 127 : c);
    return static_cast<signed char>(c);
  };
  return make_char4(q(v.x), q(v.y), q(v.z), q(v.w));
}

__device__ __forceinline__ float amax4(float4 v) {
  return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}

__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

__device__ __forceinline__ float4 swiglu4(float4 g, float4 u) {
  return make_float4(silu_mul(g.x, u.x), silu_mul(g.y, u.y), silu_mul(g.z, u.z),
                     silu_mul(g.w, u.w));
}

// width % 4 == 0, width <= 4 * CACHE * kThreads.  CACHE (float4 per
// thread) is the smallest that holds the row, so registers, and with them
// occupancy and loads in flight, follow the row width.
template <int CACHE>
__global__ void __launch_bounds__(kThreads)
    rmsnorm_quant_kernel(int width, float eps, const float* __restrict__ x,
                         const float* __restrict__ gain, int8_t* __restrict__ xq,
                         long long ldq, float* __restrict__ xs) {
  __shared__ float red[32];
  const long long row = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + row * width);
  const float4* gr = reinterpret_cast<const float4*>(gain);
  const int n4 = width >> 2;
  float4 c[CACHE];
  float ss = 0.0f;
#pragma unroll
  for (int i = 0; i < CACHE; ++i) {
    const int idx = threadIdx.x + i * kThreads;
    if (idx < n4) {
      c[i] = __ldg(xr + idx);
      ss += c[i].x * c[i].x + c[i].y * c[i].y + c[i].z * c[i].z + c[i].w * c[i].w;
    }
  }
  ss = block_sum(ss, red);
  const float r = 1.0f / sqrtf(ss / static_cast<float>(width) + eps);
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < CACHE; ++i) {
    const int idx = threadIdx.x + i * kThreads;
    if (idx < n4) {
      const float4 g = __ldg(gr + idx);
      c[i] = make_float4(c[i].x * r * g.x, c[i].y * r * g.y, c[i].z * r * g.z, c[i].w * r * g.w);
      m = fmaxf(m, amax4(c[i]));
    }
  }
  m = block_max(m, red);
  const float scale = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
  if (threadIdx.x == 0) xs[row] = scale;
  char4* out = reinterpret_cast<char4*>(xq + row * ldq);
#pragma unroll
  for (int i = 0; i < CACHE; ++i) {
    const int idx = threadIdx.x + i * kThreads;
    if (idx < n4) out[idx] = q8x4(c[i], scale);
  }
}

// gu [rows][2*ffn]: gate in [0, ffn), up in [ffn, 2 ffn).  ffn % 4 == 0.
// row_max == nullptr: quantise with this row's own maximum; else with the
// given (all-reduced) maximum.
template <int CACHE>
__global__ void __launch_bounds__(kThreads)
    swiglu_quant_kernel(int ffn, const float* __restrict__ gu, const float* __restrict__ row_max,
                        int8_t* __restrict__ xq, long long ldq, float* __restrict__ xs) {
  __shared__ float red[32];
  const long long row = blockIdx.x;
  const float4* g4 = reinterpret_cast<const float4*>(gu + row * 2 * ffn);
  const float4* u4 = g4 + (ffn >> 2);
  const int n4 = ffn >> 2;
  float4 c[CACHE];
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < CACHE; ++i) {
    const int idx = threadIdx.x + i * kThreads;
    if (idx < n4) {
      c[i] = swiglu4(__ldg(g4 + idx), __ldg(u4 + idx));
      m = fmaxf(m, amax4(c[i]));
    }
  }
  const float mx = row_max != nullptr ? row_max[row] : block_max(m, red);
  const float scale = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
  if (threadIdx.x == 0) xs[row] = scale;
  char4* out = reinterpret_cast<char4*>(xq + row * ldq);
#pragma unroll
  for (int i = 0; i < CACHE; ++i) {
    const int idx = threadIdx.x + i * kThreads;
    if (idx < n4) out[idx] = q8x4(c[i], scale);
  }
}

__global__ void __launch_bounds__(kThreads)
    swiglu_absmax_kernel(int ffn, const float* __restrict__ gu, float* __restrict__ row_max) {
  __shared__ float red[32];
  const long long row = blockIdx.x;
  const float4* g4 = reinterpret_cast<const float4*>(gu + row * 2 * ffn);
  const float4* u4 = g4 + (ffn >> 2);
  float m = 0.0f;
  for (int idx = threadIdx.x; idx < (ffn >> 2); idx += kThreads)
    m = fmaxf(m, amax4(swiglu4(__ldg(g4 + idx), __ldg(u4 + idx))));
  m = block_max(m, red);
  if (threadIdx.x == 0) row_max[row] = m;
}

}  // namespace

// Smallest supported per-thread cache (float4) that holds n4 float4.
static int cache_for(int n4) {
  const int per = (n4 + kThreads - 1) / kThreads;
  for (int c : {1, 2, 4, 6, 8, 12, 16})
    if (per <= c) return c;
  return 0;
}

#define REEF_DISPATCH_CACHE(c, KERNEL, ...)                                   \
  switch (c) {                                                              \
    case 1: KERNEL<1><<<grid, kThreads, 0, stream>>>(__VA_ARGS__); break;   \
    case 2: KERNEL<2><<<grid, kThreads, 0, stream>>>(__VA_ARGS__); break;   \
    case 4: KERNEL<4><<<grid, kThreads, 0, stream>>>(__VA_ARGS__); break;   \
    case 6: KERNEL<6><<<grid, kThreads, 0, stream>>>(__VA_ARGS__); break;   \
    case 8: KERNEL<8><<<grid, kThreads, 0, stream>>>(__VA_ARGS__); break;   \
    case 12: KERNEL<12><<<grid, kThreads, 0, stream>>>(__VA_ARGS__); break; \
    default: KERNEL<16><<<grid, kThreads, 0, stream>>>(__VA_ARGS__); break; \
  }

int rmsnorm_quant(long long rows, int width, float eps, const float* x, const float* gain,
                  int8_t* x_q, float* x_scale, cudaStream_t stream) {
  if (rows == 0) return kOk;
  const int c = cache_for(width / 4);
  if (width <= 0 || width % 4 != 0 || c == 0) return kErrInvalid;
  const unsigned grid = static_cast<unsigned>(rows);
  REEF_DISPATCH_CACHE(c, rmsnorm_quant_kernel, width, eps, x, gain, x_q,
                      static_cast<long long>(width), x_scale);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int swiglu_quant(long long rows, int ffn, const float* gu, const float* row_max, int8_t* x_q,
                 float* x_scale, cudaStream_t stream) {
  if (rows == 0) return kOk;
  const int c = cache_for(ffn / 4);
  if (ffn <= 0 || ffn % 4 != 0 || c == 0) return kErrInvalid;
  const unsigned grid = static_cast<unsigned>(rows);
  REEF_DISPATCH_CACHE(c, swiglu_quant_kernel, ffn, gu, row_max, x_q,
                      static_cast<long long>(ffn), x_scale);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int swiglu_absmax(long long rows, int ffn, const float* gu, float* row_max, cudaStream_t stream) {
  if (rows == 0) return kOk;
  if (ffn <= 0 || ffn % 4 != 0) return kErrInvalid;
  swiglu_absmax_kernel<<<static_cast<unsigned>(rows), kThreads, 0, stream>>>(ffn, gu, row_max);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace reef
