// quant.cu -- per-token activation quantisation and int8 repacking.
//
// quantize_rows follows reef's quant.hpp:90-133 bit for bit:
//   scale = max|x| > 0 ? max|x| / 127 : 1          (int8_scale, :51-57)
//   q     = clamp(nearbyint(x / scale), -127, 127)  (quantize_int8, :68-81)
// The maximum is order-free; x / scale is one IEEE division (__fdiv_rn) and
// nearbyint in the default mode is round-half-to-even (__float2int_rn).
// These passes are HBM-bound: one read of x (4 B/elem) and one write of
// x_q (1 B/elem); each CTA owns one row and keeps it in registers when it
// fits, so x is read from HBM once.
#include "common.cuh"
#include "ops.h"

#include <algorithm>

namespace reef {

namespace {

constexpr int kQuantThreads = 256;

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

// reef's int8 code (quant.hpp:68-81) through quant_code (common.cuh): the
// quotient by the reciprocal, with the correctly rounded division wherever it
// could round differently, so the same code as rint(x / scale) always.
__device__ __forceinline__ int8_t q8(float x, float scale, float rcp) {
  return static_cast<int8_t>(quant_code(x, scale, rcp));
}

// One CTA per row.  row_max (optional) supplies a precomputed max |x| per
// row (the all-reduced maximum of a tensor-parallel shard).  CACHE float4
// per thread stay in registers (the smallest that holds the row, so
// registers and occupancy follow the width); longer rows re-read the rest.
// kMulti: the int8 row goes to every destination of xq (the all-gather plan's
// peer copies); otherwise only to xq.p[0], named by a constant index so the
// pointer list stays in the parameter space instead of a local-memory copy.
template <int CACHE, bool kMulti>
__global__ void __launch_bounds__(kQuantThreads)
    quantize_rows_vec4(int in, const float* __restrict__ x, PeerDst xq, long long ldq,
                       float* __restrict__ xs, const float* __restrict__ row_max) {
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const long long row = blockIdx.x;
  const float4* xr = reinterpret_cast<const float4*>(x + row * in);
  const int n4 = in >> 2;
  float4 cache[CACHE];
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < CACHE; ++i) {
    const int idx = threadIdx.x + i * kQuantThreads;
    if (idx < n4) {
      cache[i] = __ldg(xr + idx);
      m = fmaxf(m, fmaxf(fmaxf(fabsf(cache[i].x), fabsf(cache[i].y)),
                         fmaxf(fabsf(cache[i].z), fabsf(cache[i].w))));
    }
  }
  for (int idx = threadIdx.x + CACHE * kQuantThreads; idx < n4; idx += kQuantThreads) {
    const float4 v = __ldg(xr + idx);
    m = fmaxf(m, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
  }
  float mx;
  if (row_max != nullptr) {
    mx = row_max[row];
  } else {
    mx = block_max(m, red);
  }
  const float scale = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
  const float rcp = __frcp_rn(scale);
  if (threadIdx.x == 0) xs[row] = scale;
  // each int8 row goes to every destination
#pragma unroll
  for (int i = 0; i < CACHE; ++i) {
    const int idx = threadIdx.x + i * kQuantThreads;
    if (idx < n4) {
      const float4 v = cache[i];
      const char4 q = make_char4(q8(v.x, scale, rcp), q8(v.y, scale, rcp), q8(v.z, scale, rcp),
                                 q8(v.w, scale, rcp));
      if constexpr (kMulti) {
        for (int d = 0; d < xq.n; ++d)
          reinterpret_cast<char4*>(static_cast<int8_t*>(xq.p[d]) + row * ldq)[idx] = q;
      } else {
        reinterpret_cast<char4*>(static_cast<int8_t*>(xq.p[0]) + row * ldq)[idx] = q;
      }
    }
  }
  for (int idx = threadIdx.x + CACHE * kQuantThreads; idx < n4; idx += kQuantThreads) {
    const float4 v = __ldg(xr + idx);
    const char4 q = make_char4(q8(v.x, scale, rcp), q8(v.y, scale, rcp), q8(v.z, scale, rcp),
                               q8(v.w, scale, rcp));
    if constexpr (kMulti) {
      for (int d = 0; d < xq.n; ++d)
        reinterpret_cast<char4*>(static_cast<int8_t*>(xq.p[d]) + row * ldq)[idx] = q;
    } else {
      reinterpret_cast<char4*>(static_cast<int8_t*>(xq.p[0]) + row * ldq)[idx] = q;
    }
  }
  // zero the stride padding [in, ldq)
  for (long long c = in + threadIdx.x; c < ldq; c += kQuantThreads) {
    if constexpr (kMulti) {
      for (int d = 0; d < xq.n; ++d) static_cast<int8_t*>(xq.p[d])[row * ldq + c] = 0;
    } else {
      static_cast<int8_t*>(xq.p[0])[row * ldq + c] = 0;
    }
  }
}

// Any width / alignment.
__global__ void __launch_bounds__(kQuantThreads)
    quantize_rows_scalar(int in, const float* __restrict__ x, int8_t* __restrict__ xq,
                         long long ldq, float* __restrict__ xs,
                         const float* __restrict__ row_max) {
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const long long row = blockIdx.x;
  const float* xr = x + row * in;
  float m = 0.0f;
  for (int c = threadIdx.x; c < in; c += kQuantThreads) m = fmaxf(m, fabsf(xr[c]));
  const float mx = row_max != nullptr ? row_max[row] : block_max(m, red);
  const float scale = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
  const float rcp = __frcp_rn(scale);
  if (threadIdx.x == 0) xs[row] = scale;
  for (long long c = threadIdx.x; c < ldq; c += kQuantThreads)
    xq[row * ldq + c] = c < in ? q8(xr[c], scale, rcp) : static_cast<int8_t>(0);
}

__global__ void __launch_bounds__(kQuantThreads)
    row_absmax_kernel(int in, const float* __restrict__ x, PeerDst out) {
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const float* xr = x + static_cast<long long>(blockIdx.x) * in;
  float m = 0.0f;
  for (int c = threadIdx.x; c < in; c += kQuantThreads) m = fmaxf(m, fabsf(xr[c]));
  m = block_max(m, red);
  if (threadIdx.x == 0)
    for (int d = 0; d < out.n; ++d) static_cast<float*>(out.p[d])[blockIdx.x] = m;
}

// Lanes [0, f.n) signal after the system-wide fence (every earlier kernel on
// the stream has finished, and the fence orders their stores, peer stores
// included, before the increments); lanes [0, w.n) then wait on their counter, each
// with its own deadline.  The increments come first so that two ranks that
// each signal and then wait for the other cannot both wait.  Once a wait on
// this device has given up (the error word holds kDevTimeoutPeer until the
// host reads it), the ranks are out of step and every later wait would run
// out too: those return at once, so a dead peer costs one deadline, not one
// per step.
__global__ void signal_and_wait_kernel(PeerFlags f, CounterWaits w, unsigned long long limit_ns,
                                       int* err) {
  if (f.n > 0) {
    __threadfence_system();
    for (int i = threadIdx.x; i < f.n; i += blockDim.x) atomicAdd_system(f.p[i], 1u);
  }
  const int i = threadIdx.x;
  if (i >= w.n) return;
  const unsigned int target = w.target[i];
  const unsigned long long start = globaltimer();
  unsigned int spin = 0;
  while (true) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(w.p[i]) : "memory");
    if (static_cast<int>(v - target) >= 0) break;
    if ((++spin & 63u) == 0) {
      if (err != nullptr && *reinterpret_cast<volatile int*>(err) == kDevTimeoutPeer) break;
      if (globaltimer() - start > limit_ns) {
        record_error(err, kDevTimeoutPeer);
        break;
      }
    }
    __nanosleep(32);
  }
}

__global__ void zero_f32_kernel(long long n, float* __restrict__ p) {
  pdl_wait();
  pdl_trigger();
  for (long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<long long>(gridDim.x) * blockDim.x)
    p[i] = 0.0f;
}

__global__ void push_f32_kernel(long long n, const float* __restrict__ src, PeerDst dst) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const float v = src[i];
  for (int d = 0; d < dst.n; ++d) static_cast<float*>(dst.p[d])[i] = v;
}

// out[r] = max over s of in[s][r] (row maxima gathered from `segs` ranks).
__global__ void max_segments_kernel(int segs, long long rows, const float* __restrict__ in,
                                    float* __restrict__ out) {
  const long long r = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  float m = in[r];
  for (int s = 1; s < segs; ++s) m = fmaxf(m, in[s * rows + r]);
  out[r] = m;
}

// [in][out] (Coral's transposed layout, kernels.hpp:15-16) -> [out][ldw].
__global__ void pack_weight_kernel(int in, int out, const int8_t* __restrict__ wt,
                                   int8_t* __restrict__ w, long long ldw) {
  __shared__ int8_t tile[32][33];
  const int k0 = blockIdx.x * 32, n0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
  for (int i = ty; i < 32; i += 8) {
    const int k = k0 + i, n = n0 + tx;
    tile[i][tx] = (k < in && n < out) ? wt[static_cast<long long>(k) * out + n] : 0;
  }
  __syncthreads();
  for (int i = ty; i < 32; i += 8) {
    const int n = n0 + i, k = k0 + tx;
    if (n < out && k < ldw) w[static_cast<long long>(n) * ldw + k] = k < in ? tile[tx][i] : 0;
  }
}

__global__ void pad_rows_kernel(long long rows, int in, const int8_t* __restrict__ x,
                                long long ldx, int8_t* __restrict__ y, long long ldy) {
  const long long row = blockIdx.x;
  for (long long c = threadIdx.x; c < ldy; c += blockDim.x)
    y[row * ldy + c] = c < in ? x[row * ldx + c] : static_cast<int8_t>(0);
}

__global__ void w8a8_epilogue_kernel(long long rows, int out, const int32_t* __restrict__ acc,
                                     const float* __restrict__ xs,
                                     const float* __restrict__ ws,
                                     const float* __restrict__ bias,
                                     const float* __restrict__ residual, float* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= rows * out) return;
  const long long r = i / out;
  const int c = static_cast<int>(i - r * out);
  float v = __fmul_rn(__int2float_rn(acc[i]), __fmul_rn(xs[r], ws[c]));
  if (bias != nullptr) v = __fadd_rn(v, bias[c]);
  if (residual != nullptr) v = __fadd_rn(residual[i], v);
  y[i] = v;
}

}  // namespace

static int quantize_vec4(long long rows, long long in, const float* x, const PeerDst& x_q,
                         long long ldq, float* x_scale, const float* row_max,
                         cudaStream_t stream) {
  const int per = static_cast<int>((in / 4 + kQuantThreads - 1) / kQuantThreads);
  const unsigned grid = static_cast<unsigned>(rows);
  const int ii = static_cast<int>(in);
  const dim3 g(grid), t(kQuantThreads);
#define REEF_QUANT_VEC4(C)                                                                       \
  return x_q.n > 1                                                                               \
             ? launch_k(quantize_rows_vec4<C, true>, g, t, 0, stream, ii, x, x_q, ldq, x_scale,  \
                        row_max)                                                                 \
             : launch_k(quantize_rows_vec4<C, false>, g, t, 0, stream, ii, x, x_q, ldq, x_scale, \
                        row_max)
  if (per <= 1) REEF_QUANT_VEC4(1);
  if (per <= 2) REEF_QUANT_VEC4(2);
  if (per <= 4) REEF_QUANT_VEC4(4);
  if (per <= 8) REEF_QUANT_VEC4(8);
  if (per <= 12) REEF_QUANT_VEC4(12);
  REEF_QUANT_VEC4(16);
#undef REEF_QUANT_VEC4
}

int quantize_rows(long long rows, long long in, const float* x, int8_t* x_q, long long ldq,
                  float* x_scale, const float* row_max, cudaStream_t stream) {
  if (rows == 0) return kOk;
  if (in <= 0 || ldq < in || x == nullptr || x_q == nullptr || x_scale == nullptr)
    return kErrInvalid;
  const bool vec = (in % 4 == 0) && (ldq % 4 == 0) &&
                   (reinterpret_cast<uintptr_t>(x) % 16 == 0) &&
                   (reinterpret_cast<uintptr_t>(x_q) % 4 == 0);
  if (vec) return quantize_vec4(rows, in, x, one_dst(x_q), ldq, x_scale, row_max, stream);
  return launch_k(quantize_rows_scalar, dim3(static_cast<unsigned>(rows)), dim3(kQuantThreads), 0,
                  stream, static_cast<int>(in), x, x_q, ldq, x_scale, row_max);
}

int quantize_rows_to(long long rows, long long in, const float* x, const PeerDst& x_q,
                     long long ldq, float* x_scale, const float* row_max, cudaStream_t stream) {
  if (rows == 0) return kOk;
  if (in <= 0 || ldq < in || in % 4 != 0 || ldq % 4 != 0 || x == nullptr || x_scale == nullptr ||
      !dst_ok(x_q) || reinterpret_cast<uintptr_t>(x) % 16 != 0)
    return kErrInvalid;
  for (int d = 0; d < x_q.n; ++d)
    if (reinterpret_cast<uintptr_t>(x_q.p[d]) % 4 != 0) return kErrInvalid;
  return quantize_vec4(rows, in, x, x_q, ldq, x_scale, row_max, stream);
}

int signal_and_wait(const PeerFlags& f, const CounterWaits& w, unsigned long long limit_ns,
                    cudaStream_t stream) {
  if (f.n < 0 || f.n > kMaxFlags || w.n < 0 || w.n > kMaxWaits || limit_ns == 0)
    return kErrInvalid;
  if (f.n == 0 && w.n == 0) return kOk;
  for (int i = 0; i < f.n; ++i)
    if (f.p[i] == nullptr) return kErrInvalid;
  for (int i = 0; i < w.n; ++i)
    if (w.p[i] == nullptr) return kErrInvalid;
  signal_and_wait_kernel<<<1, 32, 0, stream>>>(f, w, limit_ns, device_error_ptr());
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int zero_f32(long long n, float* p, cudaStream_t stream) {
  if (n == 0) return kOk;
  if (n < 0 || p == nullptr) return kErrInvalid;
  const long long blocks = std::min<long long>((n + 255) / 256, 1024);
  return launch_k(zero_f32_kernel, dim3(static_cast<unsigned>(blocks)), dim3(256), 0, stream, n, p);
}

int push_f32(long long n, const float* src, const PeerDst& dst, cudaStream_t stream) {
  if (n == 0) return kOk;
  if (n < 0 || src == nullptr || !dst_ok(dst)) return kErrInvalid;
  push_f32_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(n, src, dst);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int row_absmax_to(long long rows, long long in, const float* x, const PeerDst& row_max,
                  cudaStream_t stream) {
  if (rows == 0) return kOk;
  if (in <= 0 || x == nullptr || !dst_ok(row_max)) return kErrInvalid;
  return launch_k(row_absmax_kernel, dim3(static_cast<unsigned>(rows)), dim3(kQuantThreads), 0,
                  stream, static_cast<int>(in), x, row_max);
}

int row_absmax(long long rows, long long in, const float* x, float* row_max,
               cudaStream_t stream) {
  if (row_max == nullptr) return kErrInvalid;
  return row_absmax_to(rows, in, x, one_dst(row_max), stream);
}

int max_segments(int segs, long long rows, const float* in, float* out, cudaStream_t stream) {
  if (rows == 0) return kOk;
  if (segs < 1 || in == nullptr || out == nullptr) return kErrInvalid;
  max_segments_kernel<<<static_cast<unsigned>((rows + 255) / 256), 256, 0, stream>>>(segs, rows,
                                                                                     in, out);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int pack_weight_i8(long long in, long long out, const int8_t* wt, int8_t* w, long long ldw,
                   cudaStream_t stream) {
  if (in <= 0 || out <= 0 || ldw < in || wt == nullptr || w == nullptr) return kErrInvalid;
  dim3 grid(static_cast<unsigned>((ldw + 31) / 32), static_cast<unsigned>((out + 31) / 32));
  pack_weight_kernel<<<grid, dim3(32, 8), 0, stream>>>(static_cast<int>(in),
                                                       static_cast<int>(out), wt, w, ldw);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int pad_rows_i8(long long rows, long long in, const int8_t* x, long long ldx, int8_t* y,
                long long ldy, cudaStream_t stream) {
  if (rows == 0) return kOk;
  if (in <= 0 || ldy < in || ldx < in || x == nullptr || y == nullptr) return kErrInvalid;
  pad_rows_kernel<<<static_cast<unsigned>(rows), 128, 0, stream>>>(rows, static_cast<int>(in),
                                                                   x, ldx, y, ldy);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int w8a8_epilogue_i32(long long rows, long long out, const int32_t* acc, const float* x_scale,
                      const float* w_scale, const float* bias, const float* residual, float* y,
                      cudaStream_t stream) {
  if (rows == 0) return kOk;
  const long long n = rows * out;
  return launch_k(w8a8_epilogue_kernel, dim3(static_cast<unsigned>((n + 255) / 256)), dim3(256), 0,
                  stream, rows, static_cast<int>(out), acc, x_scale, w_scale, bias, residual, y);
}

}  // namespace reef
