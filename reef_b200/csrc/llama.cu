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
//   swiglu_partials y = silu(gate) * up = gate / (1 + e^-gate) * up on the decode
//                   gate/up GEMM's split-K partials -> int8 + scale
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

// reef's int8 codes (quant.hpp:68-81) of four values through quant_code
// (common.cuh): the same codes as rint(x / scale), clamped
__device__ __forceinline__ char4 q8x4(float4 v, float scale) {
  const float rcp = __frcp_rn(scale);
  auto q = [scale, rcp](float x) { return static_cast<signed char>(quant_code(x, scale, rcp)); };
  return make_char4(q(v.x), q(v.y), q(v.z), q(v.w));
}

__device__ __forceinline__ float amax4(float4 v) {
  return fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
}

__device__ __forceinline__ float4 swiglu4(float4 g, float4 u) {
  return make_float4(silu_mul(g.x, u.x), silu_mul(g.y, u.y), silu_mul(g.z, u.z),
                     silu_mul(g.w, u.w));
}

// ---- RMSNorm, defined to be identical at every tensor-parallel degree ----------
//
// The row's sum of squares is the fixed tree ((c0+c1)+(c2+c3))+((c4+c5)+(c6+c7))
// of 8 chunk sums (chunk c = columns [c*W/8, (c+1)*W/8)); a chunk sum is
// computed by 128 threads (thread i: float4s i, i+128, ... of the chunk, in
// order), an xor-shuffle tree per warp and ((w0+w1)+w2)+w3 over the chunk's 4
// warps.  A rank of a tensor-parallel group holding 8/N of the chunks computes
// the same chunk sums, so the all-gathered chunk sums give the same total.
// y = (x * gain) * r with r = 1 / sqrt(total / W + eps), and since rounding is
// monotonic, max|y| = (max|x * gain|) * r exactly, so shards combine their
// maxima with a max and get the scale TP=1 gets.
constexpr int kChunks = 8;
constexpr int kChunkThreads = 128;

__device__ __forceinline__ float sumsq4(float4 v) {
  return ((v.x * v.x + v.y * v.y) + v.z * v.z) + v.w * v.w;
}

__device__ __forceinline__ float warp_sum_tree(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float chunk_tree(const float* c) {
  return ((c[0] + c[1]) + (c[2] + c[3])) + ((c[4] + c[5]) + (c[6] + c[7]));
}

__device__ __forceinline__ float4 mul4(float4 a, float4 b) {
  return make_float4(a.x * b.x, a.y * b.y, a.z * b.z, a.w * b.w);
}

__device__ __forceinline__ float4 scale4(float4 a, float r) {
  return make_float4(a.x * r, a.y * r, a.z * r, a.w * r);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// One warp computes a chunk's sum exactly as the 128-thread definition above
// does: lane l plays threads l, 32 + l, 64 + l and 96 + l (the chunk's four
// warps), each summing its float4s l + 32 w + 128 k (k < P) in order, then
// runs each of those warps' xor-shuffle trees (an xor butterfly leaves the
// same sum in every lane) and adds ((w0 + w1) + w2) + w3.  v (when given)
// keeps x * gain, m the max of |x * gain|.
template <int P, bool kKeep, typename Load>
__device__ __forceinline__ float chunk_sum_of(Load load, const float4* __restrict__ gr, int n4,
                                              int l, float4 (&v)[4][P], float& m) {
  float ws[4];
#pragma unroll
  for (int w = 0; w < 4; ++w) {
    float s = 0.0f;
#pragma unroll
    for (int k = 0; k < P; ++k) {
      const int idx = l + 32 * w + kChunkThreads * k;
      if (idx < n4) {
        const float4 x4 = load(w, k, idx);
        s = s + sumsq4(x4);
        const float4 y4 = mul4(x4, __ldg(gr + idx));
        m = fmaxf(m, amax4(y4));
        if (kKeep) v[w][k] = y4;
      }
    }
    ws[w] = warp_sum_tree(s);
  }
  return ((ws[0] + ws[1]) + ws[2]) + ws[3];
}

template <int P, bool kKeep>
__device__ __forceinline__ float chunk_sum(const float4* __restrict__ xr,
                                           const float4* __restrict__ gr, int n4, int l,
                                           float4 (&v)[4][P], float& m) {
  return chunk_sum_of<P, kKeep>([&](int, int, int idx) { return __ldg(xr + idx); }, gr, n4, l, v,
                                m);
}

// TP=1: one CTA of 8 warps per row, warp c the chunk c; P float4 per lane
// and virtual thread.
template <int P>
__global__ void __launch_bounds__(kChunks * 32)
    rmsnorm_quant_kernel(int width, float eps, const float* __restrict__ x,
                         const float* __restrict__ gain, int8_t* __restrict__ xq,
                         long long ldq, float* __restrict__ xs) {
  __shared__ float csum[kChunks];
  __shared__ float cmax[kChunks];
  pdl_wait();
  pdl_trigger();
  const long long row = blockIdx.x;
  const int c = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int n4 = width / (4 * kChunks);  // float4 per chunk
  const float4* xr = reinterpret_cast<const float4*>(x + row * width) + c * n4;
  const float4* gr = reinterpret_cast<const float4*>(gain) + c * n4;
  float4 v[4][P];
  float m = 0.0f;
  const float cs = chunk_sum<P, true>(xr, gr, n4, l, v, m);
  m = warp_max(m);
  if (l == 0) {
    csum[c] = cs;
    cmax[c] = m;
  }
  __syncthreads();
  const float r = 1.0f / sqrtf(chunk_tree(csum) / static_cast<float>(width) + eps);
  float mm = cmax[0];
#pragma unroll
  for (int j = 1; j < kChunks; ++j) mm = fmaxf(mm, cmax[j]);
  const float mx = mm * r;
  const float scale = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
  if (threadIdx.x == 0) xs[row] = scale;
  char4* out = reinterpret_cast<char4*>(xq + row * ldq) + c * n4;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
#pragma unroll
    for (int k = 0; k < P; ++k) {
      const int idx = l + 32 * w + kChunkThreads * k;
      if (idx < n4) out[idx] = q8x4(scale4(v[w][k], r), scale);
    }
  }
}

// The decode step's o-proj output and the MLP's pre-norm in one pass, one
// CTA of 8 warps per token row: h = residual + float(sum of the split-K
// partials) * (x_scale * w_scale) (the skinny reduce's W8A8 epilogue,
// linear.hpp:125-127, then the residual add), written to h_out (the MLP's
// residual), and rmsnorm_quant_kernel's exact steps on it (the same thread
// layout and summation order), so x_q / xs_out hold the bits rmsnorm_quant
// would give on h.  part: [splits][rows][width] int32, token-major.
template <int P>
__global__ void __launch_bounds__(kChunks * 32)
    reduce_rmsnorm_quant_kernel(int width, int splits, const int32_t* __restrict__ part,
                                const float* __restrict__ xs_in, const float* __restrict__ ws,
                                const float* __restrict__ residual, float* __restrict__ h_out,
                                float eps, const float* __restrict__ gain,
                                int8_t* __restrict__ xq, float* __restrict__ xs_out) {
  __shared__ float csum[kChunks];
  __shared__ float cmax[kChunks];
  pdl_wait();
  pdl_trigger();
  const long long row = blockIdx.x;
  const int c = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int n4 = width / (4 * kChunks);  // float4 per chunk
  const long long total = static_cast<long long>(gridDim.x) * width;
  const long long base = row * width + static_cast<long long>(c) * n4 * 4;  // elements
  const float rs = xs_in[row];
  const float4* ws4 = reinterpret_cast<const float4*>(ws) + c * n4;
  const float4* res4 = reinterpret_cast<const float4*>(residual + base);
  float4* h4 = reinterpret_cast<float4*>(h_out + base);
  // every load first (the partials, scales and residual of this thread's
  // float4s), then h and its stores: nothing the stores touch is read after
  float4 hv[4][P];
  int4 acc[4][P];
#pragma unroll
  for (int w = 0; w < 4; ++w)
#pragma unroll
    for (int k = 0; k < P; ++k) {
      const int idx = l + 32 * w + kChunkThreads * k;
      acc[w][k] = idx < n4 ? *reinterpret_cast<const int4*>(part + base + 4ll * idx)
                           : make_int4(0, 0, 0, 0);
    }
  for (int sp = 1; sp < splits; ++sp)
#pragma unroll
    for (int w = 0; w < 4; ++w)
#pragma unroll
      for (int k = 0; k < P; ++k) {
        const int idx = l + 32 * w + kChunkThreads * k;
        if (idx < n4) {
          const int4 b = *reinterpret_cast<const int4*>(part + sp * total + base + 4ll * idx);
          acc[w][k].x += b.x;
          acc[w][k].y += b.y;
          acc[w][k].z += b.z;
          acc[w][k].w += b.w;
        }
      }
#pragma unroll
  for (int w = 0; w < 4; ++w)
#pragma unroll
    for (int k = 0; k < P; ++k) {
      const int idx = l + 32 * w + kChunkThreads * k;
      if (idx < n4) {
        const float4 wv = ws4[idx], r = res4[idx];
        const int4 a = acc[w][k];
        hv[w][k] = make_float4(__fadd_rn(r.x, __fmul_rn(__int2float_rn(a.x), __fmul_rn(rs, wv.x))),
                               __fadd_rn(r.y, __fmul_rn(__int2float_rn(a.y), __fmul_rn(rs, wv.y))),
                               __fadd_rn(r.z, __fmul_rn(__int2float_rn(a.z), __fmul_rn(rs, wv.z))),
                               __fadd_rn(r.w, __fmul_rn(__int2float_rn(a.w), __fmul_rn(rs, wv.w))));
      }
    }
#pragma unroll
  for (int w = 0; w < 4; ++w)
#pragma unroll
    for (int k = 0; k < P; ++k) {
      const int idx = l + 32 * w + kChunkThreads * k;
      if (idx < n4) h4[idx] = hv[w][k];
    }
  const float4* gr = reinterpret_cast<const float4*>(gain) + c * n4;
  float4 v[4][P];
  float m = 0.0f;
  const float cs = chunk_sum_of<P, true>([&](int w, int k, int) { return hv[w][k]; }, gr, n4, l,
                                         v, m);
  m = warp_max(m);
  if (l == 0) {
    csum[c] = cs;
    cmax[c] = m;
  }
  __syncthreads();
  const float r = 1.0f / sqrtf(chunk_tree(csum) / static_cast<float>(width) + eps);
  float mm = cmax[0];
#pragma unroll
  for (int j = 1; j < kChunks; ++j) mm = fmaxf(mm, cmax[j]);
  const float mx = mm * r;
  const float scale = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
  if (threadIdx.x == 0) xs_out[row] = scale;
  char4* out = reinterpret_cast<char4*>(xq + row * static_cast<long long>(width)) + c * n4;
#pragma unroll
  for (int w = 0; w < 4; ++w) {
#pragma unroll
    for (int k = 0; k < P; ++k) {
      const int idx = l + 32 * w + kChunkThreads * k;
      if (idx < n4) out[idx] = q8x4(scale4(v[w][k], r), scale);
    }
  }
}

// TP>1, pass 1: this rank's chunk sums and max|x * gain| over its columns.
// x [rows][width_local], width_local = (chunks_local / 8) * width; stats
// [rows][chunks_local + 1].  One CTA of chunks_local warps per row.
template <int P>
__global__ void __launch_bounds__(kChunks * 32)
    rms_stats_kernel(int width, int chunks_local, const float* __restrict__ x,
                     const float* __restrict__ gain, PeerDst stats) {
  __shared__ float cmax[kChunks];
  const long long row = blockIdx.x;
  const int c = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int n4 = width / (4 * kChunks);
  const int wl = chunks_local * (width / kChunks);
  const float4* xr = reinterpret_cast<const float4*>(x + row * wl) + c * n4;
  const float4* gr = reinterpret_cast<const float4*>(gain) + c * n4;
  float4 unused[4][P];
  float m = 0.0f;
  const float cs = chunk_sum<P, false>(xr, gr, n4, l, unused, m);
  m = warp_max(m);
  const long long off = row * (chunks_local + 1);
  if (l == 0) {
    for (int d = 0; d < stats.n; ++d) static_cast<float*>(stats.p[d])[off + c] = cs;
    cmax[c] = m;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float mm = cmax[0];
    for (int j = 1; j < chunks_local; ++j) mm = fmaxf(mm, cmax[j]);
    for (int d = 0; d < stats.n; ++d) static_cast<float*>(stats.p[d])[off + chunks_local] = mm;
  }
}

// TP>1, pass 2: from the all-gathered stats [ranks][rows][chunks_local + 1],
// the row's r and scale (identical on every rank and to TP=1), then this
// rank's columns quantised.  One CTA of chunks_local warps per row.
template <int P>
__global__ void __launch_bounds__(kChunks * 32)
    rms_apply_kernel(int width, int chunks_local, int ranks, long long rows, float eps,
                     const float* __restrict__ x, const float* __restrict__ gain,
                     const float* __restrict__ stats_all, PeerDst xq, float* __restrict__ xs) {
  __shared__ float rs[2];
  const long long row = blockIdx.x;
  const int c = threadIdx.x >> 5, l = threadIdx.x & 31;
  const int S = chunks_local + 1;
  if (threadIdx.x == 0) {
    float cs[kChunks];
    float mx = 0.0f;
    for (int g = 0; g < ranks; ++g) {
      const float* st = stats_all + (static_cast<long long>(g) * rows + row) * S;
      for (int j = 0; j < chunks_local; ++j) cs[g * chunks_local + j] = st[j];
      mx = fmaxf(mx, st[chunks_local]);
    }
    const float r = 1.0f / sqrtf(chunk_tree(cs) / static_cast<float>(width) + eps);
    const float m = mx * r;
    rs[0] = r;
    rs[1] = m > 0.0f ? __fdiv_rn(m, 127.0f) : 1.0f;
    xs[row] = rs[1];
  }
  __syncthreads();
  const float r = rs[0], scale = rs[1];
  const int n4 = width / (4 * kChunks);
  const int wl = chunks_local * (width / kChunks);
  const float4* xr = reinterpret_cast<const float4*>(x + row * wl) + c * n4;
  const float4* gr = reinterpret_cast<const float4*>(gain) + c * n4;
  const long long off = row * wl + static_cast<long long>(c) * n4 * 4;  // bytes
#pragma unroll
  for (int k = 0; k < 4 * P; ++k) {
    const int idx = l + 32 * k;
    if (idx < n4) {
      const char4 q = q8x4(scale4(mul4(__ldg(xr + idx), __ldg(gr + idx)), r), scale);
      for (int d = 0; d < xq.n; ++d)
        reinterpret_cast<char4*>(static_cast<int8_t*>(xq.p[d]) + off)[idx] = q;
    }
  }
}

// SwiGLU on the split-K partials of the gate/up projection (one CTA per
// row): g and u are the W8A8 epilogue values of columns n and ffn + n
// (float(sum) * (x_scale * w_scale), linear.hpp:125-127), h = silu_mul(g, u)
// as everywhere else.  row_max_out: write max |h| only.  Else quantise with
// row_max_in, or the row's own max when it is null.
template <int CACHE>
__global__ void __launch_bounds__(kThreads)
    swiglu_partials_kernel(int ffn, int splits, const int32_t* __restrict__ part,
                           const float* __restrict__ xs, const float* __restrict__ ws,
                           const float* __restrict__ row_max_in, float* __restrict__ row_max_out,
                           int8_t* __restrict__ xq, long long ldq, float* __restrict__ qs) {
  __shared__ float red[32];
  pdl_wait();
  pdl_trigger();
  const long long row = blockIdx.x;
  const long long stride = static_cast<long long>(gridDim.x) * 2 * ffn;
  const int4* p4 = reinterpret_cast<const int4*>(part + row * 2 * ffn);
  const float4* ws4 = reinterpret_cast<const float4*>(ws);
  const int n4 = ffn >> 2;
  const float rs = xs[row];
  float4 c[CACHE];
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < CACHE; ++i) {
    const int idx = threadIdx.x + i * kThreads;
    if (idx < n4) {
      int4 g = p4[idx], u = p4[n4 + idx];
      for (int s = 1; s < splits; ++s) {
        const int4 g2 = p4[s * stride / 4 + idx], u2 = p4[s * stride / 4 + n4 + idx];
        g.x += g2.x; g.y += g2.y; g.z += g2.z; g.w += g2.w;
        u.x += u2.x; u.y += u2.y; u.z += u2.z; u.w += u2.w;
      }
      const float4 wg = ws4[idx], wu = ws4[n4 + idx];
      const float4 gf = make_float4(__fmul_rn(__int2float_rn(g.x), __fmul_rn(rs, wg.x)),
                                    __fmul_rn(__int2float_rn(g.y), __fmul_rn(rs, wg.y)),
                                    __fmul_rn(__int2float_rn(g.z), __fmul_rn(rs, wg.z)),
                                    __fmul_rn(__int2float_rn(g.w), __fmul_rn(rs, wg.w)));
      const float4 uf = make_float4(__fmul_rn(__int2float_rn(u.x), __fmul_rn(rs, wu.x)),
                                    __fmul_rn(__int2float_rn(u.y), __fmul_rn(rs, wu.y)),
                                    __fmul_rn(__int2float_rn(u.z), __fmul_rn(rs, wu.z)),
                                    __fmul_rn(__int2float_rn(u.w), __fmul_rn(rs, wu.w)));
      c[i] = swiglu4(gf, uf);
      m = fmaxf(m, amax4(c[i]));
    }
  }
  if (row_max_out != nullptr) {
    m = block_max(m, red);
    if (threadIdx.x == 0) row_max_out[row] = m;
    return;
  }
  const float mx = row_max_in != nullptr ? row_max_in[row] : block_max(m, red);
  const float scale = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
  if (threadIdx.x == 0) qs[row] = scale;
  char4* out = reinterpret_cast<char4*>(xq + row * ldq);
#pragma unroll
  for (int i = 0; i < CACHE; ++i) {
    const int idx = threadIdx.x + i * kThreads;
    if (idx < n4) out[idx] = q8x4(c[i], scale);
  }
}

}  // namespace

// Smallest supported per-thread cache (float4) that holds n4 float4.
static int cache_for(int n4) {
  const int per = (n4 + kThreads - 1) / kThreads;
  for (int c : {1, 2, 4, 6, 8, 12, 16})
    if (per <= c) return c;
  return 0;
}

static int per_thread(int width) {  // float4 per thread in the chunked RMSNorm
  const int n4 = width / (4 * kChunks);
  return (n4 + kChunkThreads - 1) / kChunkThreads;
}

int rmsnorm_quant(long long rows, int width, float eps, const float* x, const float* gain,
                  int8_t* x_q, float* x_scale, cudaStream_t stream) {
  if (rows == 0) return kOk;
  if (width <= 0 || width % (4 * kChunks) != 0) return kErrInvalid;
  const unsigned grid = static_cast<unsigned>(rows);
  const int P = per_thread(width);
  const dim3 T(kChunks * 32);
  const long long ld = width;
  if (P <= 1) return launch_k(rmsnorm_quant_kernel<1>, dim3(grid), T, 0, stream, width, eps, x, gain, x_q, ld, x_scale);
  if (P <= 2) return launch_k(rmsnorm_quant_kernel<2>, dim3(grid), T, 0, stream, width, eps, x, gain, x_q, ld, x_scale);
  if (P <= 4) return launch_k(rmsnorm_quant_kernel<4>, dim3(grid), T, 0, stream, width, eps, x, gain, x_q, ld, x_scale);
  return kErrInvalid;
}

int reduce_rmsnorm_quant(long long rows, int width, int splits, const int32_t* part,
                         const float* x_scale, const float* w_scale, const float* residual,
                         float* h, float eps, const float* gain, int8_t* x_q, float* q_scale,
                         cudaStream_t stream) {
  if (rows == 0) return kOk;
  if (width <= 0 || width % (4 * kChunks) != 0 || splits < 1 || !part || !x_scale || !w_scale ||
      !residual || !h || !gain || !x_q || !q_scale)
    return kErrInvalid;
  if ((reinterpret_cast<uintptr_t>(part) | reinterpret_cast<uintptr_t>(w_scale) |
       reinterpret_cast<uintptr_t>(residual) | reinterpret_cast<uintptr_t>(h) |
       reinterpret_cast<uintptr_t>(gain)) & 15u)
    return kErrAlignment;
  const dim3 grid(static_cast<unsigned>(rows)), T(kChunks * 32);
  const int P = per_thread(width);
  if (P <= 1) return launch_k(reduce_rmsnorm_quant_kernel<1>, grid, T, 0, stream, width, splits, part, x_scale, w_scale, residual, h, eps, gain, x_q, q_scale);
  if (P <= 2) return launch_k(reduce_rmsnorm_quant_kernel<2>, grid, T, 0, stream, width, splits, part, x_scale, w_scale, residual, h, eps, gain, x_q, q_scale);
  if (P <= 4) return launch_k(reduce_rmsnorm_quant_kernel<4>, grid, T, 0, stream, width, splits, part, x_scale, w_scale, residual, h, eps, gain, x_q, q_scale);
  return kErrInvalid;
}

int rms_stats(long long rows, int width, int ranks, const float* x_local, const float* gain_local,
              const PeerDst& stats, cudaStream_t stream) {
  if (rows == 0) return kOk;
  if (width % (4 * kChunks) != 0 || kChunks % ranks != 0 || !dst_ok(stats)) return kErrInvalid;
  const int cl = kChunks / ranks, P = per_thread(width);
  const unsigned grid = static_cast<unsigned>(rows);
  const int T = cl * 32;
  if (P <= 1) rms_stats_kernel<1><<<grid, T, 0, stream>>>(width, cl, x_local, gain_local, stats);
  else if (P <= 2) rms_stats_kernel<2><<<grid, T, 0, stream>>>(width, cl, x_local, gain_local, stats);
  else if (P <= 4) rms_stats_kernel<4><<<grid, T, 0, stream>>>(width, cl, x_local, gain_local, stats);
  else return kErrInvalid;
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int rms_apply_quant(long long rows, int width, int ranks, float eps, const float* x_local,
                    const float* gain_local, const float* stats_all, const PeerDst& x_q,
                    float* x_scale, cudaStream_t stream) {
  if (rows == 0) return kOk;
  if (width % (4 * kChunks) != 0 || kChunks % ranks != 0 || !dst_ok(x_q)) return kErrInvalid;
  const int cl = kChunks / ranks, P = per_thread(width);
  const unsigned grid = static_cast<unsigned>(rows);
  const int T = cl * 32;
  if (P <= 1)
    rms_apply_kernel<1><<<grid, T, 0, stream>>>(width, cl, ranks, rows, eps, x_local, gain_local, stats_all, x_q, x_scale);
  else if (P <= 2)
    rms_apply_kernel<2><<<grid, T, 0, stream>>>(width, cl, ranks, rows, eps, x_local, gain_local, stats_all, x_q, x_scale);
  else if (P <= 4)
    rms_apply_kernel<4><<<grid, T, 0, stream>>>(width, cl, ranks, rows, eps, x_local, gain_local, stats_all, x_q, x_scale);
  else return kErrInvalid;
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int swiglu_partials(long long rows, int ffn, const int32_t* part, int splits, const float* x_scale,
                    const float* w_scale, const float* row_max_in, float* row_max_out,
                    int8_t* x_q, float* q_scale, cudaStream_t stream) {
  if (rows == 0) return kOk;
  const int c = cache_for(ffn / 4);
  if (ffn <= 0 || ffn % 4 != 0 || c == 0 || splits < 1 || !part || !x_scale || !w_scale)
    return kErrInvalid;
  if (row_max_out == nullptr && (x_q == nullptr || q_scale == nullptr)) return kErrInvalid;
  if ((reinterpret_cast<uintptr_t>(part) | reinterpret_cast<uintptr_t>(w_scale)) & 15u)
    return kErrAlignment;
  const dim3 grid(static_cast<unsigned>(rows)), block(kThreads);
  const long long ld = ffn;
#define REEF_SWIGLU_PARTIALS(C)                                                               \
  return launch_k(swiglu_partials_kernel<C>, grid, block, 0, stream, ffn, splits, part, x_scale, \
                  w_scale, row_max_in, row_max_out, x_q, ld, q_scale)
  switch (c) {
    case 1: REEF_SWIGLU_PARTIALS(1);
    case 2: REEF_SWIGLU_PARTIALS(2);
    case 4: REEF_SWIGLU_PARTIALS(4);
    case 6: REEF_SWIGLU_PARTIALS(6);
    case 8: REEF_SWIGLU_PARTIALS(8);
    case 12: REEF_SWIGLU_PARTIALS(12);
    default: REEF_SWIGLU_PARTIALS(16);
  }
#undef REEF_SWIGLU_PARTIALS
}

}  // namespace reef
