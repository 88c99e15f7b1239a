// lm_head.cu -- GPT-Neo's token input, output projection and greedy token
// choice.
//
// embedding_f32 is reef's embedding (embedding.hpp:31-66 lookup_token_embeddings
// then add_position_embeddings; the firmware's embedding_f32, kernels.hpp:81-84):
// y[t][c] = wte[id_t][c] + wpe[first_position + t][c], one rounded float add.
// The ids are read on the device (the previous step's argmax), so a decode
// loop needs no host round trip.  The engine throws on an id outside the
// vocabulary or a non-finite sum; here the first records kDevBadToken (and
// the row is written as zeros) and the second kDevNonFinite.
//
// matvec_rows_f32 is reef's float linear(x, wte) for one row
// (operator/linear.hpp:75-84 through tensor.hpp:179-192): every logit starts
// from 0 and adds the products x[k] * w[c][k] one after another, k = 0, 1,
// ..., each product and each sum rounded to float on its own (no fused
// multiply-add), so the result is bit-identical to the engine.  The engine
// throws std::overflow_error when a product or a sum is infinite or NaN
// (util.hpp:81-131); here that is recorded in the device error word.
//
// Work: in * out products, one read of w (out * in * 4 bytes): HBM-bound.
// One thread owns one output row and must add its products in order, so the
// CTA's 128 rows are staged through shared memory 32 columns at a time with
// coalesced loads (rows padded to 33 floats: each thread then reads its own
// row without bank conflicts).
//
// argmax_f32 is reef's argmax (model.hpp:32-42): the index of the first
// largest value, found by a scan that replaces the best index only on a
// strictly greater value.  So ties keep the lowest index, a NaN never
// replaces the best, and when x[0] is NaN nothing compares greater and the
// answer is 0.  One CTA reduces (value, index) pairs with exactly that order.
#include "common.cuh"
#include "ops.h"

#include <cmath>
#include <cstdint>

namespace reef {

namespace {

constexpr int kRows = 128;   // output rows per CTA, one per thread
constexpr int kCols = 32;    // columns staged per pass
constexpr int kArgThreads = 1024;

__global__ void __launch_bounds__(kRows)
    matvec_rows_f32_kernel(long long out, long long in, const float* __restrict__ w,
                           const float* __restrict__ x, float* __restrict__ y, int* err) {
  __shared__ float tile[kRows][kCols + 1];
  __shared__ float xs[kCols];
  const long long r0 = static_cast<long long>(blockIdx.x) * kRows;
  const int tid = threadIdx.x;
  float sum = 0.0f;
  bool finite = true;
  for (long long k0 = 0; k0 < in; k0 += kCols) {
    const int kc = static_cast<int>(in - k0 < kCols ? in - k0 : kCols);
    // 32 consecutive threads read 32 consecutive floats of one row
    for (int i = tid; i < kRows * kCols; i += kRows) {
      const int rr = i / kCols, kk = i % kCols;
      const long long row = r0 + rr;
      tile[rr][kk] = (row < out && kk < kc) ? w[row * in + k0 + kk] : 0.0f;
    }
    if (tid < kCols) xs[tid] = tid < kc ? x[k0 + tid] : 0.0f;
    __syncthreads();
    for (int kk = 0; kk < kc; ++kk) {
      const float p = __fmul_rn(xs[kk], tile[tid][kk]);
      sum = __fadd_rn(sum, p);
      finite = finite && isfinite(p) && isfinite(sum);
    }
    __syncthreads();
  }
  if (r0 + tid < out) {
    y[r0 + tid] = sum;
    if (!finite) record_error(err, kDevNonFinite);
  }
}

// (value, index) with the scan's order: a beats b when it is greater, or
// equal with a lower index.  NaN values never enter (they never replace the
// best in the scan); index ~0 marks "no value yet".
struct Best {
  float v;
  unsigned long long i;
};

__device__ __forceinline__ Best better(Best a, Best b) {
  if (a.i == ~0ull) return b;
  if (b.i == ~0ull) return a;
  if (a.v > b.v || (a.v == b.v && a.i < b.i)) return a;
  return b;
}

__global__ void __launch_bounds__(kArgThreads)
    argmax_f32_kernel(long long n, const float* __restrict__ x, uint32_t* __restrict__ index) {
  __shared__ float sv[kArgThreads / 32];
  __shared__ unsigned long long si[kArgThreads / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  Best b{-INFINITY, ~0ull};
  for (long long i = tid; i < n; i += kArgThreads) {
    const float v = x[i];
    if (!isnan(v)) b = better(b, Best{v, static_cast<unsigned long long>(i)});
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const Best o{__shfl_xor_sync(0xffffffffu, b.v, off), __shfl_xor_sync(0xffffffffu, b.i, off)};
    b = better(b, o);
  }
  if (lane == 0) {
    sv[warp] = b.v;
    si[warp] = b.i;
  }
  __syncthreads();
  if (tid == 0) {
    Best r{sv[0], si[0]};
    for (int w = 1; w < kArgThreads / 32; ++w) r = better(r, Best{sv[w], si[w]});
    // x[0] NaN: nothing compares greater than it, so the scan keeps 0; with
    // every value NaN the same holds
    *index = (isnan(x[0]) || r.i == ~0ull) ? 0u : static_cast<uint32_t>(r.i);
  }
}

__global__ void embedding_f32_kernel(int width, const uint32_t* __restrict__ ids,
                                     long long first_position, long long vocab,
                                     long long positions, const float* __restrict__ wte,
                                     const float* __restrict__ wpe, float* __restrict__ y,
                                     int* err) {
  const long long t = blockIdx.x;
  const uint32_t id = ids[t];
  const long long pos = first_position + t;
  float* yr = y + t * width;
  if (id >= vocab || pos >= positions) {
    if (threadIdx.x == 0) record_error(err, id >= vocab ? kDevBadToken : kDevBadPosition);
    for (int c = threadIdx.x; c < width; c += blockDim.x) yr[c] = 0.0f;
    return;
  }
  const float* a = wte + static_cast<long long>(id) * width;
  const float* b = wpe + pos * width;
  bool finite = true;
  for (int c = threadIdx.x; c < width; c += blockDim.x) {
    const float v = __fadd_rn(a[c], b[c]);
    finite = finite && isfinite(v);
    yr[c] = v;
  }
  if (!finite) record_error(err, kDevNonFinite);
}

}  // namespace

int embedding_f32(int width, long long count, const uint32_t* ids, long long first_position,
                  long long vocab, long long positions, const float* wte, const float* wpe,
                  float* y, cudaStream_t stream) {
  if (width <= 0 || count <= 0 || vocab <= 0 || positions <= 0 || first_position < 0 ||
      ids == nullptr || wte == nullptr || wpe == nullptr || y == nullptr)
    return kErrInvalid;
  if (count > 0x7fffffffLL) return kErrTooLarge;
  embedding_f32_kernel<<<static_cast<unsigned>(count), 128, 0, stream>>>(
      width, ids, first_position, vocab, positions, wte, wpe, y, device_error_ptr());
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int matvec_rows_f32(long long out, long long in, const float* w, const float* x, float* y,
                    cudaStream_t stream) {
  if (out <= 0 || in <= 0 || w == nullptr || x == nullptr || y == nullptr) return kErrInvalid;
  const long long blocks = (out + kRows - 1) / kRows;
  if (blocks > 0x7fffffffLL) return kErrTooLarge;
  matvec_rows_f32_kernel<<<static_cast<unsigned>(blocks), kRows, 0, stream>>>(
      out, in, w, x, y, device_error_ptr());
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int argmax_f32(long long n, const float* x, uint32_t* index, cudaStream_t stream) {
  if (n <= 0 || x == nullptr || index == nullptr) return kErrInvalid;
  if (n > 0xffffffffLL) return kErrTooLarge;
  argmax_f32_kernel<<<1, kArgThreads, 0, stream>>>(n, x, index);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace reef
