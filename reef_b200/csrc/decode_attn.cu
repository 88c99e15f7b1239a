// decode_attn.cu -- int8 attention for decode (one new query per sequence)
// over an int8 KV cache, split across CTAs along the cached keys.
//
// The head is reef's attend_head (attention.hpp:117-123) for a query at the
// last cached position (it sees every cached key), on int8 q / k / v with one
// fp32 scale per (token, head), a score scale, and GQA: the G = Hq / Hkv
// query heads of one KV head share its K / V stream, so each cache byte is
// read from HBM once for all of them.  Checked against the float head on the
// dequantised inputs within 1e-2.
//
// HBM-bound: each launch reads the cache once (K + V + scales); the math is
// G x 128 int8 dot products per key (dp4a) and G x 128 FMAs per key for P.V.
//
// Kernel 1 (grid: chunks x (batch * Hkv), 256 threads): one CTA stages a
// chunk of <= 256 keys of K and V in shared memory (rows 144 bytes apart, so
// the 16-byte row reads below are bank-conflict free), computes the G score
// rows (thread = key), the chunk's max and sum per head (block reductions),
// and O_h = sum_j exp(s_hj - max_h) * v_scale_j * v_j, (thread = head x 4
// dims), then writes (max, sum, O) for its chunk.
// Kernel 2 (grid: batch * Hq, 128 threads): merges the chunks of one head.
#include "common.cuh"
#include "ops.h"

namespace reef {

namespace {

constexpr int kDThreads = 256;
constexpr int kChunk = 256;       // keys per CTA (max)
constexpr int kRow = 144;         // bytes between staged rows (128 + 16)
constexpr int kMaxGroup = 16;     // query heads per KV head
constexpr float kLog2e = 1.4426950408889634f;

struct DecodeArgs {
  int batch, heads_q, heads_kv, group, max_len, chunks;
  float sm_scale;
  const int8_t* q8;        // [B][Hq][128]
  const float* q_scale;    // [B][Hq]
  const int8_t* k_cache;   // [B][Hkv][max_len][128]
  const float* k_scale;    // [B][Hkv][max_len]
  const int8_t* v_cache;
  const float* v_scale;
  const int* lens;         // [B] keys per sequence, or null
  int len;                 // keys per sequence when lens is null
  float* part;             // [chunks][B][Hq][2 + 128]
  float* out;              // [B][Hq][128]
};

template <int G>
__global__ void __launch_bounds__(kDThreads)
    decode_split_kernel(DecodeArgs a) {
  extern __shared__ __align__(16) uint8_t sm[];
  uint8_t* ks = sm;                                  // [kChunk][kRow]
  uint8_t* vs = ks + kChunk * kRow;                  // [kChunk][kRow]
  float* ksc = reinterpret_cast<float*>(vs + kChunk * kRow);  // [kChunk]
  float* vsc = ksc + kChunk;                         // [kChunk]
  float* p = vsc + kChunk;                           // [G][kChunk]
  float* red = p + G * kChunk;                       // [8 warps][G]
  float* stat = red + 8 * G;                         // [2][G]: max, sum
  int* qw = reinterpret_cast<int*>(stat + 2 * G);    // [G][32] q words

  const int chunk = blockIdx.x;
  const int bk = blockIdx.y;  // b * Hkv + hkv
  const int b = bk / a.heads_kv, hkv = bk % a.heads_kv;
  const int len = a.lens != nullptr ? a.lens[b] : a.len;
  const int key0 = chunk * kChunk;
  const int nkeys = min(kChunk, len - key0);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int h0 = hkv * G;  // first query head of this KV head
  float* part = a.part + ((static_cast<long long>(chunk) * a.batch + b) * a.heads_q + h0) * 130;
  if (nkeys <= 0) {  // chunk past this sequence's end: an empty partial
    for (int i = tid; i < G * 130; i += kDThreads) part[i] = (i % 130 == 0) ? -INFINITY : 0.0f;
    return;
  }

  // stage q (G x 128 int8), K and V rows, and the per-key scales
  const int* q32 = reinterpret_cast<const int*>(a.q8 + (static_cast<long long>(b) * a.heads_q + h0) * 128);
  for (int i = tid; i < G * 32; i += kDThreads) qw[i] = q32[i];
  const long long row0 = (static_cast<long long>(bk) * a.max_len + key0);
  const uint4* kg = reinterpret_cast<const uint4*>(a.k_cache + row0 * 128);
  const uint4* vg = reinterpret_cast<const uint4*>(a.v_cache + row0 * 128);
  for (int i = tid; i < nkeys * 8; i += kDThreads) {
    const int r = i >> 3, c = i & 7;
    *reinterpret_cast<uint4*>(ks + r * kRow + c * 16) = __ldg(kg + i);
    *reinterpret_cast<uint4*>(vs + r * kRow + c * 16) = __ldg(vg + i);
  }
  for (int i = tid; i < nkeys; i += kDThreads) {
    ksc[i] = a.k_scale[row0 + i];
    vsc[i] = a.v_scale[row0 + i];
  }
  __syncthreads();

  // scores: thread = key, G heads
  float s[G];
#pragma unroll
  for (int h = 0; h < G; ++h) s[h] = -INFINITY;
  const float base = a.sm_scale * kLog2e;
  float qs[G];
#pragma unroll
  for (int h = 0; h < G; ++h) qs[h] = a.q_scale[static_cast<long long>(b) * a.heads_q + h0 + h] * base;
  float mloc[G];
#pragma unroll
  for (int h = 0; h < G; ++h) mloc[h] = -INFINITY;
  if (tid < nkeys) {
    int acc[G];
#pragma unroll
    for (int h = 0; h < G; ++h) acc[h] = 0;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const uint4 k4 = *reinterpret_cast<const uint4*>(ks + tid * kRow + c * 16);
      const int kw[4] = {static_cast<int>(k4.x), static_cast<int>(k4.y), static_cast<int>(k4.z),
                         static_cast<int>(k4.w)};
#pragma unroll
      for (int h = 0; h < G; ++h) {
#pragma unroll
        for (int e = 0; e < 4; ++e) acc[h] = __dp4a(kw[e], qw[h * 32 + c * 4 + e], acc[h]);
      }
    }
    const float kscale = ksc[tid];
#pragma unroll
    for (int h = 0; h < G; ++h) {
      s[h] = static_cast<float>(acc[h]) * qs[h] * kscale;
      mloc[h] = s[h];
    }
  }
  // chunk max per head
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float v = mloc[h];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (lane == 0) red[warp * G + h] = v;
  }
  __syncthreads();
  if (tid < G) {
    float v = -INFINITY;
    for (int w = 0; w < kDThreads / 32; ++w) v = fmaxf(v, red[w * G + tid]);
    stat[tid] = v;
  }
  __syncthreads();
  // probabilities (relative to the chunk max) and their sum per head
  float sum[G];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    const float e = tid < nkeys ? exp2f(s[h] - stat[h]) : 0.0f;
    sum[h] = e;
    if (tid < kChunk) p[h * kChunk + tid] = e * (tid < nkeys ? vsc[tid] : 0.0f);
  }
#pragma unroll
  for (int h = 0; h < G; ++h) {
    float v = sum[h];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    __syncwarp();
    if (lane == 0) red[warp * G + h] = v;
  }
  __syncthreads();
  if (tid < G) {
    float v = 0.0f;
    for (int w = 0; w < kDThreads / 32; ++w) v += red[w * G + tid];
    stat[G + tid] = v;
  }
  __syncthreads();

  // O_h[d..d+3] = sum_j p'_hj * v_j[d..d+3]; thread = (head, 4 dims), looping
  // over heads when G > 8
  for (int hd = tid; hd < G * 32; hd += kDThreads) {
    const int h = hd >> 5, dq = hd & 31;
    float o0 = 0.f, o1 = 0.f, o2 = 0.f, o3 = 0.f;
    const float* ph = p + h * kChunk;
    for (int j = 0; j < nkeys; ++j) {
      // int8 -> float without the conversion pipe: flip the sign bit (byte
      // b becomes b + 128), place it in the mantissa of 2^23, subtract
      // 2^23 + 128 (exact for every byte)
      const uint32_t w = *reinterpret_cast<const uint32_t*>(vs + j * kRow + dq * 4) ^ 0x80808080u;
      const float pj = ph[j];
      const float v0 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540)) - 8388736.0f;
      const float v1 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7541)) - 8388736.0f;
      const float v2 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7542)) - 8388736.0f;
      const float v3 = __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7543)) - 8388736.0f;
      o0 = __fmaf_rn(pj, v0, o0);
      o1 = __fmaf_rn(pj, v1, o1);
      o2 = __fmaf_rn(pj, v2, o2);
      o3 = __fmaf_rn(pj, v3, o3);
    }
    float* ph_out = part + h * 130;
    *reinterpret_cast<float2*>(ph_out + 2 + dq * 4) = make_float2(o0, o1);
    *reinterpret_cast<float2*>(ph_out + 4 + dq * 4) = make_float2(o2, o3);
    if (dq == 0) {
      ph_out[0] = stat[h];
      ph_out[1] = stat[G + h];
    }
  }
}

__global__ void decode_combine_kernel(DecodeArgs a) {
  const int bh = blockIdx.x;  // b * Hq + h
  const int d = threadIdx.x;  // 128
  float m = -INFINITY;
  for (int c = 0; c < a.chunks; ++c) m = fmaxf(m, a.part[(static_cast<long long>(c) * a.batch * a.heads_q + bh) * 130]);
  float l = 0.0f, o = 0.0f;
  for (int c = 0; c < a.chunks; ++c) {
    const float* pc = a.part + (static_cast<long long>(c) * a.batch * a.heads_q + bh) * 130;
    const float mc = pc[0];
    if (mc == -INFINITY) continue;
    const float w = exp2f(mc - m);
    l += w * pc[1];
    o += w * pc[2 + d];
  }
  a.out[static_cast<long long>(bh) * 128 + d] = o / l;
}

template <int G>
size_t split_smem() {
  return static_cast<size_t>(kChunk) * kRow * 2 + kChunk * 4 * 2 + G * kChunk * 4 + 8 * G * 4 +
         2 * G * 4 + G * 32 * 4;
}

template <int G>
int launch_split(const DecodeArgs& a, cudaStream_t st) {
  const size_t smem = split_smem<G>();
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(decode_split_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess)
      return kErrCuda;
    configured[dev] = true;
  }
  dim3 grid(static_cast<unsigned>(a.chunks), static_cast<unsigned>(a.batch * a.heads_kv));
  decode_split_kernel<G><<<grid, kDThreads, smem, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

// One decode step's q / k / v: one warp per (sequence, head) of the QKV
// projection output qkv [B][(Hq + 2 Hkv) * 128].  q and k get rotate-half
// RoPE at the sequence's position; every head row is quantised with reef's
// rule (quant.hpp:51-81); q goes to q8 / q_scale, k and v are appended to the
// cache at row `pos`, and lens[b] = pos + 1.  A position outside the cache is
// recorded in the device error word and the row is skipped.
__global__ void decode_rope_append_kernel(int batch, int hq, int hkv, int max_len, float base,
                                          const int* __restrict__ positions,
                                          const float* __restrict__ qkv, int8_t* __restrict__ q8,
                                          float* __restrict__ q_scale, int8_t* __restrict__ k_cache,
                                          float* __restrict__ k_scale, int8_t* __restrict__ v_cache,
                                          float* __restrict__ v_scale, int* __restrict__ lens,
                                          int* err) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int heads = hq + 2 * hkv;
  if (gw >= batch * heads) return;
  const int b = gw / heads, hh = gw % heads;
  const int pos = positions[b];
  if (pos < 0 || pos >= max_len) {
    if (lane == 0 && hh == 0) record_error(err, 0x201);
    return;
  }
  if (hh == 0 && lane == 0) lens[b] = pos + 1;
  const float* x = qkv + static_cast<long long>(b) * heads * 128 + hh * 128;
  float v[4] = {x[lane], x[lane + 32], x[lane + 64], x[lane + 96]};
  if (hh < hq + hkv) {  // q or k: rotate-half RoPE, pairs (i, i + 64)
#pragma unroll
    for (int p = 0; p < 2; ++p) {
      const int i = lane + 32 * p;
      const float inv_freq = powf(base, -static_cast<float>(2 * i) / 128.0f);
      float sn, cs;
      sincosf(static_cast<float>(pos) * inv_freq, &sn, &cs);
      const float lo = v[p], hi = v[p + 2];
      v[p] = lo * cs - hi * sn;
      v[p + 2] = hi * cs + lo * sn;
    }
  }
  float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float scale = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
  int8_t* dst;
  if (hh < hq) {
    dst = q8 + (static_cast<long long>(b) * hq + hh) * 128;
    if (lane == 0) q_scale[static_cast<long long>(b) * hq + hh] = scale;
  } else {
    const bool is_k = hh < hq + hkv;
    const int kh = is_k ? hh - hq : hh - hq - hkv;
    const long long row = (static_cast<long long>(b) * hkv + kh) * max_len + pos;
    dst = (is_k ? k_cache : v_cache) + row * 128;
    if (lane == 0) (is_k ? k_scale : v_scale)[row] = scale;
  }
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    int c = __float2int_rn(__fdiv_rn(v[p], scale));
    c = c < -127 ? -127 : (c > 127 ? 127 : c);
    dst[lane + 32 * p] = static_cast<int8_t>(c);
  }
}

}  // namespace

int decode_rope_append(int batch, int heads_q, int heads_kv, int max_len, float rope_base,
                       const int* positions, const float* qkv, int8_t* q8, float* q_scale,
                       int8_t* k_cache, float* k_scale, int8_t* v_cache, float* v_scale, int* lens,
                       cudaStream_t stream) {
  const long long warps = static_cast<long long>(batch) * (heads_q + 2 * heads_kv);
  decode_rope_append_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, stream>>>(
      batch, heads_q, heads_kv, max_len, rope_base, positions, qkv, q8, q_scale, k_cache, k_scale,
      v_cache, v_scale, lens, device_error_ptr());
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

size_t decode_attn_partial_floats(int batch, int heads_q, int max_len) {
  const int chunks = (max_len + kChunk - 1) / kChunk;
  return static_cast<size_t>(chunks) * batch * heads_q * 130;
}

int decode_attn_i8(const DecodeProblem& p, cudaStream_t st) {
  if (p.batch <= 0 || p.heads_q <= 0 || p.heads_kv <= 0 || p.max_len <= 0) return kErrInvalid;
  if (p.heads_q % p.heads_kv != 0) return kErrInvalid;
  const int G = p.heads_q / p.heads_kv;
  if (G > kMaxGroup) return kErrInvalid;
  DecodeArgs a{};
  a.batch = p.batch;
  a.heads_q = p.heads_q;
  a.heads_kv = p.heads_kv;
  a.group = G;
  a.max_len = p.max_len;
  a.chunks = (p.max_len + kChunk - 1) / kChunk;
  a.sm_scale = p.sm_scale;
  a.q8 = p.q8;
  a.q_scale = p.q_scale;
  a.k_cache = p.k_cache;
  a.k_scale = p.k_scale;
  a.v_cache = p.v_cache;
  a.v_scale = p.v_scale;
  a.lens = p.lens;
  a.len = p.len;
  a.part = p.partial;
  a.out = p.out;
  int rc;
  switch (G) {
    case 1: rc = launch_split<1>(a, st); break;
    case 2: rc = launch_split<2>(a, st); break;
    case 4: rc = launch_split<4>(a, st); break;
    case 8: rc = launch_split<8>(a, st); break;
    case 16: rc = launch_split<16>(a, st); break;
    default: return kErrInvalid;
  }
  if (rc) return rc;
  decode_combine_kernel<<<static_cast<unsigned>(p.batch * p.heads_q), 128, 0, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace reef
