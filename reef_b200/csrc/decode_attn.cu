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
// HBM-bound by design, and built so that the per-byte instruction count is
// small enough for the copies to set the pace:
//   * a CTA streams its split of one (sequence, KV head) in 128-key tiles
//     through a 3-stage ring: K and V by TMA (128-byte swizzle, so the
//     tensor-core fragment loads below hit every bank once), their scales by
//     bulk copies, all completing on one mbarrier per stage; thread 0
//     refills a stage once the eight warps have released it (a second
//     mbarrier per stage), so there is no CTA-wide barrier per tile;
//   * warp w owns keys [16w, 16w + 16) of every tile and keeps its own
//     online-softmax state: S = q . K^T for the G heads (padded to 16 rows)
//     by int8 mma.sync m16n8k32 with q resident in registers; the scores,
//     the running max and the exponentials stay in the accumulator
//     registers, whose layout is the A operand of the P . V mma (f16
//     m16n8k16), so P never goes through shared memory;
//   * V reaches the P . V mma from the int8 tile with ldmatrix .trans on
//     byte pairs: a thread receives two dims of two keys and splits them into
//     two f16 pairs (exact, by byte permutes under the 0x64 exponent), so the
//     warp's 16 n-tiles are the even and odd dims of each 16-dim chunk;
//   * at the end the eight warps' (max, sum, O) merge through shared memory
//     into the split's partial; a second kernel merges the splits.
#include "common.cuh"
#include "ops.h"

#include <cuda_fp16.h>

#include <algorithm>

namespace reef {

namespace {

constexpr int kDThreads = 256;   // eight warps
constexpr int kDWarps = kDThreads / 32;
constexpr int kChunk = 256;      // sizing unit of the partial buffer (keys)
constexpr int kTileKeys = 128;   // keys per tile
constexpr int kWarpKeys = kTileKeys / kDWarps;  // 16 keys per warp per tile
constexpr int kStages = 3;
constexpr int kMaxGroup = 16;    // query heads per KV head
constexpr int kORow = 132;       // floats per head row of the merge area
constexpr float kLog2e = 1.4426950408889634f;
static_assert(kWarpKeys == 16, "one m16n8k16 k-step of keys per warp");

struct DecodeArgs {
  int batch, heads_q, heads_kv, group, max_len, chunks;
  int keys_per_split;
  float sm_scale;
  const int8_t* q8;        // [B][Hq][128]
  const float* q_scale;    // [B][Hq]
  const float* k_scale;    // [B][Hkv][max_len]
  const float* v_scale;
  const int* lens;         // [B] keys per sequence, or null
  int len;                 // keys per sequence when lens is null
  float* part;             // [chunks][B][Hq][2 + 128]
  float* out;              // [B][Hq][128]
  int* err;
};

struct DL {  // shared memory layout (bytes from a 1024-aligned base)
  static constexpr int kStageK = 0;                         // int8 [128][128], SW128
  static constexpr int kStageV = kTileKeys * 128;           // int8 [128][128], SW128
  static constexpr int kStageKs = 2 * kTileKeys * 128;      // f32 [128]
  static constexpr int kStageVs = kStageKs + kTileKeys * 4; // f32 [128]
  static constexpr int kStage = 34 * 1024;                  // 33 KB used, 1024-aligned
  static constexpr int kBars = kStages * kStage;            // full[kStages], empty[kStages]
  static constexpr int kEnd = kBars + 2 * kStages * 8;
  static constexpr int kBytes = kEnd + 1024;                // + alignment slack
  // after the last tile: per warp m[16], l[16], O[16][kORow] (reuses the stages)
  static constexpr int kMergeWarp = (32 + kMaxGroup * kORow) * 4;
};
static_assert(DL::kStageVs + kTileKeys * 4 <= DL::kStage, "stage fits");
static_assert(kDWarps * DL::kMergeWarp <= DL::kBars, "merge area fits in the stages");
static_assert(DL::kBytes <= 232448 / 2 - 1024, "two CTAs per SM");

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// D (16x8 s32) += A (16x32 s8, row) x B (32x8 s8, col)
__device__ __forceinline__ void mma_s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                             uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// D (16x8 f32) += A (16x16 f16, row) x B (16x8 f16, col)
__device__ __forceinline__ void mma_f16_16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0,
                                              uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, "
      "{%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A word of an ldmatrix .trans over int8 pairs holds bytes (k0, d), (k0, d+1),
// (k1, d), (k1, d+1) for keys k0 < k1 and dims d, d + 1.  Split it into the
// f16 pairs {(k0, d), (k1, d)} and {(k0, d+1), (k1, d+1)}, exactly: byte b
// becomes the f16 1024 + (b + 128) by placing b ^ 0x80 under the exponent
// byte 0x64, and 1152 is subtracted.
__device__ __forceinline__ void split_i8_pairs(uint32_t w, uint32_t& even, uint32_t& odd) {
  const uint32_t u = w ^ 0x80808080u;
  const uint32_t e = __byte_perm(u, 0x64646464u, 0x4240);
  const uint32_t o = __byte_perm(u, 0x64646464u, 0x4341);
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));
  const __half2 x = __hsub2(*reinterpret_cast<const __half2*>(&e), bias);
  const __half2 y = __hsub2(*reinterpret_cast<const __half2*>(&o), bias);
  even = *reinterpret_cast<const uint32_t*>(&x);
  odd = *reinterpret_cast<const uint32_t*>(&y);
}

// int32 -> fp32, exact for |v| < 2^22 (an int8 dot over 128 dims is at most
// 128 * 127 * 127 < 2^21): v + 1.5 * 2^23 as float bits, minus 1.5 * 2^23
__device__ __forceinline__ float small_i2f(int v) {
  return __fadd_rn(__int_as_float(v + 0x4B400000), -12582912.0f);
}

// byte offset of (row, 16-byte chunk) in a tile written by TMA with the
// 128-byte swizzle (rows of 128 bytes, 1024-aligned tile)
__device__ __forceinline__ uint32_t sw128(int row, int chunk) {
  return static_cast<uint32_t>(row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <int G>
__global__ void __launch_bounds__(kDThreads, 2)
    decode_mma_kernel(const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, DecodeArgs a) {
  extern __shared__ uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + DL::kBars);
  uint64_t* empty = full + kStages;

  const int split = blockIdx.x;
  const int bk = blockIdx.y;  // b * Hkv + hkv
  const int b = bk / a.heads_kv, hkv = bk % a.heads_kv;
  const int len = a.lens != nullptr ? a.lens[b] : a.len;
  const int k_begin = split * a.keys_per_split;
  const int k_end = min(len, k_begin + a.keys_per_split);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int h0 = hkv * G;  // first query head of this KV head
  float* part = a.part + ((static_cast<long long>(split) * a.batch + b) * a.heads_q + h0) * 130;
  if (k_end <= k_begin) {  // split past this sequence's end: an empty partial
    for (int i = tid; i < G * 130; i += kDThreads) part[i] = (i % 130 == 0) ? -INFINITY : 0.0f;
    return;
  }
  const int ntiles = (k_end - k_begin + kTileKeys - 1) / kTileKeys;
  const long long srow0 = static_cast<long long>(bk) * a.max_len + k_begin;  // scale index

  if (tid == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();

  // tile t into stage t % kStages (thread 0).  The TMA boxes are always
  // whole (rows past max_len arrive as zeros); the scales cover the tile's
  // keys inside the sequence, rounded up to whole 16-byte groups (max_len is
  // a multiple of 4, so the groups stay inside the row of scales).
  auto issue = [&](int t) {
    const int s = t % kStages;
    uint8_t* st = sm + s * DL::kStage;
    const int key0 = t * kTileKeys;
    const int n = min(kTileKeys, k_end - k_begin - key0);
    const int n4 = (n + 3) & ~3;
    mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(2 * kTileKeys * 128 + 2 * n4 * 4));
    tma_load_3d(st + DL::kStageK, &kmap, &full[s], 0, k_begin + key0, bk);
    tma_load_3d(st + DL::kStageV, &vmap, &full[s], 0, k_begin + key0, bk);
    bulk_load(st + DL::kStageKs, a.k_scale + srow0 + key0, n4 * 4, &full[s]);
    bulk_load(st + DL::kStageVs, a.v_scale + srow0 + key0, n4 * 4, &full[s]);
  };
  int issued = 0;  // tiles issued (thread 0)
  if (tid == 0)
    for (; issued < kStages && issued < ntiles; ++issued) issue(issued);

  // q as the A operand of the score mma: rows g and g + 8 (heads; rows at or
  // past G are zero), k-step s covering dims [32 s, 32 s + 32)
  uint32_t qa[4][4];
  {
    const uint32_t* q32 = reinterpret_cast<const uint32_t*>(
        a.q8 + (static_cast<long long>(b) * a.heads_q + h0) * 128);
#pragma unroll
    for (int s = 0; s < 4; ++s) {
      qa[s][0] = g < G ? q32[g * 32 + 8 * s + tig] : 0u;
      qa[s][1] = g + 8 < G ? q32[(g + 8) * 32 + 8 * s + tig] : 0u;
      qa[s][2] = g < G ? q32[g * 32 + 8 * s + 4 + tig] : 0u;
      qa[s][3] = g + 8 < G ? q32[(g + 8) * 32 + 8 * s + 4 + tig] : 0u;
    }
  }
  const float base = a.sm_scale * kLog2e;
  const float qs_lo = g < G ? a.q_scale[static_cast<long long>(b) * a.heads_q + h0 + g] * base : 0.0f;
  const float qs_hi =
      g + 8 < G ? a.q_scale[static_cast<long long>(b) * a.heads_q + h0 + g + 8] * base : 0.0f;

  // O for rows g (e 0, 1) and g + 8 (e 2, 3): n-tile 4c + 2p + q covers the
  // dims of 16-dim chunk 2c + p with parity q
  float o[16][4];
#pragma unroll
  for (int i = 0; i < 16; ++i)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[i][e] = 0.0f;
  float m_lo = -INFINITY, m_hi = -INFINITY;  // running max (log2 units) of rows g, g + 8
  float l_lo = 0.0f, l_hi = 0.0f;            // this thread's share of the running sums
  bool ok = true;
  int waited = 0;  // tiles whose stage thread 0 saw complete

  const int wk = warp * kWarpKeys;  // this warp's first key in a tile
  for (int t = 0; t < ntiles; ++t) {
    const int s = t % kStages;
    uint8_t* st = sm + s * DL::kStage;
    if (ok) ok = mbar_wait(&full[s], (t / kStages) & 1, a.err, kDevTimeoutFull);
    if (ok && tid == 0) waited = t + 1;
    const int n = min(kTileKeys, k_end - k_begin - t * kTileKeys);  // keys of the tile
    if (ok && wk < n) {
      // ---- S = q . K^T over this warp's 16 keys: n-tile j = keys wk + 8 j + [0, 8)
      int c[2][4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) c[j][e] = 0;
      }
      const uint32_t kb = smem_u32(st + DL::kStageK);
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int row = wk + 8 * j + (lane & 7);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {  // dims [64 hh, 64 hh + 64): chunks 4 hh + (lane >> 3)
          uint32_t b0, b1, b2, b3;
          ldsm_x4(kb + sw128(row, 4 * hh + (lane >> 3)), b0, b1, b2, b3);
          mma_s8_16832(c[j], qa[2 * hh], b0, b1);
          mma_s8_16832(c[j], qa[2 * hh + 1], b2, b3);
        }
      }
      // ---- scores (log2 units), masked past the tile's keys
      const float2* ks2 = reinterpret_cast<const float2*>(st + DL::kStageKs);
      const float2* vs2 = reinterpret_cast<const float2*>(st + DL::kStageVs);
      float sc[2][4];
      float2 vsc[2];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int k0 = wk + 8 * j + 2 * tig;  // keys k0, k0 + 1
        const float2 ks = ks2[k0 >> 1];
        vsc[j] = vs2[k0 >> 1];
        const bool v0 = k0 < n, v1 = k0 + 1 < n;
        sc[j][0] = v0 ? small_i2f(c[j][0]) * qs_lo * ks.x : -INFINITY;
        sc[j][1] = v1 ? small_i2f(c[j][1]) * qs_lo * ks.y : -INFINITY;
        sc[j][2] = v0 ? small_i2f(c[j][2]) * qs_hi * ks.x : -INFINITY;
        sc[j][3] = v1 ? small_i2f(c[j][3]) * qs_hi * ks.y : -INFINITY;
        if (!v0) vsc[j].x = 0.0f;
        if (!v1) vsc[j].y = 0.0f;
      }
      // ---- online softmax per row over the warp's keys (the four lanes of a
      // row hold its 16 keys)
      float t_lo = fmaxf(fmaxf(sc[0][0], sc[0][1]), fmaxf(sc[1][0], sc[1][1]));
      float t_hi = fmaxf(fmaxf(sc[0][2], sc[0][3]), fmaxf(sc[1][2], sc[1][3]));
      t_lo = fmaxf(t_lo, __shfl_xor_sync(0xffffffffu, t_lo, 1));
      t_lo = fmaxf(t_lo, __shfl_xor_sync(0xffffffffu, t_lo, 2));
      if (G > 8) {
        t_hi = fmaxf(t_hi, __shfl_xor_sync(0xffffffffu, t_hi, 1));
        t_hi = fmaxf(t_hi, __shfl_xor_sync(0xffffffffu, t_hi, 2));
      }
      const float mn_lo = fmaxf(m_lo, t_lo), mn_hi = fmaxf(m_hi, t_hi);
      // reference points: a row with no visible key yet keeps 0 (its p are 0)
      const float r_lo = mn_lo == -INFINITY ? 0.0f : mn_lo;
      const float r_hi = mn_hi == -INFINITY ? 0.0f : mn_hi;
      if (__any_sync(0xffffffffu, mn_lo != m_lo || (G > 8 && mn_hi != m_hi))) {
        const float al_lo = exp2f(m_lo - r_lo);  // 0 while the row was empty
        const float al_hi = G > 8 ? exp2f(m_hi - r_hi) : 1.0f;
        l_lo *= al_lo;
        l_hi *= al_hi;
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          o[i][0] *= al_lo;
          o[i][1] *= al_lo;
          if (G > 8) {
            o[i][2] *= al_hi;
            o[i][3] *= al_hi;
          }
        }
        m_lo = mn_lo;
        m_hi = mn_hi;
      }
      // P = 2^(s - max) (summed unscaled), times the key's V scale, as the
      // f16 A operand of P . V: a0 / a1 keys wk + 2 tig (+1) rows g / g + 8,
      // a2 / a3 the same 8 keys on
      uint32_t pa[4];
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const float p0 = exp2f(sc[j][0] - r_lo), p1 = exp2f(sc[j][1] - r_lo);
        l_lo += p0 + p1;
        const __half2 lo = __floats2half2_rn(p0 * vsc[j].x, p1 * vsc[j].y);
        pa[2 * j] = *reinterpret_cast<const uint32_t*>(&lo);
        if (G > 8) {
          const float p2 = exp2f(sc[j][2] - r_hi), p3 = exp2f(sc[j][3] - r_hi);
          l_hi += p2 + p3;
          const __half2 hi = __floats2half2_rn(p2 * vsc[j].x, p3 * vsc[j].y);
          pa[2 * j + 1] = *reinterpret_cast<const uint32_t*>(&hi);
        } else {
          pa[2 * j + 1] = 0u;
        }
      }
      // ---- O += P . V over the warp's 16 keys: ldmatrix .trans of int8
      // pairs; matrices (keys wk + [0, 8), chunk 2c), (keys wk + [8, 16),
      // chunk 2c), then chunk 2c + 1
      const uint32_t vb = smem_u32(st + DL::kStageV);
      const int vrow = wk + ((lane >> 3) & 1) * 8 + (lane & 7);
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t r0, r1, r2, r3;
        ldsm_x4_t(vb + sw128(vrow, 2 * cc + (lane >> 4)), r0, r1, r2, r3);
        uint32_t e0, d0, e1, d1, e2, d2, e3, d3;
        split_i8_pairs(r0, e0, d0);
        split_i8_pairs(r1, e1, d1);
        split_i8_pairs(r2, e2, d2);
        split_i8_pairs(r3, e3, d3);
        mma_f16_16816(o[4 * cc + 0], pa, e0, e1);
        mma_f16_16816(o[4 * cc + 1], pa, d0, d1);
        mma_f16_16816(o[4 * cc + 2], pa, e2, e3);
        mma_f16_16816(o[4 * cc + 3], pa, d2, d3);
      }
    }
    // ---- release the stage; thread 0 refills it once every warp has
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (tid == 0 && ok && t + kStages < ntiles) {
      ok = mbar_wait(&empty[s], (t / kStages) & 1, a.err, kDevTimeoutEmpty);
      if (ok) issue(issued++);
    }
  }
  // copies still in flight land before the stages are reused (only after a
  // timeout can any remain)
  if (tid == 0 && !ok) {
    for (int t = waited; t < issued; ++t)
      mbar_wait(&full[t % kStages], (t / kStages) & 1, a.err, kDevTimeoutDrain);
  }
  __syncthreads();  // every warp is done with the stages

  // ---- merge the eight warps' states: per warp m[16], l[16], O[16][kORow]
  float* mw = reinterpret_cast<float*>(sm + warp * DL::kMergeWarp);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  if (tig == 0) {
    if (g < G) {
      mw[g] = m_lo;
      mw[16 + g] = l_lo;
    }
    if (g + 8 < G) {
      mw[8 + g] = m_hi;
      mw[24 + g] = l_hi;
    }
  }
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) {
#pragma unroll
    for (int p = 0; p < 2; ++p) {  // chunk 2 cc + p: dims 32 cc + 16 p + 4 tig + [0, 4)
      const int d = 32 * cc + 16 * p + 4 * tig;
      const float* ev = o[4 * cc + 2 * p];
      const float* od = o[4 * cc + 2 * p + 1];
      if (g < G)
        *reinterpret_cast<float4*>(mw + 32 + g * kORow + d) = make_float4(ev[0], od[0], ev[1], od[1]);
      if (g + 8 < G)
        *reinterpret_cast<float4*>(mw + 32 + (g + 8) * kORow + d) =
            make_float4(ev[2], od[2], ev[3], od[3]);
    }
  }
  __syncthreads();
  for (int i = tid; i < G * 128; i += kDThreads) {
    const int h = i >> 7, d = i & 127;
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDWarps; ++w)
      m = fmaxf(m, reinterpret_cast<const float*>(sm + w * DL::kMergeWarp)[h]);
    float l = 0.0f, acc = 0.0f;
#pragma unroll
    for (int w = 0; w < kDWarps; ++w) {
      const float* ww = reinterpret_cast<const float*>(sm + w * DL::kMergeWarp);
      const float mw_h = ww[h];
      if (mw_h == -INFINITY) continue;  // the warp saw no key of this split
      const float sc = exp2f(mw_h - m);
      l += sc * ww[16 + h];
      acc += sc * ww[32 + h * kORow + d];
    }
    part[h * 130 + 2 + d] = acc;
    if (d == 0) {
      part[h * 130] = m;
      part[h * 130 + 1] = l;
    }
  }
}

// Merge the splits of one (sequence, query head): weights 2^(m_c - max) per
// split, computed once per block of 128 splits in shared memory.
__global__ void __launch_bounds__(128) decode_combine_kernel(DecodeArgs a) {
  __shared__ float wsm[128];
  __shared__ float red[4];
  const int bh = blockIdx.x;  // b * Hq + h
  const int d = threadIdx.x;  // 128
  const long long stride = static_cast<long long>(a.batch) * a.heads_q * 130;
  const float* pb = a.part + static_cast<long long>(bh) * 130;
  float m = -INFINITY;
  for (int c = d; c < a.chunks; c += 128) m = fmaxf(m, pb[c * stride]);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
  if ((d & 31) == 0) red[d >> 5] = m;
  __syncthreads();
  m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
  float lp = 0.0f, o = 0.0f;
  for (int c0 = 0; c0 < a.chunks; c0 += 128) {
    __syncthreads();
    const int c = c0 + d;
    float w = 0.0f;
    if (c < a.chunks) {
      const float mc = pb[c * stride];
      if (mc != -INFINITY) {
        w = exp2f(mc - m);
        lp += w * pb[c * stride + 1];
      }
    }
    wsm[d] = w;
    __syncthreads();
    const int nc = min(128, a.chunks - c0);
    const float* pc = pb + c0 * stride + 2 + d;
#pragma unroll 4
    for (int i = 0; i < nc; ++i) o += wsm[i] * pc[i * stride];
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) lp += __shfl_xor_sync(0xffffffffu, lp, off);
  __syncthreads();
  if ((d & 31) == 0) red[d >> 5] = lp;
  __syncthreads();
  const float l = (red[0] + red[1]) + (red[2] + red[3]);
  a.out[static_cast<long long>(bh) * 128 + d] = o / l;
}

// CTAs of decode_mma_kernel<G> resident per SM (0 on an error); the shared
// memory opt-in is made on the first call per device
template <int G>
int tile_ctas_per_sm() {
  static int per_sm[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return 0;
  if (per_sm[dev] == 0) {
    int n = 0;
    if (cudaFuncSetAttribute(decode_mma_kernel<G>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             DL::kBytes) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_mma_kernel<G>, kDThreads,
                                                      DL::kBytes) != cudaSuccess)
      return 0;
    per_sm[dev] = n;
  }
  return per_sm[dev];
}

template <int G>
int launch_tiles(const CUtensorMap& km, const CUtensorMap& vm, const DecodeArgs& a, int splits,
                 cudaStream_t st) {
  dim3 grid(static_cast<unsigned>(splits), static_cast<unsigned>(a.batch * a.heads_kv));
  decode_mma_kernel<G><<<grid, kDThreads, DL::kBytes, st>>>(km, vm, a);
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
  // the bulk copies read cache rows and scale groups of 16 bytes
  if (p.max_len % 4 != 0 ||
      ((reinterpret_cast<uintptr_t>(p.k_cache) | reinterpret_cast<uintptr_t>(p.v_cache) |
        reinterpret_cast<uintptr_t>(p.k_scale) | reinterpret_cast<uintptr_t>(p.v_scale)) & 15u) != 0)
    return kErrAlignment;
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
  a.k_scale = p.k_scale;
  a.v_scale = p.v_scale;
  a.lens = p.lens;
  a.len = p.len;
  a.part = p.partial;
  a.out = p.out;
  a.err = device_error_ptr();
  // Splits along the keys: at most one wave of CTAs (every CTA resident at
  // once, so none waits for a second wave), each split a whole number of
  // tiles; never more splits than the partial buffer holds (one per 256
  // keys).
  int per_sm = 0;
  switch (G) {
    case 1: per_sm = tile_ctas_per_sm<1>(); break;
    case 2: per_sm = tile_ctas_per_sm<2>(); break;
    case 4: per_sm = tile_ctas_per_sm<4>(); break;
    case 8: per_sm = tile_ctas_per_sm<8>(); break;
    case 16: per_sm = tile_ctas_per_sm<16>(); break;
    default: return kErrInvalid;
  }
  if (per_sm <= 0) return kErrCuda;
  const int pairs = p.batch * p.heads_kv;
  // K and V as [pairs][max_len][128] int8, 128-key boxes with the 128-byte
  // swizzle (rows past max_len read as zeros)
  CUtensorMap km, vm;
  const long long seg = static_cast<long long>(p.max_len) * 128;
  if (int rc = make_tma_3d_i8(&km, p.k_cache, p.max_len, 128, 128, pairs, seg, 128, kTileKeys))
    return rc;
  if (int rc = make_tma_3d_i8(&vm, p.v_cache, p.max_len, 128, 128, pairs, seg, 128, kTileKeys))
    return rc;
  const int tiles = (p.max_len + kTileKeys - 1) / kTileKeys;
  int splits = std::max(1, per_sm * num_sms() / pairs);
  splits = std::min({splits, tiles, a.chunks});
  const int tiles_per = (tiles + splits - 1) / splits;
  a.keys_per_split = tiles_per * kTileKeys;
  splits = (tiles + tiles_per - 1) / tiles_per;
  a.chunks = splits;
  int rc;
  switch (G) {
    case 1: rc = launch_tiles<1>(km, vm, a, splits, st); break;
    case 2: rc = launch_tiles<2>(km, vm, a, splits, st); break;
    case 4: rc = launch_tiles<4>(km, vm, a, splits, st); break;
    case 8: rc = launch_tiles<8>(km, vm, a, splits, st); break;
    case 16: rc = launch_tiles<16>(km, vm, a, splits, st); break;
    default: return kErrInvalid;
  }
  if (rc) return rc;
  decode_combine_kernel<<<static_cast<unsigned>(p.batch * p.heads_q), 128, 0, st>>>(a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace reef
