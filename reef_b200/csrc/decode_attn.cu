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
//   * work is cut into units of (sequence x KV head, 128-key tile) and
//     spread evenly over one wave of CTAs; a CTA may end one sequence and
//     start the next, writing one partial (max, sum, O) per sequence it
//     touched;
//   * a CTA streams its units through a 3-stage ring: K and V by TMA
//     (128-byte swizzle, so the fragment loads below hit every bank once),
//     their scales by bulk copies, completing on one mbarrier per stage;
//     thread 0 refills a stage once the eight warps have released it (a
//     second mbarrier per stage), so there is no CTA-wide barrier per tile;
//   * warp w owns keys [16w, 16w + 16) of every tile with its own
//     online-softmax state.  Both products run transposed so the heads are
//     the n = 8 side of the mma and no row is padding: S^T = K . q^T by int8
//     mma.sync m16n8k32 (q resident in registers), O^T = V^T . P^T by f16
//     m16n8k16, P^T reaching the B operand through movmatrix;
//   * V^T comes from the int8 tile by ldmatrix .trans on byte pairs: a
//     thread receives dims (d, d + 1) of keys (k, k + 1) and permutes them
//     into the f16 pairs {(d, k), (d, k + 1)} and {(d + 1, k), (d + 1, k + 1)}
//     under the exponent byte 0x64, i.e. the exact values v + 1152; the
//     offset is removed at the end with the column sums of P, which one more
//     mma (A = ones) accumulates alongside;
//   * the running max is raised only when a tile exceeds it by more than
//     2^kLazy, so the accumulators are rarely rescaled (P stays below
//     2^kLazy times the key's V scale).
//   A second kernel merges the partials of each sequence.
#include "common.cuh"
#include "ops.h"

#include <cuda_fp16.h>

#include <algorithm>

namespace reef {

namespace {

constexpr int kDThreads = 256;   // eight warps
constexpr int kDWarps = kDThreads / 32;
constexpr int kTileKeys = 128;   // keys per unit of work
constexpr int kWarpKeys = kTileKeys / kDWarps;  // 16 keys per warp per tile
constexpr int kStages = 3;
constexpr int kMaxGroup = 16;    // query heads per KV head
constexpr int kPartRow = 132;    // floats per head of a partial: m, l, 2 unused, O[128]
constexpr int kMaxCtasPerSm = 4; // bound used to size the partial buffer
constexpr int kMaxRowsPerPair = 64;  // CTAs sharing one (sequence, KV head) at most
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLazy = 4.0f;    // log2 of the largest P / v_scale
constexpr float kVBias = 1152.0f;
static_assert(kWarpKeys == 16, "one m16n8k16 k-step of keys per warp");

struct DecodeArgs {
  int batch, heads_q, heads_kv, max_len;
  int tiles;         // units per (sequence, KV head): ceil(max_len / 128)
  int ctas;          // CTAs launched
  long long units;   // batch * heads_kv * tiles
  float sm_scale;
  const int8_t* q8;        // [B][Hq][128]
  const float* q_scale;    // [B][Hq]
  const float* k_scale;    // [B][Hkv][max_len]
  const float* v_scale;
  const int* lens;         // [B] keys per sequence, or null
  const int* positions;    // [B] rows appended this step (lens - 1), or null
  int len;                 // keys per sequence when lens is null
  float* part;             // [ctas + B*Hkv][G][kPartRow]: row c + pair
  float* out;              // [B][Hq][128]
  int* err;
};

struct DL {  // shared memory layout (bytes from a 1024-aligned base)
  static constexpr int kKV = 2 * kTileKeys * 128;            // K then V, int8 [128][128] SW128
  static constexpr int kScales = kStages * kKV;              // per stage ks[128], vs[128]
  static constexpr int kWarpM = kScales + kStages * 1024;    // m[8][16], then l[8][16]
  static constexpr int kBars = kWarpM + 2 * kDWarps * kMaxGroup * 4;  // full[], empty[]
  static constexpr int kEnd = kBars + 2 * kStages * 8;
  // The merge of the eight warps' O ([8][G][128] fp32) reuses the K / V
  // buffers of the stage just consumed when it fits there (G <= 8); G = 16
  // has its own area after kEnd.
  __host__ __device__ static constexpr int merge_bytes(int g) { return kDWarps * g * 128 * 4; }
  __host__ __device__ static constexpr int bytes(int g) {
    return (merge_bytes(g) <= kKV ? kEnd : kEnd + merge_bytes(g)) + 1024;  // + alignment slack
  }
};
static_assert(DL::merge_bytes(8) <= DL::kKV, "G <= 8 merges inside a stage");
static_assert(DL::bytes(8) <= 232448 / 2 - 1024, "two CTAs per SM up to G = 8");
static_assert(DL::bytes(16) <= 232448 - 1024, "one CTA per SM at G = 16");

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t (&r)[4]) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
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

// A word of an ldmatrix .trans over int8 pairs: bytes (k, d), (k, d+1),
// (k+1, d), (k+1, d+1).  Out: the f16 pairs {(k, d), (k+1, d)} and
// {(k, d+1), (k+1, d+1)}, each value v + 1152 exactly (byte v ^ 0x80 = v +
// 128 as the mantissa under the exponent byte 0x64, i.e. 1024 + v + 128).
__device__ __forceinline__ void split_biased(uint32_t w, uint32_t& even, uint32_t& odd) {
  const uint32_t u = w ^ 0x80808080u;
  even = __byte_perm(u, 0x64646464u, 0x4240);
  odd = __byte_perm(u, 0x64646464u, 0x4341);
}

// 2^x (ex2.approx.ftz: 2 ulp; -inf -> 0, results below 2^-126 flush to 0)
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
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

__device__ __forceinline__ int seq_len(const DecodeArgs& a, int b) {
  return a.lens != nullptr ? a.lens[b] : a.len;
}

// the CTA whose units include unit x
__device__ __forceinline__ int cta_of(const DecodeArgs& a, long long x) {
  return static_cast<int>(((x + 1) * a.ctas - 1) / a.units);
}

// G query heads per KV head; NT = n-tiles of 8 heads
template <int G>
__global__ void __launch_bounds__(kDThreads, G > 8 ? 1 : 2)  // 16 heads: twice the accumulators
    decode_mma_kernel(const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, DecodeArgs a) {
  constexpr int NT = (G + 7) / 8;
  extern __shared__ uint8_t sm_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(sm_raw) + 1023) &
                                           ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + DL::kBars);
  uint64_t* empty = full + kStages;
  float* warp_m = reinterpret_cast<float*>(sm + DL::kWarpM);    // [8][16]
  float* warp_l = warp_m + kDWarps * kMaxGroup;                 // [8][16]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, tig = lane & 3;
  const int cta = blockIdx.x;
  const long long u0 = static_cast<long long>(cta) * a.units / a.ctas;
  const long long u1 = static_cast<long long>(cta + 1) * a.units / a.ctas;
  const int nunits = static_cast<int>(u1 - u0);

  if (tid == 0) {
    prefetch_tensormap(&kmap);
    prefetch_tensormap(&vmap);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], kDWarps);
    }
    fence_barrier_init();
  }
  // Before waiting for the kernel ahead (which appends this step's rows and
  // writes q and lens), thread 0 requests the K / V tiles of its first units
  // that lie wholly below the row each sequence appends: nothing running
  // writes them.  Their scales, and every other tile, follow the wait.
  uint32_t pre = 0;  // bit j: unit j's K / V were requested early
  if (tid == 0 && a.positions != nullptr) {
    for (int j = 0; j < kStages && j < nunits; ++j) {
      const long long u = u0 + j;
      const int pair = static_cast<int>(u / a.tiles);
      const int key0 = static_cast<int>(u % a.tiles) * kTileKeys;
      if (key0 + kTileKeys > a.positions[pair / a.heads_kv]) continue;
      uint8_t* kv = sm + j * DL::kKV;
      mbar_expect_tx(&full[j], static_cast<uint32_t>(2 * kTileKeys * 128));
      tma_load_3d(kv, &kmap, &full[j], 0, key0, pair);
      tma_load_3d(kv + kTileKeys * 128, &vmap, &full[j], 0, key0, pair);
      pre |= 1u << j;
    }
  }
  pdl_wait();
  // the combine kernel may be scheduled now; it waits for this grid's
  // completion (and its memory) before reading the partials
  pdl_trigger();
  __syncthreads();

  // unit j of this CTA into stage j % kStages (thread 0).  The TMA boxes are
  // whole (rows past max_len arrive as zeros); the scales cover the tile's
  // keys inside the sequence, rounded up to whole 16-byte groups (max_len is
  // a multiple of 4, so they stay inside the sequence's row of scales).  A
  // tile wholly past the sequence's end loads nothing.
  const int pair0 = static_cast<int>(u0 / a.tiles), tile0 = static_cast<int>(u0 % a.tiles);
  int ipair = pair0, itile = tile0;  // next unit to issue (thread 0)
  auto issue = [&](int j) {
    const int s = j % kStages;
    const int pair = ipair;
    const int key0 = itile * kTileKeys;
    if (++itile == a.tiles) {
      itile = 0;
      ++ipair;
    }
    const int n = min(kTileKeys, seq_len(a, pair / a.heads_kv) - key0);
    if (n <= 0) {
      mbar_arrive(&full[s]);
      return;
    }
    const int n4 = (n + 3) & ~3;
    const long long srow = static_cast<long long>(pair) * a.max_len + key0;
    uint8_t* kv = sm + s * DL::kKV;
    float* sc = reinterpret_cast<float*>(sm + DL::kScales + s * 1024);
    if (j < kStages && ((pre >> j) & 1u)) {  // K / V already requested
      mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(2 * n4 * 4));
    } else {
      mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(2 * kTileKeys * 128 + 2 * n4 * 4));
      tma_load_3d(kv, &kmap, &full[s], 0, key0, pair);
      tma_load_3d(kv + kTileKeys * 128, &vmap, &full[s], 0, key0, pair);
    }
    bulk_load(sc, a.k_scale + srow, n4 * 4, &full[s]);
    bulk_load(sc + kTileKeys, a.v_scale + srow, n4 * 4, &full[s]);
  };
  int issued = 0;  // units issued (thread 0)
  if (tid == 0)
    for (; issued < kStages && issued < nunits; ++issued) issue(issued);

  const float base = a.sm_scale * kLog2e;
  const int wk = warp * kWarpKeys;  // this warp's first key in a tile
  // fragment rows of this lane in the ldmatrix loads (keys wk + [0, 16))
  const int frow = wk + ((lane >> 3) & 1) * 8 + (lane & 7);
  const uint32_t ones = 0x3C003C00u;  // f16 pair (1, 1)
  const uint32_t ones_a[4] = {ones, ones, ones, ones};

  // per-sequence state: q as the B operand of S^T (dims x heads, k-step s =
  // dims [32 s, 32 s + 32)); the score scale of heads nt*8 + 2 tig + {0, 1};
  // O^T accumulators o[c][nt] for 16-dim chunk c (rows g: dim 16c + 2g,
  // rows g + 8: dim 16c + 2g + 1; columns: heads nt*8 + 2 tig + {0, 1}); the
  // column sums of P (os); the running max and this thread's share of the
  // sums per head column
  uint32_t qb[4][NT][2];
  float qsc[NT][2];
  float o[8][NT][4];
  float os[NT][4];
  float m[NT][2], l[NT][2];
  int pair = pair0, tile = tile0, len = 0;  // the unit being consumed
  bool ok = true;
  int waited = 0;  // units whose stage thread 0 saw complete

  for (int j = 0; j < nunits; ++j) {
    const int s = j % kStages;
    if (j == 0 || tile == 0) {  // a new (sequence, KV head): load q, reset the state
      const int b = pair / a.heads_kv, hkv = pair % a.heads_kv;
      len = seq_len(a, b);
      const long long qrow = static_cast<long long>(b) * a.heads_q + hkv * G;
      const uint32_t* q32 = reinterpret_cast<const uint32_t*>(a.q8 + qrow * 128);
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const int h = nt * 8 + g;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          qb[ks][nt][0] = h < G ? q32[h * 32 + 8 * ks + tig] : 0u;
          qb[ks][nt][1] = h < G ? q32[h * 32 + 8 * ks + 4 + tig] : 0u;
        }
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int hc = nt * 8 + 2 * tig + e;
          qsc[nt][e] = hc < G ? a.q_scale[qrow + hc] * base : 0.0f;
          m[nt][e] = -INFINITY;
          l[nt][e] = 0.0f;
        }
#pragma unroll
        for (int e = 0; e < 4; ++e) os[nt][e] = 0.0f;
#pragma unroll
        for (int c = 0; c < 8; ++c)
#pragma unroll
          for (int e = 0; e < 4; ++e) o[c][nt][e] = 0.0f;
      }
    }
    if (ok) ok = mbar_wait(&full[s], (j / kStages) & 1, a.err, kDevTimeoutFull);
    if (ok && tid == 0) waited = j + 1;
    const int n = min(kTileKeys, len - tile * kTileKeys);  // keys of the tile
    if (ok && wk < n) {
      const uint8_t* kv = sm + s * DL::kKV;
      const float* ksc = reinterpret_cast<const float*>(sm + DL::kScales + s * 1024);
      // ---- S^T = K . q^T: rows keys wk + g (c 0, 1), wk + g + 8 (c 2, 3)
      int c[NT][4], c2[NT][4];  // k-steps 0, 2 and 1, 3: two independent mma chains
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) c[nt][e] = c2[nt][e] = 0;
      const uint32_t kb = smem_u32(kv);
#pragma unroll
      for (int ks = 0; ks < 4; ++ks) {
        uint32_t ka[4];
        ldsm_x4(kb + sw128(frow, 2 * ks + (lane >> 4)), ka);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
          mma_s8_16832((ks & 1) ? c2[nt] : c[nt], ka, qb[ks][nt][0], qb[ks][nt][1]);
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) c[nt][e] += c2[nt][e];
      // ---- scores in log2 units; keys past the tile's end masked
      const bool val_lo = wk + g < n, val_hi = wk + g + 8 < n;
      const float ks_lo = ksc[wk + g], ks_hi = ksc[wk + g + 8];
      const float vs_lo = val_lo ? ksc[kTileKeys + wk + g] : 0.0f;
      const float vs_hi = val_hi ? ksc[kTileKeys + wk + g + 8] : 0.0f;
      float sc[NT][4];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        sc[nt][0] = val_lo ? small_i2f(c[nt][0]) * qsc[nt][0] * ks_lo : -INFINITY;
        sc[nt][1] = val_lo ? small_i2f(c[nt][1]) * qsc[nt][1] * ks_lo : -INFINITY;
        sc[nt][2] = val_hi ? small_i2f(c[nt][2]) * qsc[nt][0] * ks_hi : -INFINITY;
        sc[nt][3] = val_hi ? small_i2f(c[nt][3]) * qsc[nt][1] * ks_hi : -INFINITY;
      }
      // ---- the running max per head column stays while no score passes it
      // by more than 2^kLazy (one vote); otherwise the tile's max over the
      // warp's 16 keys (the eight lanes of one tig) replaces it where it
      // passed, and the accumulators are rescaled
      bool need = false;
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) need |= fmaxf(sc[nt][e], sc[nt][e + 2]) > m[nt][e] + kLazy;
      if (__any_sync(0xffffffffu, need)) {
#pragma unroll
        for (int nt = 0; nt < NT; ++nt)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            float x = fmaxf(sc[nt][e], sc[nt][e + 2]);
            x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 4));
            x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 8));
            x = fmaxf(x, __shfl_xor_sync(0xffffffffu, x, 16));
            const bool up = x > m[nt][e] + kLazy;
            const float al = up ? fast_exp2(m[nt][e] - x) : 1.0f;  // 0 from -inf
            if (up) m[nt][e] = x;
            l[nt][e] *= al;
            os[nt][e] *= al;
            os[nt][e + 2] *= al;
#pragma unroll
            for (int cc = 0; cc < 8; ++cc) {
              o[cc][nt][e] *= al;
              o[cc][nt][e + 2] *= al;
            }
          }
      }
      // ---- P = 2^(s - m) (summed unscaled), times the key's V scale, as
      // f16 pairs (key; heads 2 tig, 2 tig + 1), transposed into the B
      // operand (keys 2 tig, 2 tig + 1; head g)
      uint32_t pb[NT][2];
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) {
        const float r0 = m[nt][0] == -INFINITY ? 0.0f : m[nt][0];
        const float r1 = m[nt][1] == -INFINITY ? 0.0f : m[nt][1];
        const float p0 = fast_exp2(sc[nt][0] - r0), p1 = fast_exp2(sc[nt][1] - r1);
        const float p2 = fast_exp2(sc[nt][2] - r0), p3 = fast_exp2(sc[nt][3] - r1);
        l[nt][0] += p0 + p2;
        l[nt][1] += p1 + p3;
        const __half2 x0 = __floats2half2_rn(p0 * vs_lo, p1 * vs_lo);
        const __half2 x1 = __floats2half2_rn(p2 * vs_hi, p3 * vs_hi);
        pb[nt][0] = movmatrix_t(*reinterpret_cast<const uint32_t*>(&x0));
        pb[nt][1] = movmatrix_t(*reinterpret_cast<const uint32_t*>(&x1));
      }
      // ---- O^T += (V + 1152)^T . P^T; ldmatrix .trans matrices (keys
      // wk + [0, 8), chunk 2cc), (keys wk + [8, 16), chunk 2cc), then 2cc + 1
      const uint32_t vb = smem_u32(kv + kTileKeys * 128);
#pragma unroll
      for (int cc = 0; cc < 4; ++cc) {
        uint32_t r[4];
        ldsm_x4_t(vb + sw128(frow, 2 * cc + (lane >> 4)), r);
        uint32_t va[4], vc[4];
        split_biased(r[0], va[0], va[1]);
        split_biased(r[1], va[2], va[3]);
        split_biased(r[2], vc[0], vc[1]);
        split_biased(r[3], vc[2], vc[3]);
#pragma unroll
        for (int nt = 0; nt < NT; ++nt) {
          mma_f16_16816(o[2 * cc][nt], va, pb[nt][0], pb[nt][1]);
          mma_f16_16816(o[2 * cc + 1][nt], vc, pb[nt][0], pb[nt][1]);
        }
      }
#pragma unroll
      for (int nt = 0; nt < NT; ++nt) mma_f16_16816(os[nt], ones_a, pb[nt][0], pb[nt][1]);
    }
    // ---- release the stage; thread 0 refills it once every warp has (after
    // the merge below when this unit ends a sequence: the merge uses it)
    const bool last = j + 1 == nunits || tile + 1 == a.tiles;
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (tid == 0 && ok && !last && j + kStages < nunits) {
      ok = mbar_wait(&empty[s], (j / kStages) & 1, a.err, kDevTimeoutEmpty);
      if (ok) issue(issued++);
    }

    // ---- end of this (sequence, KV head) in this CTA: merge the eight
    // warps into the partial row cta + pair.  Each warp weighs its state by
    // 2^(m_w - max) and writes it to its own slot; the slots are then summed
    // in warp order (a fixed order for every dim).
    if (last) {
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float x = l[nt][e];
          x += __shfl_xor_sync(0xffffffffu, x, 4);
          x += __shfl_xor_sync(0xffffffffu, x, 8);
          x += __shfl_xor_sync(0xffffffffu, x, 16);
          l[nt][e] = x;
          const int h = nt * 8 + 2 * tig + e;
          if (g == 0 && h < G) warp_m[warp * kMaxGroup + h] = m[nt][e];
        }
      __syncthreads();  // every warp's m is in, and every warp is done with stage s
      float* mrg = reinterpret_cast<float*>(DL::merge_bytes(G) <= DL::kKV ? sm + s * DL::kKV
                                                                        : sm + DL::kEnd);
      float* mine = mrg + warp * G * 128;  // [G][128]
#pragma unroll
      for (int nt = 0; nt < NT; ++nt)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int h = nt * 8 + 2 * tig + e;
          if (h >= G) continue;
          float mx = -INFINITY;
#pragma unroll
          for (int w = 0; w < kDWarps; ++w) mx = fmaxf(mx, warp_m[w * kMaxGroup + h]);
          const float ws = m[nt][e] == -INFINITY ? 0.0f : exp2f(m[nt][e] - mx);
          if (g == 0) warp_l[warp * kMaxGroup + h] = l[nt][e] * ws;
          const float bias = kVBias * os[nt][e];
#pragma unroll
          for (int cc = 0; cc < 8; ++cc)
            *reinterpret_cast<float2*>(mine + h * 128 + 16 * cc + 2 * g) =
                make_float2((o[cc][nt][e] - bias) * ws, (o[cc][nt][e + 2] - bias) * ws);
        }
      __syncthreads();
      float* prow = a.part + (static_cast<long long>(cta) + pair) * G * kPartRow;
      for (int i = tid; i < G * 128; i += kDThreads) {
        const int h = i >> 7, d = i & 127;
        float acc = 0.0f;
#pragma unroll
        for (int w = 0; w < kDWarps; ++w) acc += mrg[w * G * 128 + i];
        prow[h * kPartRow + 4 + d] = acc;
      }
      if (tid < G) {
        float mx = -INFINITY, ls = 0.0f;
#pragma unroll
        for (int w = 0; w < kDWarps; ++w) {
          mx = fmaxf(mx, warp_m[w * kMaxGroup + tid]);
          ls += warp_l[w * kMaxGroup + tid];
        }
        prow[tid * kPartRow] = mx;
        prow[tid * kPartRow + 1] = ls;
      }
      __syncthreads();  // the merge area and warp_m / warp_l are free again
      if (tid == 0 && ok && j + kStages < nunits) {  // the refill held back above
        fence_proxy_async_smem();  // the merge's stores before the copy's writes
        ok = mbar_wait(&empty[s], (j / kStages) & 1, a.err, kDevTimeoutEmpty);
        if (ok) issue(issued++);
      }
    }
    if (++tile == a.tiles) {
      tile = 0;
      ++pair;
    }
  }
  // copies still in flight land before exit (only after a timeout can any
  // remain)
  if (tid == 0 && !ok) {
    for (int j = waited; j < issued; ++j)
      mbar_wait(&full[j % kStages], (j / kStages) & 1, a.err, kDevTimeoutDrain);
  }
}


// Merge the partials of one (sequence, query head): rows cta + pair for the
// CTAs that worked on the pair.  Warp w takes rows w, w + 8, ... (a lane
// holds 4 dims); the eight warp sums are added in a fixed order.
template <int G>
__global__ void __launch_bounds__(256) decode_combine_kernel(DecodeArgs a) {
  __shared__ float4 osm[kDWarps][32];
  __shared__ float lsm[kDWarps], red[kDWarps];
  const int bh = blockIdx.x;  // b * Hq + h
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = bh / a.heads_q, h = bh % a.heads_q;
  const int pair = b * a.heads_kv + h / G, hg = h % G;
  const int c0 = cta_of(a, static_cast<long long>(pair) * a.tiles);
  const int nc = cta_of(a, static_cast<long long>(pair + 1) * a.tiles - 1) - c0 + 1;
  const long long stride = static_cast<long long>(G) * kPartRow;  // one row
  const float* pb = a.part + (static_cast<long long>(c0) + pair) * stride + hg * kPartRow;
  // launched early (programmatic dependent launch): wait for the main
  // kernel's completion and memory before reading its partials
  pdl_wait();
  pdl_trigger();
  // one pass over the rows: warp w holds rows w, w + 8, ... (m, l and a
  // float4 of O per lane) in registers while the block finds the max
  constexpr int kRows = (kMaxRowsPerPair + kDWarps - 1) / kDWarps;
  float mr[kRows], lr[kRows];
  float4 vr[kRows];
  float m = -INFINITY;
#pragma unroll
  for (int i = 0; i < kRows; ++i) {
    const int c = warp + i * kDWarps;
    mr[i] = -INFINITY;
    if (c < nc) {
      const float* pr = pb + c * stride;
      mr[i] = pr[0];
      lr[i] = pr[1];
      vr[i] = reinterpret_cast<const float4*>(pr + 4)[lane];
      m = fmaxf(m, mr[i]);
    }
  }
  if (lane == 0) red[warp] = m;
  __syncthreads();
#pragma unroll
  for (int w = 0; w < kDWarps; ++w) m = fmaxf(m, red[w]);
  float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  float l = 0.0f;
#pragma unroll
  for (int i = 0; i < kRows; ++i) {
    // a CTA whose tiles all lay past the sequence's end has m = -inf
    if (mr[i] == -INFINITY) continue;
    const float w = exp2f(mr[i] - m);
    l += w * lr[i];
    o.x += w * vr[i].x;
    o.y += w * vr[i].y;
    o.z += w * vr[i].z;
    o.w += w * vr[i].w;
  }
  osm[warp][lane] = o;
  if (lane == 0) lsm[warp] = l;
  __syncthreads();
  if (tid < 128) {
    float acc = 0.0f, ls = 0.0f;
#pragma unroll
    for (int w = 0; w < kDWarps; ++w) {
      acc += reinterpret_cast<const float*>(&osm[w][0])[tid];
      ls += lsm[w];
    }
    a.out[static_cast<long long>(bh) * 128 + tid] = acc / ls;
  }
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
                             DL::bytes(G)) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, decode_mma_kernel<G>, kDThreads,
                                                      DL::bytes(G)) != cudaSuccess)
      return 0;
    per_sm[dev] = std::min(n, kMaxCtasPerSm);
  }
  return per_sm[dev];
}

template <int G>
int launch_decode(const CUtensorMap& km, const CUtensorMap& vm, DecodeArgs& a, cudaStream_t st) {
  const int per_sm = tile_ctas_per_sm<G>();
  if (per_sm <= 0) return kErrCuda;
  // one wave, and at most kMaxRowsPerPair CTAs on any (sequence, KV head)
  const long long pairs = static_cast<long long>(a.batch) * a.heads_kv;
  a.ctas = static_cast<int>(std::min({static_cast<long long>(per_sm) * num_sms(), a.units,
                                      pairs * (kMaxRowsPerPair - 1)}));
  if (int rc = launch_k(decode_mma_kernel<G>, dim3(static_cast<unsigned>(a.ctas)), dim3(kDThreads),
                        DL::bytes(G), st, km, vm, a))
    return rc;
  // the combine launches as a programmatic dependent of the main kernel, so
  // its launch overlaps the main kernel's tail
  PdlScope pdl;
  return launch_k(decode_combine_kernel<G>, dim3(static_cast<unsigned>(a.batch * a.heads_q)),
                  dim3(kDThreads), 0, st, a);
}

// One decode step's q / k / v: one warp per (sequence, head) of the QKV
// projection output qkv [B][(Hq + 2 Hkv) * 128].  q and k get rotate-half
// RoPE at the sequence's position; every head row is quantised with reef's
// rule (quant.hpp:51-81); q goes to q8 / q_scale, k and v are appended to the
// cache at row `pos`, and lens[b] = pos + 1.  A position outside the cache is
// recorded in the device error word and the row is skipped.
// The projection comes either as fp32 rows qkv [B][(Hq + 2 Hkv) * 128], or
// (kPartials) as the skinny GEMM's int32 split-K partials part[s][B][...]
// (`splits` of them, B * (Hq + 2 Hkv) * 128 apart) that this kernel sums and
// dequantises itself with the W8A8 epilogue (linear.hpp:125-127: float(sum) *
// (x_scale[b] * w_scale[n])), the values a separate reduce would have stored.
template <bool kPartials>
__global__ void decode_rope_append_kernel(int batch, int hq, int hkv, int max_len, float base,
                                          const int* __restrict__ positions,
                                          const float* __restrict__ qkv,
                                          const int32_t* __restrict__ part, int splits,
                                          const float* __restrict__ xs,
                                          const float* __restrict__ ws, int8_t* __restrict__ q8,
                                          float* __restrict__ q_scale, int8_t* __restrict__ k_cache,
                                          float* __restrict__ k_scale, int8_t* __restrict__ v_cache,
                                          float* __restrict__ v_scale, int* __restrict__ lens,
                                          int* err) {
  pdl_wait();
  pdl_trigger();
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int heads = hq + 2 * hkv;
  if (gw >= batch * heads) return;
  const int b = gw / heads, hh = gw % heads;
  const int pos = positions[b];
  if (pos < 0 || pos >= max_len) {
    if (lane == 0 && hh == 0) record_error(err, kDevBadPosition);
    return;
  }
  if (hh == 0 && lane == 0) lens[b] = pos + 1;
  float v[4];
  if constexpr (kPartials) {
    const long long stride = static_cast<long long>(batch) * heads * 128;
    const int32_t* base = part + static_cast<long long>(b) * heads * 128 + hh * 128 + lane;
    const float rs = xs[b];
    // the splits' sums, eight splits' loads in flight at a time (the
    // partials sit in L2: the loads' latency, not bandwidth, sets the pace)
    int32_t acc[4] = {0, 0, 0, 0};
    int sp = 0;
    for (; sp + 8 <= splits; sp += 8) {
      int32_t t[8][4];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int32_t* ps = base + (sp + u) * stride;
#pragma unroll
        for (int p = 0; p < 4; ++p) t[u][p] = ps[32 * p];
      }
#pragma unroll
      for (int u = 0; u < 8; ++u)
#pragma unroll
        for (int p = 0; p < 4; ++p) acc[p] += t[u][p];
    }
    for (; sp < splits; ++sp) {
      const int32_t* ps = base + sp * stride;
#pragma unroll
      for (int p = 0; p < 4; ++p) acc[p] += ps[32 * p];
    }
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const int n = hh * 128 + lane + 32 * p;
      v[p] = __fmul_rn(__int2float_rn(acc[p]), __fmul_rn(rs, ws[n]));
    }
  } else {
    const float* x = qkv + static_cast<long long>(b) * heads * 128 + hh * 128;
    v[0] = x[lane];
    v[1] = x[lane + 32];
    v[2] = x[lane + 64];
    v[3] = x[lane + 96];
  }
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

int decode_rope_append_partials(int batch, int heads_q, int heads_kv, int max_len,
                                float rope_base, const int* positions, const int32_t* part,
                                int splits, const float* x_scale, const float* w_scale,
                                int8_t* q8, float* q_scale, int8_t* k_cache, float* k_scale,
                                int8_t* v_cache, float* v_scale, int* lens, cudaStream_t stream) {
  if (part == nullptr || splits < 1 || x_scale == nullptr || w_scale == nullptr)
    return kErrInvalid;
  const long long warps = static_cast<long long>(batch) * (heads_q + 2 * heads_kv);
  // two warps per block, so the (sequence, head) rows spread over every SM
  return launch_k(decode_rope_append_kernel<true>,
                  dim3(static_cast<unsigned>((warps * 32 + 63) / 64)), dim3(64), 0, stream,
                  batch, heads_q, heads_kv, max_len, rope_base, positions,
                  static_cast<const float*>(nullptr), part, splits, x_scale, w_scale, q8, q_scale,
                  k_cache, k_scale, v_cache, v_scale, lens, device_error_ptr());
}


// the partial rows cta + pair of G heads each: at most (ctas + pairs) * G
// <= (ctas + batch) * heads_q head rows
size_t decode_attn_partial_floats(int batch, int heads_q, int max_len) {
  (void)max_len;
  return static_cast<size_t>(kMaxCtasPerSm * num_sms() + batch) * heads_q * kPartRow;
}

int decode_attn_i8(const DecodeProblem& p, cudaStream_t st) {
  if (p.batch <= 0 || p.heads_q <= 0 || p.heads_kv <= 0 || p.max_len <= 0) return kErrInvalid;
  if (p.heads_q % p.heads_kv != 0) return kErrInvalid;
  if (p.out == nullptr) return kErrInvalid;
  // the bulk copies read scale groups of 16 bytes; TMA wants 16-byte bases
  if (p.max_len % 4 != 0 ||
      ((reinterpret_cast<uintptr_t>(p.k_cache) | reinterpret_cast<uintptr_t>(p.v_cache) |
        reinterpret_cast<uintptr_t>(p.k_scale) | reinterpret_cast<uintptr_t>(p.v_scale)) & 15u) != 0)
    return kErrAlignment;
  const int G = p.heads_q / p.heads_kv;
  if (G > kMaxGroup) return kErrInvalid;
  const int pairs = p.batch * p.heads_kv;
  DecodeArgs a{};
  a.batch = p.batch;
  a.heads_q = p.heads_q;
  a.heads_kv = p.heads_kv;
  a.max_len = p.max_len;
  a.tiles = (p.max_len + kTileKeys - 1) / kTileKeys;
  a.units = static_cast<long long>(pairs) * a.tiles;
  a.sm_scale = p.sm_scale;
  a.q8 = p.q8;
  a.q_scale = p.q_scale;
  a.k_scale = p.k_scale;
  a.v_scale = p.v_scale;
  a.lens = p.lens;
  a.positions = p.lens != nullptr ? p.positions : nullptr;
  a.len = p.len;
  a.part = p.partial;
  a.out = p.out;
  a.err = device_error_ptr();
  // K and V as [pairs][max_len][128] int8, 128-key boxes with the 128-byte
  // swizzle (rows past max_len read as zeros)
  CUtensorMap km, vm;
  const long long seg = static_cast<long long>(p.max_len) * 128;
  if (int rc = make_tma_3d_i8(&km, p.k_cache, p.max_len, 128, 128, pairs, seg, 128, kTileKeys))
    return rc;
  if (int rc = make_tma_3d_i8(&vm, p.v_cache, p.max_len, 128, 128, pairs, seg, 128, kTileKeys))
    return rc;
  switch (G) {
    case 1: return launch_decode<1>(km, vm, a, st);
    case 2: return launch_decode<2>(km, vm, a, st);
    case 4: return launch_decode<4>(km, vm, a, st);
    case 8: return launch_decode<8>(km, vm, a, st);
    case 16: return launch_decode<16>(km, vm, a, st);
    default: return kErrInvalid;
  }
}

}  // namespace reef
