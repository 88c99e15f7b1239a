// flash_attn.cu -- int8 flash attention for prefill on sm_100a.
//
// The head reef's engine computes (attend_head, attention.hpp:117-123):
// softmax over the visible keys of q.k, then P.v; here with int8 q / k, one
// fp32 scale per (token, head) for each, Llama's 1/sqrt(head_dim) score
// scale, causal visibility (causal_visibility with query_start 0), GQA
// (query head h reads key/value head h / (Hq / Hkv)).  V arrives dequantised
// to f16 (v8 * v_scale, rounded once), transposed.  Checked against the
// engine's float head on the dequantised inputs within 1e-2.
//
//   S   = (q8 . k8^T) * k_scale[j] * (q_scale[i] * sm_scale * log2 e)
//   P   = 2^(S - rowmax)                  (online, fp32, one thread per row)
//   O   = sum_j P[i][j] * v[j]            (f16 x f16 -> fp32)
//   out = O / sum_j P[i][j]
//
// One CTA per (pair of 128-query tiles, batch, head): the two tiles share
// every K / V tile the CTA loads.  TMEM holds, per query tile x, an int32
// score tile S_x (128 columns) and the fp32 accumulator O_x (128 columns);
// P_x (f16) is written back over the first 64 columns of S_x and the P.V
// product reads it from there, so P never touches shared memory.  12 warps:
//   warp 0      TMA: lane 0 loads both Q tiles, then the K ring (int8, 128
//               keys x 128 B); lane 1 the V^T ring (f16 [128 dims][128 keys]
//               as two 64-key boxes).
//   warp 1      TMEM allocation; one thread issues, per key tile j and query
//               tile x, O_x += P_x(j) V(j) (kind::f16, A from TMEM) as soon as
//               the softmax group has written P_x(j), then S_x(j+1) =
//               Q_x K(j+1)^T (kind::i8) into the same columns.  The tensor
//               pipe runs one thread's MMAs in order, so S_x(j+1) overwrites
//               P_x(j) only after the product has read it, and S_x(j+1)
//               complete means O_x holds every P.V up to j.
//   warps 4..7  softmax of query tile A, warps 8..11 of query tile B: each
//               thread owns one row (its TMEM lane).  The two groups take turns
//               at the exponentials (the MUFU-bound phase): A's k-th turn
//               follows B's (k-1)-th, B's k-th follows A's k-th, through two
//               named barriers, so one group loads scores and takes its
//               maxima while the other exponentiates.
// Per score: int32 -> fp32 exactly by adding the bit pattern of 1.5 * 2^23
// (|q.k| < 2^22 for 128 int8 products) and subtracting 1.5 * 2^23, times the
// key's scale, a 3-input max, and one ex2; masks run only on the diagonal and
// tail tiles.  The row max in O is refreshed lazily: O and the row sum are
// rescaled only when the max grows by more than 2^8, so P stays below 256,
// far inside f16.  The output leaves through shared memory (the dead Q tile)
// as asynchronous TMA stores.
// Every mbarrier wait is bounded; after a timeout a thread keeps walking the
// same barrier sequence without waiting, so the CTA still exits.
#include "common.cuh"
#include "ops.h"

#include <cuda_fp16.h>

namespace reef {

namespace {

constexpr int kFThreads = 384;
// Registers: 168 a thread at launch (384 x 168 = 64512); the control
// warpgroup (warps 0-3) drops to 96 and each softmax warpgroup rises to 200,
// which holds a row's 128 scores without spilling.
constexpr uint32_t kRegsLaunch = 168, kRegsControl = 96;
constexpr uint32_t kRegsSoftmax = (kFThreads * kRegsLaunch - 128 * kRegsControl) / 256 / 8 * 8;
static_assert(128 * kRegsControl + 256 * kRegsSoftmax <= kFThreads * kRegsLaunch,
              "register split exceeds the launch allocation");
constexpr int kTile = 128;
constexpr int kHeadDim = 128;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.0f;
// 1.5 * 2^23: for |x| < 2^22, the float with bits (x + kMagicBits) is
// exactly kMagic + x.
constexpr int kMagicBits = 0x4B400000;
constexpr float kMagic = 12582912.0f;

constexpr int kKStages = 4;  // K tiles in flight (16 KB each)
constexpr int kVStages = 3;  // V^T tiles in flight (32 KB each)
struct FL {
  static constexpr int kQ = 0;                            // 2 x 16 KB (then output staging)
  static constexpr int kK = 32768;                        // kKStages x 16 KB
  static constexpr int kV = kK + kKStages * 16384;        // kVStages x 32 KB
  static constexpr int kScales = kV + kVStages * 32768;   // [8 warps][2 bufs][128] float
  static constexpr int kBars = kScales + 8 * 2 * 128 * 4;
  static constexpr int kNumBars = 8 + 2 * kKStages + 2 * kVStages;
  static constexpr int kTmemSlot = kBars + kNumBars * 8;
  static constexpr int kAlloc = kTmemSlot + 16 + 1024;
};
static_assert(FL::kAlloc <= 232448, "flash smem budget");
static_assert(FL::kK % 1024 == 0 && FL::kV % 1024 == 0, "swizzled tiles need 1 KB alignment");

struct FlashArgs {
  int batch, heads_q, heads_kv, seq, causal;
  float sm_scale;
  const float* q_scale;  // [B][Hq][S]
  const float* k_scale;  // [B][Hkv][S]
  int* err;
};

__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x by the hardware approximation (ex2.approx.ftz; 2^-inf = 0)
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ int tiles_for(int q_tile, int num_kv, int causal) {
  return causal ? min(q_tile + 1, num_kv) : num_kv;
}

// exact int32 -> fp32 (|x| < 2^22), times the key scale: one rounding
__device__ __forceinline__ float score(uint32_t acc, float ks) {
  return __fmul_rn(__fadd_rn(__int_as_float(static_cast<int>(acc) + kMagicBits), -kMagic), ks);
}

__global__ void __launch_bounds__(kFThreads, 1)
    flash_prefill_kernel(const __grid_constant__ CUtensorMap tq,
                         const __grid_constant__ CUtensorMap tk,
                         const __grid_constant__ CUtensorMap tv,
                         const __grid_constant__ CUtensorMap to, FlashArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + FL::kBars);
  uint64_t* q_full = bars + 0;
  uint64_t* s_full = bars + 1;    // [2] per query tile: S_x(j) and all before it done
  uint64_t* p_full = bars + 3;    // [2] per query tile (128 arrivals)
  uint64_t* o_done = bars + 5;    // [2] per query tile: its last P.V done
  uint64_t* drain = bars + 7;
  uint64_t* k_full = bars + 8;                                // [kKStages]
  uint64_t* k_empty = k_full + kKStages;                      // [kKStages]
  uint64_t* v_full = k_empty + kKStages;                      // [kVStages]
  uint64_t* v_empty = v_full + kVStages;                      // [kVStages]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + FL::kTmemSlot);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.seq;
  const int num_q_tiles = (S + kTile - 1) / kTile;
  const int num_pairs = (num_q_tiles + 1) / 2;
  // head-major order: the tiles of one head run together and share its K / V
  // in L2; within a head the longest (causal) pairs start first
  const int bh = static_cast<int>(blockIdx.x / num_pairs);
  const int pair = num_pairs - 1 - static_cast<int>(blockIdx.x % num_pairs);
  const int b = bh / a.heads_q, h = bh % a.heads_q;
  const int hkv = h / (a.heads_q / a.heads_kv);
  const int num_kv = (S + kTile - 1) / kTile;
  const bool has_b = 2 * pair + 1 < num_q_tiles;
  const int n_a = tiles_for(2 * pair, num_kv, a.causal);
  const int n_b = has_b ? tiles_for(2 * pair + 1, num_kv, a.causal) : 0;
  const int n = max(n_a, n_b);  // key tiles this CTA loads
  int* err = a.err;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tq);
    prefetch_tensormap(&tk);
    prefetch_tensormap(&tv);
    prefetch_tensormap(&to);
    mbar_init(q_full, 1);
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < kVStages; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  // everything above touches only this CTA's shared memory: as a programmatic
  // dependent it overlaps the kernel ahead, which must finish before q, k, v
  // or their scales are read
  pdl_wait();
  pdl_trigger();
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  // columns: S_A [0,128), S_B [128,256), O_A [256,384), O_B [384,512);
  // P_x over the first 64 columns of S_x
  const uint32_t tS = tmem;
  const uint32_t tO = tmem + 256;

  if (warp < 4) {
    setmaxnreg_dec<kRegsControl>();
    if (warp == 0) {
      // ---------------- TMA producers ----------------
      // lane 0: Q, then the K ring; lane 1: the V ring.  Independent threads,
      // so a V refill waiting for P.V never holds back the next K tile.
      const int vrow = (b * a.heads_kv + hkv) * kHeadDim;
      if (lane == 0) {
        mbar_arrive_expect_tx(q_full, has_b ? 32768 : 16384);
        tma_load_2d(smem + FL::kQ, &tq, q_full, h * kHeadDim, b * S + 2 * pair * kTile);
        if (has_b)
          tma_load_2d(smem + FL::kQ + 16384, &tq, q_full, h * kHeadDim,
                      b * S + (2 * pair + 1) * kTile);
        int issued = 0;
        for (int j = 0; j < n; ++j) {
          const int s = j % kKStages;
          if (!mbar_wait(&k_empty[s], ((j / kKStages) & 1) ^ 1u, err, kDevTimeoutEmpty)) break;
          mbar_arrive_expect_tx(&k_full[s], 16384);
          tma_load_2d(smem + FL::kK + s * 16384, &tk, &k_full[s], hkv * kHeadDim, b * S + j * kTile);
          issued = j + 1;
        }
        // let in-flight copies land before exit
        mbar_wait(q_full, 0, err, kDevTimeoutDrain);
        for (int j = issued > kKStages ? issued - kKStages : 0; j < issued; ++j)
          mbar_wait(&k_full[j % kKStages], (j / kKStages) & 1, err, kDevTimeoutDrain);
      } else if (lane == 1) {
        int issued = 0;
        for (int j = 0; j < n; ++j) {
          const int s = j % kVStages;
          if (!mbar_wait(&v_empty[s], ((j / kVStages) & 1) ^ 1u, err, kDevTimeoutEmpty)) break;
          mbar_arrive_expect_tx(&v_full[s], 32768);
          uint8_t* vs = smem + FL::kV + s * 32768;
          tma_load_2d(vs, &tv, &v_full[s], j * kTile, vrow);
          tma_load_2d(vs + 16384, &tv, &v_full[s], j * kTile + 64, vrow);
          issued = j + 1;
        }
        for (int j = issued > kVStages ? issued - kVStages : 0; j < issued; ++j)
          mbar_wait(&v_full[j % kVStages], (j / kVStages) & 1, err, kDevTimeoutDrain);
      }
    } else if (warp == 1) {
      if (lane == 0) {
        // ---------------- MMA issuer ----------------
        constexpr uint32_t kIdescS = idesc_i8(128, 128);
        constexpr uint32_t kIdescO = idesc_f16(128, 128);
        bool ok = mbar_wait(q_full, 0, err, kDevTimeoutFull);
        const uint32_t sq = smem_u32(smem + FL::kQ);
        auto issue_s = [&](int x, int j) {
          const uint32_t sk = smem_u32(smem + FL::kK + (j % kKStages) * 16384);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_i8(tS + x * 128, smem_desc_k_sw128(sq + x * 16384 + kk * 32),
                   smem_desc_k_sw128(sk + kk * 32), kIdescS, kk > 0 ? 1u : 0u);
          mma_commit(&s_full[x]);
        };
        if (ok) ok = mbar_wait(&k_full[0], 0, err, kDevTimeoutFull);
        tc_fence_after();
        if (ok) {
          issue_s(0, 0);
          if (n_b > 0) issue_s(1, 0);
          mma_commit(&k_empty[0]);
        }
        for (int j = 0; j < n && ok; ++j) {
          const int vs = j % kVStages;
          if (!mbar_wait(&v_full[vs], (j / kVStages) & 1, err, kDevTimeoutFull)) { ok = false; break; }
          if (j + 1 < n &&
              !mbar_wait(&k_full[(j + 1) % kKStages], ((j + 1) / kKStages) & 1, err, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          const uint32_t sv = smem_u32(smem + FL::kV + vs * 32768);
          for (int x = 0; x < 2; ++x) {
            const int nx = x ? n_b : n_a;
            if (j >= nx) continue;
            if (!mbar_wait(&p_full[x], j & 1, err, kDevTimeoutFull)) { ok = false; break; }
            tc_fence_after();
#pragma unroll
            for (int kk = 0; kk < 8; ++kk) {  // 16 keys per step: 8 columns of P
              const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
              mma_f16_tmem_a(tO + x * 128, tS + x * 128 + kk * 8, smem_desc_k_sw128(sv + off),
                             kIdescO, (j > 0 || kk > 0) ? 1u : 0u);
            }
            if (j + 1 < nx) {
              issue_s(x, j + 1);
            } else {
              mma_commit(&o_done[x]);
            }
          }
          if (!ok) break;
          mma_commit(&v_empty[vs]);
          if (j + 1 < n) mma_commit(&k_empty[(j + 1) % kKStages]);
        }
        mma_commit(drain);
        mbar_wait(drain, 0, err, kDevTimeoutDrain);
      }
    }
  } else {
    setmaxnreg_inc<kRegsSoftmax>();
    // ---------------- softmax / epilogue, query tile x ----------------
    // warp w reads TMEM lanes [32 (w % 4), +32): warps 4..7 and 8..11 each
    // cover all 128 rows
    const int x = (warp - 4) >> 2;
    const int nx = x ? n_b : n_a;
    const int q_tile = 2 * pair + x;
    const int t = (warp & 3) * 32 + lane;  // query row within the tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t tSx = tS + x * 128 + lane_off, tOx = tO + x * 128 + lane_off;
    const int row = q_tile * kTile + t;
    const bool row_ok = row < S;
    // rows past the end see finite scores (scale 1) and are never stored
    const float qs = row_ok ? a.q_scale[(static_cast<long long>(b) * a.heads_q + h) * S + row] : 1.0f;
    const float amul = qs * a.sm_scale * kLog2e;  // > 0
    const int last_key = a.causal ? min(row, S - 1) : S - 1;
    const long long kv_base = (static_cast<long long>(b) * a.heads_kv + hkv) * S;
    // this warp's copy of the tile's key scales: [2 bufs][128] float
    float* ksw = reinterpret_cast<float*>(smem + FL::kScales) + (warp - 4) * 256;
    float m = 0.0f, l = 0.0f;
    bool ok = true;
    // Turn-taking (hardware barriers 3 and 4, 256 threads: one group syncs,
    // the other arrives).  A syncs on 3 before each of its n_a turns and
    // arrives on 4 after; B arrives on 3 once up front and after each turn j
    // with j + 1 < n_a, and syncs on 4 before its turns j < n_a (its extra
    // causal tile runs alone).  Both barriers then see n_a completions with
    // at most one outstanding, for n_b >= n_a; otherwise the groups do not
    // take turns.  The sequence is walked whether or not a wait timed out.
    const bool turns = n_b >= n_a && n_b > 0;
    constexpr int kTurnA = 3, kTurnB = 4;
    if (turns && x == 1) named_arrive(kTurnA, 256);
    // lane l stages keys [4l, 4l+4) of each tile, loaded a tile ahead (seq is
    // a multiple of 8, so four keys are all in range or all past the end)
    const float4* ks4 = reinterpret_cast<const float4*>(a.k_scale + kv_base);
    float4 nk = (nx > 0 && 4 * lane < S) ? __ldg(ks4 + lane) : make_float4(0.f, 0.f, 0.f, 0.f);
    for (int j = 0; j < nx; ++j) {
      const uint32_t ph = j & 1;
      reinterpret_cast<float4*>(ksw + ph * 128)[lane] = nk;
      __syncwarp();
      {
        const int key_n = (j + 1) * kTile + 4 * lane;
        nk = (j + 1 < nx && key_n < S) ? __ldg(ks4 + (j + 1) * 32 + lane)
                                       : make_float4(0.f, 0.f, 0.f, 0.f);
      }
      // S_x(j) complete: also every P.V before it, so O_x and the P columns
      // are free
      if (ok) ok = mbar_wait(&s_full[x], ph, err, kDevTimeoutAccFull);
      ok = __all_sync(0xffffffffu, ok);  // reconverge before warp-collective tcgen05.ld
      tc_fence_after();
      uint32_t r[128];
#pragma unroll
      for (int c = 0; c < 4; ++c)
        tmem_ld_32x32b_x32(tSx + c * 32, *reinterpret_cast<uint32_t(*)[32]>(&r[c * 32]));
      tmem_ld_wait();
      // scores in units of q_scale * sm_scale * log2 e
      const float4* skv = reinterpret_cast<const float4*>(ksw + ph * 128);
      float mx0 = -INFINITY, mx1 = -INFINITY;
      const bool mask = (a.causal && j == q_tile) || (j + 1) * kTile > S;
      if (!mask) {
#pragma unroll
        for (int e = 0; e < 128; e += 4) {
          const float4 c = skv[e >> 2];
          const float f0 = score(r[e], c.x), f1 = score(r[e + 1], c.y);
          const float f2 = score(r[e + 2], c.z), f3 = score(r[e + 3], c.w);
          mx0 = max3(mx0, f0, f1);
          mx1 = max3(mx1, f2, f3);
          r[e] = __float_as_uint(f0);
          r[e + 1] = __float_as_uint(f1);
          r[e + 2] = __float_as_uint(f2);
          r[e + 3] = __float_as_uint(f3);
        }
      } else {
        const int lim = last_key - j * kTile;  // keys e > lim are not visible
#pragma unroll
        for (int e = 0; e < 128; e += 4) {
          const float4 c = skv[e >> 2];
          const float f0 = e > lim ? -INFINITY : score(r[e], c.x);
          const float f1 = e + 1 > lim ? -INFINITY : score(r[e + 1], c.y);
          const float f2 = e + 2 > lim ? -INFINITY : score(r[e + 2], c.z);
          const float f3 = e + 3 > lim ? -INFINITY : score(r[e + 3], c.w);
          mx0 = max3(mx0, f0, f1);
          mx1 = max3(mx1, f2, f3);
          r[e] = __float_as_uint(f0);
          r[e + 1] = __float_as_uint(f1);
          r[e + 2] = __float_as_uint(f2);
          r[e + 3] = __float_as_uint(f3);
        }
      }
      // every visited tile has a visible key in every row, so the max is finite
      const float mt = fmaxf(mx0, mx1) * amul;
      // The rescale runs warp-collective tcgen05.ld/st, so the decision is
      // per warp: when any row of the warp needs it, every row of the warp
      // moves to its own new maximum (alpha = 1 for rows whose max held).
      float alpha = 1.0f;
      bool rescale = false;
      if (j == 0) {
        m = mt;
      } else if (__any_sync(0xffffffffu, mt > m + kRescaleLog2)) {
        const float m_new = fmaxf(m, mt);
        alpha = ex2(m - m_new);
        m = m_new;
        rescale = true;
      }
      if (turns) {
        if (x == 0) {
          named_barrier(kTurnA, 256);
        } else if (j < n_a) {
          named_barrier(kTurnB, 256);
        }
      }
      // P = 2^(score - m) as f16 pairs, packed into r[0..63] (each pair
      // overwrites scores already consumed)
      const float nm = -m;
      float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
      for (int k0 = 0; k0 < 128; k0 += 2) {
        const float p0 = ex2(__fmaf_rn(__uint_as_float(r[k0]), amul, nm));
        const float p1 = ex2(__fmaf_rn(__uint_as_float(r[k0 + 1]), amul, nm));
        if (k0 & 2) {
          ps1 += p0 + p1;
        } else {
          ps0 += p0 + p1;
        }
        const __half2 hv = __floats2half2_rn(p0, p1);
        r[k0 >> 1] = *reinterpret_cast<const uint32_t*>(&hv);
      }
      if (turns) {
        if (x == 0) {
          named_arrive(kTurnB, 256);
        } else if (j + 1 < n_a) {
          named_arrive(kTurnA, 256);
        }
      }
      l = __fmaf_rn(l, alpha, ps0 + ps1);
      tmem_st_32x32b_x32(tSx, *reinterpret_cast<uint32_t(*)[32]>(&r[0]));
      tmem_st_32x32b_x32(tSx + 32, *reinterpret_cast<uint32_t(*)[32]>(&r[32]));
      if (rescale) {
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tOx + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st_32x32b_x32(tOx + c * 32, o);
        }
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[x]);
    }
    // ---------------- epilogue: out = O / l, via TMA stores ----------------
    // Staged 32 columns at a time in this tile's Q buffer (its last reader,
    // S_x(n_x - 1), is done before o_done), 128-byte swizzled rows.
    if (nx > 0) {
      if (ok) ok = mbar_wait(&o_done[x], 0, err, kDevTimeoutAccFull);
      ok = __all_sync(0xffffffffu, ok);
      tc_fence_after();
      const float inv = 1.0f / l;
      uint8_t* stage = smem + FL::kQ + x * 16384;
      for (int c = 0; c < 4; ++c) {
        uint32_t o[32];
        tmem_ld_32x32b_x32(tOx + c * 32, o);
        tmem_ld_wait();
        if (c > 0) {
          // the previous chunk's store has read the staging tile
          if (t == 0) bulk_wait_group_read0();
          named_barrier(1 + x, 128);
        }
#pragma unroll
        for (int k = 0; k < 8; ++k)
          *reinterpret_cast<float4*>(stage + t * 128 + ((k ^ (t & 7)) << 4)) =
              make_float4(__uint_as_float(o[4 * k]) * inv, __uint_as_float(o[4 * k + 1]) * inv,
                          __uint_as_float(o[4 * k + 2]) * inv, __uint_as_float(o[4 * k + 3]) * inv);
        fence_proxy_async_smem();
        named_barrier(1 + x, 128);
        if (t == 0) {
          tma_store_3d(&to, stage, h * kHeadDim + c * 32, q_tile * kTile, b);
          bulk_commit_group();
        }
      }
      if (t == 0) bulk_wait_group_read0();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ---- Q / K: RoPE, then int8 per (token, head) -----------------------------------
//
// One warp per (token, head) of the QKV projection output [T][(Hq+2Hkv)*128]:
// Llama rotate-half RoPE on q and k (theta_i = pos * base^(-2i/128), pairs
// (i, i+64)), then the head's 128 values quantised with reef's rule
// (quant.hpp:51-81: scale = max|x|/127, rne, clamp).  Outputs: q8 [T][Hq*128],
// k8 [T][Hkv*128] token-major (the int8 cache rows) and scales [B][H][S].
// (cos, sin) of pos * base^(-2i/128) for pos < seq, i < 64: computed once per
// forward so the per-element RoPE is two table loads.  i-major: table[i][pos],
// so a warp of consecutive tokens reads one contiguous run per i.
__global__ void rope_table_kernel(int seq, float base, float2* __restrict__ table) {
  pdl_wait();
  pdl_trigger();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= seq * 64) return;
  const int i = idx / seq, pos = idx - i * seq;
  const float inv_freq = powf(base, -static_cast<float>(2 * i) / kHeadDim);
  float sn, cs;
  sincosf(static_cast<float>(pos) * inv_freq, &sn, &cs);
  table[idx] = make_float2(cs, sn);
}

__global__ void rope_qk_quant_kernel(int tokens, int seq, int hq, int hkv, float base,
                                     const float2* __restrict__ table,
                                     const float* __restrict__ qkv, int8_t* __restrict__ q8,
                                     int8_t* __restrict__ k8, float* __restrict__ qs,
                                     float* __restrict__ ks) {
  const int gw = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int heads = hq + hkv;
  if (gw >= tokens * heads) return;
  const int tok = gw / heads, hh = gw % heads;
  const int pos = tok % seq, bidx = tok / seq;
  const int width = (hq + 2 * hkv) * kHeadDim;
  const float* x = qkv + static_cast<long long>(tok) * width + hh * kHeadDim;
  float v[4];
  float lo0 = x[lane], lo1 = x[lane + 32], hi0 = x[lane + 64], hi1 = x[lane + 96];
#pragma unroll
  for (int p = 0; p < 2; ++p) {
    const int i = lane + 32 * p;
    float sn, cs;
    if (table != nullptr) {
      const float2 t = __ldg(table + static_cast<long long>(i) * seq + pos);
      cs = t.x;
      sn = t.y;
    } else {
      const float inv_freq = powf(base, -static_cast<float>(2 * i) / kHeadDim);
      sincosf(static_cast<float>(pos) * inv_freq, &sn, &cs);
    }
    const float lo = p == 0 ? lo0 : lo1, hi = p == 0 ? hi0 : hi1;
    v[p] = lo * cs - hi * sn;
    v[p + 2] = hi * cs + lo * sn;
  }
  float mx = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  const float scale = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
  int8_t* dst;
  if (hh < hq) {
    dst = q8 + static_cast<long long>(tok) * hq * kHeadDim + hh * kHeadDim;
    if (lane == 0) qs[(static_cast<long long>(bidx) * hq + hh) * seq + pos] = scale;
  } else {
    const int kh = hh - hq;
    dst = k8 + static_cast<long long>(tok) * hkv * kHeadDim + kh * kHeadDim;
    if (lane == 0) ks[(static_cast<long long>(bidx) * hkv + kh) * seq + pos] = scale;
  }
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    int c = __float2int_rn(__fdiv_rn(v[p], scale));
    c = c < -127 ? -127 : (c > 127 ? 127 : c);
    dst[lane + 32 * p] = static_cast<int8_t>(c);
  }
}

// ---- V: int8 per (token, head), plus the transposed f16 copy ----------------------
//
// CTA = 64 tokens x 1 kv head (256 threads).  v8 [T][Hkv*128] token-major (the
// int8 cache rows) and vs [B][Hkv][S]; vt [B][Hkv][128][S] f16 holds the
// dequantised values f16(code * scale), transposed so the P.V MMA reads it
// K-major.  The transposed write stores 64 positions (128 bytes) per row.
constexpr int kVTokens = 64;
__global__ void __launch_bounds__(256) v_quant_kernel(int tokens, int seq, int hq, int hkv,
                                                      const float* __restrict__ qkv,
                                                      int8_t* __restrict__ v8,
                                                      float* __restrict__ vs,
                                                      __half* __restrict__ vt) {
  // odd row pitch (in halves): the transposed reads of rows 2l and 2l+1 hit
  // distinct banks across the warp
  __shared__ __half tile[kVTokens][kHeadDim + 1];
  const int kh = blockIdx.y;
  const int tok0 = blockIdx.x * kVTokens;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int width = (hq + 2 * hkv) * kHeadDim;
  for (int tt = warp; tt < kVTokens; tt += 8) {
    const int tok = tok0 + tt;
    if (tok >= tokens) break;
    const float* x = qkv + static_cast<long long>(tok) * width + (hq + hkv + kh) * kHeadDim;
    float v[4];
    float mx = 0.0f;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      v[p] = x[lane + 32 * p];
      mx = fmaxf(mx, fabsf(v[p]));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float scale = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
    const int pos = tok % seq, bidx = tok / seq;
    if (lane == 0) vs[(static_cast<long long>(bidx) * hkv + kh) * seq + pos] = scale;
    int8_t* dst = v8 + static_cast<long long>(tok) * hkv * kHeadDim + kh * kHeadDim;
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      int c = __float2int_rn(__fdiv_rn(v[p], scale));
      c = c < -127 ? -127 : (c > 127 ? 127 : c);
      dst[lane + 32 * p] = static_cast<int8_t>(c);
      tile[tt][lane + 32 * p] = __float2half_rn(__fmul_rn(static_cast<float>(c), scale));
    }
  }
  __syncthreads();
  // transposed write: vt[b][kh][d][pos], a pair of positions per thread (seq
  // is even, so a pair never straddles two sequences)
  const int tok = tok0 + 2 * lane;
  if (tok < tokens) {
    const int pos = tok % seq, bidx = tok / seq;
    __half* col = vt + (static_cast<long long>(bidx) * hkv + kh) * kHeadDim * seq + pos;
    for (int d = warp; d < kHeadDim; d += 8)
      *reinterpret_cast<__half2*>(col + static_cast<long long>(d) * seq) =
          __halves2half2(tile[2 * lane][d], tile[2 * lane + 1][d]);
  }
}

}  // namespace

int flash_prefill_i8(const FlashProblem& p, cudaStream_t stream) {
  if (p.batch <= 0 || p.heads_q <= 0 || p.heads_kv <= 0 || p.seq <= 0) return kErrInvalid;
  if (p.head_dim != kHeadDim || p.heads_q % p.heads_kv != 0) return kErrInvalid;
  if (p.seq % 8 != 0) return kErrAlignment;  // V^T rows must be 16-byte strided
  if ((reinterpret_cast<uintptr_t>(p.k_scale) & 15u) != 0) return kErrAlignment;  // float4 loads
  CUtensorMap mq, mk, mv;
  const long long tokens = static_cast<long long>(p.batch) * p.seq;
  int rc = make_tma_2d_i8(&mq, p.q8, tokens, static_cast<long long>(p.heads_q) * kHeadDim,
                          static_cast<long long>(p.heads_q) * kHeadDim, 128, 128);
  if (rc) return rc;
  rc = make_tma_2d_i8(&mk, p.k8, tokens, static_cast<long long>(p.heads_kv) * kHeadDim,
                      static_cast<long long>(p.heads_kv) * kHeadDim, 128, 128);
  if (rc) return rc;
  rc = make_tma_2d(&mv, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, p.vt,
                   static_cast<long long>(p.batch) * p.heads_kv * kHeadDim, p.seq, p.seq, 64,
                   128, CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  // out as [B][S][Hq*128] fp32 so that rows past a sequence's end are clipped
  CUtensorMap mo;
  rc = make_tma_3d(&mo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, p.out,
                   static_cast<long long>(p.heads_q) * kHeadDim, p.seq, p.batch, p.out_ld * 4,
                   static_cast<long long>(p.seq) * p.out_ld * 4, 32, 128,
                   CU_TENSOR_MAP_SWIZZLE_128B);
  if (rc) return rc;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(flash_prefill_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             FL::kAlloc) != cudaSuccess)
      return kErrCuda;
    configured[dev] = true;
  }
  FlashArgs a{};
  a.batch = p.batch;
  a.heads_q = p.heads_q;
  a.heads_kv = p.heads_kv;
  a.seq = p.seq;
  a.causal = p.causal;
  a.sm_scale = p.sm_scale;
  a.q_scale = p.q_scale;
  a.k_scale = p.k_scale;
  a.err = device_error_ptr();
  const int grid = (((p.seq + kTile - 1) / kTile + 1) / 2) * p.batch * p.heads_q;
  return launch_k(flash_prefill_kernel, dim3(static_cast<unsigned>(grid)), dim3(kFThreads),
                  FL::kAlloc, stream, mq, mk, mv, mo, a);
}

int rope_table(int seq, float rope_base, void* table, cudaStream_t stream) {
  if (seq <= 0 || table == nullptr) return kErrInvalid;
  return launch_k(rope_table_kernel, dim3(static_cast<unsigned>((seq * 64 + 255) / 256)), dim3(256),
                  0, stream, seq, rope_base, static_cast<float2*>(table));
}

int rope_qkv_quant(int batch, int seq, int heads_q, int heads_kv, float rope_base,
                   const float* qkv, int8_t* q8, int8_t* k8, int8_t* v8, float* q_scale,
                   float* k_scale, float* v_scale, void* vt, void* rope_table,
                   cudaStream_t stream) {
  const int tokens = batch * seq;
  if (tokens <= 0 || heads_q <= 0 || heads_kv <= 0) return kErrInvalid;
  float2* table = static_cast<float2*>(rope_table);
  if (table != nullptr)
    rope_table_kernel<<<(seq * 64 + 255) / 256, 256, 0, stream>>>(seq, rope_base, table);
  const long long warps = static_cast<long long>(tokens) * (heads_q + heads_kv);
  rope_qk_quant_kernel<<<static_cast<unsigned>((warps * 32 + 255) / 256), 256, 0, stream>>>(
      tokens, seq, heads_q, heads_kv, rope_base, table, qkv, q8, k8, q_scale, k_scale);
  if (seq % 2 != 0) return kErrAlignment;
  dim3 grid(static_cast<unsigned>((tokens + kVTokens - 1) / kVTokens),
            static_cast<unsigned>(heads_kv));
  v_quant_kernel<<<grid, 256, 0, stream>>>(tokens, seq, heads_q, heads_kv, qkv, v8, v_scale,
                                           static_cast<__half*>(vt));
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace reef
