// flash_attn.cu -- int8 flash attention for prefill on sm_100a.
//
// The head reef's engine computes (attend_head, attention.hpp:117-123):
// softmax over the visible keys of q.k, then P.v; here with int8 q / k / v,
// one fp32 scale per (token, head) for each, Llama's 1/sqrt(head_dim) score
// scale, causal visibility (causal_visibility with query_start 0), GQA
// (query head h reads key/value head h / (Hq / Hkv)).  Checked against the
// engine's float head on the dequantised inputs within 1e-2.
//
//   S   = (q8 . k8^T)  * q_scale[i] * k_scale[j] * sm_scale  (int32 -> fp32)
//   P   = exp(S - rowmax)                 (online, fp32, one thread per row)
//   O   = sum_j P[i][j] * v_scale[j] * v8[j]   (f16 x f16 -> fp32)
//   out = O / sum_j P[i][j]
//
// One CTA per (128-query tile, batch, head); 8 warps:
//   warp 0      TMA: Q tile once; K tiles (int8, 128 keys x 128 B) and V^T
//               tiles (f16, [128 dims][128 keys], two 64-key boxes) through
//               two-stage rings with separate K and V release.
//   warp 1      TMEM (512 columns: two int32 score buffers, one fp32 O);
//               one thread issues S = Q K^T (tcgen05 kind::i8, 128x128x32 x4)
//               into alternating score buffers, and O += P V^T (kind::f16,
//               128x128x16 x8) with P from shared memory.
//   warps 4..7  softmax: thread t owns query row t (TMEM lane t): loads its
//               128 scores, masks, keeps the running max / sum in registers,
//               writes P (f16, scaled by v_scale) into the 128-byte-swizzled
//               K-major layout the MMA reads, and rescales O in TMEM only when
//               the row max grows by more than 2^8 (lazy rescale: P stays
//               below 256, far inside f16).  Finally O / sum -> out.
// Every mbarrier wait is bounded; after a timeout a thread keeps walking the
// same barrier sequence without waiting, so the CTA still exits.
#include "common.cuh"
#include "ops.h"

#include <cuda_fp16.h>

namespace reef {

namespace {

constexpr int kFThreads = 256;
constexpr int kTile = 128;
constexpr int kHeadDim = 128;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.0f;

constexpr int kKStages = 4;  // K tiles in flight (16 KB each)
struct FL {
  static constexpr int kQ = 0;                            // 16 KB
  static constexpr int kK = 16384;                        // kKStages x 16 KB
  static constexpr int kV = kK + kKStages * 16384;        // 2 x 32 KB
  static constexpr int kP = kV + 2 * 32768;               // 2 x 32 KB
  static constexpr int kScales = kP + 2 * 32768;          // sk[2][128], sv[2][128]
  static constexpr int kBars = kScales + 4 * 128 * 4;
  static constexpr int kNumBars = 14 + 2 * kKStages;
  static constexpr int kTmemSlot = kBars + kNumBars * 8;
  static constexpr int kAlloc = kTmemSlot + 16 + 1024;
};
static_assert(FL::kAlloc <= 232448, "flash smem budget");

struct FlashArgs {
  int batch, heads_q, heads_kv, seq, causal;
  float sm_scale;
  const float* q_scale;  // [B][Hq][S]
  const float* k_scale;  // [B][Hkv][S]
  const float* v_scale;  // [B][Hkv][S]
  float* out;            // [B*S][out_ld]
  long long out_ld;
  int* err;
};

// byte offset of element e (f16) of row r in a [128][128] f16 K-major tile
// stored as two 128-byte-swizzled [128][64] blocks
__device__ __forceinline__ uint32_t p_offset(int r, int chunk16) {
  const int kb = chunk16 >> 3;  // 8 chunks of 16 B per 128-byte row
  const int c = chunk16 & 7;
  return static_cast<uint32_t>(kb * 16384 + r * 128 + ((c ^ (r & 7)) << 4));
}

__global__ void __launch_bounds__(kFThreads, 1)
    flash_prefill_kernel(const __grid_constant__ CUtensorMap tq,
                         const __grid_constant__ CUtensorMap tk,
                         const __grid_constant__ CUtensorMap tv, FlashArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + FL::kBars);
  uint64_t* q_full = bars + 0;
  uint64_t* v_full = bars + 1;   // [2]
  uint64_t* v_empty = bars + 3;  // [2]
  uint64_t* s_full = bars + 5;   // [2]
  uint64_t* s_empty = bars + 7;  // [2]
  uint64_t* p_full = bars + 9;   // [2]
  uint64_t* o_ready = bars + 11; // [2]
  uint64_t* drain = bars + 13;
  uint64_t* k_full = bars + 14;              // [kKStages]
  uint64_t* k_empty = bars + 14 + kKStages;  // [kKStages]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + FL::kTmemSlot);
  float* sk_s = reinterpret_cast<float*>(smem + FL::kScales);  // [2][128]
  float* sv_s = sk_s + 256;                                    // [2][128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int S = a.seq;
  const int num_q_tiles = (S + kTile - 1) / kTile;
  // head-major order: the query tiles of one head run together and share its
  // K / V in L2; within a head the longest (causal) tiles start first
  const int bh = static_cast<int>(blockIdx.x / num_q_tiles);
  const int q_tile = num_q_tiles - 1 - static_cast<int>(blockIdx.x % num_q_tiles);
  const int b = bh / a.heads_q, h = bh % a.heads_q;
  const int hkv = h / (a.heads_q / a.heads_kv);
  const int q0 = q_tile * kTile;
  const int num_kv = (S + kTile - 1) / kTile;
  const int n = a.causal ? min(q_tile + 1, num_kv) : num_kv;
  int* err = a.err;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tq);
    prefetch_tensormap(&tk);
    prefetch_tensormap(&tv);
    mbar_init(q_full, 1);
    for (int i = 0; i < kKStages; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_empty[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_ready[i], 1);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t tS = tmem;        // score buffers: columns [0,128) and [128,256)
  const uint32_t tO = tmem + 256;  // O: columns [256, 384)

  if (warp == 0) {
    // ---------------- TMA producers ----------------
    // lane 0: Q, then the K ring; lane 1: the V ring.  Independent threads,
    // so a V refill waiting for P.V never holds back the next K tile.
    const int vrow = (b * a.heads_kv + hkv) * kHeadDim;
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, 16384);
      tma_load_2d(smem + FL::kQ, &tq, q_full, h * kHeadDim, b * S + q0);
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
        const int s = j & 1;
        if (!mbar_wait(&v_empty[s], ((j >> 1) & 1) ^ 1u, err, kDevTimeoutEmpty)) break;
        mbar_arrive_expect_tx(&v_full[s], 32768);
        uint8_t* vs = smem + FL::kV + s * 32768;
        tma_load_2d(vs, &tv, &v_full[s], j * kTile, vrow);
        tma_load_2d(vs + 16384, &tv, &v_full[s], j * kTile + 64, vrow);
        issued = j + 1;
      }
      for (int j = issued > 2 ? issued - 2 : 0; j < issued; ++j)
        mbar_wait(&v_full[j & 1], (j >> 1) & 1, err, kDevTimeoutDrain);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t kIdescS = idesc_i8(128, 128);
      constexpr uint32_t kIdescO = idesc_f16(128, 128);
      bool ok = mbar_wait(q_full, 0, err, kDevTimeoutFull);
      tc_fence_after();
      const uint32_t sq = smem_u32(smem + FL::kQ);
      auto issue_s = [&](int j) -> bool {
        const int ks = j % kKStages;  // K ring slot
        const int sb = j & 1;         // TMEM score buffer
        if (!mbar_wait(&k_full[ks], (j / kKStages) & 1, err, kDevTimeoutFull)) return false;
        tc_fence_after();
        const uint32_t sk = smem_u32(smem + FL::kK + ks * 16384);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          mma_i8(tS + sb * 128, smem_desc_k_sw128(sq + kk * 32), smem_desc_k_sw128(sk + kk * 32),
                 kIdescS, kk > 0 ? 1u : 0u);
        mma_commit(&k_empty[ks]);
        mma_commit(&s_full[sb]);
        return true;
      };
      if (ok) ok = issue_s(0);
      if (ok && n > 1) ok = issue_s(1);
      for (int j = 0; j < n && ok; ++j) {
        const int bb = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&p_full[bb], ph, err, kDevTimeoutFull)) { ok = false; break; }
        if (!mbar_wait(&v_full[bb], ph, err, kDevTimeoutFull)) { ok = false; break; }
        tc_fence_after();
        const uint32_t sp = smem_u32(smem + FL::kP + bb * 32768);
        const uint32_t sv = smem_u32(smem + FL::kV + bb * 32768);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          mma_f16(tO, smem_desc_k_sw128(sp + off), smem_desc_k_sw128(sv + off), kIdescO,
                  (j > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&v_empty[bb]);
        mma_commit(&o_ready[bb]);
        if (j + 2 < n) {
          if (!mbar_wait(&s_empty[bb], ph, err, kDevTimeoutAccEmpty)) { ok = false; break; }
          tc_fence_after();
          if (!issue_s(j + 2)) { ok = false; break; }
        }
      }
      mma_commit(drain);
      mbar_wait(drain, 0, err, kDevTimeoutDrain);
    }
  } else if (warp >= 4) {
    // ---------------- softmax / epilogue ----------------
    const int t = threadIdx.x - 128;  // query row within the tile == TMEM lane
    const uint32_t lane_off = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int row = q0 + t;
    const bool row_ok = row < S;
    const float qs = row_ok ? a.q_scale[(static_cast<long long>(b) * a.heads_q + h) * S + row] : 0.0f;
    const float amul = qs * a.sm_scale * kLog2e;
    const long long kv_base = (static_cast<long long>(b) * a.heads_kv + hkv) * S;
    float m = -INFINITY, l = 0.0f;
    bool ok = true;
    // per-key scales of the next tile are loaded a tile ahead, into registers
    float nk = t < S ? __ldg(a.k_scale + kv_base + t) : 0.0f;
    float nv = t < S ? __ldg(a.v_scale + kv_base + t) : 0.0f;
    for (int j = 0; j < n; ++j) {
      const int bb = j & 1;
      const uint32_t ph = (j >> 1) & 1;
      sk_s[bb * 128 + t] = nk;
      sv_s[bb * 128 + t] = nv;
      named_barrier(1, 128);
      {
        const int key_n = (j + 1) * kTile + t;
        const bool has = j + 1 < n && key_n < S;
        nk = has ? __ldg(a.k_scale + kv_base + key_n) : 0.0f;
        nv = has ? __ldg(a.v_scale + kv_base + key_n) : 0.0f;
      }
      if (ok) ok = mbar_wait(&s_full[bb], ph, err, kDevTimeoutAccFull);
      ok = __all_sync(0xffffffffu, ok);  // reconverge before warp-collective tcgen05.ld
      tc_fence_after();
      uint32_t r[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld_32x32b_x32(tS + lane_off + bb * 128 + c * 32, r[c]);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(&s_empty[bb]);
      float mt = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int key = j * kTile + c * 32 + e;
          float v = static_cast<float>(static_cast<int32_t>(r[c][e])) * amul * sk_s[bb * 128 + c * 32 + e];
          if (key >= S || (a.causal && key > row)) v = -INFINITY;
          r[c][e] = __float_as_uint(v);
          mt = fmaxf(mt, v);
        }
      }
      // The rescale runs warp-collective tcgen05.ld/st, so the decision is
      // per warp: when any row of the warp needs it, every row of the warp
      // moves to its own new maximum (alpha = 1 for rows whose max held).
      if (j == 0) {
        m = mt;
      } else if (__any_sync(0xffffffffu, mt > m + kRescaleLog2)) {
        // O holds PV of tiles < j at the old max: rescale it once PV_{j-1} is done
        const float m_new = fmaxf(m, mt);
        const float alpha = exp2f(m - m_new);
        mt = m_new;
        const int pb = (j - 1) & 1;
        if (ok) ok = mbar_wait(&o_ready[pb], ((j - 1) >> 1) & 1, err, kDevTimeoutAccFull);
        ok = __all_sync(0xffffffffu, ok);
        tc_fence_after();
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(tO + lane_off + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st_32x32b_x32(tO + lane_off + c * 32, o);
        }
        tmem_st_wait();
        l *= alpha;
        m = mt;
      }
      // P buffer bb was last read by PV_{j-2}
      if (j >= 2 && ok) ok = mbar_wait(&o_ready[bb], ((j - 2) >> 1) & 1, err, kDevTimeoutAccFull);
      uint8_t* pbuf = smem + FL::kP + bb * 32768;
      float psum = 0.0f;
#pragma unroll
      for (int c16 = 0; c16 < 16; ++c16) {  // 16 chunks of 8 keys
        uint32_t packed[4];
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) {
          const int k0 = c16 * 8 + e2 * 2;
          const float p0 = exp2f(__uint_as_float(r[k0 >> 5][k0 & 31]) - m);
          const float p1 = exp2f(__uint_as_float(r[(k0 + 1) >> 5][(k0 + 1) & 31]) - m);
          psum += p0 + p1;
          const __half2 hv = __floats2half2_rn(p0 * sv_s[bb * 128 + k0], p1 * sv_s[bb * 128 + k0 + 1]);
          packed[e2] = *reinterpret_cast<const uint32_t*>(&hv);
        }
        *reinterpret_cast<uint4*>(pbuf + p_offset(t, c16)) =
            make_uint4(packed[0], packed[1], packed[2], packed[3]);
      }
      l += psum;
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[bb]);
    }
    // ---------------- epilogue: out = O / l ----------------
    if (ok) ok = mbar_wait(&o_ready[(n - 1) & 1], ((n - 1) >> 1) & 1, err, kDevTimeoutAccFull);
    ok = __all_sync(0xffffffffu, ok);
    tc_fence_after();
    const float inv = 1.0f / l;
    float* orow = a.out + (static_cast<long long>(b) * S + row) * a.out_ld + h * kHeadDim;
#pragma unroll 1
    for (int c = 0; c < 4; ++c) {
      uint32_t o[32];
      tmem_ld_32x32b_x32(tO + lane_off + c * 32, o);
      tmem_ld_wait();
      if (row_ok) {
#pragma unroll
        for (int e = 0; e < 32; e += 4)
          *reinterpret_cast<float4*>(orow + c * 32 + e) =
              make_float4(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv,
                          __uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
      }
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
// forward so the per-element RoPE is two table loads.
__global__ void rope_table_kernel(int seq, float base, float2* __restrict__ table) {
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= seq * 64) return;
  const int pos = idx >> 6, i = idx & 63;
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
      const float2 t = __ldg(table + pos * 64 + i);
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
// CTA = 32 tokens x 1 kv head (128 threads).  v8 [T][Hkv*128] token-major (the
// int8 cache rows) and vs [B][Hkv][S]; vt [B][Hkv][128][S] f16 holds the same
// int8 codes (exact in f16), transposed so the P.V MMA reads it K-major.
__global__ void v_quant_kernel(int tokens, int seq, int hq, int hkv, const float* __restrict__ qkv,
                               int8_t* __restrict__ v8, float* __restrict__ vs,
                               __half* __restrict__ vt) {
  __shared__ int8_t tile[32][kHeadDim + 4];
  const int kh = blockIdx.y;
  const int tok0 = blockIdx.x * 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int width = (hq + 2 * hkv) * kHeadDim;
  for (int tt = warp; tt < 32; tt += 4) {
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
      tile[tt][lane + 32 * p] = static_cast<int8_t>(c);
    }
  }
  __syncthreads();
  // transposed write: vt[b][kh][d][pos], 32 consecutive positions per d
  for (int d = warp; d < kHeadDim; d += 4) {
    const int tok = tok0 + lane;
    if (tok < tokens) {
      const int pos = tok % seq, bidx = tok / seq;
      vt[((static_cast<long long>(bidx) * hkv + kh) * kHeadDim + d) * seq + pos] =
          __int2half_rn(tile[lane][d]);
    }
  }
}

}  // namespace

int flash_prefill_i8(const FlashProblem& p, cudaStream_t stream) {
  if (p.batch <= 0 || p.heads_q <= 0 || p.heads_kv <= 0 || p.seq <= 0) return kErrInvalid;
  if (p.head_dim != kHeadDim || p.heads_q % p.heads_kv != 0) return kErrInvalid;
  if (p.seq % 8 != 0) return kErrAlignment;  // V^T rows must be 16-byte strided
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
  a.v_scale = p.v_scale;
  a.out = p.out;
  a.out_ld = p.out_ld;
  a.err = device_error_ptr();
  const int grid = ((p.seq + kTile - 1) / kTile) * p.batch * p.heads_q;
  flash_prefill_kernel<<<grid, kFThreads, FL::kAlloc, stream>>>(mq, mk, mv, a);
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
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
  dim3 grid(static_cast<unsigned>((tokens + 31) / 32), static_cast<unsigned>(heads_kv));
  v_quant_kernel<<<grid, 128, 0, stream>>>(tokens, seq, heads_q, heads_kv, qkv, v8, v_scale,
                                           static_cast<__half*>(vt));
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

}  // namespace reef
