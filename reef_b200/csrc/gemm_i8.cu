// gemm_i8.cu -- int8 x int8 -> int32 GEMM on sm_100a tensor cores
// (tcgen05.mma kind::i8) with fused requantisation epilogues.
//
//   D[m][n] = sum_k A[m][k] * B[n][k]       A: [M][lda] int8, B: [N][ldb] int8
//
// Both operands are K-major, which is the engine's own layout: activations
// are rows of in_features, weights are QuantizedWeight [out][in]
// (quant.hpp:38-43 of reef's inference engine).  Integer sums are
// order-free, so the accumulation order of the tensor cores gives exactly the
// sums of matmul<int8,int32> (tensor.hpp:178-246).
//
// Epilogues (all read the int32 accumulator from TMEM):
//   kF32W8A8  y = float(acc) * (x_scale[m] * w_scale[n])  [+ bias[n]]
//             -- linear() W8A8, operator/linear.hpp:122-130, each step a
//                single round-to-nearest IEEE operation (__fmul_rn/__fadd_rn).
//   kI8Shift  y = sat8(rounding_shift(acc [+ bias32[n]], shift))
//             -- linear_int8, int8.hpp:74-101.
//   kI32      y = acc   (the raw partial sums of a row-parallel shard)
//   kQkvRope  the kF32W8A8 values of a QKV projection, then per (token,
//             head) in the epilogue: rotate-half RoPE on q / k heads and
//             reef's int8 quantiser (quant.hpp:51-81) -> q8 / k8 / v8 rows,
//             their scales, and the f16 V^T copy the flash head reads.  A
//             BN = 256 tile is two whole heads; each epilogue thread holds one
//             token's 128 values of a head (TMEM lane = token).
//   kSwiGLU   y = silu(g) * u, g / u the kF32W8A8 values of the gate / up
//             weight rows n and b_up + n: each B stage holds BN/2 gate rows
//             and the BN/2 matching up rows (two TMA boxes), so one tile
//             yields BN/2 outputs; the row maxima of |y| go to row_max by
//             atomic max (the scale of the int8 activation that follows).
//
// Kernel structure (one CTA per SM, persistent over output tiles):
//   warp 0      TMA producer: 128 x 128-byte A tile and BN x 128-byte B tile
//               per stage, 128-byte swizzle, STAGES-deep mbarrier ring.
//   warp 1      allocates TMEM; one elected thread issues tcgen05.mma
//               (128 x BN x 32 per instruction, 4 per stage) into one of two
//               TMEM accumulators, commits stage frees and accumulator-ready
//               to mbarriers.
//   warps 2..5  epilogue: tcgen05.ld of the accumulator (warp w reads TMEM
//               lanes 32*(w%4)...), requantise, transpose through shared
//               memory so each store instruction writes contiguous bytes of
//               one output row, then release the accumulator.
// Double-buffered accumulators let the epilogue of tile i overlap the MMAs of
// tile i+1.  No TMA multicast anywhere.
#include "common.cuh"
#include "exact_math.cuh"
#include "ops.h"

#include <cuda_fp16.h>

#include <algorithm>
#include <cstdlib>

namespace reef {

namespace {

constexpr int kBM = 128;         // UMMA M (TMEM lanes)
constexpr int kBK = 128;         // bytes of K per stage (one 128-byte swizzle row)
constexpr int kUmmaK = 32;       // K per tcgen05.mma kind::i8
constexpr int kThreads = 192;    // 6 warps
constexpr int kEpiWarps = 4;
// The QKV epilogue runs 8 warps: warps 2..5 take the tile's first head,
// warps 6..9 its second (two warps per TMEM lane quadrant).
template <int EPI>
__host__ __device__ constexpr int epi_warps() { return EPI == kEpiQkvRope ? 8 : kEpiWarps; }
template <int EPI>
__host__ __device__ constexpr int threads_for() { return 64 + 32 * epi_warps<EPI>(); }
constexpr int kTransposeWords = 32 * 36;  // per epilogue warp

template <int BN, int STAGES>
struct Layout {
  static constexpr int kABytes = kBM * kBK;
  static constexpr int kBBytes = BN * kBK;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kTransposeOff = STAGES * kStageBytes;
  static constexpr int kRowScaleOff = kTransposeOff + kEpiWarps * kTransposeWords * 4;
  static constexpr int kBarOff = kRowScaleOff + kEpiWarps * 32 * 4;
  // full[STAGES], empty[STAGES], acc_full[2], acc_empty[2], drain
  static constexpr int kNumBars = 2 * STAGES + 5;
  static constexpr int kTmemSlotOff = kBarOff + kNumBars * 8;
  static constexpr int kBytes = kTmemSlotOff + 16;
  static constexpr int kAlloc = kBytes + 1024;  // slack to align the base
  static_assert(kAlloc <= 232448, "shared memory budget");
  static_assert((kStageBytes % 1024) == 0, "stages stay 1024-byte aligned");
};

__device__ __forceinline__ void tile_coords(int t, int num_m, int num_n, int group,
                                            int& mb, int& nb) {
  // Grouped raster: `group` m-blocks walk the n-blocks together, so the CTAs
  // in flight share B tiles (weights) and A tiles in L2.
  const int per_group = group * num_n;
  const int g = t / per_group;
  const int first_m = g * group;
  const int gsize = min(group, num_m - first_m);
  const int r = t - g * per_group;
  mb = first_m + r % gsize;
  nb = r / gsize;
}

// One unit of a CTA's work: k-blocks [kb0, kb1) of output tile (mb, nb),
// written to partial slot `slot` (its K split).
struct Item {
  int mb, nb, kb0, kb1, slot;
};

// The CTA's idx-th item, or false when it has no more: (tile, split) items
// dealt round-robin over the persistent grid; split s of `splits` takes
// k-blocks [s nk / splits, (s + 1) nk / splits).  (A stream-K cut -- every
// CTA an equal range of the tiles' k-blocks, crossing tile boundaries --
// measured slower for the decode GEMMs: a CTA's second piece adds a whole
// item's epilogue and hand-off at the end.)
__device__ __forceinline__ bool get_item(const GemmArgs& args, int num_m, int num_n, int num_k,
                                         int splits, int idx, Item& it) {
  const int t = static_cast<int>(blockIdx.x) + idx * static_cast<int>(gridDim.x);
  if (t >= num_m * num_n * splits) return false;
  tile_coords(t / splits, num_m, num_n, args.group_m, it.mb, it.nb);
  const int split = t % splits;
  it.kb0 = split * num_k / splits;
  it.kb1 = (split + 1) * num_k / splits;
  it.slot = split;
  return true;
}

template <int BN, int STAGES, int EPI>
__global__ void __launch_bounds__(threads_for<EPI>(), 1)
    gemm_i8_kernel(const __grid_constant__ CUtensorMap tma_a,
                   const __grid_constant__ CUtensorMap tma_b, GemmArgs args) {
  using L = Layout<BN, STAGES>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  uint64_t* acc_full = bars + 2 * STAGES;
  uint64_t* acc_empty = bars + 2 * STAGES + 2;
  uint64_t* drain = bars + 2 * STAGES + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + L::kTmemSlotOff);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int M = args.M, N = args.N, K = args.K;
  constexpr int kOut = EPI == kEpiSwiGLU ? BN / 2 : BN;  // output columns per tile
  const int num_m = (M + kBM - 1) / kBM;
  const int num_n = (N + kOut - 1) / kOut;
  // K may come in `segs` equal segments read through 3-D tensor maps (an
  // all-gathered activation is rank-major [segs][rows][K]); k-block kb is
  // block kb % kbs of segment kb / kbs.  One segment for plain row-major.
  const int segs = args.k_segments > 1 ? args.k_segments : 1;
  const int kbs = (K + kBK - 1) / kBK;
  const int num_k = kbs * segs;
  const int splits = args.k_splits > 1 ? args.k_splits : 1;
  int* err = args.err;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tma_a);
    prefetch_tensormap(&tma_b);
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], epi_warps<EPI>() * 32);
    }
    mbar_init(drain, 1);
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 2 * BN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      long long issued = 0;
      bool ok = true;
      // When A depends on no earlier kernel (the weights of a swap-AB skinny
      // GEMM), the first item's leading k-blocks of A are requested before
      // waiting for the kernel before this one (a programmatic dependent
      // launch lets the two overlap); their B halves follow the wait.  The
      // ring is fresh, so those stages need no "empty" wait.
      int pre = 0;
      Item first;
      if (args.a_first && get_item(args, num_m, num_n, num_k, splits, 0, first)) {
        const int mb = first.mb, kb0 = first.kb0;
        pre = min(STAGES, first.kb1 - kb0);
        for (int i = 0; i < pre; ++i) {
          const int kb = kb0 + i, seg = kb / kbs, kx = (kb - seg * kbs) * kBK;
          mbar_arrive_expect_tx(&full[i], L::kStageBytes);
          if (args.a_tiles != nullptr)
            bulk_load(smem + i * L::kStageBytes,
                      args.a_tiles + (static_cast<long long>(mb) * kbs + kb) * L::kABytes,
                      L::kABytes, &full[i]);
          else
            tma_load_3d(smem + i * L::kStageBytes, &tma_a, &full[i], kx, mb * kBM, seg);
        }
      }
      pdl_wait();
      // a programmatic dependent may be scheduled now; it waits for this
      // grid's completion and memory before reading the outputs
      pdl_trigger();
      Item it;
      for (int idx = 0; ok && get_item(args, num_m, num_n, num_k, splits, idx, it); ++idx) {
        const int mb = it.mb, nb = it.nb, kb0 = it.kb0, kb1 = it.kb1;
        for (int kb = kb0; kb < kb1; ++kb) {
          const bool prefetched = idx == 0 && kb - kb0 < pre;
          if (!prefetched && !mbar_wait(&empty[stage], phase ^ 1u, err, kDevTimeoutEmpty)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + stage * L::kStageBytes;
          uint8_t* sb = sa + L::kABytes;
          const int seg = kb / kbs, kx = (kb - seg * kbs) * kBK;
          if (!prefetched) {
            mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
            if (args.a_tiles != nullptr)
              bulk_load(sa, args.a_tiles + (static_cast<long long>(mb) * kbs + kb) * L::kABytes,
                        L::kABytes, &full[stage]);
            else
              tma_load_3d(sa, &tma_a, &full[stage], kx, mb * kBM, seg);
          }
          if constexpr (EPI == kEpiSwiGLU) {
            tma_load_3d(sb, &tma_b, &full[stage], kx, nb * kOut, seg);
            tma_load_3d(sb + kOut * kBK, &tma_b, &full[stage], kx,
                        static_cast<int>(args.b_up) + nb * kOut, seg);
          } else {
            tma_load_3d(sb, &tma_b, &full[stage], kx, nb * BN, seg);
          }
          ++issued;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      // Copies still in flight land before the CTA may exit: wait (bounded)
      // for the last load issued into each stage.
      const long long tail = issued < STAGES ? issued : STAGES;
      for (long long i = 0; i < tail; ++i) {
        // walk back from the most recent issue
        int s = stage - 1 - static_cast<int>(i);
        uint32_t ph = phase;
        while (s < 0) {
          s += STAGES;
          ph ^= 1u;
        }
        mbar_wait(&full[s], ph, err, kDevTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      constexpr uint32_t kIdesc = idesc_i8(kBM, BN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      Item it;
      for (int idx = 0; ok && get_item(args, num_m, num_n, num_k, splits, idx, it); ++idx) {
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1u, err, kDevTimeoutAccEmpty)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + static_cast<uint32_t>(acc * BN);
        const int kb0 = it.kb0, kb1 = it.kb1;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, err, kDevTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + stage * L::kStageBytes);
          const uint32_t sb = sa + L::kABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / kUmmaK; ++kk) {
            mma_i8(d_tmem, smem_desc_k_sw128(sa + kk * kUmmaK),
                   smem_desc_k_sw128(sb + kk * kUmmaK), kIdesc,
                   (kb > kb0 || kk != 0) ? 1u : 0u);
          }
          mma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        mma_commit(&acc_full[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
      }
      // Every MMA issued by this thread completes before TMEM is released.
      mma_commit(drain);
      mbar_wait(drain, 0, err, kDevTimeoutDrain);
    }
  } else {
    // ---------------- epilogue ----------------
    // Per 32-column chunk: tcgen05.ld gives thread `lane` row (row0 + lane);
    // the raw int32 values go through this warp's shared-memory buffer
    // (row stride 36 words: 16-byte accesses are bank-conflict free both
    // ways), then each thread requantises 4 consecutive columns of 8 rows,
    // so a store instruction writes 4 rows x 32 contiguous columns and the
    // per-column scale / bias are loaded once per chunk.
    // the epilogue reads scales and residuals and writes outputs that the
    // kernel before this one may touch
    pdl_wait();
    const int q = warp & 3;  // TMEM lane quadrant this warp may read
    uint32_t* tbuf = reinterpret_cast<uint32_t*>(smem + L::kTransposeOff) +
                     (warp - 2) * kTransposeWords;
    float* rs_s = reinterpret_cast<float*>(smem + L::kRowScaleOff) + (warp - 2) * 32;
    const int sub_row = lane >> 3;       // 0..3
    const int sub_col = (lane & 7) * 4;  // 0, 4, ..., 28
    int acc = 0;
    uint32_t acc_phase = 0;
    Item it;
    for (int idx = 0; get_item(args, num_m, num_n, num_k, splits, idx, it); ++idx) {
      const int mb = it.mb, nb = it.nb;
      // K-split partial outputs land in their own slice of y
      const long long y_off = static_cast<long long>(it.slot) * args.split_stride;
      // warp-uniform outcome: the tcgen05.ld below is warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait(&acc_full[acc], acc_phase, err, kDevTimeoutAccFull)))
        break;
      tc_fence_after();
      const int row0 = mb * kBM + q * 32;  // first output row of this warp
      if constexpr (EPI == kEpiF32W8A8 || EPI == kEpiSwiGLU) {
        const int my_row = row0 + lane;
        rs_s[lane] = my_row < M ? args.x_scale[my_row] : 0.0f;
      }
      if constexpr (EPI == kEpiQkvRope) {
        // One head (128 columns) of the tile per warp, 32 tokens (its TMEM
        // lane quadrant): pass 1 dequantises, rotates and takes max |x|,
        // writing the values back over the accumulator columns; pass 2 reads
        // them again to quantise and store.
        const QkvOut& qo = args.qkv;
        const int hl = (warp - 2) >> 2;
        const int hh = nb * (BN / 128) + hl;
        const int heads = qo.heads_q + 2 * qo.heads_kv;
        const int m = row0 + lane;  // this thread's token
        const bool mok = m < M;
        if (hh < heads) {  // warp-uniform
          const int pos = mok ? m % qo.seq : 0, bidx = mok ? m / qo.seq : 0;
          const float rsv = mok ? args.x_scale[m] : 0.0f;
          float* wsb = reinterpret_cast<float*>(smem + L::kTransposeOff) + (warp - 2) * 128;
#pragma unroll
          for (int i = 0; i < 4; ++i) wsb[lane + 32 * i] = args.w_scale[hh * 128 + lane + 32 * i];
          __syncwarp();
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                 static_cast<uint32_t>(acc * BN + hl * 128);
          const bool rope = hh < qo.heads_q + qo.heads_kv;
          // i-major table: a warp's consecutive tokens read one run per i
          const float2* tr = qo.rope + pos;
          float mx0 = 0.0f, mx1 = 0.0f;
#pragma unroll 1
          for (int h = 0; h < 2; ++h) {  // columns [32h, 32h+32) and [64+32h, 96+32h)
            uint32_t lo[32], hi[32];
            tmem_ld_32x32b_x32(taddr + h * 32, lo);
            tmem_ld_32x32b_x32(taddr + 64 + h * 32, hi);
            tmem_ld_wait();
#pragma unroll
            for (int k0 = 0; k0 < 32; k0 += 16) {
              float2 cs[16];
              if (rope) {
#pragma unroll
                for (int k = 0; k < 16; ++k)
                  cs[k] = __ldg(tr + static_cast<long long>(h * 32 + k0 + k) * qo.seq);
              }
              // linear.hpp:125-127: float(sum) * (row_scale * w_scale[c])
#pragma unroll
              for (int k = 0; k < 16; ++k) {
                const int kk = k0 + k;
                float a = __fmul_rn(__int2float_rn(static_cast<int32_t>(lo[kk])),
                                    __fmul_rn(rsv, wsb[h * 32 + kk]));
                float b = __fmul_rn(__int2float_rn(static_cast<int32_t>(hi[kk])),
                                    __fmul_rn(rsv, wsb[64 + h * 32 + kk]));
                if (rope) {
                  // rotate-half RoPE, pair (i, i + 64): the packing kernel's expressions
                  const float a2 = a * cs[k].x - b * cs[k].y;
                  b = b * cs[k].x + a * cs[k].y;
                  a = a2;
                }
                mx0 = fmaxf(mx0, fabsf(a));
                mx1 = fmaxf(mx1, fabsf(b));
                lo[kk] = __float_as_uint(a);
                hi[kk] = __float_as_uint(b);
              }
            }
            tmem_st_32x32b_x32(taddr + h * 32, lo);
            tmem_st_32x32b_x32(taddr + 64 + h * 32, hi);
          }
          tmem_st_wait();
          const float mx = fmaxf(mx0, mx1);
          const float scale = mx > 0.0f ? __fdiv_rn(mx, 127.0f) : 1.0f;
          const float rcp = __frcp_rn(scale);
          int8_t* dst = nullptr;
          float* sdst = nullptr;
          const bool is_v = !rope;
          const int kh = hh - qo.heads_q - (is_v ? qo.heads_kv : 0);
          if (hh < qo.heads_q) {
            dst = qo.q8 + static_cast<long long>(m) * qo.heads_q * 128 + hh * 128;
            sdst = qo.qs + (static_cast<long long>(bidx) * qo.heads_q + hh) * qo.seq + pos;
          } else if (!is_v) {
            dst = qo.k8 + static_cast<long long>(m) * qo.heads_kv * 128 + kh * 128;
            sdst = qo.ks + (static_cast<long long>(bidx) * qo.heads_kv + kh) * qo.seq + pos;
          } else {
            if (qo.v8 != nullptr) dst = qo.v8 + static_cast<long long>(m) * qo.heads_kv * 128 + kh * 128;
            if (qo.vs != nullptr)
              sdst = qo.vs + (static_cast<long long>(bidx) * qo.heads_kv + kh) * qo.seq + pos;
          }
          if (mok && sdst != nullptr) *sdst = scale;
          __half* vt = is_v ? static_cast<__half*>(qo.vt) +
                                  (static_cast<long long>(bidx) * qo.heads_kv + kh) * 128 * qo.seq + pos
                            : nullptr;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            uint32_t v[32];
            tmem_ld_32x32b_x32(taddr + c * 32, v);
            tmem_ld_wait();
            // reef's code rint(x / scale), clamped: fast by the reciprocal,
            // the division only for chunks holding a near-tie (see quant_code)
            bool exact = false;
            int code[32];
#pragma unroll
            for (int k = 0; k < 32; ++k) {
              const float x = __uint_as_float(v[k]);
              const float qf = __fmul_rn(x, rcp);
              const float r = rintf(qf);
              exact |= !(fabsf(qf) < 128.0f && fabsf(qf - r) < 0.49993896f);
              code[k] = __float2int_rn(r);
            }
            if (__any_sync(0xffffffffu, exact)) {
#pragma unroll
              for (int k = 0; k < 32; ++k)
                code[k] = __float2int_rn(__fdiv_rn(__uint_as_float(v[k]), scale));
            }
#pragma unroll
            for (int k = 0; k < 32; ++k) code[k] = code[k] < -127 ? -127 : (code[k] > 127 ? 127 : code[k]);
            if (mok) {
              if (dst != nullptr) {
                uint32_t pk[8];
#pragma unroll
                for (int w = 0; w < 8; ++w)
                  pk[w] = (code[4 * w] & 0xff) | ((code[4 * w + 1] & 0xff) << 8) |
                          ((code[4 * w + 2] & 0xff) << 16) |
                          (static_cast<uint32_t>(code[4 * w + 3] & 0xff) << 24);
                *reinterpret_cast<uint4*>(dst + c * 32) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                *reinterpret_cast<uint4*>(dst + c * 32 + 16) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
              }
              if (is_v) {
                // vt[b][kh][d][pos] = f16(code * scale): a warp's 32 tokens are
                // consecutive positions, so each d is one contiguous run
#pragma unroll
                for (int k = 0; k < 32; ++k)
                  vt[static_cast<long long>(c * 32 + k) * qo.seq] =
                      __float2half_rn(__fmul_rn(static_cast<float>(code[k]), scale));
              }
            }
          }
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
        continue;
      }
      if constexpr (EPI == kEpiSwiGLU) {
        // gate chunk c and up chunk c (accumulator columns c*32 and BN/2 + c*32)
        // each pass through the transpose buffer; thread (sub_row, sub_col)
        // then owns 4 columns of 8 rows of both
        float rmax[8];
#pragma unroll
        for (int it = 0; it < 8; ++it) rmax[it] = 0.0f;
#pragma unroll 1
        for (int c = 0; c < kOut / 32; ++c) {
          const int col0 = nb * kOut + c * 32;
          const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                 static_cast<uint32_t>(acc * BN + c * 32);
          uint32_t r[32];
          uint4 gv[8], uv[8];
          tmem_ld_32x32b_x32(taddr, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<uint4*>(&tbuf[lane * 36 + j]) =
                make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
          __syncwarp();
#pragma unroll
          for (int it = 0; it < 8; ++it)
            gv[it] = *reinterpret_cast<const uint4*>(&tbuf[(it * 4 + sub_row) * 36 + sub_col]);
          __syncwarp();
          tmem_ld_32x32b_x32(taddr + kOut, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<uint4*>(&tbuf[lane * 36 + j]) =
                make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
          __syncwarp();
#pragma unroll
          for (int it = 0; it < 8; ++it)
            uv[it] = *reinterpret_cast<const uint4*>(&tbuf[(it * 4 + sub_row) * 36 + sub_col]);
          __syncwarp();
          if (col0 >= N) continue;  // warp-uniform
          const int n = col0 + sub_col;
          float wg[4], wu[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int nn = n + e < N ? n + e : N - 1;
            wg[e] = args.w_scale[nn];
            wu[e] = args.w_scale[args.b_up + nn];
          }
          const bool full_vec = args.vec_ok && (n + 3 < N);
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int rl = it * 4 + sub_row;
            const int m = row0 + rl;
            if (m < M && n < N) {
              const float rsv = rs_s[rl];
              const uint32_t ga[4] = {gv[it].x, gv[it].y, gv[it].z, gv[it].w};
              const uint32_t ua[4] = {uv[it].x, uv[it].y, uv[it].z, uv[it].w};
              float o[4];
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                // the gate / up values of the unfused W8A8 linear, then SwiGLU
                const float g = __fmul_rn(__int2float_rn(static_cast<int32_t>(ga[e])),
                                          __fmul_rn(rsv, wg[e]));
                const float u = __fmul_rn(__int2float_rn(static_cast<int32_t>(ua[e])),
                                          __fmul_rn(rsv, wu[e]));
                o[e] = silu_mul(g, u);
              }
              float* y = static_cast<float*>(args.y) + static_cast<long long>(m) * args.ldy + n;
              if (full_vec) {
                *reinterpret_cast<float4*>(y) = make_float4(o[0], o[1], o[2], o[3]);
                rmax[it] = fmaxf(rmax[it], fmaxf(fmaxf(fabsf(o[0]), fabsf(o[1])),
                                                 fmaxf(fabsf(o[2]), fabsf(o[3]))));
              } else {
                for (int e = 0; e < 4 && n + e < N; ++e) {
                  y[e] = o[e];
                  rmax[it] = fmaxf(rmax[it], fabsf(o[e]));
                }
              }
            }
          }
        }
        // the 8 lanes of a sub-row hold its 32 columns: reduce, one atomic
        // per row (|y| >= 0, so the int order of the bits is the float order)
#pragma unroll
        for (int it = 0; it < 8; ++it) {
          float v = rmax[it];
          v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
          v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
          v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
          const int m = row0 + it * 4 + sub_row;
          if ((lane & 7) == 0 && m < M)
            atomicMax(reinterpret_cast<int*>(args.row_max) + m, __float_as_int(v));
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
        continue;
      }
      if constexpr (EPI == kEpiI32T) {
        // split-K partials of a swap-AB GEMM, token-major: y[split][n][m],
        // straight from the accumulator (lane = row m, so a token's 32 rows
        // are one contiguous 128-byte store)
        int32_t* yp = static_cast<int32_t*>(args.y) + y_off;
        const int m = row0 + lane;
#pragma unroll 1
        for (int c = 0; c < BN / 32; ++c) {
          const int col0 = nb * BN + c * 32;
          if (col0 >= N) break;  // warp-uniform
          uint32_t r[32];
          tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                                 static_cast<uint32_t>(acc * BN + c * 32),
                             r);
          tmem_ld_wait();
          if (m < M) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (col0 + j < N) yp[static_cast<long long>(col0 + j) * args.ldy + m] = static_cast<int32_t>(r[j]);
          }
        }
        tc_fence_before();
        mbar_arrive(&acc_empty[acc]);
        acc ^= 1;
        if (acc == 0) acc_phase ^= 1u;
        continue;
      }
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        const int col0 = nb * BN + c * 32;
        uint32_t r[32];
        tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(q * 32) << 16) +
                               static_cast<uint32_t>(acc * BN + c * 32),
                           r);
        tmem_ld_wait();
        if (col0 < N) {  // warp-uniform
#pragma unroll
          for (int j = 0; j < 32; j += 4)
            *reinterpret_cast<uint4*>(&tbuf[lane * 36 + j]) =
                make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
          __syncwarp();
          const int n = col0 + sub_col;
          float ws[4] = {0.f, 0.f, 0.f, 0.f}, bf[4] = {0.f, 0.f, 0.f, 0.f};
          int32_t bi[4] = {0, 0, 0, 0};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int nn = n + e < N ? n + e : N - 1;
            if constexpr (EPI == kEpiF32W8A8) {
              ws[e] = args.w_scale[nn];
              if (args.bias_f != nullptr) bf[e] = args.bias_f[nn];
            } else if constexpr (EPI == kEpiI8Shift) {
              if (args.bias_i != nullptr) bi[e] = args.bias_i[nn];
            }
          }
          const bool full_vec = args.vec_ok && (n + 3 < N);
          // The residual rows of this chunk are loaded before any store: y may
          // alias nothing, but the compiler cannot know, and loads ordered
          // behind stores would serialise on memory latency.
          float4 res[8];
          if constexpr (EPI == kEpiF32W8A8) {
            if (args.residual != nullptr) {
#pragma unroll
              for (int it = 0; it < 8; ++it) {
                const int m = row0 + it * 4 + sub_row;
                res[it] = make_float4(0.f, 0.f, 0.f, 0.f);
                if (m < M && n < N) {
                  const float* rp = args.residual + static_cast<long long>(m) * args.ldy + n;
                  if (full_vec) {
                    res[it] = __ldg(reinterpret_cast<const float4*>(rp));
                  } else {
                    float t4[4] = {0.f, 0.f, 0.f, 0.f};
                    for (int e = 0; e < 4 && n + e < N; ++e) t4[e] = __ldg(rp + e);
                    res[it] = make_float4(t4[0], t4[1], t4[2], t4[3]);
                  }
                }
              }
            }
          }
#pragma unroll
          for (int it = 0; it < 8; ++it) {
            const int rl = it * 4 + sub_row;
            const int m = row0 + rl;
            const uint4 a4 = *reinterpret_cast<const uint4*>(&tbuf[rl * 36 + sub_col]);
            if (m < M && n < N) {
              const uint32_t av[4] = {a4.x, a4.y, a4.z, a4.w};
              const long long off = static_cast<long long>(m) * args.ldy + n;
              if constexpr (EPI == kEpiF32W8A8) {
                const float rsv = rs_s[rl];
                float o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                  // linear.hpp:125-127: float(sum) * (row_scale * w_scale[c])
                  o[e] = __fmul_rn(__int2float_rn(static_cast<int32_t>(av[e])),
                                   __fmul_rn(rsv, ws[e]));
                  if (args.bias_f != nullptr) o[e] = __fadd_rn(o[e], bf[e]);
                  if (args.gelu) o[e] = gelu_dev(o[e]);  // MLP c_fc + gelu, mlp.hpp:108-133
                }
                if (args.residual != nullptr) {  // residual_add(input, sublayer), block.hpp:27-39
                  o[0] = __fadd_rn(res[it].x, o[0]);
                  o[1] = __fadd_rn(res[it].y, o[1]);
                  o[2] = __fadd_rn(res[it].z, o[2]);
                  o[3] = __fadd_rn(res[it].w, o[3]);
                }
                float* y = static_cast<float*>(args.y) + off;
                if (full_vec) {
                  *reinterpret_cast<float4*>(y) = make_float4(o[0], o[1], o[2], o[3]);
                } else {
                  for (int e = 0; e < 4 && n + e < N; ++e) y[e] = o[e];
                }
              } else if constexpr (EPI == kEpiI8Shift) {
                int8_t o[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  o[e] = requant_rnu_sat8(static_cast<int32_t>(av[e]) + bi[e], args.shift);
                int8_t* y = static_cast<int8_t*>(args.y) + off;
                if (full_vec) {
                  *reinterpret_cast<char4*>(y) = make_char4(o[0], o[1], o[2], o[3]);
                } else {
                  for (int e = 0; e < 4 && n + e < N; ++e) y[e] = o[e];
                }
              } else {
                int32_t* y = static_cast<int32_t*>(args.y) + y_off + off;
                if (full_vec) {
                  *reinterpret_cast<uint4*>(y) = a4;
                } else {
                  for (int e = 0; e < 4 && n + e < N; ++e) y[e] = static_cast<int32_t>(av[e]);
                }
              }
            }
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[acc]);
      acc ^= 1;
      if (acc == 0) acc_phase ^= 1u;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * BN);
  }
}

// M-blocks per raster group when the caller leaves it open.  A group walks
// all n-blocks together, so B is streamed from DRAM once per group while
// the group's A rows stay in L2.
// * B small enough to stay in L2 beside the streaming A and outputs (at most
//   44 MiB: config 3's o-proj and down weights): group 1, every n-block of
//   one m-block before the next, so B is read from DRAM once and A once (the
//   down projection read B eight times over with group 16).
// * Else the largest power of two from 8 to 64 whose A rows (group x 128 x K
//   bytes) fit in 32 MiB: B is read M / (128 group) times.  Measured on
//   config 3 under the power cap: group 8 -> 64 takes the gate/up GEMM (B
//   90 MB) from 1.09 to 1.00 ms.
// REEF_B200_GEMM_GROUP fixes it instead.
int default_group_m(long long K, long long b_bytes) {
  static int fixed = -1;
  if (fixed < 0) {
    int x = 0;
    if (const char* e = std::getenv("REEF_B200_GEMM_GROUP")) {
      const int y = std::atoi(e);
      if (y >= 1 && y <= 1024) x = y;
    }
    fixed = x;
  }
  if (fixed > 0) return fixed;
  if (b_bytes <= (44ll << 20)) return 1;
  int g = 64;
  while (g > 8 && static_cast<long long>(g) * kBM * K > (32ll << 20)) g /= 2;
  return g;
}

template <int BN, int STAGES, int EPI>
int launch(const GemmProblem& p, cudaStream_t stream) {
  using L = Layout<BN, STAGES>;
  CUtensorMap ma, mb;
  const int segs = p.args.k_segments > 1 ? p.args.k_segments : 1;
  int rc = make_tma_3d_i8(&ma, p.a, p.M, p.K, p.lda, segs, p.a_seg, kBK, kBM);
  if (rc) return rc;
  if constexpr (EPI == kEpiSwiGLU) {
    rc = make_tma_3d_i8(&mb, p.b, p.args.b_up + p.N, p.K, p.ldb, segs, p.b_seg, kBK, BN / 2);
  } else {
    rc = make_tma_3d_i8(&mb, p.b, p.N, p.K, p.ldb, segs, p.b_seg, kBK, BN);
  }
  if (rc) return rc;
  auto kernel = gemm_i8_kernel<BN, STAGES, EPI>;
  static bool configured[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !configured[dev]) {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             L::kAlloc) != cudaSuccess)
      return kErrCuda;
    configured[dev] = true;
  }
  constexpr int kOut = EPI == kEpiSwiGLU ? BN / 2 : BN;
  const int num_tiles = ((p.M + kBM - 1) / kBM) * ((p.N + kOut - 1) / kOut);
  const int splits = p.args.k_splits > 1 ? p.args.k_splits : 1;
  const int ctas = p.args.max_ctas > 0 ? std::min(p.args.max_ctas, num_sms()) : num_sms();
  const int grid = std::min(num_tiles * splits, ctas);
  GemmArgs args = p.args;
  args.M = p.M;
  args.N = p.N;
  args.K = p.K;
  // A's K spans every segment of an all-gathered operand
  if (args.group_m <= 0) {
    const long long k_all = static_cast<long long>(p.K) * std::max(1, p.args.k_segments);
    const long long b_rows = EPI == kEpiSwiGLU ? p.args.b_up + p.N : p.N;
    args.group_m = default_group_m(k_all, b_rows * k_all);
  }
  args.err = device_error_ptr();
  // gelu is an option of the fp32 epilogue of whole (unsplit) outputs only
  if (args.gelu && (EPI != kEpiF32W8A8 || splits > 1)) return kErrInvalid;
  {
    const uintptr_t y = reinterpret_cast<uintptr_t>(args.y);
    const int align = EPI == kEpiI8Shift ? 4 : 16;
    const uintptr_t r = reinterpret_cast<uintptr_t>(args.residual);
    args.vec_ok = (y % align == 0) && (r % 16 == 0) && (args.ldy % 4 == 0) ? 1 : 0;
  }
  return launch_k(kernel, dim3(static_cast<unsigned>(grid)), dim3(threads_for<EPI>()), L::kAlloc,
                  stream, ma, mb, args);
}

// Sums the K-split partials part[s][m][n] (token-major, m * n apart) and
// applies the epilogue: y[m][n].  kVec: four consecutive outputs per thread
// (n % 4 == 0), else one.  Launched as a programmatic dependent of the GEMM
// that writes the partials.
template <int EPI, bool kVec>
__global__ void __launch_bounds__(256)
    skinny_reduce_kernel(int splits, int M, int N, const int32_t* __restrict__ part,
                         const float* __restrict__ xs, const float* __restrict__ ws,
                         const float* __restrict__ bias, const float* __restrict__ residual,
                         void* __restrict__ y) {
  pdl_wait();
  pdl_trigger();
  const long long total = static_cast<long long>(M) * N;
  constexpr int V = kVec ? 4 : 1;
  const long long i = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * V;
  if (i >= total) return;
  int32_t a[V];
  if constexpr (kVec) {
    int4 v = *reinterpret_cast<const int4*>(part + i);
    for (int s = 1; s < splits; ++s) {
      const int4 w = *reinterpret_cast<const int4*>(part + static_cast<long long>(s) * total + i);
      v.x += w.x;
      v.y += w.y;
      v.z += w.z;
      v.w += w.w;
    }
    a[0] = v.x;
    a[1] = v.y;
    a[2] = v.z;
    a[3] = v.w;
  } else {
    int32_t v = part[i];
    for (int s = 1; s < splits; ++s) v += part[static_cast<long long>(s) * total + i];
    a[0] = v;
  }
  const int m = static_cast<int>(i / N), n = static_cast<int>(i % N);
  if constexpr (EPI == kEpiF32W8A8) {
    const float rs = xs[m];
    float o[V];
#pragma unroll
    for (int e = 0; e < V; ++e) {
      // linear.hpp:125-127: float(sum) * (row_scale * w_scale[c]), then + bias
      o[e] = __fmul_rn(__int2float_rn(a[e]), __fmul_rn(rs, ws[n + e]));
      if (bias != nullptr) o[e] = __fadd_rn(o[e], bias[n + e]);
      if (residual != nullptr) o[e] = __fadd_rn(residual[i + e], o[e]);
    }
    if constexpr (kVec)
      *reinterpret_cast<float4*>(static_cast<float*>(y) + i) = make_float4(o[0], o[1], o[2], o[3]);
    else
      static_cast<float*>(y)[i] = o[0];
  } else {
    if constexpr (kVec)
      *reinterpret_cast<int4*>(static_cast<int32_t*>(y) + i) = make_int4(a[0], a[1], a[2], a[3]);
    else
      static_cast<int32_t*>(y)[i] = a[0];
  }
}

// K splits for the skinny GEMM.  When the tiles fit on the SMs, split K so
// that tiles x splits fills one wave without passing the SM count (at least
// two k-blocks per split): a second, partial wave gives some CTAs two items,
// and measured slower than one wave even with more, shorter items.  When
// there are more tiles than SMs (a wide weight), the persistent grid deals
// (tile, split) items round-robin, so the slowest CTA runs ceil(items / SMs)
// items of ceil(k-blocks / splits) blocks (+1 for the per-item hand-off),
// and the partials add splits * m * 4 bytes per weight row against k bytes of
// weights: take the split count (<= 16) that minimises that product.
int skinny_splits(int m, int n, int k) {
  const int tiles = (n + kBM - 1) / kBM;
  const int nk = (k + kBK - 1) / kBK;
  const int sms = num_sms();
  if (tiles <= sms) return std::max(1, std::min(sms / tiles, std::max(1, nk / 2)));
  int best = 1;
  double best_cost = 0.0;
  for (int s = 1; s <= 16; ++s) {
    if (s > 1 && nk / s < 2) break;
    const long long items = static_cast<long long>(tiles) * s;
    const long long waves = (items + sms - 1) / sms;
    const double cost = static_cast<double>(waves) * ((nk + s - 1) / s + 1) *
                        (1.0 + 4.0 * s * m / static_cast<double>(k));
    if (s == 1 || cost < best_cost * (1.0 - 1e-9)) {
      best = s;
      best_cost = cost;
    }
  }
  return best;
}

}  // namespace

size_t skinny_partial_bytes(int m, int n, int k) {
  return static_cast<size_t>(skinny_splits(m, n, k)) * n * m * sizeof(int32_t);
}

int skinny_split_count(int m, int n, int k) { return skinny_splits(m, n, k); }

int gemm_i8_skinny_partials(int m, int n, int k, const int8_t* x, const int8_t* w,
                            int32_t* part, cudaStream_t stream, const int8_t* w_tiles) {
  if (m <= 0 || n <= 0 || k <= 0 || m > 128 || part == nullptr || x == nullptr || w == nullptr)
    return kErrInvalid;
  if (w_tiles != nullptr && (reinterpret_cast<uintptr_t>(w_tiles) & 1023u) != 0)
    return kErrAlignment;  // the swizzle pattern repeats every 1024 bytes
  const int splits = skinny_splits(m, n, k);
  GemmProblem p{};
  p.M = n;  // weight rows on the MMA's M side (swap-AB)
  p.N = m;  // tokens on its N side
  p.K = k;
  p.a = w;
  p.lda = static_cast<long long>(kpad(k));
  p.b = x;
  p.ldb = static_cast<long long>(kpad(k));
  p.args.k_splits = splits;
  p.args.split_stride = static_cast<long long>(n) * m;
  p.args.y = part;
  p.args.ldy = n;
  p.args.a_first = 1;  // the weights: no earlier kernel writes them
  p.args.a_tiles = w_tiles;
  return m <= 64 ? launch<64, 8, kEpiI32T>(p, stream) : launch<128, 6, kEpiI32T>(p, stream);
}

namespace {
// One thread per 16-byte chunk of the tiled layout (see ops.h).
__global__ void pack_weight_tiles_kernel(long long rows, long long in, const int8_t* __restrict__ w,
                                         long long ldw, int kb_count, long long chunks,
                                         uint4* __restrict__ tiles) {
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= chunks) return;
  const long long tile = i >> 10;        // 1024 chunks of 16 bytes per tile
  const int r = static_cast<int>((i >> 3) & 127), cp = static_cast<int>(i & 7);
  const int c = cp ^ (r & 7);            // the logical chunk stored at this position
  const long long rb = tile / kb_count, kb = tile - rb * kb_count;
  const long long row = rb * kBM + r, col = kb * kBK + c * 16;
  uint8_t b[16];
#pragma unroll
  for (int j = 0; j < 16; ++j)
    b[j] = (row < rows && col + j < in) ? static_cast<uint8_t>(w[row * ldw + col + j]) : 0;
  uint4 v;
  v.x = b[0] | (b[1] << 8) | (b[2] << 16) | (static_cast<uint32_t>(b[3]) << 24);
  v.y = b[4] | (b[5] << 8) | (b[6] << 16) | (static_cast<uint32_t>(b[7]) << 24);
  v.z = b[8] | (b[9] << 8) | (b[10] << 16) | (static_cast<uint32_t>(b[11]) << 24);
  v.w = b[12] | (b[13] << 8) | (b[14] << 16) | (static_cast<uint32_t>(b[15]) << 24);
  tiles[i] = v;
}
}  // namespace

size_t weight_tiles_bytes(long long rows, long long in) {
  if (rows <= 0 || in <= 0) return 0;
  const long long rbs = (rows + kBM - 1) / kBM, kbs = (in + kBK - 1) / kBK;
  return static_cast<size_t>(rbs * kbs) * kBM * kBK;
}

int pack_weight_tiles(long long rows, long long in, const int8_t* w, long long ldw, int8_t* tiles,
                      cudaStream_t stream) {
  if (rows <= 0 || in <= 0 || ldw < in || w == nullptr || tiles == nullptr) return kErrInvalid;
  if ((reinterpret_cast<uintptr_t>(tiles) & 1023u) != 0) return kErrAlignment;
  const int kbs = static_cast<int>((in + kBK - 1) / kBK);
  const long long chunks = static_cast<long long>(weight_tiles_bytes(rows, in) / 16);
  pack_weight_tiles_kernel<<<static_cast<unsigned>((chunks + 255) / 256), 256, 0, stream>>>(
      rows, in, w, ldw, kbs, chunks, reinterpret_cast<uint4*>(tiles));
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

int skinny_reduce(int m, int n, int splits, const int32_t* part, int epilogue,
                  const float* x_scale, const float* w_scale, const float* bias,
                  const float* residual, void* y, cudaStream_t stream) {
  if (m <= 0 || n <= 0 || splits < 1 || part == nullptr || y == nullptr) return kErrInvalid;
  if (epilogue == kEpiF32W8A8 && (x_scale == nullptr || w_scale == nullptr)) return kErrInvalid;
  if (epilogue != kEpiF32W8A8 && epilogue != kEpiI32) return kErrInvalid;
  const bool vec = n % 4 == 0 && (reinterpret_cast<uintptr_t>(part) & 15u) == 0 &&
                   (reinterpret_cast<uintptr_t>(y) & 15u) == 0;
  const long long total = static_cast<long long>(m) * n;
  const long long threads = vec ? total / 4 : total;
  const dim3 grid(static_cast<unsigned>((threads + 255) / 256)), block(256);
  if (epilogue == kEpiF32W8A8)
    return vec ? launch_k(skinny_reduce_kernel<kEpiF32W8A8, true>, grid, block, 0, stream, splits,
                          m, n, part, x_scale, w_scale, bias, residual, y)
               : launch_k(skinny_reduce_kernel<kEpiF32W8A8, false>, grid, block, 0, stream, splits,
                          m, n, part, x_scale, w_scale, bias, residual, y);
  const float* none = nullptr;
  return vec ? launch_k(skinny_reduce_kernel<kEpiI32, true>, grid, block, 0, stream, splits, m, n,
                        part, none, none, none, none, y)
             : launch_k(skinny_reduce_kernel<kEpiI32, false>, grid, block, 0, stream, splits, m, n,
                        part, none, none, none, none, y);
}

int gemm_i8_skinny(int m, int n, int k, const int8_t* x, const int8_t* w, int epilogue,
                   const float* x_scale, const float* w_scale, const float* bias,
                   const float* residual, void* y, void* partial, cudaStream_t stream,
                   const int8_t* w_tiles) {
  if (m <= 0 || n <= 0 || k <= 0 || m > 128 || partial == nullptr || y == nullptr)
    return kErrInvalid;
  if (epilogue != kEpiF32W8A8 && epilogue != kEpiI32) return kErrInvalid;
  int32_t* part = static_cast<int32_t*>(partial);
  if (int rc = gemm_i8_skinny_partials(m, n, k, x, w, part, stream, w_tiles)) return rc;
  // the reduce launches as a programmatic dependent of the GEMM, so its launch
  // overlaps the GEMM's tail
  PdlScope pdl;
  return skinny_reduce(m, n, skinny_splits(m, n, k), part, epilogue, x_scale, w_scale, bias,
                       residual, y, stream);
}

int gemm_i8(const GemmProblem& p, int epilogue, cudaStream_t stream) {
  if (p.M <= 0 || p.N <= 0 || p.K <= 0) return kErrInvalid;
  const bool wide = p.N > 128;
  switch (epilogue) {
    case kEpiF32W8A8:
      return wide ? launch<256, 4, kEpiF32W8A8>(p, stream)
                  : launch<128, 6, kEpiF32W8A8>(p, stream);
    case kEpiI8Shift:
      return wide ? launch<256, 4, kEpiI8Shift>(p, stream)
                  : launch<128, 6, kEpiI8Shift>(p, stream);
    case kEpiI32:
      return wide ? launch<256, 4, kEpiI32>(p, stream)
                  : launch<128, 6, kEpiI32>(p, stream);
    case kEpiSwiGLU:
      if (p.args.row_max == nullptr || p.args.b_up < p.N) return kErrInvalid;
      return launch<256, 4, kEpiSwiGLU>(p, stream);
    case kEpiQkvRope: {
      const QkvOut& q = p.args.qkv;
      if (q.seq <= 0 || q.heads_q <= 0 || q.heads_kv <= 0 || q.rope == nullptr || !q.q8 ||
          !q.k8 || !q.qs || !q.ks || !q.vt || p.N != (q.heads_q + 2 * q.heads_kv) * 128 ||
          p.M % q.seq != 0)
        return kErrInvalid;
      return launch<256, 4, kEpiQkvRope>(p, stream);
    }
    default:
      return kErrInvalid;
  }
}

}  // namespace reef
