// common.cuh -- device helpers shared by the reef_b200 sm_100a kernels.
//
// Every wait on an mbarrier is bounded: after kWaitLimitNs of %globaltimer
// time the waiting thread records an error code in the launch's device error
// word and gives up, so a broken pipeline ends the kernel instead of hanging
// the GPU.  The host reads the word back through reef_b200_device_error().
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace reef {

// ---- error word -------------------------------------------------------------

enum DeviceError : int {
  kDevOk = 0,
  kDevTimeoutFull = 0x101,     // consumer waited too long for a TMA stage
  kDevTimeoutEmpty = 0x102,    // producer waited too long for a free stage
  kDevTimeoutAccFull = 0x103,  // epilogue waited too long for an accumulator
  kDevTimeoutAccEmpty = 0x104, // MMA waited too long for the epilogue
  kDevTimeoutDrain = 0x105,    // final drain of the MMA pipe
  kDevTimeoutPeer = 0x106,     // a peer flag never arrived
  kDevBadPosition = 0x201,     // a decode position outside the cache
  kDevBadToken = 0x202,        // a token id outside the vocabulary
  kDevNonFinite = 0x301,       // a float product or sum the engine would reject
};

// A wait gives up after this long (ns of %globaltimer).
constexpr unsigned long long kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

// ---- programmatic dependent launch ----------------------------------------------
//
// A kernel launched as a programmatic dependent (launch_k under a PdlScope,
// ops.h) may start while the kernel before it in the stream still runs.
// pdl_wait() returns once that kernel has completed and its memory is
// visible (at once for an ordinary launch); every such kernel calls it before
// it touches anything an earlier kernel writes, and calls pdl_trigger() only
// after it, so the next kernel's early part overlaps this kernel alone, never
// an older one.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- shared-memory addresses ------------------------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier -----------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.release.cta.shared::cta.b64 st, [%0];\n\t}" ::"r"(
          smem_u32(bar))
      : "memory");
}

// Raise the bytes the current phase expects without arriving (the arrival,
// and any more bytes, follow with mbar_arrive_expect_tx).
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.expect_tx.relaxed.cta.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 st, [%0], %1;\n\t}" ::
          "r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns
// false (after recording `code`) when `limit_ns` of %globaltimer pass.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity,
                                          int* err, int code,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long start = globaltimer();
  for (uint32_t spin = 1;; ++spin) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((spin & 255u) == 0 && globaltimer() - start > limit_ns) {
      record_error(err, code);
      return false;
    }
  }
}

// ---- TMA (cp.async.bulk.tensor), no multicast --------------------------------

__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map,
                                            uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map,
                                            uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1),
      "r"(c2)
      : "memory");
}

// Global -> shared bulk copy (not a tensor map, no multicast): `bytes` (a
// multiple of 16; both addresses 16-byte aligned), completing on `bar`.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gsrc, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(gsrc)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Shared -> global tile store (bulk-group completion).  The tensor map
// clips rows outside its extent.
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* smem_src, int c0,
                                             int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(smem_src)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// Wait until every committed bulk store has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map))
               : "memory");
}

// ---- tcgen05 -------------------------------------------------------------------

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::
                   "r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::
                   : "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] x B[smem]^T, int8 x int8 -> int32, one CTA.
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc,
                                       uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem] x B[smem]^T, f16 x f16 -> f32, one CTA.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc,
                                        uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] x B[smem]^T, f16 x f16 -> f32, one CTA.  A is M rows
// (TMEM lanes) of K f16 values packed two to a 32-bit column, element 2c in
// the low half of column c.
__device__ __forceinline__ void mma_f16_tmem_a(uint32_t d_tmem, uint32_t a_tmem,
                                               uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::
          "r"(smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp receives
// lane (quadrant*32 + t), columns [col, col+32).
__device__ __forceinline__ void tmem_ld_32x32b_x32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
        "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
        "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]),
        "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 16 consecutive 32-bit columns, store from registers.
__device__ __forceinline__ void tmem_st_32x32b_x16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
      "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]),
      "r"(r[14]), "r"(r[15])
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns, store from registers.
__device__ __forceinline__ void tmem_st_32x32b_x32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::
          "r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
      "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]),
      "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]),
      "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Warpgroup register reconfiguration: every thread of the warpgroup runs the
// same call.  The block's total (threads x registers at launch) is fixed, so
// the decreases of some warpgroups must cover the increases of the others.
template <uint32_t kRegs>
__device__ __forceinline__ void setmaxnreg_dec() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegs));
}
template <uint32_t kRegs>
__device__ __forceinline__ void setmaxnreg_inc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegs));
}

// Generic-proxy writes to shared memory become visible to the async proxy
// (tcgen05.mma operand reads, TMA) of this CTA.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Barrier among `count` threads (a multiple of 32) on hardware barrier `id`.
__device__ __forceinline__ void named_barrier(int id, int count) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Arrive on hardware barrier `id` (expecting `count` threads) without waiting.
__device__ __forceinline__ void named_arrive(int id, int count) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart
// (stride byte offset), leading byte offset unused for this layout,
// descriptor version 1 (sm_100), layout type 2 = SWIZZLE_128B.
__device__ __forceinline__ uint64_t smem_desc_k_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);  // start address
  d |= static_cast<uint64_t>(1u) << 16;                     // LBO (16 B, unused)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;             // SBO = 1024 B
  d |= static_cast<uint64_t>(1u) << 46;                     // version
  d |= static_cast<uint64_t>(2u) << 61;                     // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::i8: signed int8 A and B, int32 D, both
// K-major, M x N tile.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n, bool a_unsigned = false,
                                                bool b_unsigned = false) {
  return (2u << 4)                                   // D format: s32
         | ((a_unsigned ? 0u : 1u) << 7)             // A: s8 (1) / u8 (0)
         | ((b_unsigned ? 0u : 1u) << 10)            // B: s8 (1) / u8 (0)
         | (static_cast<uint32_t>(n >> 3) << 17)     // N >> 3
         | (static_cast<uint32_t>(m >> 4) << 24);    // M >> 4
}

// Instruction descriptor, kind::f16: f16 A and B, f32 D, A K-major, B with
// the given major-ness (false = K-major, true = MN-major).
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n, bool b_mn_major = false) {
  return (1u << 4)                                   // D format: f32
         | (0u << 7) | (0u << 10)                    // A, B: f16
         | ((b_mn_major ? 1u : 0u) << 16)            // B major-ness
         | (static_cast<uint32_t>(n >> 3) << 17)
         | (static_cast<uint32_t>(m >> 4) << 24);
}

// ---- small math ----------------------------------------------------------------

// reef's int8 code of x at `scale` (quant.hpp:51-81): rint(x / scale)
// clamped to +-127, with x / scale the correctly rounded quotient
// (__fdiv_rn).  rcp = __frcp_rn(scale).  Fast path: q = fl(x * rcp) differs
// from x / scale by at most |q| * 1.5 * 2^-23 (two roundings of 2^-24), i.e.
// < 2.3e-5 when |q| < 128, so whenever q lies further than 6.1e-5 from a
// half-integer the correctly rounded quotient rounds to the same integer.
// Anything else (near a tie, |q| >= 128, a non-finite q) takes the division.
__device__ __forceinline__ int quant_code(float x, float scale, float rcp) {
  const float q = __fmul_rn(x, rcp);
  const float r = rintf(q);
  const int c = (fabsf(q) < 128.0f && fabsf(q - r) < 0.49993896f)
                    ? __float2int_rn(r)
                    : __float2int_rn(__fdiv_rn(x, scale));
  return c < -127 ? -127 : (c > 127 ? 127 : c);
}

// silu(g) * u = g / (1 + e^-g) * u, the one definition every SwiGLU uses.
__device__ __forceinline__ float silu_mul(float g, float u) {
  return __fdividef(g, 1.0f + __expf(-g)) * u;
}

// rounding_shift then saturate_int8 (reef int8.hpp:43-60): floor(v / 2^s + 1/2)
// clamped to [-128, 127].
__device__ __forceinline__ int8_t requant_rnu_sat8(int32_t v, uint32_t shift) {
  int32_t r = v;
  if (shift > 0) r = (v >> shift) + ((v >> (shift - 1)) & 1);
  r = r < -128 ? -128 : (r > 127 ? 127 : r);
  return static_cast<int8_t>(r);
}

}  // namespace reef
