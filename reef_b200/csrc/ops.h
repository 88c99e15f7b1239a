// ops.h -- internal C++ interface of libreef_b200 (kernel launchers).
//
// The public surface is the C ABI in include/reef_b200.h; capi.cpp validates
// arguments and forwards here.  Every launcher returns a status code from the
// enum below (the same values as REEF_B200_* in the public header).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace reef {

enum Status : int {
  kOk = 0,
  kErrInvalid = 1,
  kErrAlignment = 2,
  kErrCuda = 3,
  kErrUnsupported = 4,
  kErrNccl = 5,
  kErrTimeout = 6,
  kErrTooLarge = 7,
};

enum Epilogue : int {
  kEpiF32W8A8 = 0,  // y = float(acc) * (x_scale[m] * w_scale[n]) [+ bias[n]]
  kEpiI8Shift = 1,  // y = sat8(rnu_shift(acc [+ bias32[n]], shift))
  kEpiI32 = 2,      // y = acc
  // y = silu(g) * u with g, u the kEpiF32W8A8 values of B rows n and b_up + n;
  // row_max[m] = max(row_max[m], max_n |y|) (atomic; zero it first)
  kEpiSwiGLU = 3,
  // the kEpiF32W8A8 values of a QKV projection (heads of 128 columns: q, then
  // k, then v), then RoPE on q / k and int8 per (token, head): see QkvOut
  kEpiQkvRope = 4,
  // y = acc, the split-K partials of a swap-AB skinny GEMM stored
  // token-major: y[split][n][m] (n: the kernel's N, a token; m: its M, a
  // weight row), row stride ldy = M
  kEpiI32T = 5,
};

// kEpiQkvRope outputs (the layout rope_qkv_quant writes).  Rows are tokens
// b * seq + pos.
struct QkvOut {
  const float2* rope;  // [64][seq] (cos, sin) of pos * base^(-2i/128), i-major
  int seq, heads_q, heads_kv;
  int8_t* q8;          // [T][Hq*128]
  int8_t* k8;          // [T][Hkv*128]
  int8_t* v8;          // [T][Hkv*128] or null
  float* qs;           // [B][Hq][S]
  float* ks;           // [B][Hkv][S]
  float* vs;           // [B][Hkv][S] or null
  void* vt;            // [B][Hkv][128][S] f16, f16(v code * v scale)
};

// ---- launches --------------------------------------------------------------------
//
// While a PdlScope lives on a host thread, the kernels that thread launches
// through launch_k go out as programmatic dependents of the kernel before
// them in the stream: their launch and set-up (and, in the skinny GEMM, the
// weight loads, which no earlier kernel writes) overlap that kernel's work.
// Each such kernel waits for its predecessor (pdl_wait, common.cuh) before
// reading or writing anything the predecessor may touch.  Without a scope,
// launch_k is an ordinary launch.
extern thread_local bool t_pdl;
struct PdlScope {
  bool prev;
  PdlScope() : prev(t_pdl) { t_pdl = true; }
  ~PdlScope() { t_pdl = prev; }
  PdlScope(const PdlScope&) = delete;
  PdlScope& operator=(const PdlScope&) = delete;
};

template <typename... KArgs, typename... Args>
int launch_k(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
             Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = t_pdl ? attr : nullptr;
  cfg.numAttrs = t_pdl ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...) != cudaSuccess) return kErrCuda;
  return cudaGetLastError() == cudaSuccess ? kOk : kErrCuda;
}

// Row stride (bytes) of every int8 matrix the tensor cores read: TMA needs
// 16-byte aligned row strides.
inline size_t kpad(size_t in) { return (in + 15) / 16 * 16; }

struct GemmArgs {
  int M, N, K;
  const float* x_scale;   // [M]   (kEpiF32W8A8)
  const float* w_scale;   // [N]   (kEpiF32W8A8)
  const float* bias_f;    // [N] or null (kEpiF32W8A8)
  const int32_t* bias_i;  // [N] or null (kEpiI8Shift)
  const float* residual;  // [M][ldy] or null (kEpiF32W8A8): y = residual + y
  void* y;                // [M][ldy] output
  long long ldy;          // elements
  uint32_t shift;         // kEpiI8Shift
  int group_m;            // raster group (0 = default)
  int k_segments;         // > 1: K arrives as this many segments (3-D tensor maps)
  int k_splits;           // > 1: K split across CTAs; split s writes y + s * split_stride
  long long b_up;         // kEpiSwiGLU: first B row of the "up" half
  float* row_max;         // kEpiSwiGLU: [M] running max |y| per row
  QkvOut qkv;             // kEpiQkvRope
  long long split_stride; // elements between the partial outputs of two splits
  int vec_ok;             // 16-byte (int8: 4-byte) output stores allowed (launcher)
  int max_ctas;           // > 0: at most this many persistent CTAs (SMs left to others)
  int gelu;               // kEpiF32W8A8: y = gelu(dequant + bias), reef's tanh form, before any residual
  // A depends on no earlier kernel (the weights of a swap-AB GEMM): its first
  // stages are requested before the kernel waits for its predecessor
  int a_first;
  // A in the tiled layout of pack_weight_tiles (one contiguous, pre-swizzled
  // 16 KiB block per 128-row x 128-byte stage, read by one bulk copy) instead
  // of through the tensor map; one K segment only
  const int8_t* a_tiles;
  int* err;               // device error word (set by the launcher)
};

struct GemmProblem {
  int M, N, K;      // K: per segment (args.k_segments segments; 1 = plain)
  const int8_t* a;  // [segs][M][lda]
  long long lda;    // bytes, multiple of 16
  const int8_t* b;  // [segs][N][ldb] (segment strides below)
  long long ldb;    // bytes, multiple of 16
  long long a_seg;  // bytes between A segments (multiple of 16; any value for 1 segment)
  long long b_seg;  // bytes between B segments
  GemmArgs args;
};

// ---- device plumbing (device.cu) ----------------------------------------------
int num_sms();
int* device_error_ptr();               // this device's error word
int check_device();
// Failure-detection self-test: a bounded wait that nothing satisfies (see device.cu).
int selftest_wait_timeout(unsigned long long limit_ns, int* done, cudaStream_t stream);                    // kOk on sm_100, else kErrUnsupported
int read_device_error(int* code);      // synchronizes, returns and clears
int make_tma_2d_i8(CUtensorMap* map, const void* base, long long rows,
                   long long cols, long long ld_bytes, int box_cols, int box_rows);
int make_tma_3d(CUtensorMap* map, CUtensorMapDataType type, const void* base, long long d0,
                long long d1, long long d2, long long s1, long long s2, int box0, int box1,
                CUtensorMapSwizzle swizzle);
int make_tma_3d_i8(CUtensorMap* map, const void* base, long long rows, long long cols,
                   long long ld_bytes, long long segs, long long seg_bytes, int box_cols,
                   int box_rows);
int make_tma_2d(CUtensorMap* map, CUtensorMapDataType type, int elem_bytes,
                const void* base, long long rows, long long cols, long long ld_elems,
                int box_cols, int box_rows, CUtensorMapSwizzle swizzle);

// ---- kernels ------------------------------------------------------------------
int gemm_i8(const GemmProblem& p, int epilogue, cudaStream_t stream);
// Gate/up projection with SwiGLU in the epilogue (layer.cpp): h [rows][ffn]
// fp32 and row_max [rows] = max |h| of each row.
int linear_w8a8_swiglu(long long rows, int in, int ffn, const int8_t* xq, const float* xs,
                       const int8_t* w_gu, const float* ws, float* h, float* row_max,
                       cudaStream_t st);
// QKV projection with RoPE + per-(token, head) int8 in the epilogue
// (layer.cpp): the outputs of rope_qkv_quant on the projection.  `out.rope`
// is filled here from rope_base (it must point at [64][seq] float2 scratch).
int linear_w8a8_qkv_rope(long long rows, int in, const int8_t* xq, const float* xs,
                         const int8_t* w_qkv, const float* ws, float rope_base, QkvOut out,
                         cudaStream_t st);

// Skinny GEMM for few tokens (decode): y[m][n] = epi(sum_k x[m][k] w[n][k]) with
// the weights as the 128-row MMA operand (swap-AB), tokens (m <= 128) on the
// MMA's N side, and K split across CTAs into int32 partials in `partial`
// (skinny_partial_bytes() of scratch), reduced and requantised by a second
// kernel.  epilogue: kEpiF32W8A8 (x_scale, w_scale, bias, residual -> y fp32)
// or kEpiI32 (y int32 [m][n], the sums of a row-parallel shard).
size_t skinny_partial_bytes(int m, int n, int k);
int gemm_i8_skinny(int m, int n, int k, const int8_t* x, const int8_t* w, int epilogue,
                   const float* x_scale, const float* w_scale, const float* bias,
                   const float* residual, void* y, void* partial, cudaStream_t stream,
                   const int8_t* w_tiles = nullptr);
// The two halves of gemm_i8_skinny, for consumers that fold the split-K sum
// into their own pass: the GEMM writes skinny_split_count(m, n, k) int32
// partials part[s][m][n] (token-major, m * n apart); skinny_reduce sums them
// and applies the epilogue (kEpiF32W8A8: dequant [+ bias] [+ residual] ->
// fp32 y; kEpiI32: the int32 sums), y [m][n].
int skinny_split_count(int m, int n, int k);
// w_tiles (optional): the same weights in pack_weight_tiles' layout, streamed
// as contiguous 16 KiB blocks instead of 128-byte row pieces
int gemm_i8_skinny_partials(int m, int n, int k, const int8_t* x, const int8_t* w,
                            int32_t* part, cudaStream_t stream, const int8_t* w_tiles = nullptr);
// The decode layout of a K-major int8 weight w [rows][ldw]: 16 KiB tiles of
// 128 rows x 128 bytes of K, each stored as the tensor cores read it
// (128-byte swizzle: 16-byte chunk c of tile row r at r * 128 + ((c ^ (r & 7))
// * 16)), the tiles of one 128-row block consecutive along K: tile (rb, kb)
// at ((rb * KB + kb) * 16384), KB = ceil(in / 128).  Bytes past the matrix
// are zero.
size_t weight_tiles_bytes(long long rows, long long in);
int pack_weight_tiles(long long rows, long long in, const int8_t* w, long long ldw,
                      int8_t* tiles, cudaStream_t stream);
int skinny_reduce(int m, int n, int splits, const int32_t* part, int epilogue,
                  const float* x_scale, const float* w_scale, const float* bias,
                  const float* residual, void* y, cudaStream_t stream);

// One output written alike to up to kMaxDst places: the same offset in every
// rank's symmetric arena, so an exchanged activation goes from the kernel that
// produces it straight into every peer's memory over NVLink (no separate copy).
constexpr int kMaxDst = 8;
struct PeerDst {
  int n = 0;
  void* p[kMaxDst] = {};
};
inline PeerDst one_dst(void* p) {
  PeerDst d;
  d.n = 1;
  d.p[0] = p;
  return d;
}
// 1..kMaxDst destinations, none null
inline bool dst_ok(const PeerDst& d) {
  if (d.n < 1 || d.n > kMaxDst) return false;
  for (int i = 0; i < d.n; ++i)
    if (d.p[i] == nullptr) return false;
  return true;
}

// Counters in peers' memory that one warp increments (system-scope atomics,
// after a system-wide fence): a step's "delivered" / "consumed" signals.
constexpr int kMaxFlags = 32;
struct PeerFlags {
  int n = 0;
  unsigned int* p[kMaxFlags] = {};
};

// Local counters a stream waits on before its next kernels: lane i of one
// warp spins (system-scope acquire loads) until counter p[i] reaches
// target[i] (wrap-around >=, as the counters only grow), or until `limit_ns`
// of %globaltimer pass, in which case it records kDevTimeoutPeer in the
// device error word and returns, so no wait outlives its limit (the host
// reads REEF_B200_ERR_TIMEOUT).  While the word holds kDevTimeoutPeer (until
// the host reads it), later waits return at once.
constexpr int kMaxWaits = 8;
struct CounterWaits {
  int n = 0;
  const unsigned int* p[kMaxWaits] = {};
  unsigned int target[kMaxWaits] = {};
};
// One launch: signal `f` (a system-wide fence, then the increments), then
// wait for `w`.  Either may be empty; nothing is launched when both are.
int signal_and_wait(const PeerFlags& f, const CounterWaits& w, unsigned long long limit_ns,
                    cudaStream_t stream);

// lm_head.cu -- the token embedding, reef's float linear(x, w) for one row
// (bit-identical) and argmax
int embedding_f32(int width, long long count, const uint32_t* ids, long long first_position,
                  long long vocab, long long positions, const float* wte, const float* wpe,
                  float* y, cudaStream_t stream);
int matvec_rows_f32(long long out, long long in, const float* w, const float* x, float* y,
                    cudaStream_t stream);
int argmax_f32(long long n, const float* x, uint32_t* index, cudaStream_t stream);

// gptneo.cu -- reef's float layernorm, bit for bit (one row per CTA)
int layernorm_exact(long long rows, int width, float eps, const float* x, const float* gain,
                    const float* shift, float* y, cudaStream_t stream);
// layernorm_exact then quantize_rows (quant.hpp:112-133) in one pass: x_q
// [rows][ldq] int8 (padding zeroed) and x_scale [rows], the same bits
int layernorm_exact_quant(long long rows, int width, float eps, const float* x, const float* gain,
                          const float* shift, int8_t* x_q, long long ldq, float* x_scale,
                          cudaStream_t stream);

// elementwise.cu -- the rest of reef's Coral operators, bit for bit
int linear_f32(long long rows, int in, int out, const float* x, const float* wt,
               const float* bias, float* y, cudaStream_t stream);
enum UnaryExactOp { kUnaryExp = 0, kUnaryTanh = 1, kUnaryGelu = 2 };
int unary_exact(int op, long long n, const float* x, float* y, cudaStream_t stream);
int add_f32(long long n, const float* a, const float* b, float* y, cudaStream_t stream);
int gelu_int8(long long n, const int8_t* x, const int8_t* table, int8_t* y, cudaStream_t stream);
int add_int8(long long n, const int8_t* a, const int8_t* b, int8_t* y, cudaStream_t stream);
int embedding_int8(int width, long long count, const uint32_t* ids, long long first_position,
                   long long vocab, long long positions, const int8_t* wte, const int8_t* wpe,
                   int8_t* y, cudaStream_t stream);
int layernorm_int8(long long rows, int width, const int8_t* x, const int8_t* gain,
                   const int8_t* shift, int8_t* y, cudaStream_t stream);

// quant.cu
int quantize_rows(long long rows, long long in, const float* x, int8_t* x_q,
                  long long ldq, float* x_scale, const float* row_max,
                  cudaStream_t stream);
// quantize_rows with the int8 rows written to every destination (in and ldq
// multiples of 4, x 16-byte aligned; x_scale local)
int quantize_rows_to(long long rows, long long in, const float* x, const PeerDst& x_q,
                     long long ldq, float* x_scale, const float* row_max, cudaStream_t stream);
// src [n] fp32 copied to every destination by SM stores
int push_f32(long long n, const float* src, const PeerDst& dst, cudaStream_t stream);
// p[0, n) = 0 by a kernel (a link of a programmatic-dependent chain, where a
// memset node would make the next kernel wait for the whole one before)
int zero_f32(long long n, float* p, cudaStream_t stream);
// out[r] = max_s in[s][r] for in [segs][rows]
int max_segments(int segs, long long rows, const float* in, float* out, cudaStream_t stream);
int row_absmax(long long rows, long long in, const float* x, float* row_max,
               cudaStream_t stream);
int row_absmax_to(long long rows, long long in, const float* x, const PeerDst& row_max,
                  cudaStream_t stream);
int pack_weight_i8(long long in, long long out, const int8_t* wt, int8_t* w,
                   long long ldw, cudaStream_t stream);
int pad_rows_i8(long long rows, long long in, const int8_t* x, long long ldx,
                int8_t* y, long long ldy, cudaStream_t stream);
int w8a8_epilogue_i32(long long rows, long long out, const int32_t* acc,
                      const float* x_scale, const float* w_scale, const float* bias,
                      const float* residual, float* y, cudaStream_t stream);

// llama.cu -- fused RMSNorm / SwiGLU + per-token quantisation
int rmsnorm_quant(long long rows, int width, float eps, const float* x, const float* gain,
                  int8_t* x_q, float* x_scale, cudaStream_t stream);
// skinny_reduce (kEpiF32W8A8 + residual) into h, then rmsnorm_quant on h, in
// one pass (one CTA per row): the same h, x_q and scales as the two kernels.
// part [splits][rows][width] int32; x_q [rows][width]; 16-byte alignment.
int reduce_rmsnorm_quant(long long rows, int width, int splits, const int32_t* part,
                         const float* x_scale, const float* w_scale, const float* residual,
                         float* h, float eps, const float* gain, int8_t* x_q, float* q_scale,
                         cudaStream_t stream);
// SwiGLU of the gate/up projection's split-K partials (token-major int32
// sums part[s][row][2 ffn], splits of them, rows * 2 ffn apart), dequantised
// with the W8A8 epilogue: h = silu(g) * u, one CTA per row.  row_max_out set:
// write max |h| per row and nothing else.  Otherwise quantise h to x_q / x_scale
// with row_max_in (the all-reduced maximum) or, when it is null, the row's
// own maximum.
int swiglu_partials(long long rows, int ffn, const int32_t* part, int splits, const float* x_scale,
                    const float* w_scale, const float* row_max_in, float* row_max_out,
                    int8_t* x_q, float* q_scale, cudaStream_t stream);
// TP-sharded RMSNorm (columns split over `ranks`): per-rank stats, all-gather,
// then quantise this rank's columns with the full row's scale.
// stats and x_q go to every destination of their PeerDst (x_scale is local).
int rms_stats(long long rows, int width, int ranks, const float* x_local, const float* gain_local,
              const PeerDst& stats, cudaStream_t stream);
int rms_apply_quant(long long rows, int width, int ranks, float eps, const float* x_local,
                    const float* gain_local, const float* stats_all, const PeerDst& x_q,
                    float* x_scale, cudaStream_t stream);

// attention_exact.cu -- reef's integer and float heads, bit for bit.
// Scores stay in shared memory, which bounds the key length.
constexpr int kMaxKeysExact = 32768;

struct AttnHeadArgs {
  int heads;            // heads in this launch (blockIdx.y)
  int query_len, key_len, head_dim, window;
  long long query_start;
  long long q_stride, q_head;      // elements between query rows / heads
  long long kv_stride, kv_head;    // elements between key rows / heads
  long long out_stride, out_head;  // elements between output rows / heads
};

int attention_head_int8(const AttnHeadArgs& a, const int8_t* q, const int8_t* k,
                        const int8_t* v, uint32_t score_shift, const uint16_t* table,
                        uint32_t out_shift, int8_t* out, cudaStream_t stream);
int attention_head_f32(const AttnHeadArgs& a, const float* q, const float* k, const float* v,
                       float* out, cudaStream_t stream);
int softmax_int8_rows(long long rows, int n, const int32_t* scores, uint32_t shift,
                      const uint16_t* table, uint8_t* probs, cudaStream_t stream);

// flash_attn.cu -- int8 flash attention (prefill) and its input packing.
struct FlashProblem {
  int batch, heads_q, heads_kv, seq, head_dim, causal;
  float sm_scale;
  const int8_t* q8;       // [B*S][Hq*128]  token-major
  const int8_t* k8;       // [B*S][Hkv*128] token-major
  const void* vt;         // [B][Hkv][128][S] f16, dequantised v
  const float* q_scale;   // [B][Hq][S]
  const float* k_scale;   // [B][Hkv][S]
  float* out;             // [B*S][out_ld]
  long long out_ld;
};
int flash_prefill_i8(const FlashProblem& p, cudaStream_t stream);
int rope_qkv_quant(int batch, int seq, int heads_q, int heads_kv, float rope_base,
                   const float* qkv, int8_t* q8, int8_t* k8, int8_t* v8, float* q_scale,
                   float* k_scale, float* v_scale, void* vt, void* rope_table,
                   cudaStream_t stream);  // rope_table: [64][seq] float2 scratch or null
// (cos, sin) of pos * base^(-2i/128), pos < seq, i < 64, into table [64][seq] float2
int rope_table(int seq, float rope_base, void* table, cudaStream_t stream);

// decode_attn.cu -- int8 decode attention over an int8 KV cache (split-KV)
struct DecodeProblem {
  int batch, heads_q, heads_kv, max_len;
  float sm_scale;
  const int8_t* q8;       // [B][Hq][128]
  const float* q_scale;   // [B][Hq]
  const int8_t* k_cache;  // [B][Hkv][max_len][128]
  const float* k_scale;   // [B][Hkv][max_len]
  const int8_t* v_cache;
  const float* v_scale;
  const int* lens;        // [B] cached keys per sequence (device), or null
  // [B] device, or null: the row each sequence appends in this step (lens =
  // positions + 1), unchanged while the step runs.  Lets the kernel request
  // the K / V tiles wholly below it before the kernel ahead of it (the one
  // that appends those rows) has finished.
  const int* positions;
  int len;                // cached keys of every sequence when lens is null
  float* partial;         // decode_attn_partial_floats() floats of scratch
  float* out;             // [B][Hq][128]
};
size_t decode_attn_partial_floats(int batch, int heads_q, int max_len);
// The decode step's q / k / v from the QKV projection's split-K partials (the
// skinny GEMM's token-major int32 sums, gemm_i8_skinny_partials), summed and
// dequantised here, so no separate reduce runs: RoPE at each sequence's
// position, q quantised per head into q8 / q_scale, k and v quantised per head
// and appended to the cache at row positions[b], lens[b] = positions[b] + 1.
int decode_rope_append_partials(int batch, int heads_q, int heads_kv, int max_len,
                                float rope_base, const int* positions, const int32_t* part,
                                int splits, const float* x_scale, const float* w_scale,
                                int8_t* q8, float* q_scale, int8_t* k_cache, float* k_scale,
                                int8_t* v_cache, float* v_scale, int* lens, cudaStream_t stream);
int decode_attn_i8(const DecodeProblem& p, cudaStream_t stream);

}  // namespace reef
