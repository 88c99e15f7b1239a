// layer.cpp -- decoder layers assembled from the sm_100a kernels, with
// Megatron tensor parallelism over the NCCL communicator of comm.cpp.
//
// reef runs one GPT-Neo block per layer on one core (operator/block.hpp
// :97-108) and has no tensor parallelism.  Here a layer is sharded across TP
// ranks (one process or thread per GPU):
//   column-parallel  q/k/v (by heads), FFN up / gate / c_fc (by FFN columns):
//                    each rank owns output rows of W; no communication, and
//                    every output column equals TP=1's bit for bit.
//   row-parallel     attention output and FFN down / c_proj (by K): the
//                    rank's K-slice of the activation is quantised with the
//                    FULL row's scale (all-reduce MAX of the row maxima), its
//                    int32 partial sums are all-reduced (SUM, exact), and the
//                    dequant epilogue adds the bias once and the residual.
// So y is identical on every rank and bit-identical to TP=1 for the W8A8
// GEMMs; the GPT-Neo block is bit-identical to reef's Block<float>.
#include "../../include/reef_b200.h"

#include "comm.h"
#include "ops.h"

#include <algorithm>
#include <cstdlib>
#include <vector>
#include <cstdint>

namespace reef {

namespace {

#define REEF_TRY(expr)            \
  do {                            \
    const int rc_ = (expr);       \
    if (rc_ != kOk) return rc_;   \
  } while (0)

// Bump allocator over the caller's workspace (256-byte aligned pieces).
struct Carve {
  uint8_t* base;
  size_t used = 0;
  size_t cap;
  explicit Carve(void* b, size_t c) : base(static_cast<uint8_t*>(b)), cap(c) {}
  template <typename T>
  T* take(size_t count) {
    used = (used + 255) & ~static_cast<size_t>(255);
    T* p = reinterpret_cast<T*>(base ? base + used : nullptr);
    used += count * sizeof(T);
    return p;
  }
  bool fits() const { return base == nullptr || used <= cap; }
};

GemmProblem problem(long long rows, int in, int out, const int8_t* a, const int8_t* w) {
  GemmProblem p{};
  p.M = static_cast<int>(rows);
  p.N = out;
  p.K = in;
  p.a = a;
  p.lda = static_cast<long long>(kpad(in));
  p.b = w;
  p.ldb = static_cast<long long>(kpad(in));
  return p;
}

int gemm_w8a8_f32(long long rows, int in, int out, const int8_t* xq, const float* xs,
                  const int8_t* w, const float* ws, const float* bias, const float* residual,
                  float* y, cudaStream_t st, bool gelu = false) {
  GemmProblem p = problem(rows, in, out, xq, w);
  p.args.x_scale = xs;
  p.args.w_scale = ws;
  p.args.bias_f = bias;
  p.args.residual = residual;
  p.args.y = y;
  p.args.ldy = out;
  p.args.gelu = gelu ? 1 : 0;
  return gemm_i8(p, kEpiF32W8A8, st);
}

}  // namespace

// Gate/up projection fused with SwiGLU: h = silu(x W_g^T) * (x W_u^T), W_gu
// [2*ffn][in] (gate rows, then up rows), plus row_max[m] = max |h[m]| (this
// rank's columns).
int linear_w8a8_swiglu(long long rows, int in, int ffn, const int8_t* xq, const float* xs,
                       const int8_t* w_gu, const float* ws, float* h, float* row_max,
                       cudaStream_t st) {
  if (rows == 0) return kOk;
  REEF_TRY(zero_f32(rows, row_max, st));  // the epilogue's atomic maxima start at 0
  GemmProblem p = problem(rows, in, ffn, xq, w_gu);
  p.args.x_scale = xs;
  p.args.w_scale = ws;
  p.args.y = h;
  p.args.ldy = ffn;
  p.args.b_up = ffn;
  p.args.row_max = row_max;
  return gemm_i8(p, kEpiSwiGLU, st);
}

int linear_w8a8_qkv_rope(long long rows, int in, const int8_t* xq, const float* xs,
                         const int8_t* w_qkv, const float* ws, float rope_base, QkvOut out,
                         cudaStream_t st) {
  if (rows == 0) return kOk;
  REEF_TRY(rope_table(out.seq, rope_base, const_cast<float2*>(out.rope), st));
  GemmProblem p = problem(rows, in, (out.heads_q + 2 * out.heads_kv) * 128, xq, w_qkv);
  p.args.x_scale = xs;
  p.args.w_scale = ws;
  p.args.qkv = out;
  return gemm_i8(p, kEpiQkvRope, st);
}

// Row-parallel W8A8 linear.  `quant` fills xq/xs from the local input given
// the full-row maximum (or computes it itself when row_max is null);
// `absmax` writes the local row maxima.
// Optional instrumentation: record ev[0] / ev[1] around one kernel launch.
struct Span {
  cudaEvent_t* ev;
  cudaStream_t st;
  Span(cudaEvent_t* e, cudaStream_t s) : ev(e), st(s) {
    if (ev) cudaEventRecord(ev[0], st);
  }
  ~Span() {
    if (ev) cudaEventRecord(ev[1], st);
  }
};

template <typename Quant, typename AbsMax>
int rowpar_linear(Comm* c, long long rows, int in_local, int out, Quant quant, AbsMax absmax,
                  const int8_t* w, const float* ws, const float* bias, const float* residual,
                  int8_t* xq, float* xs, float* row_max, int32_t* acc, float* y,
                  cudaStream_t st, cudaEvent_t* ev = nullptr) {
  if (comm_world(c) == 1) {
    REEF_TRY(quant(static_cast<const float*>(nullptr)));
    Span sp(ev, st);
    return gemm_w8a8_f32(rows, in_local, out, xq, xs, w, ws, bias, residual, y, st);
  }
  REEF_TRY(absmax(row_max));
  REEF_TRY(allreduce_max_f32(c, row_max, static_cast<size_t>(rows), st));
  REEF_TRY(quant(static_cast<const float*>(row_max)));
  GemmProblem p = problem(rows, in_local, out, xq, w);
  p.args.y = acc;
  p.args.ldy = out;
  {
    Span sp(ev, st);
    REEF_TRY(gemm_i8(p, kEpiI32, st));
  }
  REEF_TRY(allreduce_sum_i32(c, acc, static_cast<size_t>(rows) * out, st));
  return w8a8_epilogue_i32(rows, out, acc, xs, ws, bias, residual, y, st);
}

// Row-parallel linear for few rows (decode): the skinny split-K GEMM.
template <typename Quant, typename AbsMax>
int rowpar_skinny(Comm* c, int rows, int in_local, int out, Quant quant, AbsMax absmax,
                  const int8_t* w, const float* ws, const float* residual, int8_t* xq, float* xs,
                  float* row_max, int32_t* acc, void* partial, float* y, cudaStream_t st,
                  const int8_t* w_tiles = nullptr) {
  if (comm_world(c) == 1) {
    REEF_TRY(quant(static_cast<const float*>(nullptr)));
    return gemm_i8_skinny(rows, out, in_local, xq, w, kEpiF32W8A8, xs, ws, nullptr, residual, y,
                          partial, st, w_tiles);
  }
  REEF_TRY(absmax(row_max));
  REEF_TRY(allreduce_max_f32(c, row_max, static_cast<size_t>(rows), st));
  REEF_TRY(quant(static_cast<const float*>(row_max)));
  REEF_TRY(gemm_i8_skinny(rows, out, in_local, xq, w, kEpiI32, nullptr, nullptr, nullptr, nullptr,
                          acc, partial, st, w_tiles));
  REEF_TRY(allreduce_sum_i32(c, acc, static_cast<size_t>(rows) * out, st));
  return w8a8_epilogue_i32(rows, out, acc, xs, ws, nullptr, residual, y, st);
}

}  // namespace reef

using namespace reef;

namespace {

inline cudaStream_t S(reef_b200_stream_t s) { return reinterpret_cast<cudaStream_t>(s); }
inline Comm* C(reef_b200_comm* c) { return reinterpret_cast<Comm*>(c); }

// ---- Llama-shape layer ----------------------------------------------------------

// The QKV epilogue's outputs in the layer's buffers (the int8 v rows and v
// scales are not needed by the flash head, which reads V^T).
QkvOut qkv_out(const reef_b200_llama_layer* L, int hq, int hkv, int8_t* q8, int8_t* k8,
               float* qs, float* ks, void* vt, void* rope) {
  QkvOut o{};
  o.rope = static_cast<const float2*>(rope);
  o.seq = static_cast<int>(L->seq);
  o.heads_q = hq;
  o.heads_kv = hkv;
  o.q8 = q8;
  o.k8 = k8;
  o.qs = qs;
  o.ks = ks;
  o.vt = vt;
  return o;
}

struct LlamaBufs {
  int8_t* xq;
  float* xs;
  float* row_max;
  float* big;     // SwiGLU output h [T][ffn]
  int8_t* q8;
  int8_t* k8;
  float* qs;
  float* ks;
  void* vt;
  float* attn;
  float* h;
  int32_t* acc;
  void* rope;     // [64][seq] (cos, sin)
};

size_t llama_carve(const reef_b200_llama_layer* L, void* ws, LlamaBufs* b) {
  const size_t T = L->batch * L->seq;
  const size_t H = L->hidden, hq = L->heads_q, hkv = L->heads_kv, F = L->ffn, D = 128;
  Carve c(ws, ~static_cast<size_t>(0));
  const size_t widest = std::max({kpad(H), kpad(hq * D), kpad(F)});
  b->xq = c.take<int8_t>(T * widest);
  b->xs = c.take<float>(T);
  b->row_max = c.take<float>(T);
  b->big = c.take<float>(T * F);
  b->q8 = c.take<int8_t>(T * hq * D);
  b->k8 = c.take<int8_t>(T * hkv * D);
  b->qs = c.take<float>(T * hq);
  b->ks = c.take<float>(T * hkv);
  b->vt = c.take<uint16_t>(T * hkv * D);
  b->attn = c.take<float>(T * hq * D);
  b->h = c.take<float>(T * H);
  b->acc = c.take<int32_t>(L->comm != nullptr ? T * H : 0);
  b->rope = c.take<float>(L->seq * 64 * 2);
  return c.used + 256;
}

// Chunks of whole sequences the all-gather plan pipelines over: 2 when the
// batch divides (measured on config 3 at TP=2 and TP=4: 2.04 / 1.55 ms per
// layer against 2.11 / 1.68 with 4), else 1 (no pipelining).
// REEF_B200_TP_CHUNKS (1, 2 or 4) sets the cap.
int ag_chunks(const reef_b200_llama_layer* L) {
  int cap = 2;
  if (const char* e = std::getenv("REEF_B200_TP_CHUNKS")) cap = std::max(1, std::min(4, std::atoi(e)));
  for (int c : {4, 2})
    if (c <= cap && L->batch % static_cast<size_t>(c) == 0) return c;
  return 1;
}

// SMs the pipelined all-gather plan's GEMMs may occupy (0: all): the rest
// stay free for the neighbouring chunk's NVLink-writing kernels, which would
// otherwise wait for the persistent GEMM to leave the SMs.
// REEF_B200_TP_GEMM_SMS overrides the default.
int ag_gemm_sms() {
  static int v = -1;
  if (v < 0) {
    int x = 0;
    if (const char* e = std::getenv("REEF_B200_TP_GEMM_SMS")) x = std::max(0, std::atoi(e));
    v = x;
  }
  return v;
}

// Whether the TP=1 prefill forward launches its kernels as programmatic
// dependents of one another: off unless REEF_B200_PREFILL_PDL=1.  Measured
// on config 3 under the power cap, the chain made the layer slower (4.16 and
// 4.26 ms against 4.03 and 4.05 ms without, same box, interleaved runs): the
// dependents' CTAs that fit beside a persistent GEMM's wait there, and the
// GEMMs leave no tail worth overlapping.
bool prefill_pdl() {
  static int v = -1;
  if (v < 0) {
    const char* e = std::getenv("REEF_B200_PREFILL_PDL");
    v = (e != nullptr && e[0] == '1') ? 1 : 0;
  }
  return v == 1;
}

bool llama_allgather(const reef_b200_llama_layer* L) {
  return L->comm != nullptr && comm_world(reinterpret_cast<Comm*>(L->comm)) > 1 &&
         L->tp_mode == REEF_B200_TP_ALLGATHER;
}

struct LlamaAgBufs {
  float* stats;
  float* stats_all;
  int8_t* xq;
  int8_t* xq_all;
  float* xs;
  float* row_max;
  float* big;     // SwiGLU output h [T][ffn]
  int8_t* q8;
  int8_t* k8;
  float* qs;
  float* ks;
  void* vt;
  float* attn;
  float* h;
  void* rope;
};

size_t llama_ag_carve(const reef_b200_llama_layer* L, int world, void* ws, LlamaAgBufs* b) {
  const size_t T = L->batch * L->seq, N = static_cast<size_t>(world);
  const size_t H = L->hidden, hq = L->heads_q, hkv = L->heads_kv, F = L->ffn, D = 128;
  const size_t Hl = H / N, S = 8 / N + 1;
  const size_t kmax = std::max({Hl, hq * D, F});
  Carve c(ws, ~static_cast<size_t>(0));
  b->stats = c.take<float>(T * S);
  b->stats_all = c.take<float>(N * T * S);
  b->xq = c.take<int8_t>(T * kmax);
  b->xq_all = c.take<int8_t>(N * T * kmax);
  b->xs = c.take<float>(T);
  b->row_max = c.take<float>(T);
  b->big = c.take<float>(T * F);
  b->q8 = c.take<int8_t>(T * hq * D);
  b->k8 = c.take<int8_t>(T * hkv * D);
  b->qs = c.take<float>(T * hq);
  b->ks = c.take<float>(T * hkv);
  b->vt = c.take<uint16_t>(T * hkv * D);
  b->attn = c.take<float>(T * hq * D);
  b->h = c.take<float>(T * Hl);
  b->rope = c.take<float>(L->seq * 64 * 2);
  return c.used + 256;
}

// Widths far above any model's, and small enough that no workspace size or
// index built from them (tokens x width x 4 bytes) can overflow.
int dims_in_range(size_t hidden, size_t ffn, size_t heads_a, size_t heads_b) {
  if (hidden > (1u << 20) || ffn > (1u << 22) || heads_a > 4096 || heads_b > 4096)
    return REEF_B200_ERR_INVALID;
  return REEF_B200_OK;
}

int llama_check(const reef_b200_llama_layer* L) {
  if (L == nullptr) return REEF_B200_ERR_INVALID;
  if (L->batch == 0 || L->seq == 0 || L->hidden == 0 || L->heads_q == 0 || L->heads_kv == 0 ||
      L->ffn == 0 || L->head_dim != 128 || L->heads_q % L->heads_kv != 0 ||
      L->hidden % 16 != 0 || L->ffn % 16 != 0 || L->seq % 8 != 0 ||
      L->batch > (1u << 30) || L->seq > (1u << 30) || L->batch * L->seq > (1u << 30))
    return REEF_B200_ERR_INVALID;
  if (int rc = dims_in_range(L->hidden, L->ffn, L->heads_q, L->heads_kv)) return rc;
  if (!L->attn_norm || !L->w_qkv || !L->s_qkv || !L->w_o || !L->s_o || !L->mlp_norm ||
      !L->w_gu || !L->s_gu || !L->w_down || !L->s_down)
    return REEF_B200_ERR_INVALID;
  return REEF_B200_OK;
}

// ---- Llama-shape decode step -------------------------------------------------------

struct DecodeBufs {
  int8_t* xq;
  float* xs;
  float* xs2;  // the gate/up projection's input scales (xs holds the o-proj's or the down's)
  float* row_max;
  float* big;
  int8_t* q8;
  float* qs;
  int* lens;
  float* attn;
  float* h;
  int32_t* acc;
  void* partial;
  float* dpart;
};

size_t decode_carve(const reef_b200_llama_layer* L, size_t max_len, void* ws, DecodeBufs* b) {
  const size_t B = L->batch;
  const size_t H = L->hidden, hq = L->heads_q, hkv = L->heads_kv, F = L->ffn, D = 128;
  Carve c(ws, ~static_cast<size_t>(0));
  b->xq = c.take<int8_t>(B * std::max({kpad(H), kpad(hq * D), kpad(F)}));
  b->xs = c.take<float>(B);
  b->xs2 = c.take<float>(B);
  b->row_max = c.take<float>(B);
  b->big = c.take<float>(B * std::max((hq + 2 * hkv) * D, 2 * F));
  b->q8 = c.take<int8_t>(B * hq * D);
  b->qs = c.take<float>(B * hq);
  b->lens = c.take<int>(B);
  b->attn = c.take<float>(B * hq * D);
  b->h = c.take<float>(B * H);
  b->acc = c.take<int32_t>(L->comm != nullptr ? B * H : 0);
  const int Bi = static_cast<int>(B);
  const size_t part = std::max({skinny_partial_bytes(Bi, static_cast<int>((hq + 2 * hkv) * D),
                                                     static_cast<int>(H)),
                                skinny_partial_bytes(Bi, static_cast<int>(H),
                                                     static_cast<int>(hq * D)),
                                skinny_partial_bytes(Bi, static_cast<int>(2 * F),
                                                     static_cast<int>(H)),
                                skinny_partial_bytes(Bi, static_cast<int>(H), static_cast<int>(F))});
  b->partial = c.take<uint8_t>(part);
  b->dpart = c.take<float>(decode_attn_partial_floats(Bi, static_cast<int>(hq),
                                                       static_cast<int>(max_len)));
  return c.used + 256;
}

int decode_check(const reef_b200_llama_layer* L, size_t max_len) {
  if (L == nullptr || max_len == 0 || max_len > (1u << 24)) return REEF_B200_ERR_INVALID;
  if (L->batch == 0 || L->batch > 128 || L->hidden == 0 || L->heads_q == 0 ||
      L->heads_kv == 0 || L->ffn == 0 || L->head_dim != 128 || L->heads_q % L->heads_kv != 0 ||
      L->hidden % 16 != 0 || L->ffn % 16 != 0)
    return REEF_B200_ERR_INVALID;
  if (int rc = dims_in_range(L->hidden, L->ffn, L->heads_q, L->heads_kv)) return rc;
  const size_t g = L->heads_q / L->heads_kv;
  if (g != 1 && g != 2 && g != 4 && g != 8 && g != 16) return REEF_B200_ERR_INVALID;
  if (!L->attn_norm || !L->w_qkv || !L->s_qkv || !L->w_o || !L->s_o || !L->mlp_norm ||
      !L->w_gu || !L->s_gu || !L->w_down || !L->s_down)
    return REEF_B200_ERR_INVALID;
  if (L->hidden % 32 != 0) return REEF_B200_ERR_INVALID;  // 8 RMSNorm chunks of float4
  for (const int8_t* t : {L->t_qkv, L->t_o, L->t_gu, L->t_down})
    if (reinterpret_cast<uintptr_t>(t) % 1024 != 0) return REEF_B200_ERR_INVALID;
  if (L->comm != nullptr && L->tp_mode != REEF_B200_TP_ALLREDUCE &&
      L->tp_mode != REEF_B200_TP_ALLGATHER)
    return REEF_B200_ERR_INVALID;
  if (llama_allgather(L)) {
    const size_t N = static_cast<size_t>(comm_world(reinterpret_cast<Comm*>(L->comm)));
    if (8 % N != 0 || L->hidden % (32 * N) != 0 || (L->hidden / N) % 16 != 0 ||
        (L->heads_q * 128) % 16 != 0)
      return REEF_B200_ERR_INVALID;
  }
  return REEF_B200_OK;
}

// ---- GPT-Neo block ------------------------------------------------------------

struct NeoBufs {
  float* h;
  float* q;
  float* k;
  float* v;
  float* ctx;
  float* a;
  float* f;
  int8_t* xq;
  float* xs;
  float* row_max;
  int32_t* acc;
};

size_t neo_carve(const reef_b200_gptneo_block* B, void* ws, NeoBufs* b) {
  const size_t T = B->seq, d = B->hidden, dl = B->heads * B->head_dim, F = B->ffn;
  Carve c(ws, ~static_cast<size_t>(0));
  b->h = c.take<float>(T * d);
  b->q = c.take<float>(T * dl);
  b->k = c.take<float>(T * dl);
  b->v = c.take<float>(T * dl);
  b->ctx = c.take<float>(T * dl);
  b->a = c.take<float>(T * d);
  b->f = c.take<float>(T * F);
  b->xq = c.take<int8_t>(T * std::max({kpad(d), kpad(dl), kpad(F)}));
  b->xs = c.take<float>(T);
  b->row_max = c.take<float>(T);
  b->acc = c.take<int32_t>(B->comm != nullptr ? T * d : 0);
  return c.used + 256;
}

int neo_check(const reef_b200_gptneo_block* B) {
  if (B == nullptr) return REEF_B200_ERR_INVALID;
  if (B->seq == 0 || B->hidden == 0 || B->heads == 0 || B->head_dim == 0 || B->ffn == 0 ||
      B->seq > static_cast<size_t>(kMaxKeysExact))
    return REEF_B200_ERR_INVALID;
  if (int rc = dims_in_range(B->hidden, B->ffn, B->heads, B->head_dim)) return rc;
  if (!B->ln1_g || !B->ln2_g || !B->wq || !B->wk || !B->wv || !B->sq || !B->sk || !B->sv ||
      !B->wo || !B->so || !B->wfc || !B->sfc || !B->wproj || !B->sproj)
    return REEF_B200_ERR_INVALID;
  return REEF_B200_OK;
}


// This layer's KV cache for a cached block: [max_tokens][heads*head_dim]
// rows, token-major; the block's `seq` new rows go at `position`.
struct NeoCache {
  float* k;
  float* v;
  size_t position;
};

int neo_forward(const reef_b200_gptneo_block* B, const float* x, float* y, const NeoCache* kv,
                void* workspace, size_t workspace_bytes, cudaStream_t st) {
  if (int rc = neo_check(B)) return rc;
  if (!x || !y || !workspace) return REEF_B200_ERR_INVALID;
  NeoBufs b;
  if (neo_carve(B, workspace, &b) > workspace_bytes) return REEF_B200_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return REEF_B200_ERR_ALIGNMENT;
  if (int rc = check_device()) return rc;
  Comm* c = C(B->comm);
  const long long T = static_cast<long long>(B->seq);
  const int d = static_cast<int>(B->hidden), dl = static_cast<int>(B->heads * B->head_dim),
            F = static_cast<int>(B->ffn);
  const long long ld = static_cast<long long>(kpad(d));

  // Attention::forward (attention.hpp:354-372): ln_1, q/k/v projections
  // (column-parallel by heads), every local head, o_proj (row-parallel) with
  // the residual of Block::forward (block.hpp:99-102) fused in.
  REEF_TRY(layernorm_exact_quant(T, d, B->eps, x, B->ln1_g, B->ln1_b, b.xq, ld, b.xs, st));
  REEF_TRY(gemm_w8a8_f32(T, d, dl, b.xq, b.xs, B->wq, B->sq, nullptr, nullptr, b.q, st));
  // with a cache the key and value rows go straight into it
  const size_t past = kv != nullptr ? kv->position : 0;
  float* kr = kv != nullptr ? kv->k + past * dl : b.k;
  float* vr = kv != nullptr ? kv->v + past * dl : b.v;
  REEF_TRY(gemm_w8a8_f32(T, d, dl, b.xq, b.xs, B->wk, B->sk, nullptr, nullptr, kr, st));
  REEF_TRY(gemm_w8a8_f32(T, d, dl, b.xq, b.xs, B->wv, B->sv, nullptr, nullptr, vr, st));
  AttnHeadArgs aa{};
  aa.heads = static_cast<int>(B->heads);
  aa.query_len = static_cast<int>(T);
  aa.key_len = static_cast<int>(past + T);
  aa.head_dim = static_cast<int>(B->head_dim);
  aa.window = static_cast<int>(B->window);
  aa.query_start = static_cast<long long>(past);
  aa.q_stride = aa.kv_stride = aa.out_stride = dl;
  aa.q_head = aa.kv_head = aa.out_head = static_cast<long long>(B->head_dim);
  REEF_TRY(attention_head_f32(aa, b.q, kv != nullptr ? kv->k : b.k, kv != nullptr ? kv->v : b.v,
                              b.ctx, st));
  {
    auto quant = [&](const float* rm) {
      return quantize_rows(T, dl, b.ctx, b.xq, static_cast<long long>(kpad(dl)), b.xs, rm, st);
    };
    auto absmax = [&](float* rm) { return row_absmax(T, dl, b.ctx, rm, st); };
    REEF_TRY(rowpar_linear(c, T, dl, d, quant, absmax, B->wo, B->so, B->bo, x, b.xq, b.xs,
                           b.row_max, b.acc, b.a, st));
  }
  // MLP::forward (mlp.hpp:108-133): ln_2, c_fc (column-parallel) with gelu
  // in its epilogue, c_proj (row-parallel) with the second residual fused in.
  REEF_TRY(layernorm_exact_quant(T, d, B->eps, b.a, B->ln2_g, B->ln2_b, b.xq, ld, b.xs, st));
  REEF_TRY(gemm_w8a8_f32(T, d, F, b.xq, b.xs, B->wfc, B->sfc, B->bfc, nullptr, b.f, st,
                         /*gelu=*/true));
  {
    auto quant = [&](const float* rm) {
      return quantize_rows(T, F, b.f, b.xq, static_cast<long long>(kpad(F)), b.xs, rm, st);
    };
    auto absmax = [&](float* rm) { return row_absmax(T, F, b.f, rm, st); };
    REEF_TRY(rowpar_linear(c, T, F, d, quant, absmax, B->wproj, B->sproj, B->bproj, b.a, b.xq,
                           b.xs, b.row_max, b.acc, y, st));
  }
  return REEF_B200_OK;
}


// ---- float GPT-Neo block ----------------------------------------------------------------

int neo_f32_check(const reef_b200_gptneo_block_f32* B) {
  if (B == nullptr || B->seq == 0 || B->hidden == 0 || B->heads == 0 || B->head_dim == 0 ||
      B->ffn == 0 || B->seq > static_cast<size_t>(kMaxKeysExact) || B->seq > 65535 ||
      !B->ln1_g || !B->wq || !B->wk || !B->wv || !B->wo || !B->ln2_g || !B->wfc || !B->wproj)
    return REEF_B200_ERR_INVALID;
  return REEF_B200_OK;
}

struct NeoF32Bufs {
  float* h;    // layernormed rows [T][d]
  float* q;    // [T][dl]
  float* ctx;  // [T][dl]
  float* t;    // a sublayer's output [T][d]
  float* a;    // x + attention [T][d]
  float* f;    // [T][ffn]
};

size_t neo_f32_carve(const reef_b200_gptneo_block_f32* B, void* ws, NeoF32Bufs* b) {
  const size_t T = B->seq, d = B->hidden, dl = B->heads * B->head_dim;
  Carve c(ws, ~static_cast<size_t>(0));
  b->h = c.take<float>(T * d);
  b->q = c.take<float>(T * dl);
  b->ctx = c.take<float>(T * dl);
  b->t = c.take<float>(T * d);
  b->a = c.take<float>(T * d);
  b->f = c.take<float>(T * B->ffn);
  return c.used + 256;
}

// The firmware's float layer (gpt_neo.cc:136-176 with Precision::kFloat32)
// on `seq` new positions of this layer's cache: every operator exact, so the
// rows equal the engine's float Block<float>::forward.
int neo_f32_forward(const reef_b200_gptneo_block_f32* B, const float* x, float* y,
                    const NeoCache& kv, void* workspace, size_t workspace_bytes,
                    cudaStream_t st) {
  if (int rc = neo_f32_check(B)) return rc;
  NeoF32Bufs b;
  if (neo_f32_carve(B, workspace, &b) > workspace_bytes) return REEF_B200_ERR_INVALID;
  const long long T = static_cast<long long>(B->seq);
  const int d = static_cast<int>(B->hidden), dl = static_cast<int>(B->heads * B->head_dim),
            F = static_cast<int>(B->ffn);
  // x + attention(ln_1(x)): q/k/v without bias, the keys and values into the cache
  REEF_TRY(layernorm_exact(T, d, B->eps, x, B->ln1_g, B->ln1_b, b.h, st));
  REEF_TRY(linear_f32(T, d, dl, b.h, B->wq, nullptr, b.q, st));
  REEF_TRY(linear_f32(T, d, dl, b.h, B->wk, nullptr, kv.k + kv.position * dl, st));
  REEF_TRY(linear_f32(T, d, dl, b.h, B->wv, nullptr, kv.v + kv.position * dl, st));
  AttnHeadArgs aa{};
  aa.heads = static_cast<int>(B->heads);
  aa.query_len = static_cast<int>(T);
  aa.key_len = static_cast<int>(kv.position + T);
  aa.head_dim = static_cast<int>(B->head_dim);
  aa.window = static_cast<int>(B->window);
  aa.query_start = static_cast<long long>(kv.position);
  aa.q_stride = aa.kv_stride = aa.out_stride = dl;
  aa.q_head = aa.kv_head = aa.out_head = static_cast<long long>(B->head_dim);
  REEF_TRY(attention_head_f32(aa, b.q, kv.k, kv.v, b.ctx, st));
  REEF_TRY(linear_f32(T, dl, d, b.ctx, B->wo, B->bo, b.t, st));
  REEF_TRY(add_f32(T * d, x, b.t, b.a, st));
  // + mlp(ln_2(.)): c_fc + bias, gelu, c_proj + bias
  REEF_TRY(layernorm_exact(T, d, B->eps, b.a, B->ln2_g, B->ln2_b, b.h, st));
  REEF_TRY(linear_f32(T, d, F, b.h, B->wfc, B->bfc, b.f, st));
  REEF_TRY(unary_exact(kUnaryGelu, T * F, b.f, b.f, st));
  REEF_TRY(linear_f32(T, F, d, b.f, B->wproj, B->bproj, b.t, st));
  return add_f32(T * d, b.a, b.t, y, st);
}

// ---- GPT-Neo model step ------------------------------------------------------------------

// the cache row width (heads * head_dim) of a model's blocks
size_t model_width(const reef_b200_gptneo_model* m) {
  return m->blocks != nullptr ? m->blocks[0].heads * m->blocks[0].head_dim
                              : m->blocks_f32[0].heads * m->blocks_f32[0].head_dim;
}

int model_check(const reef_b200_gptneo_model* m, size_t count) {
  if (m == nullptr || (m->blocks == nullptr) == (m->blocks_f32 == nullptr) || m->layers == 0 ||
      m->vocab == 0 || m->max_positions == 0 || m->hidden == 0 || count == 0 ||
      count > static_cast<size_t>(kMaxKeysExact) || !m->wte || !m->wpe || !m->ln_f_g ||
      !m->ln_f_b || m->vocab > 0xffffffffull)
    return REEF_B200_ERR_INVALID;
  const size_t dl = model_width(m);
  for (size_t l = 0; l < m->layers; ++l) {
    if (m->blocks != nullptr) {
      reef_b200_gptneo_block blk = m->blocks[l];
      blk.seq = count;
      if (blk.hidden != m->hidden || blk.heads * blk.head_dim != dl ||
          neo_check(&blk) != REEF_B200_OK)
        return REEF_B200_ERR_INVALID;
    } else {
      reef_b200_gptneo_block_f32 blk = m->blocks_f32[l];
      blk.seq = count;
      if (blk.hidden != m->hidden || blk.heads * blk.head_dim != dl ||
          neo_f32_check(&blk) != REEF_B200_OK)
        return REEF_B200_ERR_INVALID;
    }
  }
  return REEF_B200_OK;
}

struct StepBufs {
  float* x[2];       // [count][hidden], ping-pong between blocks
  float* normed;     // [hidden]
  float* logits;     // [vocab] when the caller wants only the token
  void* block_ws;    // one block's workspace for `count` rows
  size_t block_bytes;
};

size_t step_carve(const reef_b200_gptneo_model* m, size_t count, void* ws, StepBufs* b) {
  Carve c(ws, ~static_cast<size_t>(0));
  b->x[0] = c.take<float>(count * m->hidden);
  b->x[1] = c.take<float>(count * m->hidden);
  b->normed = c.take<float>(m->hidden);
  b->logits = c.take<float>(m->vocab);
  size_t need = 0;
  for (size_t l = 0; l < m->layers; ++l) {
    if (m->blocks != nullptr) {
      reef_b200_gptneo_block blk = m->blocks[l];
      blk.seq = count;
      NeoBufs nb;
      need = std::max(need, neo_carve(&blk, nullptr, &nb));
    } else {
      reef_b200_gptneo_block_f32 blk = m->blocks_f32[l];
      blk.seq = count;
      NeoF32Bufs nb;
      need = std::max(need, neo_f32_carve(&blk, nullptr, &nb));
    }
  }
  b->block_bytes = need;
  b->block_ws = c.take<uint8_t>(need);
  return c.used + 256;
}

}  // namespace

extern "C" {

// ---- communicator -----------------------------------------------------------------

size_t reef_b200_comm_unique_id_bytes(void) { return comm_unique_id_bytes(); }

int reef_b200_comm_unique_id(void* id, size_t bytes) { return comm_unique_id(id, bytes); }

int reef_b200_comm_init(int rank, int world, const void* id, double timeout_s,
                        reef_b200_comm** comm) {
  if (comm == nullptr) return REEF_B200_ERR_INVALID;
  Comm* c = nullptr;
  const int rc = comm_init(rank, world, id, timeout_s, &c);
  *comm = reinterpret_cast<reef_b200_comm*>(c);
  return rc;
}

int reef_b200_comm_destroy(reef_b200_comm* comm) { return comm_destroy(C(comm)); }

int reef_b200_comm_abort(reef_b200_comm* comm) { return comm_abort(C(comm)); }

// ---- tensor-parallel linears -----------------------------------------------------

int reef_b200_linear_w8a8_rowpar(reef_b200_comm* comm, size_t rows, size_t in_local,
                                 size_t out, const float* x_local, const int8_t* w_shard,
                                 const float* w_scale, const float* bias, int8_t* x_q,
                                 float* x_scale, float* row_max, int32_t* acc, float* y,
                                 reef_b200_stream_t stream) {
  if (rows == 0) return REEF_B200_OK;
  if (in_local == 0 || out == 0 || rows > (1u << 31) - 1 || !x_local || !w_shard || !w_scale ||
      !x_q || !x_scale || !y)
    return REEF_B200_ERR_INVALID;
  if (comm != nullptr && comm_world(C(comm)) > 1 && (!row_max || !acc))
    return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  const long long R = static_cast<long long>(rows);
  const int K = static_cast<int>(in_local), N = static_cast<int>(out);
  cudaStream_t st = S(stream);
  auto quant = [&](const float* rm) {
    return quantize_rows(R, K, x_local, x_q, static_cast<long long>(kpad(in_local)), x_scale, rm,
                         st);
  };
  auto absmax = [&](float* rm) { return row_absmax(R, K, x_local, rm, st); };
  return rowpar_linear(C(comm), R, K, N, quant, absmax, w_shard, w_scale, bias, nullptr, x_q,
                       x_scale, row_max, acc, y, st);
}

// ---- Llama-shape layer -------------------------------------------------------------

size_t reef_b200_llama_layer_workspace_bytes(const reef_b200_llama_layer* L) {
  if (llama_check(L) != REEF_B200_OK) return 0;
  if (llama_allgather(L)) {
    LlamaAgBufs b;
    return llama_ag_carve(L, comm_world(C(L->comm)), nullptr, &b);
  }
  LlamaBufs b;
  return llama_carve(L, nullptr, &b);
}

size_t reef_b200_llama_layer_kernel_launches(const reef_b200_llama_layer* L) {
  if (llama_check(L) != REEF_B200_OK) return 0;
  // rmsnorm+quant, qkv GEMM, rope table, rope q/k, quant v, flash, o-proj,
  // rmsnorm+quant, gate/up GEMM, down; a row-parallel linear is quant + GEMM
  // (TP=1) or absmax + quant + int32 GEMM + dequant epilogue (TP>1)
  // rmsnorm+quant, rope table, QKV GEMM (RoPE + q/k/V^T packing in its
  // epilogue), flash, o-proj (quant + GEMM), rmsnorm+quant, gate/up GEMM (SwiGLU
  // and its row maxima in the epilogue), quant, down GEMM.  TP>1 all-reduce
  // plan: a row-parallel linear adds an absmax pass and an int32 epilogue pass
  // (the MLP's absmax comes from the gate/up GEMM); all-gather plan: each
  // RMSNorm is two passes (stats, apply) and the o-proj input an absmax pass.
  // The all-gather plan pipelined over k chunks of sequences runs each of its
  // 12 per-token kernels once per chunk, plus the push of the SwiGLU row
  // maxima (the RoPE table once).
  if (llama_allgather(L)) return ag_chunks(L) > 1 ? 13 * ag_chunks(L) + 1 : 13;
  return L->comm != nullptr ? 13 : 10;
}

static int llama_forward(const reef_b200_llama_layer* L, const float* x, float* y,
                         void* workspace, size_t workspace_bytes, cudaEvent_t* ev,
                         reef_b200_stream_t stream);

int reef_b200_llama_layer_forward(const reef_b200_llama_layer* L, const float* x, float* y,
                                  void* workspace, size_t workspace_bytes,
                                  reef_b200_stream_t stream) {
  return llama_forward(L, x, y, workspace, workspace_bytes, nullptr, stream);
}

int reef_b200_llama_layer_forward_events(const reef_b200_llama_layer* L, const float* x,
                                         float* y, void* workspace, size_t workspace_bytes,
                                         void* const* events, reef_b200_stream_t stream) {
  if (events == nullptr) return REEF_B200_ERR_INVALID;
  cudaEvent_t ev[10];
  for (int i = 0; i < 10; ++i) {
    if (events[i] == nullptr) return REEF_B200_ERR_INVALID;
    ev[i] = static_cast<cudaEvent_t>(events[i]);
  }
  return llama_forward(L, x, y, workspace, workspace_bytes, ev, stream);
}

// Events of the pipelined forward, destroyed on every exit (a pending event
// may be destroyed; its resources go when it completes).
struct EventSet {
  std::vector<cudaEvent_t> ev;
  explicit EventSet(int n) : ev(n, nullptr) {}
  int create() {
    for (auto& e : ev)
      if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return kErrCuda;
    return kOk;
  }
  ~EventSet() {
    for (auto e : ev)
      if (e != nullptr) cudaEventDestroy(e);
  }
};

// The all-gather plan, pipelined over chunks of whole sequences.  Chunk k's
// kernels run on the communicator's compute stream k.  The data a step
// exchanges lives in the communicator's symmetric arena, one region per chunk
// and kind (int8 activations, RMSNorm chunk sums, row maxima), laid out
// [rank][rows][...]: the kernel that produces a rank's segment writes it
// straight into every rank's arena over NVLink (its stores go to the peers'
// mapped arenas; on 4 GPUs that moves ~550-620 GB/s per GPU against
// ~300-350 GB/s for copy-engine copies, and no separate transfer step waits
// in between).  The gate/up GEMM takes its row maxima with atomics locally,
// and a small kernel pushes them.  After a producing step the rank increments
// the region's "delivered" counter in every peer's arena (a system-wide fence
// orders the kernel's stores first); a consuming step waits until its local
// counter shows every peer's delivery, and afterwards increments the
// region's "consumed" counter in every peer's arena; a producing step writes
// a region only once every peer has consumed its previous contents.  Counter
// targets derive from (forward round, use), so counters only grow.  Every
// wait is a bounded spin on the device (signal_and_wait): after the
// communicator's timeout it records kDevTimeoutPeer and lets the stream go
// on, so a peer that died cannot leave this rank's streams waiting.  Steps
// are issued wavefront-wise so that every rank issues the same sequence;
// each wait depends only on steps issued earlier on some rank, so the
// pipeline cannot deadlock.  Each chunk computes exactly what the
// unpipelined plan computes for its rows, so the result is identical.
static int llama_forward_ag_pipelined(const reef_b200_llama_layer* L, const float* x, float* y,
                                      const LlamaAgBufs& b, int chunks, cudaStream_t st) {
  Comm* c = C(L->comm);
  const int N = comm_world(c), rank = comm_rank(c);
  if (chunks > kComputeStreams) return REEF_B200_ERR_INVALID;
  const int H = static_cast<int>(L->hidden), hq = static_cast<int>(L->heads_q),
            hkv = static_cast<int>(L->heads_kv), F = static_cast<int>(L->ffn), D = 128;
  const int seq = static_cast<int>(L->seq);
  const int Hl = H / N, S = 8 / N + 1, qkv_w = (hq + 2 * hkv) * D;
  const long long kmax = std::max({Hl, hq * D, F});
  const int bc = static_cast<int>(L->batch) / chunks;  // sequences per chunk
  const long long Tc = static_cast<long long>(bc) * seq;
  const float* g1 = L->attn_norm + static_cast<long long>(rank) * Hl;
  const float* g2 = L->mlp_norm + static_cast<long long>(rank) * Hl;

  // arena: per chunk [XQ: N*Tc*kmax B][ST: N*Tc*S f32][MX: N*Tc f32], 256-B aligned
  auto al = [](long long v) { return (v + 255) & ~255ll; };
  const long long xq_bytes = al(N * Tc * kmax), st_bytes = al(N * Tc * S * 4),
                  mx_bytes = al(N * Tc * 4);
  const long long chunk_bytes = xq_bytes + st_bytes + mx_bytes;
  enum Kind { kXq = 0, kSt = 1, kMx = 2 };
  constexpr int kUses[3] = {4, 2, 2};  // per forward
  REEF_TRY(comm_arena_reserve(c, static_cast<size_t>(chunk_bytes * chunks), 6 * chunks));
  uint8_t* arena = comm_arena_data(c);
  const uint32_t round = comm_next_round(c);
  auto region_off = [&](int k, Kind kind) {
    return k * chunk_bytes + (kind == kXq ? 0 : kind == kSt ? xq_bytes : xq_bytes + st_bytes);
  };
  auto data_slot = [&](int k, Kind kind) { return 6 * k + 2 * kind; };
  auto cons_slot = [&](int k, Kind kind) { return 6 * k + 2 * kind + 1; };
  auto epoch = [&](Kind kind, int use) {
    return static_cast<uint32_t>((round - 1) * kUses[kind] + use + 1);
  };
  auto xq_all = [&](int k) { return reinterpret_cast<int8_t*>(arena + region_off(k, kXq)); };
  auto st_all = [&](int k) { return reinterpret_cast<float*>(arena + region_off(k, kSt)); };
  auto mx_all = [&](int k) { return reinterpret_cast<float*>(arena + region_off(k, kMx)); };
  // this rank's segment of the row-max region here
  auto mx_mine = [&](int k) { return mx_all(k) + rank * Tc; };

  EventSet done(chunks), fork(1);
  REEF_TRY(done.create());
  REEF_TRY(fork.create());
  auto sk = [&](int k) { return comm_compute_stream(c, k); };
  REEF_TRY(rope_table(seq, L->rope_base, b.rope, st));
  if (cudaEventRecord(fork.ev[0], st) != cudaSuccess) return REEF_B200_ERR_CUDA;
  for (int k = 0; k < chunks; ++k)
    if (cudaStreamWaitEvent(sk(k), fork.ev[0], 0) != cudaSuccess) return REEF_B200_ERR_CUDA;

  // A step of chunk k on its own stream.  It waits until every peer has
  // delivered the uses of the regions it reads (`ins`) and has consumed the
  // previous use of the regions it writes (`outs`: it writes them into every
  // rank's arena, its own included); after the kernels it marks its inputs
  // consumed and its outputs delivered, on every peer: each region has a
  // "delivered" and a "consumed" counter that every peer increments once per
  // use (system-scope atomics after the step), so a step waits on one
  // counter per region instead of one flag per peer.  A peer cannot run
  // two uses ahead (producing use e + 1 needs this rank's consumption of use
  // e), so a counter never passes a target early.  Chunk k's step also
  // waits for chunk k - 1's same step, so the chunks run one step apart: the
  // NVLink-bound steps (the quantisers that write to every peer) of one
  // chunk overlap the tensor-bound steps (GEMMs, flash) of its neighbour
  // instead of running beside their own kind.
  struct Use {
    Kind kind;
    int use;
  };
  // Chunk k's signals of its last step wait to go out with the first kernel
  // of its next step: one launch increments the peers' counters (after a
  // system-wide fence) and then waits, with the communicator's deadline, for
  // this step's local counters.  A wait that runs out records
  // kDevTimeoutPeer and returns, so a peer that never signals cannot hang
  // this stream.
  std::vector<PeerFlags> pending(chunks);
  const unsigned long long limit_ns = comm_wait_limit_ns(c);
  auto step = [&](int k, std::initializer_list<Use> ins, std::initializer_list<Use> outs,
                  auto&& fn) -> int {
    const uint32_t peers = static_cast<uint32_t>(N - 1);
    CounterWaits w;
    if (static_cast<int>(ins.size() + outs.size()) > kMaxWaits) return kErrInvalid;
    for (const Use& i : ins) {
      w.p[w.n] = comm_local_counter(c, data_slot(k, i.kind));
      w.target[w.n++] = epoch(i.kind, i.use) * peers;
    }
    for (const Use& o : outs) {
      w.p[w.n] = comm_local_counter(c, cons_slot(k, o.kind));
      w.target[w.n++] = (epoch(o.kind, o.use) - 1) * peers;
    }
    REEF_TRY(signal_and_wait(pending[k], w, limit_ns, sk(k)));
    pending[k] = PeerFlags{};
    if (k > 0 && cudaStreamWaitEvent(sk(k), done.ev[k - 1], 0) != cudaSuccess) return kErrCuda;
    REEF_TRY(fn(sk(k)));
    PeerFlags& f = pending[k];
    if ((N - 1) * static_cast<int>(ins.size() + outs.size()) > kMaxFlags) return kErrInvalid;
    for (int r = 0; r < N; ++r) {
      if (r == rank) continue;
      for (const Use& i : ins) f.p[f.n++] = comm_counter(c, cons_slot(k, i.kind), r);
      for (const Use& o : outs) f.p[f.n++] = comm_counter(c, data_slot(k, o.kind), r);
    }
    return cudaEventRecord(done.ev[k], sk(k)) == cudaSuccess ? kOk : kErrCuda;
  };
  // this rank's segment of region (k, kind) in every rank's arena (the [N][Tc][w]
  // layout of the step's width w, bytes per row given)
  static_assert(kMaxDst >= 8, "the all-gather plan runs on up to 8 ranks");
  auto everywhere = [&](int k, Kind kind, long long row_bytes, bool self) {
    PeerDst d;
    for (int r = 0; r < N; ++r) {
      if (r == rank && !self) continue;
      d.p[d.n++] = comm_peer_data(c, r) + region_off(k, kind) + rank * Tc * row_bytes;
    }
    return d;
  };
  auto xq_to = [&](int k, long long kl) { return everywhere(k, kXq, kl, true); };
  auto st_to = [&](int k) { return everywhere(k, kSt, S * 4, true); };
  auto mx_to = [&](int k, bool self) { return everywhere(k, kMx, 4, self); };
  // per-chunk views of the workspace
  auto xk = [&](int k) { return x + k * Tc * Hl; };
  auto hk = [&](int k) { return b.h + k * Tc * Hl; };
  auto xsk = [&](int k) { return b.xs + k * Tc; };
  auto rmk = [&](int k) { return b.row_max + k * Tc; };
  auto attnk = [&](int k) { return b.attn + k * Tc * hq * D; };
  auto bigk = [&](int k) { return b.big + k * Tc * F; };
  // the gathered activation [N][Tc][kl] of chunk k times this rank's rows of W
  auto problem_k = [&](int k, int kl, const int8_t* w, int n, const float* ws, float* out) {
    GemmProblem p{};
    p.M = static_cast<int>(Tc);
    p.N = n;
    p.K = kl;
    p.a = xq_all(k);
    p.lda = kl;
    p.a_seg = Tc * kl;
    p.b = w;
    p.ldb = static_cast<long long>(kl) * N;
    p.b_seg = kl;
    p.args.k_segments = N;
    p.args.x_scale = xsk(k);
    p.args.w_scale = ws;
    p.args.y = out;
    p.args.ldy = n;
    p.args.max_ctas = ag_gemm_sms();
    return p;
  };

  // ---- attention block
  for (int k = 0; k < chunks; ++k)
    REEF_TRY(step(k, {}, {{kSt, 0}}, [&](cudaStream_t s) {
      return rms_stats(Tc, H, N, xk(k), g1, st_to(k), s);
    }));
  for (int k = 0; k < chunks; ++k)
    REEF_TRY(step(k, {{kSt, 0}}, {{kXq, 0}}, [&](cudaStream_t s) {
      return rms_apply_quant(Tc, H, N, L->rms_eps, xk(k), g1, st_all(k), xq_to(k, Hl), xsk(k), s);
    }));
  for (int k = 0; k < chunks; ++k)
    REEF_TRY(step(k, {{kXq, 0}}, {}, [&](cudaStream_t s) {
      uint16_t* vt = static_cast<uint16_t*>(b.vt) + static_cast<long long>(k) * bc * hkv * D * seq;
      GemmProblem p = problem_k(k, Hl, L->w_qkv, qkv_w, L->s_qkv, nullptr);
      p.args.qkv = qkv_out(L, hq, hkv, b.q8 + k * Tc * hq * D, b.k8 + k * Tc * hkv * D,
                           b.qs + static_cast<long long>(k) * bc * hq * seq,
                           b.ks + static_cast<long long>(k) * bc * hkv * seq, vt, b.rope);
      return gemm_i8(p, kEpiQkvRope, s);
    }));
  for (int k = 0; k < chunks; ++k)
    REEF_TRY(step(k, {}, {{kMx, 0}}, [&](cudaStream_t s) {
      FlashProblem fp{};
      fp.batch = bc;
      fp.heads_q = hq;
      fp.heads_kv = hkv;
      fp.seq = seq;
      fp.head_dim = D;
      fp.causal = 1;
      fp.sm_scale = 0.08838834764831845f;
      fp.q8 = b.q8 + k * Tc * hq * D;
      fp.k8 = b.k8 + k * Tc * hkv * D;
      fp.vt = static_cast<uint16_t*>(b.vt) + static_cast<long long>(k) * bc * hkv * D * seq;
      fp.q_scale = b.qs + static_cast<long long>(k) * bc * hq * seq;
      fp.k_scale = b.ks + static_cast<long long>(k) * bc * hkv * seq;
      fp.out = attnk(k);
      fp.out_ld = static_cast<long long>(hq) * D;
      REEF_TRY(flash_prefill_i8(fp, s));
      return row_absmax_to(Tc, hq * D, attnk(k), mx_to(k, true), s);
    }));
  for (int k = 0; k < chunks; ++k)
    REEF_TRY(step(k, {{kMx, 0}}, {{kXq, 1}}, [&](cudaStream_t s) {
      REEF_TRY(max_segments(N, Tc, mx_all(k), rmk(k), s));
      return quantize_rows_to(Tc, hq * D, attnk(k), xq_to(k, hq * D), hq * D, xsk(k), rmk(k), s);
    }));
  for (int k = 0; k < chunks; ++k)
    REEF_TRY(step(k, {{kXq, 1}}, {}, [&](cudaStream_t s) {
      GemmProblem p = problem_k(k, hq * D, L->w_o, Hl, L->s_o, hk(k));
      p.args.residual = xk(k);
      return gemm_i8(p, kEpiF32W8A8, s);
    }));
  // ---- MLP block
  for (int k = 0; k < chunks; ++k)
    REEF_TRY(step(k, {}, {{kSt, 1}}, [&](cudaStream_t s) {
      return rms_stats(Tc, H, N, hk(k), g2, st_to(k), s);
    }));
  for (int k = 0; k < chunks; ++k)
    REEF_TRY(step(k, {{kSt, 1}}, {{kXq, 2}}, [&](cudaStream_t s) {
      return rms_apply_quant(Tc, H, N, L->rms_eps, hk(k), g2, st_all(k), xq_to(k, Hl), xsk(k), s);
    }));
  // gate/up: the SwiGLU epilogue takes each row's max with atomics into this
  // rank's segment here; it is then pushed to the peers
  for (int k = 0; k < chunks; ++k)
    REEF_TRY(step(k, {{kXq, 2}}, {{kMx, 1}}, [&](cudaStream_t s) {
      if (cudaMemsetAsync(mx_mine(k), 0, static_cast<size_t>(Tc) * sizeof(float), s) != cudaSuccess)
        return static_cast<int>(kErrCuda);
      GemmProblem p = problem_k(k, Hl, L->w_gu, F, L->s_gu, bigk(k));
      p.args.b_up = F;
      p.args.row_max = mx_mine(k);
      REEF_TRY(gemm_i8(p, kEpiSwiGLU, s));
      return push_f32(Tc, mx_mine(k), mx_to(k, false), s);
    }));
  for (int k = 0; k < chunks; ++k)
    REEF_TRY(step(k, {{kMx, 1}}, {{kXq, 3}}, [&](cudaStream_t s) {
      REEF_TRY(max_segments(N, Tc, mx_all(k), rmk(k), s));
      return quantize_rows_to(Tc, F, bigk(k), xq_to(k, F), F, xsk(k), rmk(k), s);
    }));
  for (int k = 0; k < chunks; ++k)
    REEF_TRY(step(k, {{kXq, 3}}, {}, [&](cudaStream_t s) {
      GemmProblem p = problem_k(k, F, L->w_down, Hl, L->s_down, y + k * Tc * Hl);
      p.args.residual = hk(k);
      return gemm_i8(p, kEpiF32W8A8, s);
    }));
  // the last steps' signals, then join: the caller's stream waits for every
  // chunk's last kernel
  for (int k = 0; k < chunks; ++k) {
    REEF_TRY(signal_and_wait(pending[k], CounterWaits{}, limit_ns, sk(k)));
    if (cudaEventRecord(done.ev[k], sk(k)) != cudaSuccess) return REEF_B200_ERR_CUDA;
    if (cudaStreamWaitEvent(st, done.ev[k], 0) != cudaSuccess) return REEF_B200_ERR_CUDA;
  }
  return REEF_B200_OK;
}

// The all-gather plan (REEF_B200_TP_ALLGATHER): x, y and the residual are
// this rank's hidden/world columns; every projection reads the all-gathered
// int8 activation (rank-major [world][tokens][K/world], consumed as K
// segments by the GEMM's 3-D tensor maps) and writes this rank's output rows.
static int llama_forward_ag(const reef_b200_llama_layer* L, const float* x, float* y,
                            void* workspace, size_t workspace_bytes, cudaEvent_t* ev,
                            cudaStream_t st) {
  Comm* c = C(L->comm);
  const int N = comm_world(c), rank = comm_rank(c);
  LlamaAgBufs b;
  if (llama_ag_carve(L, N, workspace, &b) > workspace_bytes) return REEF_B200_ERR_INVALID;
  // the instrumented forward (per-kernel spans) runs the steps in sequence
  if (ev == nullptr && ag_chunks(L) > 1)
    return llama_forward_ag_pipelined(L, x, y, b, ag_chunks(L), st);
  const long long T = static_cast<long long>(L->batch * L->seq);
  const int H = static_cast<int>(L->hidden), hq = static_cast<int>(L->heads_q),
            hkv = static_cast<int>(L->heads_kv), F = static_cast<int>(L->ffn), D = 128;
  const int Hl = H / N, S = 8 / N + 1, qkv_w = (hq + 2 * hkv) * D;
  const float* g1 = L->attn_norm + static_cast<long long>(rank) * Hl;
  const float* g2 = L->mlp_norm + static_cast<long long>(rank) * Hl;

  // all-gathered activation [N][T][kl] times this rank's rows of W [n][N*kl]
  auto seg_problem = [&](int kl, const int8_t* w, int n, const float* ws, float* out) {
    GemmProblem p{};
    p.M = static_cast<int>(T);
    p.N = n;
    p.K = kl;
    p.a = b.xq_all;
    p.lda = kl;
    p.a_seg = T * kl;
    p.b = w;
    p.ldb = static_cast<long long>(kl) * N;
    p.b_seg = kl;
    p.args.k_segments = N;
    p.args.x_scale = b.xs;
    p.args.w_scale = ws;
    p.args.y = out;
    p.args.ldy = n;
    return p;
  };
  auto gemm_seg = [&](int kl, const int8_t* w, int n, const float* ws, const float* residual,
                      float* out, cudaEvent_t* e) -> int {
    GemmProblem p = seg_problem(kl, w, n, ws, out);
    p.args.residual = residual;
    Span sp(e, st);
    return gemm_i8(p, kEpiF32W8A8, st);
  };
  auto rms = [&](const float* xin, const float* g) -> int {
    REEF_TRY(rms_stats(T, H, N, xin, g, one_dst(b.stats), st));
    REEF_TRY(allgather_bytes(c, b.stats, b.stats_all, static_cast<size_t>(T) * S * 4, st));
    REEF_TRY(rms_apply_quant(T, H, N, L->rms_eps, xin, g, b.stats_all, one_dst(b.xq), b.xs, st));
    return allgather_bytes(c, b.xq, b.xq_all, static_cast<size_t>(T) * Hl, st);
  };

  REEF_TRY(rms(x, g1));
  // QKV projection with RoPE and the int8 q / k / V^T packing in its epilogue
  REEF_TRY(rope_table(static_cast<int>(L->seq), L->rope_base, b.rope, st));
  {
    GemmProblem p = seg_problem(Hl, L->w_qkv, qkv_w, L->s_qkv, nullptr);
    p.args.qkv = qkv_out(L, hq, hkv, b.q8, b.k8, b.qs, b.ks, b.vt, b.rope);
    Span sp(ev ? ev + 0 : nullptr, st);
    REEF_TRY(gemm_i8(p, kEpiQkvRope, st));
  }
  FlashProblem fp{};
  fp.batch = static_cast<int>(L->batch);
  fp.heads_q = hq;
  fp.heads_kv = hkv;
  fp.seq = static_cast<int>(L->seq);
  fp.head_dim = D;
  fp.causal = 1;
  fp.sm_scale = 0.08838834764831845f;
  fp.q8 = b.q8;
  fp.k8 = b.k8;
  fp.vt = b.vt;
  fp.q_scale = b.qs;
  fp.k_scale = b.ks;
  fp.out = b.attn;
  fp.out_ld = static_cast<long long>(hq) * D;
  {
    Span sp(ev ? ev + 2 : nullptr, st);
    REEF_TRY(flash_prefill_i8(fp, st));
  }
  // o-proj: full-row scale of the attention output, then gather its codes
  REEF_TRY(row_absmax(T, hq * D, b.attn, b.row_max, st));
  REEF_TRY(allreduce_max_f32(c, b.row_max, static_cast<size_t>(T), st));
  REEF_TRY(quantize_rows(T, hq * D, b.attn, b.xq, hq * D, b.xs, b.row_max, st));
  REEF_TRY(allgather_bytes(c, b.xq, b.xq_all, static_cast<size_t>(T) * hq * D, st));
  REEF_TRY(gemm_seg(hq * D, L->w_o, Hl, L->s_o, x, b.h, ev ? ev + 4 : nullptr));
  // MLP
  REEF_TRY(rms(b.h, g2));
  {
    // gate/up + SwiGLU in the GEMM epilogue: h [T][F] and its local row maxima
    if (cudaMemsetAsync(b.row_max, 0, static_cast<size_t>(T) * sizeof(float), st) != cudaSuccess)
      return REEF_B200_ERR_CUDA;
    GemmProblem p = seg_problem(Hl, L->w_gu, F, L->s_gu, b.big);
    p.args.b_up = F;
    p.args.row_max = b.row_max;
    Span sp(ev ? ev + 6 : nullptr, st);
    REEF_TRY(gemm_i8(p, kEpiSwiGLU, st));
  }
  REEF_TRY(allreduce_max_f32(c, b.row_max, static_cast<size_t>(T), st));
  REEF_TRY(quantize_rows(T, F, b.big, b.xq, F, b.xs, b.row_max, st));
  REEF_TRY(allgather_bytes(c, b.xq, b.xq_all, static_cast<size_t>(T) * F, st));
  return gemm_seg(F, L->w_down, Hl, L->s_down, b.h, y, ev ? ev + 8 : nullptr);
}

static int llama_forward(const reef_b200_llama_layer* L, const float* x, float* y,
                         void* workspace, size_t workspace_bytes, cudaEvent_t* ev,
                         reef_b200_stream_t stream) {
  if (int rc = llama_check(L)) return rc;
  if (llama_allgather(L)) {
    if (!x || !y || !workspace) return REEF_B200_ERR_INVALID;
    if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return REEF_B200_ERR_ALIGNMENT;
    if (int rc = check_device()) return rc;
    return llama_forward_ag(L, x, y, workspace, workspace_bytes, ev, S(stream));
  }
  if (!x || !y || !workspace) return REEF_B200_ERR_INVALID;
  LlamaBufs b;
  if (llama_carve(L, workspace, &b) > workspace_bytes) return REEF_B200_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return REEF_B200_ERR_ALIGNMENT;
  if (int rc = check_device()) return rc;
  cudaStream_t st = S(stream);
  Comm* c = C(L->comm);
  const long long T = static_cast<long long>(L->batch * L->seq);
  const int H = static_cast<int>(L->hidden), hq = static_cast<int>(L->heads_q),
            hkv = static_cast<int>(L->heads_kv), F = static_cast<int>(L->ffn), D = 128;
  const int qkv_w = (hq + 2 * hkv) * D;
  // With REEF_B200_PREFILL_PDL=1 (and no communicator, no per-kernel spans)
  // every kernel goes out as a programmatic dependent of the one before: its
  // CTAs start on the SMs the previous kernel's last CTAs free, and each
  // waits for that kernel to finish before it reads its output.
  PdlScope pdl;
  if (comm_world(c) != 1 || ev != nullptr || !prefill_pdl()) t_pdl = pdl.prev;

  // attention block: y_attn = x + o_proj(attn(rope(qkv(rmsnorm(x)))))
  REEF_TRY(rmsnorm_quant(T, H, L->rms_eps, x, L->attn_norm, b.xq, b.xs, st));
  // QKV projection with RoPE and the int8 q / k / V^T packing in its epilogue
  REEF_TRY(rope_table(static_cast<int>(L->seq), L->rope_base, b.rope, st));
  {
    GemmProblem p = problem(T, H, qkv_w, b.xq, L->w_qkv);
    p.args.x_scale = b.xs;
    p.args.w_scale = L->s_qkv;
    p.args.qkv = qkv_out(L, hq, hkv, b.q8, b.k8, b.qs, b.ks, b.vt, b.rope);
    Span sp(ev ? ev + 0 : nullptr, st);
    REEF_TRY(gemm_i8(p, kEpiQkvRope, st));
  }
  FlashProblem fp{};
  fp.batch = static_cast<int>(L->batch);
  fp.heads_q = hq;
  fp.heads_kv = hkv;
  fp.seq = static_cast<int>(L->seq);
  fp.head_dim = D;
  fp.causal = 1;
  fp.sm_scale = 0.08838834764831845f;  // 1 / sqrt(128)
  fp.q8 = b.q8;
  fp.k8 = b.k8;
  fp.vt = b.vt;
  fp.q_scale = b.qs;
  fp.k_scale = b.ks;
  fp.out = b.attn;
  fp.out_ld = static_cast<long long>(hq) * D;
  {
    Span sp(ev ? ev + 2 : nullptr, st);
    REEF_TRY(flash_prefill_i8(fp, st));
  }
  {
    auto quant = [&](const float* rm) {
      return quantize_rows(T, hq * D, b.attn, b.xq, static_cast<long long>(kpad(hq * D)), b.xs,
                           rm, st);
    };
    auto absmax = [&](float* rm) { return row_absmax(T, hq * D, b.attn, rm, st); };
    REEF_TRY(rowpar_linear(c, T, hq * D, H, quant, absmax, L->w_o, L->s_o, nullptr, x, b.xq,
                           b.xs, b.row_max, b.acc, b.h, st, ev ? ev + 4 : nullptr));
  }
  // MLP block: y = h + down(swiglu(gate_up(rmsnorm(h))))
  REEF_TRY(rmsnorm_quant(T, H, L->rms_eps, b.h, L->mlp_norm, b.xq, b.xs, st));
  {
    // gate/up + SwiGLU in the GEMM epilogue: h [T][F] and its local row maxima
    Span sp(ev ? ev + 6 : nullptr, st);
    REEF_TRY(linear_w8a8_swiglu(T, H, F, b.xq, b.xs, L->w_gu, L->s_gu, b.big, b.row_max, st));
  }
  {
    auto quant = [&](const float*) {
      return quantize_rows(T, F, b.big, b.xq, F, b.xs, b.row_max, st);
    };
    auto absmax = [&](float*) { return static_cast<int>(kOk); };  // written by the GEMM
    REEF_TRY(rowpar_linear(c, T, F, H, quant, absmax, L->w_down, L->s_down, nullptr, b.h, b.xq,
                           b.xs, b.row_max, b.acc, y, st, ev ? ev + 8 : nullptr));
  }
  return REEF_B200_OK;
}

// ---- Llama-shape decode step ---------------------------------------------------------

size_t reef_b200_llama_decode_workspace_bytes(const reef_b200_llama_layer* L, size_t max_len) {
  if (decode_check(L, max_len) != REEF_B200_OK || check_device() != kOk) return 0;
  DecodeBufs b;
  return decode_carve(L, max_len, nullptr, &b);
}

int reef_b200_llama_decode_forward(const reef_b200_llama_layer* L, const float* x, float* y,
                                   const int32_t* positions, int8_t* k_cache, float* k_scale,
                                   int8_t* v_cache, float* v_scale, size_t max_len,
                                   void* workspace, size_t workspace_bytes,
                                   reef_b200_stream_t stream) {
  if (int rc = decode_check(L, max_len)) return rc;
  if (!x || !y || !positions || !k_cache || !k_scale || !v_cache || !v_scale || !workspace)
    return REEF_B200_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0 ||
      (reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) % 16 != 0)
    return REEF_B200_ERR_ALIGNMENT;
  if (int rc = check_device()) return rc;
  DecodeBufs b;
  if (decode_carve(L, max_len, workspace, &b) > workspace_bytes) return REEF_B200_ERR_INVALID;
  cudaStream_t st = S(stream);
  Comm* c = C(L->comm);
  const int B = static_cast<int>(L->batch), H = static_cast<int>(L->hidden),
            hq = static_cast<int>(L->heads_q), hkv = static_cast<int>(L->heads_kv),
            F = static_cast<int>(L->ffn), D = 128;
  const int qkv_w = (hq + 2 * hkv) * D;
  int32_t* part = static_cast<int32_t*>(b.partial);
  // Every kernel of the step launches as a programmatic dependent of the one
  // before it: its launch and set-up, and the skinny GEMMs' weight loads (no
  // kernel writes the weights), overlap the kernel ahead.  The QKV and
  // gate/up GEMMs leave int32 split-K partials that the next kernel sums
  // itself (RoPE + cache append; SwiGLU + quantisation), so no separate
  // reduce runs between them.
  PdlScope pdl;
  REEF_TRY(rmsnorm_quant(B, H, L->rms_eps, x, L->attn_norm, b.xq, b.xs, st));
  const int s_qkv = skinny_split_count(B, qkv_w, H);
  REEF_TRY(gemm_i8_skinny_partials(B, qkv_w, H, b.xq, L->w_qkv, part, st, L->t_qkv));
  REEF_TRY(decode_rope_append_partials(B, hq, hkv, static_cast<int>(max_len), L->rope_base,
                                       positions, part, s_qkv, b.xs, L->s_qkv, b.q8, b.qs,
                                       k_cache, k_scale, v_cache, v_scale, b.lens, st));
  DecodeProblem dp{};
  dp.batch = B;
  dp.heads_q = hq;
  dp.heads_kv = hkv;
  dp.max_len = static_cast<int>(max_len);
  dp.sm_scale = 0.08838834764831845f;  // 1 / sqrt(128)
  dp.q8 = b.q8;
  dp.q_scale = b.qs;
  dp.k_cache = k_cache;
  dp.k_scale = k_scale;
  dp.v_cache = v_cache;
  dp.v_scale = v_scale;
  dp.lens = b.lens;
  dp.positions = positions;
  dp.partial = b.dpart;
  dp.out = b.attn;
  REEF_TRY(decode_attn_i8(dp, st));
  // o-proj with the residual, then the MLP's pre-norm: without a peer to
  // share the rows with, the o-proj's split-K sum, the residual and RMSNorm +
  // quant run as one kernel; the gate/up input scales go to xs2
  const int kq = static_cast<int>(hq * D);
  if (comm_world(c) == 1) {
    REEF_TRY(quantize_rows(B, kq, b.attn, b.xq, static_cast<long long>(kpad(kq)), b.xs, nullptr,
                           st));
    REEF_TRY(gemm_i8_skinny_partials(B, H, kq, b.xq, L->w_o, part, st, L->t_o));
    REEF_TRY(reduce_rmsnorm_quant(B, H, skinny_split_count(B, H, kq), part, b.xs, L->s_o, x, b.h,
                                  L->rms_eps, L->mlp_norm, b.xq, b.xs2, st));
  } else {
    auto quant = [&](const float* rm) {
      return quantize_rows(B, kq, b.attn, b.xq, static_cast<long long>(kpad(kq)), b.xs, rm, st);
    };
    auto absmax = [&](float* rm) { return row_absmax(B, kq, b.attn, rm, st); };
    REEF_TRY(rowpar_skinny(c, B, kq, H, quant, absmax, L->w_o, L->s_o, x, b.xq, b.xs, b.row_max,
                           b.acc, b.partial, b.h, st, L->t_o));
    REEF_TRY(rmsnorm_quant(B, H, L->rms_eps, b.h, L->mlp_norm, b.xq, b.xs2, st));
  }
  const int s_gu = skinny_split_count(B, 2 * F, H);
  REEF_TRY(gemm_i8_skinny_partials(B, 2 * F, H, b.xq, L->w_gu, part, st, L->t_gu));
  {
    // the down projection's input scales go back to xs (gate/up's are read
    // from xs2 meanwhile)
    auto quant = [&](const float* rm) {
      return swiglu_partials(B, F, part, s_gu, b.xs2, L->s_gu, rm, nullptr, b.xq, b.xs, st);
    };
    auto absmax = [&](float* rm) {
      return swiglu_partials(B, F, part, s_gu, b.xs2, L->s_gu, nullptr, rm, nullptr, nullptr, st);
    };
    REEF_TRY(rowpar_skinny(c, B, F, H, quant, absmax, L->w_down, L->s_down, b.h, b.xq, b.xs,
                           b.row_max, b.acc, b.partial, y, st, L->t_down));
  }
  return REEF_B200_OK;
}

// ---- GPT-Neo W8A8 block ---------------------------------------------------------------

size_t reef_b200_gptneo_block_workspace_bytes(const reef_b200_gptneo_block* B) {
  if (neo_check(B) != REEF_B200_OK) return 0;
  NeoBufs b;
  return neo_carve(B, nullptr, &b);
}

int reef_b200_gptneo_block_forward(const reef_b200_gptneo_block* B, const float* x, float* y,
                                   void* workspace, size_t workspace_bytes,
                                   reef_b200_stream_t stream) {
  return neo_forward(B, x, y, nullptr, workspace, workspace_bytes, S(stream));
}

int reef_b200_gptneo_block_forward_cached(const reef_b200_gptneo_block* B, const float* x,
                                          float* y, size_t position, float* k_cache,
                                          float* v_cache, size_t max_tokens, void* workspace,
                                          size_t workspace_bytes, reef_b200_stream_t stream) {
  if (!k_cache || !v_cache || B == nullptr || max_tokens > static_cast<size_t>(kMaxKeysExact) ||
      position > max_tokens || B->seq > max_tokens - position)
    return REEF_B200_ERR_INVALID;
  const NeoCache kv{k_cache, v_cache, position};
  return neo_forward(B, x, y, &kv, workspace, workspace_bytes, S(stream));
}

// ---- GPT-Neo decode loop ---------------------------------------------------------------

size_t reef_b200_gptneo_step_workspace_bytes(const reef_b200_gptneo_model* m, size_t count) {
  if (model_check(m, count) != REEF_B200_OK) return 0;
  StepBufs b;
  return step_carve(m, count, nullptr, &b);
}

int reef_b200_gptneo_step(const reef_b200_gptneo_model* m, const uint32_t* ids, size_t count,
                          size_t position, float* k_cache, float* v_cache, size_t max_tokens,
                          float* logits, uint32_t* next_id, void* workspace,
                          size_t workspace_bytes, reef_b200_stream_t stream) {
  if (int rc = model_check(m, count)) return rc;
  if (!ids || !k_cache || !v_cache || !workspace || max_tokens > m->max_positions ||
      max_tokens > static_cast<size_t>(kMaxKeysExact) || position > max_tokens ||
      count > max_tokens - position)
    return REEF_B200_ERR_INVALID;
  if (reinterpret_cast<uintptr_t>(workspace) % 256 != 0) return REEF_B200_ERR_ALIGNMENT;
  StepBufs b;
  if (step_carve(m, count, workspace, &b) > workspace_bytes) return REEF_B200_ERR_INVALID;
  if (int rc = check_device()) return rc;
  cudaStream_t st = S(stream);
  const size_t d = m->hidden;
  const size_t dl = model_width(m);
  // x = wte[id] + wpe[position] (gpt_neo.cc:130-133)
  REEF_TRY(embedding_f32(static_cast<int>(d), static_cast<long long>(count), ids,
                         static_cast<long long>(position), static_cast<long long>(m->vocab),
                         static_cast<long long>(m->max_positions), m->wte, m->wpe, b.x[0], st));
  // every block on this layer's cache (gpt_neo.cc:135-177)
  int cur = 0;
  for (size_t l = 0; l < m->layers; ++l) {
    const size_t layer_off = l * max_tokens * dl;
    const NeoCache kv{k_cache + layer_off, v_cache + layer_off, position};
    if (m->blocks != nullptr) {
      reef_b200_gptneo_block blk = m->blocks[l];
      blk.seq = count;
      REEF_TRY(neo_forward(&blk, b.x[cur], b.x[cur ^ 1], &kv, b.block_ws, b.block_bytes, st));
    } else {
      reef_b200_gptneo_block_f32 blk = m->blocks_f32[l];
      blk.seq = count;
      REEF_TRY(neo_f32_forward(&blk, b.x[cur], b.x[cur ^ 1], kv, b.block_ws, b.block_bytes, st));
    }
    cur ^= 1;
  }
  if (logits == nullptr && next_id == nullptr) return REEF_B200_OK;
  // logits = ln_f(x) . wte^T for the last token, then the greedy choice
  // (gpt_neo.cc:179-187)
  float* lg = logits != nullptr ? logits : b.logits;
  REEF_TRY(layernorm_exact(1, static_cast<int>(d), m->eps, b.x[cur] + (count - 1) * d, m->ln_f_g,
                           m->ln_f_b, b.normed, st));
  REEF_TRY(matvec_rows_f32(static_cast<long long>(m->vocab), static_cast<long long>(d), m->wte,
                           b.normed, lg, st));
  if (next_id != nullptr)
    REEF_TRY(argmax_f32(static_cast<long long>(m->vocab), lg, next_id, st));
  return REEF_B200_OK;
}

}  // extern "C"
