// fake_ops.cpp -- test infrastructure: host stand-ins for the kernel launchers
// (reef_b200/csrc/ops.h) that reef_b200/csrc/layer.cpp calls, so that the
// layer drivers' host logic -- above all the pipelined all-gather forward's
// step schedule and its cross-rank counters -- runs on the CPU with threads
// as ranks.  Nothing here is part of the library.
//
// The kernels that compute are no-ops: this checks the schedule, not the
// arithmetic, which the GPU tests pin.  signal_and_wait does on the host what
// its kernel does on the device: the increments first, then a spin on each
// local counter until it reaches its target (wrap-around >=) or the deadline
// passes.  A wait that runs out is counted, and after one has, later waits
// return at once, as the device error word makes them.  A stream runs its
// work at the call, so each rank executes its steps in issue order.
#include "ops.h"

#include <atomic>
#include <chrono>
#include <thread>

namespace reef {

thread_local bool t_pdl = false;

}  // namespace reef

namespace {

std::atomic<int> g_timeouts{0};
std::atomic<long> g_waits{0};
std::atomic<long> g_signals{0};
std::atomic<int> g_wait_limit_ms{3000};

}  // namespace

extern "C" int fake_ops_timeouts() { return g_timeouts.load(); }
extern "C" long fake_ops_waits() { return g_waits.load(); }
extern "C" long fake_ops_signals() { return g_signals.load(); }
extern "C" void fake_ops_reset() {
  g_timeouts = 0;
  g_waits = 0;
  g_signals = 0;
}

namespace reef {

int signal_and_wait(const PeerFlags& f, const CounterWaits& w, unsigned long long limit_ns,
                    cudaStream_t) {
  if (f.n < 0 || f.n > kMaxFlags || w.n < 0 || w.n > kMaxWaits || limit_ns == 0)
    return kErrInvalid;
  for (int i = 0; i < f.n; ++i) {
    if (f.p[i] == nullptr) return kErrInvalid;
    __atomic_fetch_add(f.p[i], 1u, __ATOMIC_SEQ_CST);
    ++g_signals;
  }
  const auto limit = std::chrono::milliseconds(g_wait_limit_ms.load());
  for (int i = 0; i < w.n; ++i) {
    if (w.p[i] == nullptr) return kErrInvalid;
    ++g_waits;
    const auto t0 = std::chrono::steady_clock::now();
    for (;;) {
      const unsigned v = __atomic_load_n(w.p[i], __ATOMIC_SEQ_CST);
      if (static_cast<int>(v - w.target[i]) >= 0) break;
      if (g_timeouts.load() > 0) break;  // an earlier wait ran out: return at once
      if (std::chrono::steady_clock::now() - t0 > limit) {
        ++g_timeouts;
        break;
      }
      std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
  }
  return kOk;
}

int check_device() { return kOk; }

// ---- kernels that compute: no-ops here ----------------------------------------------

int add_f32(long long, const float*, const float*, float*, cudaStream_t) { return kOk; }
int argmax_f32(long long, const float*, uint32_t*, cudaStream_t) { return kOk; }
int attention_head_f32(const AttnHeadArgs&, const float*, const float*, const float*, float*,
                       cudaStream_t) {
  return kOk;
}
int decode_attn_i8(const DecodeProblem&, cudaStream_t) { return kOk; }
size_t decode_attn_partial_floats(int batch, int heads_q, int max_len) {
  return static_cast<size_t>(batch) * heads_q * (max_len / 128 + 1) * 130;
}
int decode_rope_append_partials(int, int, int, int, float, const int*, const int32_t*, int,
                                const float*, const float*, int8_t*, float*, int8_t*, float*,
                                int8_t*, float*, int*, cudaStream_t) {
  return kOk;
}
int embedding_f32(int, long long, const uint32_t*, long long, long long, long long, const float*,
                  const float*, float*, cudaStream_t) {
  return kOk;
}
int flash_prefill_i8(const FlashProblem&, cudaStream_t) { return kOk; }
int gemm_i8(const GemmProblem&, int, cudaStream_t) { return kOk; }
int gemm_i8_skinny(int, int, int, const int8_t*, const int8_t*, int, const float*, const float*,
                   const float*, const float*, void*, void*, cudaStream_t, const int8_t*) {
  return kOk;
}
int gemm_i8_skinny_partials(int, int, int, const int8_t*, const int8_t*, int32_t*, cudaStream_t,
                            const int8_t*) {
  return kOk;
}
int layernorm_exact(long long, int, float, const float*, const float*, const float*, float*,
                    cudaStream_t) {
  return kOk;
}
int layernorm_exact_quant(long long, int, float, const float*, const float*, const float*,
                          int8_t*, long long, float*, cudaStream_t) {
  return kOk;
}
int linear_f32(long long, int, int, const float*, const float*, const float*, float*,
               cudaStream_t) {
  return kOk;
}
int matvec_rows_f32(long long, long long, const float*, const float*, float*, cudaStream_t) {
  return kOk;
}
int max_segments(int, long long, const float*, float*, cudaStream_t) { return kOk; }
int push_f32(long long, const float*, const PeerDst& d, cudaStream_t) {
  return dst_ok(d) ? kOk : kErrInvalid;
}
int quantize_rows(long long, long long, const float*, int8_t*, long long, float*, const float*,
                  cudaStream_t) {
  return kOk;
}
int quantize_rows_to(long long, long long, const float*, const PeerDst& d, long long, float*,
                     const float*, cudaStream_t) {
  return dst_ok(d) ? kOk : kErrInvalid;
}
int reduce_rmsnorm_quant(long long, int, int, const int32_t*, const float*, const float*,
                         const float*, float*, float, const float*, int8_t*, float*,
                         cudaStream_t) {
  return kOk;
}
int rms_apply_quant(long long, int, int, float, const float*, const float*, const float*,
                    const PeerDst& d, float*, cudaStream_t) {
  return dst_ok(d) ? kOk : kErrInvalid;
}
int rms_stats(long long, int, int, const float*, const float*, const PeerDst& d, cudaStream_t) {
  return dst_ok(d) ? kOk : kErrInvalid;
}
int rmsnorm_quant(long long, int, float, const float*, const float*, int8_t*, float*,
                  cudaStream_t) {
  return kOk;
}
int rope_table(int, float, void*, cudaStream_t) { return kOk; }
int row_absmax(long long, long long, const float*, float*, cudaStream_t) { return kOk; }
int row_absmax_to(long long, long long, const float*, const PeerDst& d, cudaStream_t) {
  return dst_ok(d) ? kOk : kErrInvalid;
}
size_t skinny_partial_bytes(int m, int n, int) { return static_cast<size_t>(m) * n * 4 * 16; }
int skinny_split_count(int, int, int) { return 1; }
int swiglu_partials(long long, int, const int32_t*, int, const float*, const float*,
                    const float*, float*, int8_t*, float*, cudaStream_t) {
  return kOk;
}
int unary_exact(int, long long, const float*, float*, cudaStream_t) { return kOk; }
int w8a8_epilogue_i32(long long, long long, const int32_t*, const float*, const float*,
                      const float*, const float*, float*, cudaStream_t) {
  return kOk;
}
int zero_f32(long long, float*, cudaStream_t) { return kOk; }

}  // namespace reef
