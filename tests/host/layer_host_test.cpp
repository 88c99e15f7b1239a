// layer_host_test.cpp -- test infrastructure: drives the Llama layer's
// tensor-parallel forward (reef_b200/csrc/layer.cpp) and its communicator
// (comm.cpp) on the CPU, threads as ranks, over the stand-ins in
// fake_cuda_nccl.cpp (CUDA runtime, NCCL) and fake_ops.cpp (kernels as
// no-ops, the cross-rank counter waits done on the host with a deadline).
// Prints one "ok <case>" line per passing case, "FAIL ..." lines otherwise;
// exits non-zero on any failure.
//
// Per world size (2, 4, 8), one communicator is driven through the sequence
// a user of several layer shapes and chunk counts produces:
//   pipelined all-gather forwards at 2 chunks, then at 4 (a larger arena),
//   the unpipelined all-gather forward (1 chunk; NCCL all-gathers), a wider
//   layer at 2 chunks (a larger arena again), the all-reduce plan, the
//   instrumented forward, and the first layer at 2 chunks once more (the arena
//   is kept).
// Then, on a new communicator per world size, the decode step under both
// plans and reef's GPT-Neo block (other_drivers_case).
// After each step: every forward returned OK, no counter wait ran out, and
// each rank's local counters add up to what the forwards since the arena was
// made must have signalled: every use of a region (per chunk: 4 int8
// activations, 2 RMSNorm sums, 2 row maxima) is delivered and consumed once by
// each of the N - 1 peers, so 16 x chunks x forwards x (N - 1).
#include "comm.h"
#include "reef_b200.h"

#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

using namespace reef;

extern "C" void fake_set_rank(int r);
extern "C" int fake_violations();
extern "C" int fake_live_allocations();
extern "C" int fake_ops_timeouts();
extern "C" void fake_ops_reset();

namespace {

std::mutex g_print;
std::atomic<int> g_fail{0};

#define CHECK(cond)                                                                    \
  do {                                                                                 \
    if (!(cond)) {                                                                     \
      std::lock_guard<std::mutex> lk(g_print);                                         \
      std::fprintf(stderr, "FAIL %s:%d: %s\n", __FILE__, __LINE__, #cond);             \
      ++g_fail;                                                                        \
    }                                                                                  \
  } while (0)

#define CHECK_EQ(a, b)                                                                 \
  do {                                                                                 \
    const long long va = static_cast<long long>(a), vb = static_cast<long long>(b);    \
    if (va != vb) {                                                                    \
      std::lock_guard<std::mutex> lk(g_print);                                         \
      std::fprintf(stderr, "FAIL %s:%d: %s == %s (%lld vs %lld)\n", __FILE__, __LINE__, \
                   #a, #b, va, vb);                                                    \
      ++g_fail;                                                                        \
    }                                                                                  \
  } while (0)

void run_ranks(int world, const std::function<void(int)>& f) {
  std::vector<std::thread> th;
  for (int r = 0; r < world; ++r)
    th.emplace_back([&f, r] {
      fake_set_rank(r);
      f(r);
    });
  for (auto& t : th) t.join();
}

// Weights and norms are never read by the no-op kernels; the descriptor only
// needs valid, aligned pointers.
alignas(256) unsigned char g_dummy[256];

struct Shape {
  size_t hidden, heads_q, heads_kv, ffn, batch, seq;
};

reef_b200_llama_layer layer_for(const Shape& s, int world, Comm* c, int mode) {
  reef_b200_llama_layer L{};
  L.batch = s.batch;
  L.seq = s.seq;
  L.hidden = s.hidden;
  L.heads_q = s.heads_q / world;
  L.heads_kv = s.heads_kv / world;
  L.head_dim = 128;
  L.ffn = s.ffn / world;
  L.rms_eps = 1e-5f;
  L.rope_base = 10000.0f;
  const auto* f = reinterpret_cast<const float*>(g_dummy);
  const auto* w = reinterpret_cast<const int8_t*>(g_dummy);
  L.attn_norm = f;
  L.w_qkv = w;
  L.s_qkv = f;
  L.w_o = w;
  L.s_o = f;
  L.mlp_norm = f;
  L.w_gu = w;
  L.s_gu = f;
  L.w_down = w;
  L.s_down = f;
  L.comm = reinterpret_cast<reef_b200_comm*>(c);
  L.tp_mode = mode;
  return L;
}

// One forward of layer L on this rank (host buffers: the no-op kernels touch
// none, the fake collectives copy within the workspace).
int forward(const reef_b200_llama_layer& L, int world, bool instrumented) {
  const size_t ws = reef_b200_llama_layer_workspace_bytes(&L);
  if (ws == 0) return -1;
  const size_t cols = L.tp_mode == REEF_B200_TP_ALLGATHER ? L.hidden / world : L.hidden;
  const size_t io = L.batch * L.seq * cols * sizeof(float);
  void* w = std::aligned_alloc(256, (ws + 255) / 256 * 256);
  auto* x = static_cast<float*>(std::aligned_alloc(256, (io + 255) / 256 * 256));
  auto* y = static_cast<float*>(std::aligned_alloc(256, (io + 255) / 256 * 256));
  int rc;
  if (instrumented) {
    cudaEvent_t ev[10];
    for (auto& e : ev) cudaEventCreateWithFlags(&e, 0);
    void* evp[10];
    for (int i = 0; i < 10; ++i) evp[i] = ev[i];
    rc = reef_b200_llama_layer_forward_events(&L, x, y, w, ws, evp, nullptr);
    for (auto& e : ev) cudaEventDestroy(e);
  } else {
    rc = reef_b200_llama_layer_forward(&L, x, y, w, ws, nullptr);
  }
  std::free(w);
  std::free(x);
  std::free(y);
  return rc;
}

unsigned long long counter_sum(Comm* c, int slots) {
  unsigned long long s = 0;
  for (int i = 0; i < slots; ++i) s += *comm_local_counter(c, i);
  return s;
}

void world_case(int world) {
  const Shape a{1024, 8, 8, 2816, 4, 256};    // 4 sequences: 1, 2 or 4 chunks
  const Shape b{2048, 16, 16, 5632, 4, 1024};  // a wider layer: a larger arena
  std::vector<unsigned char> id(comm_unique_id_bytes());
  fake_set_rank(0);
  CHECK(comm_unique_id(id.data(), id.size()) == kOk);
  std::vector<Comm*> comms(world, nullptr);
  run_ranks(world, [&](int r) {
    CHECK(comm_init(r, world, id.data(), 5.0, &comms[r]) == kOk);
  });
  for (Comm* c : comms)
    if (c == nullptr) return;
  const unsigned long long peers = static_cast<unsigned long long>(world - 1);

  // phase: (shape, plan, chunks, forwards, instrumented, counters expected
  // after it, slots to add up)
  struct Phase {
    const Shape* s;
    int mode;
    const char* chunks;
    int forwards;
    bool instrumented;
    unsigned long long want;
    int slots;
  };
  const int AG = REEF_B200_TP_ALLGATHER, AR = REEF_B200_TP_ALLREDUCE;
  const Phase phases[] = {
      {&a, AG, "2", 3, false, 16 * 2 * 3 * peers, 12},   // arena made: 12 slots
      {&a, AG, "4", 3, false, 16 * 4 * 3 * peers, 24},   // 24 slots: a new arena
      {&a, AG, "1", 2, false, 16 * 4 * 3 * peers, 24},   // NCCL all-gathers: untouched
      {&b, AG, "2", 2, false, 16 * 2 * 2 * peers, 12},   // more data: a new arena (12 slots)
      {&a, AR, "2", 1, false, 16 * 2 * 2 * peers, 12},   // all-reduce plan: untouched
      {&a, AG, "2", 1, true, 16 * 2 * 2 * peers, 12},    // instrumented: unpipelined
      {&a, AG, "2", 2, false, 16 * 2 * 4 * peers, 12},   // arena kept: counts go on
  };
  int k = 0;
  for (const Phase& p : phases) {
    ++k;
    setenv("REEF_B200_TP_CHUNKS", p.chunks, 1);
    fake_ops_reset();
    run_ranks(world, [&](int r) {
      const reef_b200_llama_layer L = layer_for(*p.s, world, comms[r], p.mode);
      for (int f = 0; f < p.forwards; ++f) CHECK_EQ(forward(L, world, p.instrumented), 0);
    });
    CHECK_EQ(fake_ops_timeouts(), 0);
    for (int r = 0; r < world; ++r) {
      fake_set_rank(r);
      if (counter_sum(comms[r], p.slots) != p.want) {
        std::lock_guard<std::mutex> lk(g_print);
        std::fprintf(stderr, "FAIL world %d phase %d rank %d: counters %llu, want %llu\n", world,
                     k, r, counter_sum(comms[r], p.slots), p.want);
        ++g_fail;
      }
    }
  }
  unsetenv("REEF_B200_TP_CHUNKS");
  run_ranks(world, [&](int r) { CHECK(comm_destroy(comms[r]) == kOk); });
  CHECK_EQ(fake_violations(), 0);
  CHECK_EQ(fake_live_allocations(), 0);
}

// The decode step (both plans) and reef's GPT-Neo block at TP = world on one
// communicator: every call returns OK and every rank issues the same
// collectives in the same order (the fake NCCL counts a mismatch as a
// violation).
void other_drivers_case(int world) {
  std::vector<unsigned char> id(comm_unique_id_bytes());
  fake_set_rank(0);
  CHECK(comm_unique_id(id.data(), id.size()) == kOk);
  std::vector<Comm*> comms(world, nullptr);
  run_ranks(world, [&](int r) {
    CHECK(comm_init(r, world, id.data(), 5.0, &comms[r]) == kOk);
  });
  for (Comm* c : comms)
    if (c == nullptr) return;
  const Shape d{1024, 16, 8, 2816, 8, 1};  // 8 sequences, one new token each
  const size_t max_len = 256;
  run_ranks(world, [&](int r) {
    for (int mode : {REEF_B200_TP_ALLREDUCE, REEF_B200_TP_ALLGATHER}) {
      const reef_b200_llama_layer L = layer_for(d, world, comms[r], mode);
      const size_t ws = reef_b200_llama_decode_workspace_bytes(&L, max_len);
      CHECK(ws != 0);
      if (ws == 0) continue;
      const size_t cache = L.batch * L.heads_kv * max_len;
      std::vector<int8_t> kc(cache * 128), vc(cache * 128);
      std::vector<float> ks(cache), vs(cache), x(L.batch * L.hidden), y(L.batch * L.hidden);
      std::vector<int32_t> pos(L.batch, 7);
      void* w = std::aligned_alloc(256, (ws + 255) / 256 * 256);
      for (int step = 0; step < 3; ++step)
        CHECK_EQ(reef_b200_llama_decode_forward(&L, x.data(), y.data(), pos.data(), kc.data(),
                                                ks.data(), vc.data(), vs.data(), max_len, w, ws,
                                                nullptr),
                 0);
      std::free(w);
    }
    // GPT-Neo (config 2's widths): heads split over the ranks
    reef_b200_gptneo_block B{};
    B.seq = 128;
    B.hidden = 256;
    B.heads = 8 / world;
    B.head_dim = 32;
    B.ffn = 1024 / world;
    B.window = 0;
    B.eps = 1e-5f;
    const auto* f = reinterpret_cast<const float*>(g_dummy);
    const auto* w8 = reinterpret_cast<const int8_t*>(g_dummy);
    B.ln1_g = B.ln1_b = B.ln2_g = B.ln2_b = f;
    B.wq = B.wk = B.wv = B.wo = B.wfc = B.wproj = w8;
    B.sq = B.sk = B.sv = B.so = B.sfc = B.sproj = f;
    B.bo = B.bfc = B.bproj = f;
    B.comm = reinterpret_cast<reef_b200_comm*>(comms[r]);
    const size_t ws = reef_b200_gptneo_block_workspace_bytes(&B);
    CHECK(ws != 0);
    if (ws == 0) return;
    std::vector<float> x(B.seq * B.hidden), y(B.seq * B.hidden);
    void* w = std::aligned_alloc(256, (ws + 255) / 256 * 256);
    for (int k = 0; k < 2; ++k)
      CHECK_EQ(reef_b200_gptneo_block_forward(&B, x.data(), y.data(), w, ws, nullptr), 0);
    std::free(w);
  });
  CHECK_EQ(fake_ops_timeouts(), 0);
  run_ranks(world, [&](int r) { CHECK(comm_destroy(comms[r]) == kOk); });
  CHECK_EQ(fake_violations(), 0);
}

}  // namespace

int main() {
  for (int world : {2, 4, 8}) {
    const int before = g_fail.load();
    world_case(world);
    if (g_fail.load() == before) std::printf("ok world %d\n", world);
  }
  for (int world : {2, 4, 8}) {
    const int before = g_fail.load();
    other_drivers_case(world);
    if (g_fail.load() == before) std::printf("ok decode and gptneo world %d\n", world);
  }
  std::fflush(stdout);
  return g_fail.load() == 0 ? 0 : 1;
}
