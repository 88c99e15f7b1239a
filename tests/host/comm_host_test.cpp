// comm_host_test.cpp -- test infrastructure: drives the communicator in
// reef_b200/csrc/comm.cpp on the CPU, threads as ranks, over the stand-ins
// in fake_cuda_nccl.cpp.  Prints one "ok <case>" line per passing case and
// "FAIL ..." lines otherwise; exits non-zero on any failure.
//
// Cases:
//   arena    the symmetric arena: zeroed counters, every rank's mapping of
//            every peer, counts that grow across forwards, a request that
//            fits keeps the arena and its round, a larger one replaces it
//            with zeroed counters and restarts the rounds, and no rank ever
//            frees memory a peer still maps (ranks drop their mappings at
//            staggered times), teardown included;
//   teardown a rank that never tears down: the others' teardown returns
//            REEF_B200_ERR_TIMEOUT after the communicator's timeout instead
//            of waiting for good;
//   reserve  a rank that never asks for the arena: the others' request
//            returns REEF_B200_ERR_TIMEOUT after the timeout.
#include "comm.h"

#include <atomic>
#include <barrier>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <functional>
#include <mutex>
#include <thread>
#include <vector>

using namespace reef;

extern "C" void fake_set_rank(int r);
extern "C" int fake_violations();
extern "C" void fake_reset_violations();
extern "C" int fake_live_allocations();
extern "C" void fake_set_close_delay_us(int us);
extern "C" void fake_set_collective_limit_ms(int ms);

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

void run_ranks(int world, const std::function<void(int)>& f) {
  std::vector<std::thread> th;
  for (int r = 0; r < world; ++r)
    th.emplace_back([&f, r] {
      fake_set_rank(r);
      f(r);
    });
  for (auto& t : th) t.join();
}

std::vector<unsigned char> new_id() {
  std::vector<unsigned char> id(comm_unique_id_bytes());
  fake_set_rank(0);
  CHECK(comm_unique_id(id.data(), id.size()) == kOk);
  return id;
}

double seconds_since(std::chrono::steady_clock::time_point t0) {
  return std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
}

void arena_case(int world) {
  const auto id = new_id();
  std::vector<uint8_t*> first(world), second(world);
  std::barrier sync(world);
  fake_set_close_delay_us(2000);  // rank r drops a mapping r x 2 ms late
  run_ranks(world, [&](int r) {
    Comm* c = nullptr;
    CHECK(comm_init(r, world, id.data(), 5.0, &c) == kOk);
    if (c == nullptr) return;
    CHECK(comm_arena_reserve(c, 1 << 20, 6) == kOk);
    for (int s = 0; s < 6; ++s) CHECK(*comm_local_counter(c, s) == 0u);
    first[r] = comm_arena_data(c);
    sync.arrive_and_wait();
    for (int q = 0; q < world; ++q) CHECK(comm_peer_data(c, q) == first[q]);
    // three forwards: a round each, and a signal to every peer's slot-0 counter
    for (uint32_t k = 1; k <= 3; ++k) {
      CHECK(comm_next_round(c) == k);
      for (int q = 0; q < world; ++q)
        if (q != r) __atomic_fetch_add(comm_counter(c, 0, q), 1u, __ATOMIC_SEQ_CST);
    }
    sync.arrive_and_wait();
    CHECK(*comm_local_counter(c, 0) == 3u * static_cast<unsigned>(world - 1));
    // a request that fits keeps the arena, its counters and its round
    CHECK(comm_arena_reserve(c, 1 << 19, 6) == kOk);
    CHECK(comm_arena_data(c) == first[r]);
    CHECK(comm_next_round(c) == 4u);
    sync.arrive_and_wait();  // every rank read its counter before any replaces
    // a larger one replaces it: zero counters, rounds from 1 again
    CHECK(comm_arena_reserve(c, 8 << 20, 12) == kOk);
    second[r] = comm_arena_data(c);
    for (int s = 0; s < 12; ++s) CHECK(*comm_local_counter(c, s) == 0u);
    CHECK(comm_next_round(c) == 1u);
    sync.arrive_and_wait();
    for (int q = 0; q < world; ++q) CHECK(comm_peer_data(c, q) == second[q]);
    CHECK(comm_destroy(c) == kOk);
  });
  fake_set_close_delay_us(0);
  CHECK(fake_violations() == 0);
  CHECK(fake_live_allocations() == 0);
}

void teardown_case() {
  const int world = 4;
  const auto id = new_id();
  std::barrier sync(world);
  std::atomic<int> finished{0};
  fake_set_collective_limit_ms(300);
  run_ranks(world, [&](int r) {
    Comm* c = nullptr;
    CHECK(comm_init(r, world, id.data(), 0.5, &c) == kOk);
    if (c == nullptr) return;
    CHECK(comm_arena_reserve(c, 1 << 20, 6) == kOk);
    sync.arrive_and_wait();
    if (r == world - 1) {  // never tears down; cleans up once the others gave up
      while (finished.load() < world - 1) std::this_thread::sleep_for(std::chrono::milliseconds(5));
      comm_abort(c);
      return;
    }
    const auto t0 = std::chrono::steady_clock::now();
    CHECK(comm_destroy(c) == kErrTimeout);
    CHECK(seconds_since(t0) < 10.0);
    ++finished;
  });
  fake_set_collective_limit_ms(2000);
  fake_reset_violations();  // a rank that gives up frees what the absent rank still maps
}

void reserve_case() {
  const int world = 2;
  const auto id = new_id();
  std::atomic<int> finished{0};
  fake_set_collective_limit_ms(300);
  run_ranks(world, [&](int r) {
    Comm* c = nullptr;
    CHECK(comm_init(r, world, id.data(), 0.5, &c) == kOk);
    if (c == nullptr) return;
    if (r == 1) {  // never asks for the arena
      while (finished.load() < 1) std::this_thread::sleep_for(std::chrono::milliseconds(5));
      comm_abort(c);
      return;
    }
    const auto t0 = std::chrono::steady_clock::now();
    CHECK(comm_arena_reserve(c, 1 << 20, 6) == kErrTimeout);
    CHECK(seconds_since(t0) < 10.0);
    ++finished;
    comm_abort(c);
  });
  fake_set_collective_limit_ms(2000);
  fake_reset_violations();
}

}  // namespace

int main() {
  struct Case {
    const char* name;
    std::function<void()> run;
  };
  const Case cases[] = {
      {"arena world 2", [] { arena_case(2); }},
      {"arena world 4", [] { arena_case(4); }},
      {"arena world 8", [] { arena_case(8); }},
      {"teardown", teardown_case},
      {"reserve", reserve_case},
  };
  for (const Case& k : cases) {
    const int before = g_fail.load();
    k.run();
    if (g_fail.load() == before) std::printf("ok %s\n", k.name);
  }
  std::fflush(stdout);
  return g_fail.load() == 0 ? 0 : 1;
}
