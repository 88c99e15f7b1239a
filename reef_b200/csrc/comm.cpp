// comm.cpp -- the tensor-parallel communicator: one NCCL communicator per
// rank (one process or thread per GPU), created non-blocking so that a rank
// that never joins turns into REEF_B200_ERR_TIMEOUT after a deadline instead
// of a hang.  Collectives are enqueued on the caller's stream (so a whole TP
// layer stays asynchronous and can be captured in a CUDA graph).
//
// Only two collectives are on the W8A8 path (a Megatron row-parallel linear,
// which reef does not have; its TP=1 result is the oracle):
//   all-reduce MAX of per-token fp32 row maxima, so every rank quantises its
//     K-shard of an activation row with the full row's scale (quant.hpp
//     :90-133 over the whole row), and
//   all-reduce SUM of int32 partial sums, exact and order-free, so the
//     result is bit-identical at every TP degree.
#include "comm.h"

#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <thread>
#include <vector>

namespace reef {

struct Comm {
  ncclComm_t nccl = nullptr;
  int rank = 0;
  int world = 1;
  double timeout_s = 60.0;
  cudaStream_t stream = nullptr;  // collectives that overlap compute
  cudaStream_t compute[kComputeStreams] = {};  // the pipelined chunks' kernels
  int ctas = 0;                   // NCCL's CTA budget
  // symmetric arena
  uint8_t* arena = nullptr;        // this rank's (cudaMalloc)
  std::vector<uint8_t*> peer;      // every rank's, mapped here (peer[rank] = arena)
  size_t arena_data = 0;           // data bytes
  int arena_slots = 0;
  uint32_t round = 0;
};

namespace {

// Drive a non-blocking NCCL operation to completion, or give up at the
// deadline (abort the communicator: the caller's ranks are out of step).
// Enqueuing a collective usually settles within microseconds, so the first
// 2 ms poll without sleeping (a sleep per collective would make the host,
// not the GPU, set the pace); after that, every 200 us.
int settle(Comm* c, ncclResult_t r) {
  if (r == ncclSuccess) return kOk;
  if (r != ncclInProgress) return kErrNccl;
  const auto start = std::chrono::steady_clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    if (ncclCommGetAsyncError(c->nccl, &st) != ncclSuccess) return kErrNccl;
    if (st == ncclSuccess) return kOk;
    if (st != ncclInProgress) return kErrNccl;
    const double waited =
        std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count();
    if (waited > c->timeout_s) return kErrTimeout;
    if (waited > 2e-3) {
      std::this_thread::sleep_for(std::chrono::microseconds(200));
    } else {
      std::this_thread::yield();
    }
  }
}

// Wait for the stream with the communicator's deadline (a collective that a
// peer never joins would otherwise block the host for good).
int sync_bounded(Comm* c, cudaStream_t s) {
  const auto start = std::chrono::steady_clock::now();
  for (;;) {
    const cudaError_t e = cudaStreamQuery(s);
    if (e == cudaSuccess) return kOk;
    if (e != cudaErrorNotReady) return kErrCuda;
    if (std::chrono::duration<double>(std::chrono::steady_clock::now() - start).count() >
        c->timeout_s)
      return kErrTimeout;
    std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

void close_peers(Comm* c) {
  for (int r = 0; r < static_cast<int>(c->peer.size()); ++r)
    if (r != c->rank && c->peer[r] != nullptr) cudaIpcCloseMemHandle(c->peer[r]);
  c->peer.clear();
}

void arena_free(Comm* c) {
  close_peers(c);
  if (c->arena != nullptr) cudaFree(c->arena);
  c->arena = nullptr;
  c->arena_data = 0;
  c->arena_slots = 0;
}

// Every rank drops its mappings of the peers' arenas, then waits until all
// ranks have (an all-reduce of one word as the barrier) before any rank frees
// its own: an exported allocation must not be freed while another process
// still has it open.  The caller has drained this rank's work, so none of its
// kernels still stores into a peer's arena.  Used where every rank takes the
// same step (a larger arena, the communicator's teardown).
int arena_release_collective(Comm* c) {
  if (c->arena == nullptr) return kOk;
  close_peers(c);
  int* word = nullptr;
  if (cudaMalloc(&word, sizeof(int)) != cudaSuccess) return kErrCuda;
  int rc = cudaMemsetAsync(word, 0, sizeof(int), c->stream) == cudaSuccess ? kOk : kErrCuda;
  if (rc == kOk) rc = settle(c, ncclAllReduce(word, word, 1, ncclInt32, ncclSum, c->nccl, c->stream));
  if (rc == kOk) rc = sync_bounded(c, c->stream);
  // after a timeout the all-reduce may still be pending on the stream: the
  // word stays allocated (cudaFree would wait for it) until the abort
  if (rc != kErrTimeout) cudaFree(word);
  if (rc != kOk) return rc;
  arena_free(c);
  return kOk;
}

size_t flag_bytes(int slots, int world) {
  return (static_cast<size_t>(slots) * world * sizeof(uint32_t) + 255) & ~static_cast<size_t>(255);
}

}  // namespace

int comm_unique_id(void* out, size_t bytes) {
  if (out == nullptr || bytes < sizeof(ncclUniqueId)) return kErrInvalid;
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return kErrNccl;
  std::memcpy(out, &id, sizeof id);
  return kOk;
}

size_t comm_unique_id_bytes() { return sizeof(ncclUniqueId); }

int comm_init(int rank, int world, const void* id_bytes, double timeout_s, Comm** out) {
  if (out == nullptr || id_bytes == nullptr || world < 1 || rank < 0 || rank >= world)
    return kErrInvalid;
  Comm* c = new Comm();
  c->rank = rank;
  c->world = world;
  c->timeout_s = timeout_s > 0 ? timeout_s : 60.0;
  ncclUniqueId id;
  std::memcpy(&id, id_bytes, sizeof id);
  // NCCL's kernels share the GPU with the layer's: cap their CTAs (a
  // persistent GEMM running beside a collective leaves this many SMs free).
  // REEF_B200_NCCL_CTAS overrides the default of 8 (2 ranks) / 16 (more).
  c->ctas = world <= 2 ? 8 : 16;
  if (const char* e = std::getenv("REEF_B200_NCCL_CTAS")) {
    const int v = std::atoi(e);
    if (v >= 1 && v <= 64) c->ctas = v;
  }
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  cfg.maxCTAs = c->ctas;
  ncclResult_t r = ncclCommInitRankConfig(&c->nccl, world, id, rank, &cfg);
  int rc = (c->nccl == nullptr && r != ncclSuccess) ? kErrNccl : settle(c, r);
  if (rc == kOk) {
    int lo = 0, hi = 0;
    cudaDeviceGetStreamPriorityRange(&lo, &hi);
    if (cudaStreamCreateWithPriority(&c->stream, cudaStreamNonBlocking, hi) != cudaSuccess)
      rc = kErrCuda;
    for (auto& s : c->compute)
      if (rc == kOk && cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess)
        rc = kErrCuda;
  }
  if (rc != kOk) {
    if (c->nccl != nullptr) ncclCommAbort(c->nccl);
    delete c;
    return rc;
  }
  *out = c;
  return kOk;
}

int comm_destroy(Comm* c) {
  if (c == nullptr) return kOk;
  int rc = kOk;
  if (c->arena != nullptr) {
    cudaDeviceSynchronize();
    // a peer that never reaches the barrier leaves its all-reduce on our
    // stream: abort (which ends it) instead of waiting on the stream
    rc = arena_release_collective(c);
    if (rc != kOk) {
      comm_abort(c);
      return rc;
    }
  }
  if (c->stream != nullptr) {
    cudaStreamSynchronize(c->stream);
    cudaStreamDestroy(c->stream);
  }
  for (auto s : c->compute)
    if (s != nullptr) {
      cudaStreamSynchronize(s);
      cudaStreamDestroy(s);
    }
  if (c->nccl != nullptr) {
    ncclResult_t r = ncclCommFinalize(c->nccl);
    rc = settle(c, r);
    if (rc == kOk) {
      ncclCommDestroy(c->nccl);
    } else {
      ncclCommAbort(c->nccl);
    }
  }
  delete c;
  return rc;
}

int comm_abort(Comm* c) {
  if (c == nullptr) return kOk;
  arena_free(c);
  if (c->nccl != nullptr) ncclCommAbort(c->nccl);
  if (c->stream != nullptr) cudaStreamDestroy(c->stream);
  for (auto s : c->compute)
    if (s != nullptr) cudaStreamDestroy(s);
  delete c;
  return kOk;
}

int comm_rank(const Comm* c) { return c ? c->rank : 0; }
int comm_world(const Comm* c) { return c ? c->world : 1; }
cudaStream_t comm_stream(const Comm* c) { return c ? c->stream : nullptr; }
cudaStream_t comm_compute_stream(const Comm* c, int i) {
  return (c && i >= 0 && i < kComputeStreams) ? c->compute[i] : nullptr;
}

int allreduce_max_f32(Comm* c, float* buf, size_t n, cudaStream_t stream) {
  if (c == nullptr || c->world == 1 || n == 0) return kOk;
  return settle(c, ncclAllReduce(buf, buf, n, ncclFloat32, ncclMax, c->nccl, stream));
}

int allreduce_sum_i32(Comm* c, int32_t* buf, size_t n, cudaStream_t stream) {
  if (c == nullptr || c->world == 1 || n == 0) return kOk;
  return settle(c, ncclAllReduce(buf, buf, n, ncclInt32, ncclSum, c->nccl, stream));
}

int allgather_bytes(Comm* c, const void* send, void* recv, size_t bytes, cudaStream_t stream) {
  if (c == nullptr || c->world == 1) {
    if (send != recv && bytes > 0)
      return cudaMemcpyAsync(recv, send, bytes, cudaMemcpyDeviceToDevice, stream) == cudaSuccess
                 ? kOk
                 : kErrCuda;
    return kOk;
  }
  if (bytes == 0) return kOk;
  return settle(c, ncclAllGather(send, recv, bytes, ncclInt8, c->nccl, stream));
}


int comm_arena_reserve(Comm* c, size_t data_bytes, int slots) {
  if (c == nullptr || c->world < 2 || slots < 1) return kErrInvalid;
  if (c->arena != nullptr && c->arena_data >= data_bytes && c->arena_slots >= slots) return kOk;
  // every rank reaches this point with the same sizes; drain before replacing
  if (cudaDeviceSynchronize() != cudaSuccess) return kErrCuda;
  if (int rc = arena_release_collective(c)) return rc;
  const size_t fb = flag_bytes(slots, c->world);
  const size_t total = fb + ((data_bytes + 255) & ~static_cast<size_t>(255));
  if (cudaMalloc(&c->arena, total) != cudaSuccess) return kErrCuda;
  // the new counters start at zero, and so do the forward rounds their
  // targets derive from
  c->round = 0;
  if (cudaMemsetAsync(c->arena, 0, fb, c->stream) != cudaSuccess) return kErrCuda;
  // exchange IPC handles (an all-gather through NCCL on the same stream as the
  // zeroing, so a peer holds this arena's handle only once its counters are
  // zero)
  cudaIpcMemHandle_t mine;
  if (cudaIpcGetMemHandle(&mine, c->arena) != cudaSuccess) return kErrCuda;
  const size_t hb = sizeof(cudaIpcMemHandle_t);
  uint8_t* dev = nullptr;
  if (cudaMalloc(&dev, hb * (c->world + 1)) != cudaSuccess) return kErrCuda;
  std::vector<cudaIpcMemHandle_t> all(c->world);
  int rc = kOk;
  if (cudaMemcpyAsync(dev + hb * c->world, &mine, hb, cudaMemcpyHostToDevice, c->stream) !=
      cudaSuccess)
    rc = kErrCuda;
  if (rc == kOk) rc = allgather_bytes(c, dev + hb * c->world, dev, hb, c->stream);
  if (rc == kOk) rc = sync_bounded(c, c->stream);
  if (rc == kOk && cudaMemcpy(all.data(), dev, hb * c->world, cudaMemcpyDeviceToHost) != cudaSuccess)
    rc = kErrCuda;
  if (rc != kErrTimeout) cudaFree(dev);  // (as in arena_release_collective)
  if (rc != kOk) return rc;
  c->peer.assign(c->world, nullptr);
  for (int r = 0; r < c->world; ++r) {
    if (r == c->rank) {
      c->peer[r] = c->arena;
      continue;
    }
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess)
      return kErrCuda;
    c->peer[r] = static_cast<uint8_t*>(p);
  }
  c->arena_data = data_bytes;
  c->arena_slots = slots;
  return kOk;
}

uint8_t* comm_arena_data(Comm* c) {
  return c && c->arena ? c->arena + flag_bytes(c->arena_slots, c->world) : nullptr;
}

uint8_t* comm_peer_data(Comm* c, int r) {
  if (c == nullptr || c->arena == nullptr || r < 0 || r >= c->world) return nullptr;
  return c->peer[r] + flag_bytes(c->arena_slots, c->world);
}

unsigned int* comm_counter(Comm* c, int slot, int r) {
  if (c == nullptr || c->arena == nullptr || slot < 0 || slot >= c->arena_slots || r < 0 ||
      r >= c->world)
    return nullptr;
  return reinterpret_cast<unsigned int*>(c->peer[r] + static_cast<size_t>(slot) * c->world *
                                                           sizeof(uint32_t));
}

unsigned int* comm_local_counter(Comm* c, int slot) {
  return c ? comm_counter(c, slot, c->rank) : nullptr;
}

unsigned long long comm_wait_limit_ns(const Comm* c) {
  const double s = c ? c->timeout_s : 60.0;
  return static_cast<unsigned long long>(s * 1e9);
}

uint32_t comm_next_round(Comm* c) { return c ? ++c->round : 0; }

}  // namespace reef
