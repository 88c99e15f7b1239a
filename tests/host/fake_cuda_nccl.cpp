// fake_cuda_nccl.cpp -- test infrastructure: host-only stand-ins for the CUDA
// runtime and NCCL calls that reef_b200/csrc/comm.cpp makes, so that the
// communicator's host logic (the symmetric arena and its replacement, the
// forward rounds, the teardown barrier, bounded waits) runs on the CPU with
// threads as ranks.  Nothing here is part of the library.
//
// Model:
// * device memory is host memory; every allocation records its owner rank and
//   the ranks that have it open through an IPC handle, and cudaFree of memory
//   another rank still has open counts a violation (CUDA documents that case
//   as undefined: an exported allocation must outlive its importers' handles);
// * threads share one address space, so an IPC handle carries the pointer and
//   "opening" it returns the same pointer;
// * work on a stream runs at the call; a stream is marked stuck when a
//   collective on it never completed (a rank did not join), and then
//   cudaStreamQuery answers cudaErrorNotReady for good, as a real stream with
//   a hung NCCL kernel would;
// * a collective is a rendezvous of the communicator's ranks: the last rank to
//   arrive computes every rank's result, so no rank returns before all data is
//   complete.  A rank that waits longer than the collective limit withdraws
//   and leaves its stream stuck.
#include <cuda_runtime.h>
#include <nccl.h>

#include <chrono>
#include <condition_variable>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <set>
#include <string>
#include <thread>
#include <vector>

struct CUstream_st {
  bool stuck = false;
};

namespace {

thread_local int t_rank = -1;

std::mutex g_mu;
struct Alloc {
  int owner;
  std::set<int> importers;
};
std::map<void*, Alloc> g_allocs;
int g_violations = 0;
int g_close_delay_us = 0;      // rank r sleeps r * this before closing a handle
int g_collective_limit_ms = 2000;

struct Group {
  int n = 0;
  std::mutex m;
  std::condition_variable cv;
  long gen = 0;
  int arrived = 0;
  struct Part {
    const void* send = nullptr;
    void* recv = nullptr;
  };
  std::vector<Part> parts;
  // the collective of the current generation (every rank must call the same)
  int kind = 0;  // 1 all-reduce, 2 all-gather
  size_t count = 0;
  ncclDataType_t type = ncclInt8;
  ncclRedOp_t op = ncclSum;
};
std::map<std::string, Group*> g_groups;
long g_next_id = 0;

size_t type_bytes(ncclDataType_t t) {
  switch (t) {
    case ncclInt8:
    case ncclUint8:
      return 1;
    case ncclFloat16:
    case ncclBfloat16:
      return 2;
    case ncclInt32:
    case ncclUint32:
    case ncclFloat32:
      return 4;
    default:
      return 8;
  }
}

void violation(const char* what) {
  std::lock_guard<std::mutex> lk(g_mu);
  ++g_violations;
  std::fprintf(stderr, "fake: violation on rank %d: %s\n", t_rank, what);
}

}  // namespace

struct ncclComm {
  Group* g;
  int rank;
  bool aborted = false;
};

namespace {

// Every rank's part is in; compute each rank's receive buffer.
void complete(Group* g) {
  const int n = g->n;
  if (g->kind == 1) {
    const size_t c = g->count;
    if (g->type == ncclInt32 && g->op == ncclSum) {
      std::vector<int64_t> acc(c, 0);
      for (int r = 0; r < n; ++r)
        for (size_t i = 0; i < c; ++i) acc[i] += static_cast<const int32_t*>(g->parts[r].send)[i];
      for (int r = 0; r < n; ++r)
        for (size_t i = 0; i < c; ++i)
          static_cast<int32_t*>(g->parts[r].recv)[i] = static_cast<int32_t>(acc[i]);
    } else if (g->type == ncclFloat32 && g->op == ncclMax) {
      std::vector<float> acc(c);
      for (size_t i = 0; i < c; ++i) acc[i] = static_cast<const float*>(g->parts[0].send)[i];
      for (int r = 1; r < n; ++r)
        for (size_t i = 0; i < c; ++i) {
          const float v = static_cast<const float*>(g->parts[r].send)[i];
          if (v > acc[i]) acc[i] = v;
        }
      for (int r = 0; r < n; ++r) std::memcpy(g->parts[r].recv, acc.data(), c * sizeof(float));
    } else {
      violation("all-reduce of an unsupported type / operation");
    }
  } else {
    const size_t b = g->count * type_bytes(g->type);
    std::vector<uint8_t> all(b * n);
    for (int r = 0; r < n; ++r) std::memcpy(all.data() + r * b, g->parts[r].send, b);
    for (int r = 0; r < n; ++r) std::memcpy(g->parts[r].recv, all.data(), b * n);
  }
}

ncclResult_t collective(ncclComm* c, int kind, const void* send, void* recv, size_t count,
                        ncclDataType_t type, ncclRedOp_t op, cudaStream_t s) {
  if (c == nullptr || c->aborted) return ncclInvalidArgument;
  Group* g = c->g;
  std::unique_lock<std::mutex> lk(g->m);
  if (g->arrived == 0) {
    g->kind = kind;
    g->count = count;
    g->type = type;
    g->op = op;
  } else if (g->kind != kind || g->count != count || g->type != type || g->op != op) {
    lk.unlock();
    violation("ranks called different collectives");
    lk.lock();
  }
  const long my = g->gen;
  g->parts[c->rank] = {send, recv};
  if (++g->arrived == g->n) {
    complete(g);
    g->arrived = 0;
    ++g->gen;
    g->cv.notify_all();
    return ncclSuccess;
  }
  if (!g->cv.wait_for(lk, std::chrono::milliseconds(g_collective_limit_ms),
                      [&] { return g->gen != my; })) {
    // a peer never joined: withdraw; the stream never completes
    --g->arrived;
    g->parts[c->rank] = {};
    if (s != nullptr) s->stuck = true;
  }
  return ncclSuccess;
}

}  // namespace

// ---- controls for the test driver ---------------------------------------------

extern "C" void fake_set_rank(int r) { t_rank = r; }
extern "C" int fake_violations() {
  std::lock_guard<std::mutex> lk(g_mu);
  return g_violations;
}
extern "C" void fake_reset_violations() {
  std::lock_guard<std::mutex> lk(g_mu);
  g_violations = 0;
}
extern "C" int fake_live_allocations() {
  std::lock_guard<std::mutex> lk(g_mu);
  return static_cast<int>(g_allocs.size());
}
extern "C" void fake_set_close_delay_us(int us) { g_close_delay_us = us; }
extern "C" void fake_set_collective_limit_ms(int ms) { g_collective_limit_ms = ms; }

// ---- CUDA runtime ------------------------------------------------------------------

cudaError_t cudaMalloc(void** p, size_t bytes) {
  void* q = std::aligned_alloc(256, (bytes + 255) / 256 * 256 + 256);
  if (q == nullptr) return cudaErrorMemoryAllocation;
  std::memset(q, 0xA5, bytes);  // not zero: the code must zero what it relies on
  std::lock_guard<std::mutex> lk(g_mu);
  g_allocs[q] = Alloc{t_rank, {}};
  *p = q;
  return cudaSuccess;
}

cudaError_t cudaFree(void* p) {
  if (p == nullptr) return cudaSuccess;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_allocs.find(p);
    if (it == g_allocs.end()) {
      ++g_violations;
      std::fprintf(stderr, "fake: rank %d frees unknown memory\n", t_rank);
      return cudaErrorInvalidValue;
    }
    if (!it->second.importers.empty()) {
      ++g_violations;
      std::fprintf(stderr, "fake: rank %d frees memory that rank %d still has open\n", t_rank,
                   *it->second.importers.begin());
    }
    g_allocs.erase(it);
  }
  std::free(p);
  return cudaSuccess;
}

cudaError_t cudaMemset(void* p, int v, size_t n) {
  std::memset(p, v, n);
  return cudaSuccess;
}

cudaError_t cudaMemsetAsync(void* p, int v, size_t n, cudaStream_t) {
  std::memset(p, v, n);
  return cudaSuccess;
}

cudaError_t cudaMemcpy(void* d, const void* s, size_t n, cudaMemcpyKind) {
  std::memcpy(d, s, n);
  return cudaSuccess;
}

cudaError_t cudaMemcpyAsync(void* d, const void* s, size_t n, cudaMemcpyKind, cudaStream_t) {
  std::memcpy(d, s, n);
  return cudaSuccess;
}

cudaError_t cudaDeviceSynchronize(void) { return cudaSuccess; }

cudaError_t cudaDeviceGetStreamPriorityRange(int* lo, int* hi) {
  *lo = 0;
  *hi = -1;
  return cudaSuccess;
}

cudaError_t cudaStreamCreateWithFlags(cudaStream_t* s, unsigned int) {
  *s = new CUstream_st();
  return cudaSuccess;
}

cudaError_t cudaStreamCreateWithPriority(cudaStream_t* s, unsigned int, int) {
  *s = new CUstream_st();
  return cudaSuccess;
}

cudaError_t cudaStreamQuery(cudaStream_t s) {
  return (s != nullptr && s->stuck) ? cudaErrorNotReady : cudaSuccess;
}

cudaError_t cudaStreamSynchronize(cudaStream_t s) {
  if (s != nullptr && s->stuck) {
    // a real stream would block for good; the test would hang, so say so
    violation("cudaStreamSynchronize on a stream that never completes");
    return cudaErrorNotReady;
  }
  return cudaSuccess;
}

cudaError_t cudaStreamDestroy(cudaStream_t s) {
  delete s;
  return cudaSuccess;
}

// Work runs at the call, so an event is complete as soon as it is recorded and
// a wait on it has nothing to order.
struct CUevent_st {
  int recorded = 0;
};

cudaError_t cudaEventCreateWithFlags(cudaEvent_t* e, unsigned int) {
  *e = new CUevent_st();
  return cudaSuccess;
}

cudaError_t cudaEventDestroy(cudaEvent_t e) {
  delete e;
  return cudaSuccess;
}

cudaError_t cudaEventRecord(cudaEvent_t e, cudaStream_t) {
  if (e == nullptr) return cudaErrorInvalidResourceHandle;
  ++e->recorded;
  return cudaSuccess;
}

cudaError_t cudaStreamWaitEvent(cudaStream_t, cudaEvent_t e, unsigned int) {
  return e == nullptr ? cudaErrorInvalidResourceHandle : cudaSuccess;
}

cudaError_t cudaIpcGetMemHandle(cudaIpcMemHandle_t* h, void* p) {
  std::memset(h, 0, sizeof *h);
  std::memcpy(h->reserved, &p, sizeof p);
  return cudaSuccess;
}

cudaError_t cudaIpcOpenMemHandle(void** p, cudaIpcMemHandle_t h, unsigned int) {
  void* q = nullptr;
  std::memcpy(&q, h.reserved, sizeof q);
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_allocs.find(q);
  if (it == g_allocs.end()) return cudaErrorInvalidResourceHandle;
  it->second.importers.insert(t_rank);
  *p = q;
  return cudaSuccess;
}

cudaError_t cudaIpcCloseMemHandle(void* p) {
  if (g_close_delay_us > 0 && t_rank > 0)
    std::this_thread::sleep_for(std::chrono::microseconds(g_close_delay_us * t_rank));
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = g_allocs.find(p);
  if (it == g_allocs.end()) return cudaErrorInvalidValue;
  it->second.importers.erase(t_rank);
  return cudaSuccess;
}

// ---- NCCL ----------------------------------------------------------------------------

ncclResult_t ncclGetUniqueId(ncclUniqueId* id) {
  std::memset(id, 0, sizeof *id);
  std::lock_guard<std::mutex> lk(g_mu);
  std::snprintf(id->internal, sizeof id->internal, "fake-%ld", g_next_id++);
  return ncclSuccess;
}

ncclResult_t ncclCommInitRankConfig(ncclComm_t* comm, int nranks, ncclUniqueId id, int rank,
                                    ncclConfig_t*) {
  std::lock_guard<std::mutex> lk(g_mu);
  Group*& g = g_groups[std::string(id.internal)];
  if (g == nullptr) {
    g = new Group();
    g->n = nranks;
    g->parts.resize(nranks);
  }
  *comm = new ncclComm{g, rank};
  return ncclSuccess;
}

ncclResult_t ncclCommGetAsyncError(ncclComm_t, ncclResult_t* st) {
  *st = ncclSuccess;
  return ncclSuccess;
}

ncclResult_t ncclCommFinalize(ncclComm_t) { return ncclSuccess; }

ncclResult_t ncclCommDestroy(ncclComm_t c) {
  delete c;
  return ncclSuccess;
}

ncclResult_t ncclCommAbort(ncclComm_t c) {
  delete c;
  return ncclSuccess;
}

ncclResult_t ncclAllReduce(const void* send, void* recv, size_t count, ncclDataType_t type,
                           ncclRedOp_t op, ncclComm_t comm, cudaStream_t s) {
  return collective(comm, 1, send, recv, count, type, op, s);
}

ncclResult_t ncclAllGather(const void* send, void* recv, size_t count, ncclDataType_t type,
                           ncclComm_t comm, cudaStream_t s) {
  return collective(comm, 2, send, recv, count, type, ncclSum, s);
}
