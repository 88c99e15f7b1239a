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
#include <cstring>
#include <thread>

namespace reef {

struct Comm {
  ncclComm_t nccl = nullptr;
  int rank = 0;
  int world = 1;
  double timeout_s = 60.0;
};

namespace {

// Drive a non-blocking NCCL operation to completion, or give up at the
// deadline (abort the communicator: the caller's ranks are out of step).
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
    std::this_thread::sleep_for(std::chrono::microseconds(200));
  }
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
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  ncclResult_t r = ncclCommInitRankConfig(&c->nccl, world, id, rank, &cfg);
  int rc = (c->nccl == nullptr && r != ncclSuccess) ? kErrNccl : settle(c, r);
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
  if (c->nccl != nullptr) ncclCommAbort(c->nccl);
  delete c;
  return kOk;
}

int comm_rank(const Comm* c) { return c ? c->rank : 0; }
int comm_world(const Comm* c) { return c ? c->world : 1; }

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

}  // namespace reef
