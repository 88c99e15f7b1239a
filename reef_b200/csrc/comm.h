// comm.h -- tensor-parallel communicator (NCCL), see comm.cpp.
#pragma once

#include "ops.h"

namespace reef {

struct Comm;

size_t comm_unique_id_bytes();
int comm_unique_id(void* out, size_t bytes);
int comm_init(int rank, int world, const void* id_bytes, double timeout_s, Comm** out);
int comm_destroy(Comm* c);
int comm_abort(Comm* c);
int comm_rank(const Comm* c);
int comm_world(const Comm* c);
int allreduce_max_f32(Comm* c, float* buf, size_t n, cudaStream_t stream);
int allreduce_sum_i32(Comm* c, int32_t* buf, size_t n, cudaStream_t stream);
// rank-major all-gather: recv = [world][bytes] (send may not alias recv)
int allgather_bytes(Comm* c, const void* send, void* recv, size_t bytes, cudaStream_t stream);

}  // namespace reef
