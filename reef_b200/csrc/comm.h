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
// The communicator's own stream (high priority) for collectives that overlap
// compute.  NCCL's kernels are capped at a few CTAs (maxCTAs: 8 at 2 ranks, 16
// above; REEF_B200_NCCL_CTAS overrides), so they leave the GPU's other SMs to
// the layer's kernels.
cudaStream_t comm_stream(const Comm* c);
// Compute streams for work pipelined against the collectives (kComputeStreams).
constexpr int kComputeStreams = 4;
cudaStream_t comm_compute_stream(const Comm* c, int i);

// ---- Symmetric arena: peer stores over NVLink, counters with bounded waits
//
// Every rank holds an arena of the same size, mapped into every peer's
// address space (CUDA IPC), laid out alike: `slots` x world uint32 flags, then
// data.  Kernels write into peers' data regions directly (comm_peer_data).
// A slot's first flag word is a counter that peers increment after their
// kernels, and that a stream waits on before its next kernels, both with
// signal_and_wait (ops.h): its wait gives up after comm_wait_limit_ns and
// records kDevTimeoutPeer, so a peer that never signals cannot hang a stream.
// Counts only grow while an arena lives, so a counter never needs resetting.
// (Re)creates the arena when it is smaller than asked; collective (every rank
// calls it with the same sizes in the same order).  A new arena's counters
// start at zero and comm_next_round starts again at 1 with them; the old one
// is freed only after every rank has dropped its mapping of it.
int comm_arena_reserve(Comm* c, size_t data_bytes, int slots);
uint8_t* comm_arena_data(Comm* c);  // this rank's data region
// rank r's data region as mapped here (r = this rank: comm_arena_data)
uint8_t* comm_peer_data(Comm* c, int r);
// The counter of `slot` in rank r's arena (for the signals), this rank's own
// counter of `slot` (for the waits), and how long a wait may last (the
// communicator's timeout).
unsigned int* comm_counter(Comm* c, int slot, int r);
unsigned int* comm_local_counter(Comm* c, int slot);
unsigned long long comm_wait_limit_ns(const Comm* c);
// A counter the pipelined forward advances once per call after reserving
// the arena (identical on all ranks, which make the same calls), from which
// the counters' targets derive; it restarts with every new arena.
uint32_t comm_next_round(Comm* c);
int allreduce_max_f32(Comm* c, float* buf, size_t n, cudaStream_t stream);
int allreduce_sum_i32(Comm* c, int32_t* buf, size_t n, cudaStream_t stream);
// rank-major all-gather: recv = [world][bytes] (send may not alias recv)
int allgather_bytes(Comm* c, const void* send, void* recv, size_t bytes, cudaStream_t stream);

}  // namespace reef
