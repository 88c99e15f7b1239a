"""Megatron tensor-parallel sharding of reef's W8A8 layers, and the
communicator bootstrap.

reef runs on one core and has no tensor parallelism; its TP=1 result is the
oracle.  The plan is Megatron's:

* column-parallel (no communication): q/k/v split by heads, FFN gate/up (or
  GPT-Neo c_fc) split by FFN columns.  A rank owns whole output rows of W,
  each with the scale reef's quantize_rows gives the FULL row, so every
  output column it computes is TP=1's, bit for bit.
* row-parallel: attention output projection and FFN down (c_proj) split by
  input features K.  A rank owns the K-slice of W (per-channel scales are
  still full-row scales, replicated); the activation slice is quantised with
  the full row's scale (all-reduce MAX), int32 partial sums are all-reduced
  (SUM, exact), and the bias is added once.

The functions here are pure index arithmetic on numpy / torch tensors, so
the CPU tests (gloo ranks) and the GPU path shard identically.
"""
from __future__ import annotations

import ctypes as C


def shard_range(total: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of this rank's equal share of `total`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    if total % world:
        raise ValueError(f"{total} does not split evenly across {world} ranks")
    n = total // world
    return rank * n, (rank + 1) * n


def qkv_rows(heads_q: int, heads_kv: int, head_dim: int, world: int, rank: int) -> list[int]:
    """Rows of a stacked [q; k; v] weight ([(Hq + 2 Hkv) * hd][hidden]) that
    this rank owns: its query heads, then its key heads, then its value heads."""
    q0, q1 = shard_range(heads_q, world, rank)
    k0, k1 = shard_range(heads_kv, world, rank)
    rows = list(range(q0 * head_dim, q1 * head_dim))
    base = heads_q * head_dim
    rows += list(range(base + k0 * head_dim, base + k1 * head_dim))
    base += heads_kv * head_dim
    rows += list(range(base + k0 * head_dim, base + k1 * head_dim))
    return rows


def gate_up_rows(ffn: int, world: int, rank: int) -> list[int]:
    """Rows of a stacked [gate; up] weight ([2 ffn][hidden]) this rank owns:
    its gate rows, then the matching up rows."""
    f0, f1 = shard_range(ffn, world, rank)
    return list(range(f0, f1)) + list(range(ffn + f0, ffn + f1))


def col_slice(total: int, world: int, rank: int) -> slice:
    """K-slice of a row-parallel weight (and of its input activation)."""
    a, b = shard_range(total, world, rank)
    return slice(a, b)


# ---- communicator bootstrap ---------------------------------------------------

class Comm:
    """A reef_b200 communicator (NCCL over NVLink) for this rank.

    The unique id is made on rank 0 and shared over the torch.distributed
    process group that launched the ranks; every rank then calls
    reef_b200_comm_init with its CUDA device current."""

    def __init__(self, rank: int, world: int, timeout_s: float = 60.0):
        import torch.distributed as dist

        from . import _lib
        L = _lib.lib()
        nbytes = L.reef_b200_comm_unique_id_bytes()
        buf = (C.c_uint8 * nbytes)()
        if rank == 0:
            _lib.call("reef_b200_comm_unique_id", C.addressof(buf), nbytes)
        obj = [bytes(buf)]
        dist.broadcast_object_list(obj, src=0)
        C.memmove(buf, obj[0], nbytes)
        handle = C.c_void_p()
        _lib.call("reef_b200_comm_init", rank, world, C.addressof(buf), timeout_s,
                  C.addressof(handle))
        self.handle = handle
        self.rank, self.world = rank, world

    @property
    def ptr(self) -> int:
        return self.handle.value

    def close(self) -> None:
        from . import _lib
        if self.handle.value:
            _lib.call("reef_b200_comm_destroy", self.handle)
            self.handle = C.c_void_p()
