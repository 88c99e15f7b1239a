"""The tensor-parallel communicator's host logic on the CPU.

reef_b200/csrc/comm.cpp is compiled with g++ together with host-only stand-ins
for the CUDA runtime and NCCL calls it makes (tests/host/fake_cuda_nccl.cpp)
and driven with threads as ranks (tests/host/comm_host_test.cpp):

* the symmetric arena: zeroed counters, every rank's mapping of every peer,
  counts that grow across forwards, a request that fits keeps the arena and
  its round, a larger one replaces it with zeroed counters and restarts the
  rounds (the counter targets of the pipelined forward derive from the
  round), and no rank frees memory a peer still has open, teardown included,
  at world 2, 4 and 8;
* a rank that never tears down, or never asks for the arena: the others'
  calls return REEF_B200_ERR_TIMEOUT after the communicator's timeout instead
  of waiting for good.

reef has no tensor parallelism (its TP=1 result is the oracle for the layer),
so this pins the communicator's own contract, not an algorithm of reef's.
Needs g++ and the CUDA and NCCL headers; skipped without them.
"""
import os
import shutil
import subprocess

import pytest

from reef_b200 import build

HERE = os.path.dirname(os.path.abspath(__file__))


def test_communicator_host_logic(tmp_path):
    cuda_inc = os.path.join(build.CUDA, "include")
    nccl_inc, _ = build._nccl_dirs()
    if shutil.which("g++") is None or not os.path.isfile(os.path.join(cuda_inc, "cuda_runtime.h")) \
            or not os.path.isfile(os.path.join(nccl_inc, "nccl.h")):
        pytest.skip("g++ or the CUDA / NCCL headers not present")
    exe = str(tmp_path / "comm_host_test")
    cmd = ["g++", "-std=c++20", "-O1", "-pthread", "-Wall", "-Werror=return-type",
           f"-I{os.path.join(build.ROOT, 'include')}", f"-I{build.CSRC}", f"-I{cuda_inc}",
           f"-I{nccl_inc}", os.path.join(build.CSRC, "comm.cpp"),
           os.path.join(HERE, "host", "fake_cuda_nccl.cpp"),
           os.path.join(HERE, "host", "comm_host_test.cpp"), "-o", exe]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    r = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr[-4000:]
    passed = {line[3:] for line in r.stdout.splitlines() if line.startswith("ok ")}
    assert passed == {"arena world 2", "arena world 4", "arena world 8", "teardown", "reserve"}
