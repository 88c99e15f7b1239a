"""The tensor-parallel communicator's and layer drivers' host logic on the CPU.

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

The Llama layer's drivers (reef_b200/csrc/layer.cpp) run the same way, with the
kernels stubbed out and the cross-rank counter waits done on the host with a
deadline (tests/host/fake_ops.cpp, tests/host/layer_host_test.cpp): at world
2, 4 and 8, one communicator goes through the pipelined all-gather forward at
2 and then 4 chunks, the unpipelined one, a wider layer, the all-reduce plan,
the instrumented forward and the first layer again; no counter wait may run
out, and each rank's counters must add up to the signals those forwards send.
The decode step under both plans and reef's GPT-Neo block run at the same
world sizes, every rank issuing the same collectives in the same order.
The communicator from before the arena fix (a new arena that kept counting
forward rounds) makes these waits run out, as it stalled the tensor-parallel
GPU test.

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


def _build_and_run(tmp_path, name: str, sources: list[str], sanitize: bool = False,
                   args: tuple[str, ...] = ()) -> set[str]:
    """Compile `sources` with the fakes into one program, run it, and return
    the names of its passing cases.  sanitize: AddressSanitizer, so a copy
    outside a host buffer (a collective into a mis-sized workspace region)
    fails the run."""
    cuda_inc = os.path.join(build.CUDA, "include")
    nccl_inc, _ = build._nccl_dirs()
    if shutil.which("g++") is None or not os.path.isfile(os.path.join(cuda_inc, "cuda_runtime.h")) \
            or not os.path.isfile(os.path.join(nccl_inc, "nccl.h")):
        pytest.skip("g++ or the CUDA / NCCL headers not present")
    exe = str(tmp_path / name)
    cmd = ["g++", "-std=c++20", "-O1", "-pthread", "-Wall", "-Werror=return-type",
           f"-I{os.path.join(build.ROOT, 'include')}", f"-I{build.CSRC}", f"-I{cuda_inc}",
           f"-I{nccl_inc}", *sources, os.path.join(HERE, "host", "fake_cuda_nccl.cpp"), "-o", exe]
    if sanitize:
        cmd.insert(1, "-fsanitize=address,undefined")
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-4000:]
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=0")
    r = subprocess.run([exe, *args], capture_output=True, text=True, timeout=180, env=env)
    assert r.returncode == 0, r.stdout + r.stderr[-4000:]
    return {line[3:] for line in r.stdout.splitlines() if line.startswith("ok ")}


def test_communicator_host_logic(tmp_path):
    passed = _build_and_run(tmp_path, "comm_host_test", [
        os.path.join(build.CSRC, "comm.cpp"), os.path.join(HERE, "host", "comm_host_test.cpp")])
    assert passed == {"arena world 2", "arena world 4", "arena world 8", "teardown", "reserve"}


def test_pipelined_forward_schedule(tmp_path):
    passed = _build_and_run(tmp_path, "layer_host_test", [
        os.path.join(build.CSRC, "layer.cpp"), os.path.join(build.CSRC, "comm.cpp"),
        os.path.join(HERE, "host", "fake_ops.cpp"),
        os.path.join(HERE, "host", "layer_host_test.cpp")], sanitize=True)
    assert passed == {"world 2", "world 4", "world 8", "decode and gptneo world 2",
                      "decode and gptneo world 4", "decode and gptneo world 8"}
