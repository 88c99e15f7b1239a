"""Failure detection on the GPU without a fault: a bounded mbarrier wait that
nothing satisfies, and the tensor-parallel forward's wait on a peer counter
that nothing increments (how a dead peer looks to a rank), each give up
after their limit, record their code in the device error word and return;
the context stays usable (a W8A8 linear right after is still bit-exact with
the oracle).
"""
import ctypes as C
import time

import numpy as np
import pytest
import torch

from oracle import oracle as ro
from reef_b200 import _lib
from reef_b200 import kernels as K

pytestmark = pytest.mark.gpu


def device_error() -> int:
    code = C.c_int(0)
    _lib.call("reef_b200_device_error", C.addressof(code))
    return code.value


def test_bounded_wait_times_out_and_context_survives():
    assert device_error() == 0  # clean before
    done = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.call("reef_b200_selftest_wait_timeout", 2000, done.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert int(done.item()) == 2          # the wait gave up
    assert device_error() == 0x101        # kDevTimeoutFull, read and cleared
    assert device_error() == 0
    # the device still computes correctly
    x = ro.normal(11, (64, 256))
    w, ws = ro.quantize_rows(ro.normal(12, (96, 256), 0, 0.02))
    y = K.linear_w8a8(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(),
                      torch.from_numpy(ws).cuda())
    want = ro.linear_w8a8(x, w, ws)
    np.testing.assert_array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_peer_counter_wait_times_out_and_context_survives():
    assert device_error() == 0
    stream = torch.cuda.current_stream().cuda_stream
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    # a counter that already reached its target: the wait returns at once
    counter.fill_(5)
    _lib.call("reef_b200_selftest_peer_wait_timeout", 2000, counter.data_ptr(), 3, stream)
    torch.cuda.synchronize()
    assert device_error() == 0
    # a counter nothing increments: the wait gives up after 2 ms
    counter.zero_()
    _lib.call("reef_b200_selftest_peer_wait_timeout", 2000, counter.data_ptr(), 1, stream)
    torch.cuda.synchronize()
    assert device_error() == 0x106        # kDevTimeoutPeer, read and cleared
    assert device_error() == 0
    x = ro.normal(13, (64, 256))
    w, ws = ro.quantize_rows(ro.normal(14, (96, 256), 0, 0.02))
    y = K.linear_w8a8(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda(),
                      torch.from_numpy(ws).cuda())
    want = ro.linear_w8a8(x, w, ws)
    np.testing.assert_array_equal(y.cpu().numpy().view(np.uint32), want.view(np.uint32))


def test_peer_wait_after_a_timeout_returns_at_once():
    """Once a peer wait has given up (0x106 in the error word, not yet read),
    later waits return at once instead of each running out its own limit: a
    wait with a 1.5 s limit on a counter nothing increments ends in well
    under that."""
    assert device_error() == 0
    stream = torch.cuda.current_stream().cuda_stream
    counter = torch.zeros(1, dtype=torch.int32, device="cuda")
    _lib.call("reef_b200_selftest_peer_wait_timeout", 2000, counter.data_ptr(), 1, stream)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    _lib.call("reef_b200_selftest_peer_wait_timeout", 1500000, counter.data_ptr(), 1, stream)
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 0.5
    assert device_error() == 0x106
    assert device_error() == 0
