"""reef_b200_linear_w8a8_noalloc against reef_b200_linear_w8a8_bias.

The no-allocation entry point serves callers that cannot allocate any device
memory (a host owning all of it through its own arena, or a port of reef's
never-allocating firmware): its quantisation scratch is a fixed array inside
the library instead of caller-provided buffers.  Its results must be
bit-identical to the scratch-taking entry point, on consecutive calls that
reuse the shared array with different shapes, and a shape whose scratch would
exceed the array must be refused with REEF_B200_ERR_TOO_LARGE.

This file sorts last so that a run stopping at the first failure has already
run every other test; it also passes alone in a fresh process.
"""
import numpy as np
import pytest
import torch

from oracle import oracle as ro
from reef_b200 import _lib
from reef_b200 import kernels as K

pytestmark = pytest.mark.gpu


def _noalloc(x, w, ws, bias):
    rows, k = x.shape
    n = w.shape[0]
    y = torch.empty((rows, n), dtype=torch.float32, device=x.device)
    _lib.call("reef_b200_linear_w8a8_noalloc", rows, k, n, x.data_ptr(), w.data_ptr(),
              ws.data_ptr(), None if bias is None else bias.data_ptr(), y.data_ptr(),
              torch.cuda.current_stream().cuda_stream)
    return y


def _case(rows, k, n, seed, with_bias):
    x = ro.normal(seed, (rows, k))
    x[rows // 2] = 0.0  # all-zero row: scale 1
    w, ws = ro.quantize_rows(ro.normal(seed + 1, (n, k), 0.0, 0.02))
    wp = np.zeros((n, K.kpad(k)), np.int8)
    wp[:, :k] = w
    b = ro.normal(seed + 2, (n,), 0.0, 0.02) if with_bias else None
    dev = lambda a: None if a is None else torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return dev(x), dev(wp), dev(ws), dev(b)


def test_noalloc_matches_scratch_entry_point_on_consecutive_calls(cuda_lib):
    # two calls in a row through the shared scratch: a wide-K call, then a
    # ragged one that leaves stale bytes of the first beyond its own rows;
    # each is compared with the scratch-taking entry point and with the oracle
    for rows, k, n, seed, with_bias in [(384, 4096, 1024, 11, True), (37, 200, 300, 12, False)]:
        x, w, ws, b = _case(rows, k, n, seed, with_bias)
        got = _noalloc(x, w, ws, b)
        want = K.linear_w8a8(x, w, ws, b)
        torch.cuda.synchronize()
        got_np = got.cpu().numpy()
        np.testing.assert_array_equal(got_np.view(np.uint32), want.cpu().numpy().view(np.uint32))
        oracle = ro.linear_w8a8(x.cpu().numpy(), w.cpu().numpy()[:, :k], ws.cpu().numpy(),
                                None if b is None else b.cpu().numpy())
        np.testing.assert_array_equal(got_np.view(np.uint32), oracle.view(np.uint32))
    K.check_device_error()


def test_noalloc_largest_accepted_shape_and_first_refused(cuda_lib):
    # at in = 4096 the scratch is rows * 4096 (a multiple of 256) + 4 * rows
    # bytes: 4092 rows need 16,777,200 of the 16,777,216 and run; 4093 rows
    # need 16,781,300 and are refused before anything is launched
    rows, k, n = 4092, 4096, 256
    x, w, ws, b = _case(rows, k, n, 21, True)
    got = _noalloc(x, w, ws, b)
    want = K.linear_w8a8(x, w, ws, b)
    torch.cuda.synchronize()
    np.testing.assert_array_equal(got.cpu().numpy().view(np.uint32),
                                  want.cpu().numpy().view(np.uint32))
    K.check_device_error()
    p = torch.empty(16, device="cuda")
    rc = _lib.lib().reef_b200_linear_w8a8_noalloc(rows + 1, k, n, p.data_ptr(), p.data_ptr(),
                                                   p.data_ptr(), None, p.data_ptr(), None)
    assert rc == 7  # REEF_B200_ERR_TOO_LARGE


def test_noalloc_rejects_shapes_beyond_its_scratch(cuda_lib):
    limit = 16 << 20
    rows, k = 5000, 4096  # 5000 * 4096 int8 > 16 MiB
    assert rows * k > limit
    p = torch.empty(16, device="cuda")
    rc = _lib.lib().reef_b200_linear_w8a8_noalloc(rows, k, 8, p.data_ptr(), p.data_ptr(),
                                                   p.data_ptr(), None, p.data_ptr(), None)
    assert rc == 7  # REEF_B200_ERR_TOO_LARGE
