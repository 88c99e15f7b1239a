"""GPT-Neo's lm_head row and the greedy argmax on the GPU, bit for bit.

reef_b200_matvec_rows_f32 must equal reef's float linear(x, wte) for one
row (the oracle, pinned to reef's kMatvec goldens and to the engine), at the
goldens' shapes, at GPT-Neo 28M's lm_head (50257 x 256) and at ragged
shapes; a product that overflows must be reported in the device error word
(the engine throws).  reef_b200_argmax_f32 must return the engine's index:
the first maximum, signed zeros equal, NaN never winning unless at index 0.
"""
import ctypes as C

import numpy as np
import pytest
import torch

from oracle import oracle as ro
from reef_b200 import _lib
from reef_b200 import kernels as K
from tests import goldens

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_lib):
    yield
    K.check_device_error()


def gpu_matvec(w, x):
    y = K.matvec_rows_f32(torch.from_numpy(np.ascontiguousarray(w)).cuda(),
                          torch.from_numpy(np.ascontiguousarray(x)).cuda())
    torch.cuda.synchronize()
    return y.cpu().numpy()


def gpu_argmax(x):
    idx = K.argmax_f32(torch.from_numpy(np.ascontiguousarray(x, np.float32)).cuda())
    torch.cuda.synchronize()
    return int(idx.cpu().numpy().view(np.uint32)[0])


def test_matvec_matches_reef_goldens():
    for c in goldens.cases("linear", "kMatvec"):
        y = gpu_matvec(c["w"].reshape(c["out"], c["in"]), c["x"])
        np.testing.assert_array_equal(y.view(np.uint32), c["y"].view(np.uint32))


@pytest.mark.parametrize("out,n", [(50257, 256), (1, 1), (129, 33), (7, 1000), (300, 31)])
def test_matvec_bit_identical_to_engine(out, n):
    rng = np.random.default_rng(out + n)
    w = rng.normal(0.0, 0.02, (out, n)).astype(np.float32)  # GPT-Neo's wte scale
    x = rng.normal(0.0, 1.0, n).astype(np.float32)
    want, ok = ro.matvec_rows_f32(w, x)
    assert ok
    np.testing.assert_array_equal(gpu_matvec(w, x).view(np.uint32), want.view(np.uint32))


def test_matvec_overflow_is_reported():
    w = np.full((130, 5), 1e30, np.float32)
    x = np.full(5, 1e30, np.float32)
    gpu_matvec(w, x)
    code = C.c_int(-1)
    assert _lib.lib().reef_b200_device_error(C.byref(code)) == 0
    assert code.value == 0x301


def test_argmax_matches_reef_goldens():
    for c in goldens.cases("elementwise", "kArgmax"):
        assert gpu_argmax(c["x"]) == c["index"]


def test_argmax_edge_cases_match_engine():
    rng = np.random.default_rng(5)
    cases = [rng.uniform(-10, 10, 50257).astype(np.float32),
             rng.uniform(-10, 10, 3_000_001).astype(np.float32),
             np.array([2.5], np.float32),
             np.array([1.0, 3.0, 3.0, 2.0], np.float32),
             np.array([0.0, -0.0], np.float32), np.array([-0.0, 0.0], np.float32),
             np.array([np.nan, 5.0, 1.0], np.float32),
             np.array([1.0, np.nan, 5.0, np.nan], np.float32),
             np.array([np.nan, np.nan], np.float32),
             np.array([-np.inf, -np.inf, -np.inf], np.float32)]
    ties = np.zeros(100_000, np.float32)
    ties[[4097, 70_000, 99_999]] = 7.0  # the first of three maxima far apart
    cases.append(ties)
    for v in cases:
        assert gpu_argmax(v) == ro.argmax_f32(v), v[:8]
