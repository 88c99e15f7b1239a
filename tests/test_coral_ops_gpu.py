"""The rest of reef's Coral operator set on the GPU, bit for bit.

Every reef_kernels function (coral/include/reef_kernels/kernels.hpp) has a
reef_b200_ entry point; the W8A8 / int8 linears, heads, lm_head, argmax and
embedding have their own tests.  Here: the float linear ± bias, layernorm,
gelu, exp_nonpositive, tanh and add of the float path, and the int8 gelu
table, layernorm, saturating add and embedding -- each against reef's own
golden vectors and, at larger sizes, against the oracle.
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


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def st():
    return torch.cuda.current_stream().cuda_stream


def fbits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def gpu_linear_f32(x, wt, bias=None):
    rows, n_in = x.shape
    out = wt.shape[1]
    y = torch.empty((rows, out), device="cuda")
    xd, wd = dev(x), dev(wt)
    if bias is None:
        _lib.call("reef_b200_linear_f32", rows, n_in, out, xd.data_ptr(), wd.data_ptr(),
                  y.data_ptr(), st())
    else:
        bd = dev(bias)
        _lib.call("reef_b200_linear_bias_f32", rows, n_in, out, xd.data_ptr(), wd.data_ptr(),
                  bd.data_ptr(), y.data_ptr(), st())
    torch.cuda.synchronize()
    return y.cpu().numpy()


def test_linear_f32_matches_reef_goldens():
    for table in ("kLinear", "kLinearBias"):
        for c in goldens.cases("linear", table):
            x = c["x"].reshape(c["rows"], c["in"])
            wt = c["wt"].reshape(c["in"], c["out"])
            y = gpu_linear_f32(x, wt, c.get("bias"))
            np.testing.assert_array_equal(fbits(y).ravel(), fbits(c["y"]))


@pytest.mark.parametrize("rows,n_in,out", [(1, 768, 3072), (5, 257, 300), (17, 64, 1)])
def test_linear_f32_bit_identical_to_engine(rows, n_in, out):
    rng = np.random.default_rng(rows + n_in + out)
    x = rng.normal(0, 1, (rows, n_in)).astype(np.float32)
    wt = rng.normal(0, 0.02, (n_in, out)).astype(np.float32)
    b = rng.normal(0, 0.02, out).astype(np.float32)
    np.testing.assert_array_equal(fbits(gpu_linear_f32(x, wt, b)),
                                  fbits(ro.linear_f32(x, wt, b)))


def test_layernorm_f32_matches_reef_goldens():
    for c in goldens.cases("layernorm", "kLayerNorm"):
        rows, w = c["rows"], c["width"]
        x, g, s = dev(c["x"]), dev(c["gain"]), dev(c["shift"])
        y = torch.empty(rows * w, device="cuda")
        _lib.call("reef_b200_layernorm_f32", rows, w, x.data_ptr(), g.data_ptr(), s.data_ptr(),
                  c["eps"], y.data_ptr(), st())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(fbits(y.cpu().numpy()), fbits(c["y"]))


@pytest.mark.parametrize("table,fn", [("kExp", "reef_b200_exp_nonpositive_f32"),
                                      ("kTanh", "reef_b200_tanh_f32"),
                                      ("kGelu", "reef_b200_gelu_f32")])
def test_unary_f32_matches_reef_goldens(table, fn):
    for c in goldens.cases("math", table):
        x = dev(c["x"])
        y = torch.empty_like(x)
        _lib.call(fn, x.numel(), x.data_ptr(), y.data_ptr(), st())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(fbits(y.cpu().numpy()), fbits(c["y"]))


def test_add_f32_matches_reef_goldens_and_reports_overflow():
    for c in goldens.cases("elementwise", "kAdd"):
        a, b = dev(c["a"]), dev(c["b"])
        y = torch.empty_like(a)
        _lib.call("reef_b200_add_f32", a.numel(), a.data_ptr(), b.data_ptr(), y.data_ptr(), st())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(fbits(y.cpu().numpy()), fbits(c["y"]))
    big = torch.full((40,), 3e38, device="cuda")
    y = torch.empty_like(big)
    _lib.call("reef_b200_add_f32", 40, big.data_ptr(), big.data_ptr(), y.data_ptr(), st())
    code = C.c_int(-1)
    assert _lib.lib().reef_b200_device_error(C.byref(code)) == 0
    assert code.value == 0x301


def test_int8_operators_match_reef_goldens():
    for c in goldens.cases("int8", "kInt8Gelu"):
        x, t = dev(c["x"]), dev(c["table"])
        y = torch.empty_like(x)
        _lib.call("reef_b200_gelu_int8", x.numel(), x.data_ptr(), t.data_ptr(), y.data_ptr(), st())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(y.cpu().numpy(), c["y"])
    for c in goldens.cases("int8", "kInt8LayerNorm"):
        x, g, s = dev(c["x"]), dev(c["gain"]), dev(c["shift"])
        y = torch.empty_like(x)
        _lib.call("reef_b200_layernorm_int8", c["rows"], c["width"], x.data_ptr(), g.data_ptr(),
                  s.data_ptr(), y.data_ptr(), st())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(y.cpu().numpy(), c["y"])
    for c in goldens.cases("int8", "kInt8Add"):
        a, b = dev(c["a"]), dev(c["b"])
        y = torch.empty_like(a)
        _lib.call("reef_b200_add_int8", a.numel(), a.data_ptr(), b.data_ptr(), y.data_ptr(), st())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(y.cpu().numpy(), c["y"])
    for c in goldens.cases("int8", "kInt8Embedding"):
        w = c["width"]
        wte, wpe = dev(c["wte"]), dev(c["wpe"])
        ids = torch.tensor([c["id"]], dtype=torch.int32, device="cuda")
        y = torch.empty(w, dtype=torch.int8, device="cuda")
        _lib.call("reef_b200_embedding_int8", w, 1, ids.data_ptr(), c["position"],
                  wte.numel() // w, wpe.numel() // w, wte.data_ptr(), wpe.data_ptr(),
                  y.data_ptr(), st())
        torch.cuda.synchronize()
        np.testing.assert_array_equal(y.cpu().numpy(), c["y"])


@pytest.mark.parametrize("rows,width", [(300, 768), (7, 4096), (2, 32767), (64, 1)])
def test_layernorm_int8_exact_at_width(rows, width):
    rng = np.random.default_rng(rows * width)
    x = rng.integers(-128, 128, (rows, width), dtype=np.int8)
    g = rng.integers(-128, 128, width, dtype=np.int8)
    s = rng.integers(-128, 128, width, dtype=np.int8)
    y = torch.empty((rows, width), dtype=torch.int8, device="cuda")
    xd, gd, sd = dev(x), dev(g), dev(s)
    _lib.call("reef_b200_layernorm_int8", rows, width, xd.data_ptr(), gd.data_ptr(),
              sd.data_ptr(), y.data_ptr(), st())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y.cpu().numpy(), ro.layernorm_int8(x, g, s))


def test_int8_elementwise_large():
    rng = np.random.default_rng(9)
    n = 3_000_001
    a = rng.integers(-128, 128, n, dtype=np.int8)
    b = rng.integers(-128, 128, n, dtype=np.int8)
    table = rng.integers(-128, 128, 256, dtype=np.int8)
    ad, bd, td = dev(a), dev(b), dev(table)
    y = torch.empty(n, dtype=torch.int8, device="cuda")
    _lib.call("reef_b200_add_int8", n, ad.data_ptr(), bd.data_ptr(), y.data_ptr(), st())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y.cpu().numpy(), ro.add_int8(a, b))
    _lib.call("reef_b200_gelu_int8", n, ad.data_ptr(), td.data_ptr(), y.data_ptr(), st())
    torch.cuda.synchronize()
    np.testing.assert_array_equal(y.cpu().numpy(), ro.gelu_int8(a, table))
