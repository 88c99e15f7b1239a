"""Parity of the tcgen05 int8 GEMM paths against reef (bit for bit).

* reef's own golden vectors (tests/golden, from gen_golden.cpp): W8A8 linear
  with and without bias (incl. the all-zero row), int8 linear with shift-1
  ties and int32 biases;
* the CPU oracle on seeded odd shapes (ragged M/N/K, partial tiles, tiny and
  wide) and on every config-5 sweep shape at full size (a row of every
  128-row block, all columns);
* the raw int32 partial-sum epilogue.
All comparisons are exact (bit patterns for fp32).
"""
import numpy as np
import pytest
import torch

from oracle import oracle as ro
from reef_b200 import kernels as K
from tests import goldens

pytestmark = pytest.mark.gpu


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def bits(a):
    a = np.asarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else a


def padk(w):
    """[n][k] -> [n][kpad(k)] zero-padded."""
    n, k = w.shape
    out = np.zeros((n, K.kpad(k)), w.dtype)
    out[:, :k] = w
    return out


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_lib):
    yield
    K.check_device_error()


# ---- reef's golden vectors -----------------------------------------------------

@pytest.mark.parametrize("table", ["kW8a8", "kW8a8Bias"])
def test_w8a8_goldens(table):
    for c in goldens.cases("linear", table):
        wt = dev(c["qt"].reshape(c["in"], c["out"]))  # Coral [in][out]
        w = K.pack_weight_i8(wt)
        x = dev(c["x"].reshape(c["rows"], c["in"]))
        b = dev(c["bias"]) if "bias" in c else None
        y = K.linear_w8a8(x, w, dev(c["qs"]), b)
        np.testing.assert_array_equal(bits(host(y).ravel()), bits(c["y"]))


@pytest.mark.parametrize("table", ["kInt8Linear", "kInt8LinearBias"])
def test_int8_goldens(table):
    for c in goldens.cases("int8", table):
        w = K.pack_weight_i8(dev(c["wt"].reshape(c["in"], c["out"])))
        x = K.pad_rows_i8(dev(c["x"].reshape(c["rows"], c["in"])))
        b = dev(c["bias"]) if "bias" in c else None
        y = K.linear_int8(x, w, c["shift"], b, in_features=c["in"])
        np.testing.assert_array_equal(host(y).ravel(), c["y"])


# ---- oracle, odd shapes ---------------------------------------------------------

SHAPES = [  # rows, in, out
    (1, 7, 5), (3, 37, 21), (2, 64, 48), (1, 256, 64), (17, 130, 33),
    (128, 128, 128), (129, 256, 257), (255, 1000, 300), (300, 384, 520),
    (1, 4096, 4096), (64, 8192, 1024), (513, 512, 2048),
]


@pytest.mark.parametrize("rows,k,n", SHAPES)
def test_w8a8_matches_oracle(rows, k, n):
    seed = rows * 1000 + k + n
    x = ro.normal(seed, (rows, k))
    x[rows // 2] = 0.0                      # all-zero row: scale 1
    x[-1, :: max(1, k // 5)] *= 1e4         # a row dominated by a few values
    w, ws = ro.quantize_rows(ro.normal(seed + 1, (n, k), 0.0, 0.02))
    bias = ro.normal(seed + 2, (n,), 0.0, 0.02)
    want = ro.linear_w8a8(x, w, ws, bias)
    got = host(K.linear_w8a8(dev(x), dev(padk(w)), dev(ws), dev(bias)))
    np.testing.assert_array_equal(bits(got), bits(want))
    want_nb = ro.linear_w8a8(x, w, ws)
    got_nb = host(K.linear_w8a8(dev(x), dev(padk(w)), dev(ws)))
    np.testing.assert_array_equal(bits(got_nb), bits(want_nb))


def test_quantize_rows_matches_oracle():
    x = ro.normal(5, (37, 1000))
    x[3] = 0.0
    x[4, 7] = 127.0 * 3.0
    # near-ties that a multiply by the reciprocal of the scale (128/127) rounds
    # the other way: the quantiser's fast path must hand them to the division
    x[5, :4] = [128.0, 5.543306827545166, 7.559054851531982, 88.18897247314453]
    x[5, 4:] = 0.0
    q, s = K.quantize_rows(dev(x))
    wq, ws = ro.quantize_rows(x)
    np.testing.assert_array_equal(host(q)[:, :1000], wq)
    assert list(host(q)[5, :4]) == [127, 6, 8, 88]
    assert not host(q)[:, 1000:].any()
    np.testing.assert_array_equal(bits(host(s)), bits(ws))


@pytest.mark.parametrize("rows,k,n,shift", [(1, 7, 5, 1), (16, 64, 64, 8),
                                            (33, 200, 130, 1), (130, 4096, 300, 12),
                                            (5, 96, 1000, 31), (7, 64, 9, 0)])
def test_int8_linear_matches_oracle(rows, k, n, shift):
    seed = 7 * rows + k + n
    x = ro.int8_uniform(seed, (rows, k))
    w = ro.int8_uniform(seed + 1, (n, k))
    bias = ro.int32_uniform(seed + 2, (n,), -4096, 4096)
    want = ro.linear_int8(x, w, shift, bias)
    got = host(K.linear_int8(dev(padk(x)), dev(padk(w)), shift, dev(bias), in_features=k))
    np.testing.assert_array_equal(got, want)


def test_random_shapes_match_oracle():
    """24 seeded random W8A8 shapes (rows 1-600, in 1-2100, out 1-700: both
    the skinny and the persistent GEMM paths, partial tiles on every side),
    each with and without bias, on activations with exact ties, zeros,
    negative zeros, denormals and all-zero rows; and 12 int8 linears with
    random shifts 0-31 and int32 biases.  Bit for bit against the oracle."""
    from tests.test_oracle import _sweep_activation
    rng = np.random.default_rng(31337)
    for case in range(24):
        rows = int(rng.integers(1, 601))
        k = int(rng.integers(1, 2101))
        n = int(rng.integers(1, 701))
        x = _sweep_activation(rng, rows, k)
        w, ws = ro.quantize_rows((rng.standard_normal((n, k)) * 0.02).astype(np.float32))
        bias = (rng.standard_normal(n) * 0.02).astype(np.float32)
        for b in (bias, None):
            want = ro.linear_w8a8(x, w, ws, b)
            got = host(K.linear_w8a8(dev(x), dev(padk(w)), dev(ws),
                                     None if b is None else dev(b)))
            np.testing.assert_array_equal(bits(got), bits(want),
                                          err_msg=f"case {case}: {rows}x{k}x{n}")
    for case in range(12):
        rows, k, n = int(rng.integers(1, 300)), int(rng.integers(1, 1500)), int(rng.integers(1, 500))
        shift = int(rng.integers(0, 32))
        x = rng.integers(-128, 128, (rows, k)).astype(np.int8)
        w = rng.integers(-128, 128, (n, k)).astype(np.int8)
        bias = rng.integers(-(1 << 20), 1 << 20, n).astype(np.int32)
        want = ro.linear_int8(x, w, shift, bias)
        got = host(K.linear_int8(dev(padk(x)), dev(padk(w)), shift, dev(bias), in_features=k))
        np.testing.assert_array_equal(got, want, err_msg=f"int8 case {case}: {rows}x{k}x{n}")


@pytest.mark.parametrize("m,n,k", [(1, 8, 16), (128, 256, 128), (200, 300, 4096),
                                   (1000, 129, 28672)])
def test_gemm_i32_matches_oracle(m, n, k):
    a = ro.int8_uniform(m + n, (m, k), -127, 127)
    b = ro.int8_uniform(m + n + 1, (n, k), -127, 127)
    got = host(K.gemm_i8_i32(dev(padk(a)), dev(padk(b)), k))
    np.testing.assert_array_equal(got, ro.gemm_i8(a, b))


# ---- config 5: the GEMM sweep at full size, a row of every 128-row block ------------

SWEEP_NK = [(4096, 4096), (11008, 4096), (4096, 11008), (28672, 8192), (8192, 28672)]
SWEEP_M = [1, 16, 128, 1024, 8192, 16384]


@pytest.mark.parametrize("n,k", SWEEP_NK)
@pytest.mark.parametrize("m", SWEEP_M)
def test_sweep_shapes_sampled(m, n, k):
    g = torch.Generator(device="cuda").manual_seed(m * 7 + n + k)
    a = torch.randint(-127, 128, (m, k), generator=g, device="cuda", dtype=torch.int8)
    b = torch.randint(-127, 128, (n, k), generator=g, device="cuda", dtype=torch.int8)
    xs = torch.rand((m,), generator=g, device="cuda") * 1e-3 + 1e-3
    ws = torch.rand((n,), generator=g, device="cuda") * 1e-3 + 1e-3
    y = K.gemm_w8a8(a, xs, b, ws)
    # one row of every 128-row block (at a seeded offset inside it) and the
    # last row, each across all N columns: every output tile of the
    # persistent, raster-grouped schedule is compared, group boundaries
    # included
    off = np.random.default_rng(m + n).integers(0, 128, (m + 127) // 128)
    rows = sorted({m - 1, *[min(m - 1, 128 * i + int(o)) for i, o in enumerate(off)]})
    idx = torch.tensor(rows, device="cuda")
    acc = ro.gemm_i8(host(a.index_select(0, idx)), host(b))
    want = ro.w8a8_epilogue(acc, host(xs)[rows], host(ws))
    np.testing.assert_array_equal(bits(host(y.index_select(0, idx))), bits(want))


# ---- skinny (decode) GEMM: swap-AB + split-K ---------------------------------------

# the config-4 decode shapes (tiles fit one wave) and wide weights with more
# 128-row tiles than SMs (the split chosen by the multi-wave cost)
@pytest.mark.parametrize("m", [1, 16, 64, 100, 128])
@pytest.mark.parametrize("n,k", [(1280, 8192), (8192, 1024), (7168, 8192), (8192, 3584),
                                 (300, 200), (19000, 1024), (28672, 2048)])
def test_skinny_gemm_matches_oracle(m, n, k):
    g = torch.Generator(device="cuda").manual_seed(m + n + k)
    a = torch.randint(-127, 128, (m, K.kpad(k)), generator=g, device="cuda", dtype=torch.int8)
    b = torch.randint(-127, 128, (n, K.kpad(k)), generator=g, device="cuda", dtype=torch.int8)
    xs = torch.rand((m,), generator=g, device="cuda") * 1e-3 + 1e-3
    ws = torch.rand((n,), generator=g, device="cuda") * 1e-3 + 1e-3
    bias = torch.rand((n,), generator=g, device="cuda")
    y = K.gemm_w8a8_skinny(a, xs, b, ws, bias, in_features=k)
    acc = ro.gemm_i8(host(a)[:, :k], host(b)[:, :k])
    want = ro.w8a8_epilogue(acc, host(xs), host(ws), host(bias))
    np.testing.assert_array_equal(bits(host(y)), bits(want))


# ---- gate/up projection with SwiGLU in the epilogue ----------------------------------

# one and many tiles, ffn not a multiple of the 128-column output tile, rows not
# a multiple of the 128-row tile, the config-3 FFN width
@pytest.mark.parametrize("rows,k,ffn", [(128, 256, 128), (300, 512, 640), (257, 1024, 136),
                                        (64, 4096, 11008), (1000, 64, 48)])
def test_swiglu_gemm(rows, k, ffn):
    """g, u: the oracle's W8A8 linear (bit-exact reference for the GEMM part);
    h = silu(g) * u within the fast exp / divide the kernel uses (a few ulp);
    row_max = max |h| of the returned h, exactly."""
    g = torch.Generator(device="cuda").manual_seed(rows + k + ffn)
    a = torch.randint(-127, 128, (rows, K.kpad(k)), generator=g, device="cuda", dtype=torch.int8)
    w = torch.randint(-127, 128, (2 * ffn, K.kpad(k)), generator=g, device="cuda",
                      dtype=torch.int8)
    xs = torch.rand((rows,), generator=g, device="cuda") * 1e-3 + 1e-4
    ws = torch.rand((2 * ffn,), generator=g, device="cuda") * 1e-3 + 1e-4
    h, row_max = K.linear_w8a8_swiglu(a, xs, w, ws, in_features=k)
    acc = ro.gemm_i8(host(a)[:, :k], host(w)[:, :k])
    gu = ro.w8a8_epilogue(acc, host(xs), host(ws), None).astype(np.float64)
    gate, up = gu[:, :ffn], gu[:, ffn:]
    want = gate / (1.0 + np.exp(-gate)) * up
    got = host(h)
    np.testing.assert_allclose(got, want, rtol=2e-5, atol=1e-6)
    np.testing.assert_array_equal(bits(host(row_max)), bits(np.abs(got).max(axis=1)))
