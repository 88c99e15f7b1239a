"""Pins the CPU oracle before anything is checked against it.

1. Against reef's own golden vectors (tests/golden, written by the reference's
   gen_golden.cpp): bit for bit.
2. Against reef's known-answer tests (inference-engine/reference/cpp/tests/
   test_quant.cpp, test_int8.cpp), restated here.
3. Against reef's engine compiled in place (oracle/_ref) on fresh seeded
   inputs, where that library was built.
No GPU is needed.
"""
import numpy as np
import pytest

from oracle import oracle as ro
from tests import goldens


def bits(a):
    a = np.asarray(a)
    return a.view(np.uint32) if a.dtype == np.float32 else a


# ---- 1. golden vectors -----------------------------------------------------

@pytest.mark.parametrize("table", ["kW8a8", "kW8a8Bias"])
def test_w8a8_linear_matches_reef_goldens(table):
    for c in goldens.cases("linear", table):
        x = c["x"].reshape(c["rows"], c["in"])
        w = c["qt"].reshape(c["in"], c["out"]).T  # [in][out] -> [out][in]
        y = ro.linear_w8a8(x, w, c["qs"], c.get("bias"))
        np.testing.assert_array_equal(bits(y.ravel()), bits(c["y"]))


@pytest.mark.parametrize("table", ["kInt8Linear", "kInt8LinearBias"])
def test_int8_linear_matches_reef_goldens(table):
    for c in goldens.cases("int8", table):
        x = c["x"].reshape(c["rows"], c["in"])
        w = c["wt"].reshape(c["in"], c["out"]).T
        y = ro.linear_int8(x, w, c["shift"], c.get("bias"))
        np.testing.assert_array_equal(y.ravel(), c["y"])


def test_softmax_int8_matches_reef_goldens():
    for c in goldens.cases("int8", "kInt8Softmax"):
        np.testing.assert_array_equal(ro.exp_table(), c["table"])
        s = c["scores"].reshape(c["rows"], c["n"])
        p = ro.softmax_int8(s, c["shift"], c["table"])
        np.testing.assert_array_equal(p.ravel(), c["probs"])


def test_attention_int8_matches_reef_goldens():
    for c in goldens.cases("int8", "kInt8Attention"):
        d = c["head_dim"]
        y = ro.attention_head_int8(
            c["q"].reshape(-1, d), c["k"].reshape(-1, d), c["v"].reshape(-1, d),
            c["query_start"], c["window"], c["score_shift"], c["out_shift"],
            c["table"])
        np.testing.assert_array_equal(y.ravel(), c["y"])


def test_attention_f32_matches_reef_goldens():
    for c in goldens.cases("attention", "kAttention"):
        d = c["head_dim"]
        y = ro.attention_head_f32(
            c["q"].reshape(-1, d), c["k"].reshape(-1, d), c["v"].reshape(-1, d),
            c["query_start"], c["window"])
        np.testing.assert_array_equal(bits(y.ravel()), bits(c["y"]))


def test_matvec_matches_reef_goldens():
    for c in goldens.cases("linear", "kMatvec"):
        y, ok = ro.matvec_rows_f32(c["w"].reshape(c["out"], c["in"]), c["x"])
        assert ok
        np.testing.assert_array_equal(bits(y), bits(c["y"]))


def test_argmax_matches_reef_goldens():
    cs = goldens.cases("elementwise", "kArgmax")
    assert len(cs) == 3  # random, ties (first of two maxima), signed zeros
    for c in cs:
        assert ro.argmax_f32(c["x"]) == c["index"]


def test_exp_tanh_gelu_match_reef_goldens():
    (e,) = goldens.cases("math", "kExp")
    np.testing.assert_array_equal(bits(ro.exp_nonpositive(e["x"])), bits(e["y"]))
    (g,) = goldens.cases("math", "kGelu")
    np.testing.assert_array_equal(bits(ro.gelu(g["x"])), bits(g["y"]))


def test_layernorm_matches_reef_goldens():
    for c in goldens.cases("layernorm", "kLayerNorm"):
        x = c["x"].reshape(c["rows"], c["width"])
        y = ro.layernorm(x, c["gain"], c["shift"], np.float32(c["eps"]))
        np.testing.assert_array_equal(bits(y.ravel()), bits(c["y"]))


# ---- 2. reef's known-answer tests -------------------------------------------

def test_quant_kats():
    # test_quant.cpp:38-53
    f = ro.lib().ro_int8_scale
    assert f(254.0) == 2.0 and f(127.0) == 1.0 and f(0.0) == 1.0
    q, s = ro.quantize_rows(np.array(
        [[254.0, 127.0, -127.0], [0, 0, 0], [1.0, -0.5, 0.25]], np.float32))
    assert list(q[0]) == [127, 64, -64] and s[0] == 2.0  # 63.5 ties to 64
    assert s[1] == 1.0 and list(q[1]) == [0, 0, 0]
    assert s[2] == np.float32(1.0) / np.float32(127.0) and q[2, 0] == 127
    q, _ = ro.quantize_rows(np.array([[2.5, 3.5, -2.5, 2.4, 127.0]], np.float32))
    assert list(q[0]) == [2, 4, -2, 2, 127]


def test_w8a8_hand_computed_kat():
    # test_quant.cpp:78-95
    x = np.array([[127.0, -2.5, 3.5]], np.float32)
    wq, ws = ro.quantize_rows(np.array(
        [[1.0, 0.0, -1.0], [254.0, 127.0, -127.0]], np.float32))
    y = ro.linear_w8a8(x, wq, ws, np.array([0.5, -1.0], np.float32))
    first = np.float32(15621.0) * (np.float32(1.0) * (np.float32(1.0) / np.float32(127.0)))
    assert y[0, 0] == first + np.float32(0.5)
    assert y[0, 1] == np.float32(15745.0) * np.float32(2.0) - np.float32(1.0)


def test_int8_kats():
    # test_int8.cpp:37-86, 117-159
    rs = ro.rounding_shift
    assert [rs(3, 1), rs(-3, 1), rs(5, 2), rs(6, 2), rs(-6, 2), rs(-7, 2),
            rs(-7, 0)] == [2, -1, 1, 2, -1, -2, -7]
    assert [ro.saturate_int8(v) for v in (127, 128, -128, -100000)] == \
        [127, 127, -128, -128]
    x = np.array([[1, 2]], np.int8)
    w = np.array([[3, -4], [127, 127]], np.int8)
    y = ro.linear_int8(x, w, 2, np.array([100, 0], np.int32))
    assert list(y[0]) == [24, 95]
    assert ro.linear_int8(x, w, 0)[0, 1] == 127
    t = ro.exp_table()
    assert t[0] == 32768 and t[16] == 12055 and t[255] == 0
    assert np.all(np.diff(t.astype(np.int32)) <= 0)
    p = ro.softmax_int8(np.array([[5, 5]], np.int32), 0)
    assert list(p[0]) == [128, 128]


# ---- 3. the engine itself, compiled in place --------------------------------

needs_ref = pytest.mark.skipif(not ro.ref_available(),
                               reason="oracle/_ref not built")


def _c(a, t):
    return a.ctypes.data_as(t)


@needs_ref
@pytest.mark.parametrize("rows,k,n,seed", [(5, 96, 40, 11), (17, 130, 33, 12),
                                           (1, 256, 64, 13)])
def test_w8a8_matches_engine(rows, k, n, seed):
    import ctypes as C
    x = ro.normal(seed, (rows, k))
    x[0] = 0.0  # the all-zero scale
    w, ws = ro.quantize_rows(ro.normal(seed + 100, (n, k), 0.0, 0.02))
    b = ro.normal(seed + 200, (n,), 0.0, 0.02)
    want = np.empty((rows, n), np.float32)
    rc = ro.ref().ref_linear_w8a8(rows, k, n, _c(x, C.POINTER(C.c_float)),
                                  _c(w, C.POINTER(C.c_int8)),
                                  _c(ws, C.POINTER(C.c_float)),
                                  _c(b, C.POINTER(C.c_float)),
                                  _c(want, C.POINTER(C.c_float)))
    assert rc == 0
    got = ro.linear_w8a8(x, w, ws, b)
    np.testing.assert_array_equal(bits(got), bits(want))


def _sweep_activation(rng, rows: int, k: int) -> np.ndarray:
    """Activations at the quantiser's hard cases: magnitudes from denormal to
    1e3, exact zeros and negative zeros, all-zero rows, and rows whose scale
    is a power of two with values at c + 1/2 exactly (ties to even)."""
    x = (rng.standard_normal((rows, k)) * 10.0 ** rng.uniform(-6, 3, (rows, 1))).astype(np.float32)
    x[rng.random((rows, k)) < 0.05] = 0.0
    x[rng.random((rows, k)) < 0.02] = -0.0
    x[rng.random((rows, k)) < 0.02] = np.float32(1e-40) * rng.choice([-1, 1])
    for r in range(rows):
        kind = rng.integers(0, 6)
        if kind == 0:
            x[r] = 0.0
        elif kind == 1:  # scale 2^e: the maximum is 127 * 2^e, the rest ties
            e = int(rng.integers(-20, 10))
            codes = rng.integers(-126, 126, k).astype(np.float32) + 0.5
            x[r] = np.ldexp(codes, e).astype(np.float32)
            x[r, int(rng.integers(0, k))] = np.float32(np.ldexp(127.0, e)) * rng.choice([-1, 1])
    return x


@needs_ref
def test_random_sweep_matches_engine():
    """120 seeded random shapes (rows 1-24, in 1-300 around the 16-byte
    padding edges, out 1-70) through quantize_rows, the W8A8 linear with and
    without bias, the int8 linear (shift 1-31, int32 bias) and the int8
    matmul: the restatement equals reef's engine bit for bit in every one."""
    import ctypes as C
    f32, i8, i32 = C.POINTER(C.c_float), C.POINTER(C.c_int8), C.POINTER(C.c_int32)
    rng = np.random.default_rng(20261202)
    R = ro.ref()
    for case in range(120):
        rows = int(rng.integers(1, 25))
        k = int(rng.choice([1, 2, 15, 16, 17, 31, 33, 64, 127, 129, int(rng.integers(1, 301))]))
        n = int(rng.integers(1, 71))
        x = _sweep_activation(rng, rows, k)
        wf = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
        # quantize_rows
        q_want = np.empty((rows, k), np.int8)
        s_want = np.empty(rows, np.float32)
        assert R.ref_quantize_rows(rows, k, _c(x, f32), _c(q_want, i8), _c(s_want, f32)) == 0
        q, sc = ro.quantize_rows(x)
        np.testing.assert_array_equal(q, q_want, err_msg=f"case {case}")
        np.testing.assert_array_equal(bits(sc), bits(s_want), err_msg=f"case {case}")
        # the W8A8 linear, with and without bias
        w, ws = ro.quantize_rows(wf)
        b = (rng.standard_normal(n) * 0.02).astype(np.float32)
        for bias in (None, b):
            want = np.empty((rows, n), np.float32)
            assert R.ref_linear_w8a8(rows, k, n, _c(x, f32), _c(w, i8), _c(ws, f32),
                                     None if bias is None else _c(bias, f32),
                                     _c(want, f32)) == 0
            got = ro.linear_w8a8(x, w, ws, bias)
            np.testing.assert_array_equal(bits(got), bits(want), err_msg=f"case {case}")
        # the int8 linear and the exact int8 matmul
        xi = rng.integers(-128, 128, (rows, k)).astype(np.int8)
        wi = rng.integers(-128, 128, (n, k)).astype(np.int8)
        shift = int(rng.integers(1, 32))
        bi = rng.integers(-(1 << 20), 1 << 20, n).astype(np.int32)
        for bias in (None, bi):
            want8 = np.empty((rows, n), np.int8)
            assert R.ref_linear_int8(rows, k, n, _c(xi, i8), _c(wi, i8), shift,
                                     None if bias is None else _c(bias, i32),
                                     _c(want8, i8)) == 0
            np.testing.assert_array_equal(ro.linear_int8(xi, wi, shift, bias), want8,
                                          err_msg=f"case {case}")
        acc = np.empty((rows, n), np.int32)
        assert R.ref_matmul_i8(rows, n, k, _c(xi, i8), _c(wi, i8), _c(acc, i32)) == 0
        np.testing.assert_array_equal(ro.gemm_i8(xi, wi), acc, err_msg=f"case {case}")


@needs_ref
def test_random_attention_sweep_matches_engine():
    """160 seeded random heads, int8 and float: query and key lengths 1-70,
    head dims 1-128, query offsets up to past the last key, windows from 1
    to wider than the keys (0 = global), score and output shifts.  The
    restatement equals reef's engine bit for bit, and refuses exactly the
    configurations the engine refuses (a query row that sees no key)."""
    import ctypes as C
    f32, i8 = C.POINTER(C.c_float), C.POINTER(C.c_int8)
    rng = np.random.default_rng(4096)
    R = ro.ref()
    refused = 0
    for case in range(160):
        ql, kl = int(rng.integers(1, 21)), int(rng.integers(1, 71))
        d = int(rng.choice([1, 4, 8, 32, 64, 128, int(rng.integers(1, 129))]))
        start = int(rng.integers(0, kl + 3))
        window = int(rng.choice([0, 0, 1, 2, int(rng.integers(1, kl + 4))]))
        if case % 2 == 0:
            q = rng.integers(-128, 128, (ql, d)).astype(np.int8)
            k = rng.integers(-128, 128, (kl, d)).astype(np.int8)
            v = rng.integers(-128, 128, (kl, d)).astype(np.int8)
            sh, osh = int(rng.integers(0, 17)), int(rng.integers(4, 13))
            want = np.empty((ql, d), np.int8)
            rc = R.ref_attend_head_int8(ql, kl, d, start, window, _c(q, i8), _c(k, i8),
                                        _c(v, i8), sh, osh, _c(want, i8))
            call = lambda: ro.attention_head_int8(q, k, v, start, window, sh, osh)
        else:
            scale = float(10.0 ** rng.uniform(-2, 1))
            q = (rng.standard_normal((ql, d)) * scale).astype(np.float32)
            k = (rng.standard_normal((kl, d)) * scale).astype(np.float32)
            v = rng.standard_normal((kl, d)).astype(np.float32)
            want = np.empty((ql, d), np.float32)
            rc = R.ref_attend_head_f32(ql, kl, d, start, window, _c(q, f32), _c(k, f32),
                                       _c(v, f32), _c(want, f32))
            call = lambda: ro.attention_head_f32(q, k, v, start, window)
        if rc != 0:
            refused += 1
            with pytest.raises(ValueError):
                call()
            continue
        got = call()
        if want.dtype == np.float32:
            np.testing.assert_array_equal(bits(got), bits(want), err_msg=f"case {case}")
        else:
            np.testing.assert_array_equal(got, want, err_msg=f"case {case}")
    assert 0 < refused < 80  # both kinds of configuration occurred


@needs_ref
def test_attention_int8_matches_engine():
    import ctypes as C
    i8 = C.POINTER(C.c_int8)
    for (ql, kl, d, qs, win, sh, seed) in [(7, 33, 32, 26, 0, 8, 1),
                                           (9, 40, 16, 31, 5, 6, 2),
                                           (64, 64, 64, 0, 0, 10, 3)]:
        q = ro.int8_uniform(seed, (ql, d))
        k = ro.int8_uniform(seed + 1, (kl, d))
        v = ro.int8_uniform(seed + 2, (kl, d))
        want = np.empty((ql, d), np.int8)
        assert ro.ref().ref_attend_head_int8(ql, kl, d, qs, win, _c(q, i8),
                                             _c(k, i8), _c(v, i8), sh, 8,
                                             _c(want, i8)) == 0
        got = ro.attention_head_int8(q, k, v, qs, win, sh, 8)
        np.testing.assert_array_equal(got, want)


@needs_ref
def test_gptneo_block_matches_engine():
    """Config 1 shape (d 256, 4 heads, FFN 1024) at a short sequence."""
    import ctypes as C
    f = C.POINTER(C.c_float)
    seq, d, heads, ffn = 16, 256, 4, 1024
    fw = block_float_weights(d, ffn, seed=70)
    x = ro.normal(69, (seq, d))
    want = np.empty((seq, d), np.float32)
    args = [fw[k] for k in ("ln1_g", "ln1_b", "wq", "wk", "wv", "wo", "bo",
                            "ln2_g", "ln2_b", "wfc", "bfc", "wproj", "bproj")]
    rc = ro.ref().ref_block_w8a8(seq, d, heads, ffn, 0, 0, np.float32(1e-5),
                                 _c(x, f), *[_c(a, f) for a in args],
                                 _c(want, f))
    assert rc == 0
    got = ro.gptneo_block_w8a8(x, ro.quantize_block(fw), heads)
    np.testing.assert_array_equal(bits(got), bits(want))


@needs_ref
def test_random_block_sweep_matches_engine():
    """Ten seeded random GPT-Neo W8A8 blocks: widths 32-96, head dims 8-32,
    FFN widths not a multiple of 16, 1-24 positions, global and local
    (windows 1, 3, 8) attention, and LayerNorm gains and shifts away from 1
    and 0.  The restatement equals Block<float>::forward bit for bit."""
    import ctypes as C
    f = C.POINTER(C.c_float)
    rng = np.random.default_rng(97)
    for case in range(10):
        d = int(rng.choice([32, 64, 96]))
        hd = int(rng.choice([8, 16, 32]))
        heads = d // hd
        ffn = int(rng.choice([40, 72, 136, 4 * d]))
        seq = int(rng.integers(1, 25))
        local = int(rng.integers(0, 2))
        window = int(rng.choice([1, 3, 8])) if local else 0
        fw = block_float_weights(d, ffn, seed=300 + 20 * case)
        for g in ("ln1_g", "ln2_g"):
            fw[g] = (1.0 + 0.3 * rng.standard_normal(d)).astype(np.float32)
        for b in ("ln1_b", "ln2_b"):
            fw[b] = (0.1 * rng.standard_normal(d)).astype(np.float32)
        x = (rng.standard_normal((seq, d)) * 2.0).astype(np.float32)
        want = np.empty((seq, d), np.float32)
        args = [fw[k] for k in ("ln1_g", "ln1_b", "wq", "wk", "wv", "wo", "bo",
                                "ln2_g", "ln2_b", "wfc", "bfc", "wproj", "bproj")]
        rc = ro.ref().ref_block_w8a8(seq, d, heads, ffn, window, local, np.float32(1e-5),
                                     _c(x, f), *[_c(a, f) for a in args], _c(want, f))
        assert rc == 0, f"case {case}"
        got = ro.gptneo_block_w8a8(x, ro.quantize_block(fw), heads, window=window)
        np.testing.assert_array_equal(bits(got), bits(want), err_msg=f"case {case}")


def block_float_weights(d, ffn, seed):
    """Config-1 block weights: projections N(0, 0.02), biases N(0, 0.02),
    LayerNorm gains 1 and shifts 0."""
    return {
        "ln1_g": np.ones(d, np.float32), "ln1_b": np.zeros(d, np.float32),
        "ln2_g": np.ones(d, np.float32), "ln2_b": np.zeros(d, np.float32),
        "wq": ro.normal(seed + 1, (d, d), 0, 0.02),
        "wk": ro.normal(seed + 2, (d, d), 0, 0.02),
        "wv": ro.normal(seed + 3, (d, d), 0, 0.02),
        "wo": ro.normal(seed + 4, (d, d), 0, 0.02),
        "bo": ro.normal(seed + 5, (d,), 0, 0.02),
        "wfc": ro.normal(seed + 6, (ffn, d), 0, 0.02),
        "bfc": ro.normal(seed + 7, (ffn,), 0, 0.02),
        "wproj": ro.normal(seed + 8, (d, ffn), 0, 0.02),
        "bproj": ro.normal(seed + 9, (d,), 0, 0.02),
    }


@needs_ref
def test_lm_head_and_argmax_match_engine():
    R = ro.ref()
    rng = np.random.default_rng(11)
    for out, n in [(1, 1), (129, 33), (500, 256)]:
        w = rng.uniform(-0.5, 0.5, (out, n)).astype(np.float32)
        x = rng.uniform(-2.0, 2.0, n).astype(np.float32)
        y, ok = ro.matvec_rows_f32(w, x)
        want = np.empty(out, np.float32)
        rc = R.ref_matvec_rows_f32(out, n, ro._p(w, ro._f32p), ro._p(x, ro._f32p),
                                   ro._p(want, ro._f32p))
        assert ok and rc == 0
        np.testing.assert_array_equal(bits(y), bits(want))
    # a product that overflows: the engine throws, the restatement says so
    w = np.full((3, 4), 1e30, np.float32)
    x = np.full(4, 1e30, np.float32)
    _, ok = ro.matvec_rows_f32(w, x)
    want = np.empty(3, np.float32)
    rc = R.ref_matvec_rows_f32(3, 4, ro._p(w, ro._f32p), ro._p(x, ro._f32p), ro._p(want, ro._f32p))
    assert not ok and rc == -2
    import ctypes as C
    cases = [rng.uniform(-10, 10, 1000).astype(np.float32),
             np.array([1.0, 3.0, 3.0, 2.0], np.float32),
             np.array([np.nan, 5.0, 1.0], np.float32),
             np.array([1.0, np.nan, 5.0, np.nan], np.float32),
             np.array([-np.inf, -np.inf], np.float32),
             np.array([0.0, -0.0], np.float32), np.array([-0.0, 0.0], np.float32)]
    for v in cases:
        idx = C.c_size_t()
        assert R.ref_argmax_f32(v.size, ro._p(v, ro._f32p), C.byref(idx)) == 0
        assert ro.argmax_f32(v) == idx.value, v


def test_embedding_and_add_match_reef_goldens():
    """kEmbedding / kAdd (gen_golden.cpp:464-503): wte[id] + wpe[position] and
    the residual add are one rounded float add each, as numpy's float32 add."""
    for c in goldens.cases("elementwise", "kEmbedding"):
        w = c["width"]
        y = c["wte"].reshape(-1, w)[c["id"]] + c["wpe"].reshape(-1, w)[c["position"]]
        np.testing.assert_array_equal(y.view(np.uint32), c["y"].view(np.uint32))
    for c in goldens.cases("elementwise", "kAdd"):
        np.testing.assert_array_equal((c["a"] + c["b"]).view(np.uint32), c["y"].view(np.uint32))


def test_coral_float_linear_matches_reef_goldens():
    """kLinear / kLinearBias (gen_golden.cpp): the float linear with Coral's
    [in][out] weight, bit for bit."""
    for table in ("kLinear", "kLinearBias"):
        for c in goldens.cases("linear", table):
            x = c["x"].reshape(c["rows"], c["in"])
            wt = c["wt"].reshape(c["in"], c["out"])
            y = ro.linear_f32(x, wt, c.get("bias"))
            np.testing.assert_array_equal(y.view(np.uint32).ravel(),
                                          c["y"].view(np.uint32))


def test_int8_elementwise_match_reef_goldens():
    """kInt8Gelu, kInt8LayerNorm, kInt8Add, kInt8Embedding (gen_golden.cpp
    write_int8): the integer-only operators, exactly."""
    for c in goldens.cases("int8", "kInt8Gelu"):
        np.testing.assert_array_equal(ro.gelu_int8(c["x"], c["table"]), c["y"])
    for c in goldens.cases("int8", "kInt8LayerNorm"):
        x = c["x"].reshape(c["rows"], c["width"])
        np.testing.assert_array_equal(ro.layernorm_int8(x, c["gain"], c["shift"]).ravel(),
                                      c["y"])
    for c in goldens.cases("int8", "kInt8Add"):
        np.testing.assert_array_equal(ro.add_int8(c["a"], c["b"]), c["y"])
    for c in goldens.cases("int8", "kInt8Embedding"):
        w = c["width"]
        y = ro.embedding_int8(c["wte"].reshape(-1, w), c["wpe"].reshape(-1, w), [c["id"]],
                              c["position"])
        np.testing.assert_array_equal(y.ravel(), c["y"])


@needs_ref
@pytest.mark.parametrize("rows,n_in,out,seed", [(3, 257, 300, 21), (1, 768, 96, 22)])
def test_float_linear_matches_engine(rows, n_in, out, seed):
    import ctypes as C
    f = C.POINTER(C.c_float)
    x = ro.normal(seed, (rows, n_in))
    wt = ro.normal(seed + 1, (n_in, out), 0.0, 0.02)
    b = ro.normal(seed + 2, (out,), 0.0, 0.02)
    for bias in (None, b):
        want = np.empty((rows, out), np.float32)
        rc = ro.ref().ref_linear_f32(rows, n_in, out, _c(x, f), _c(wt, f),
                                     None if bias is None else _c(bias, f), _c(want, f))
        assert rc == 0
        np.testing.assert_array_equal(bits(ro.linear_f32(x, wt, bias)), bits(want))


@needs_ref
def test_int8_elementwise_match_engine():
    """layernorm_int8 (widths past a warp and odd ones, negative means), the
    saturating add and the gelu table lookup against reef's engine."""
    import ctypes as C
    i8 = C.POINTER(C.c_int8)
    rng = np.random.default_rng(23)
    for rows, width in ((7, 768), (3, 37), (2, 4096)):
        x = rng.integers(-128, 128, (rows, width), dtype=np.int8)
        x[0] = -np.abs(x[0]) - 1  # a row with a negative, inexact mean
        g = rng.integers(-128, 128, width, dtype=np.int8)
        s = rng.integers(-128, 128, width, dtype=np.int8)
        want = np.empty((rows, width), np.int8)
        assert ro.ref().ref_layernorm_int8(rows, width, _c(x, i8), _c(g, i8), _c(s, i8),
                                           _c(want, i8)) == 0
        np.testing.assert_array_equal(ro.layernorm_int8(x, g, s), want)
    a = rng.integers(-128, 128, 5000, dtype=np.int8)
    b = rng.integers(-128, 128, 5000, dtype=np.int8)
    want = np.empty(5000, np.int8)
    assert ro.ref().ref_add_int8(5000, _c(a, i8), _c(b, i8), _c(want, i8)) == 0
    np.testing.assert_array_equal(ro.add_int8(a, b), want)
    table = np.empty(256, np.int8)
    assert ro.ref().ref_gelu_int8(5000, _c(a, i8), 0.05, 0.02, _c(table, i8), _c(want, i8)) == 0
    np.testing.assert_array_equal(ro.gelu_int8(a, table), want)
