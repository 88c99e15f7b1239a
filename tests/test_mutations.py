"""Mutation tests: each check the kernels are held to can fail.

reef's practice (coral/README.md:129-130) is to break a kernel once and watch
its golden test reject it.  Here the mistake is planted in a CPU restatement
(never on the GPU): every test below computes one operator the way a plausible
but wrong kernel would -- another rounding rule, another order of float
operations, another tie or window rule -- and asserts that the comparison the
parity tests use (reef's golden vectors, or the pinned oracle on the same
seeded inputs) tells it apart from the right answer.  The right restatement
passes the same comparison in tests/test_oracle.py.
"""
import numpy as np

from oracle import oracle as ro
from tests import blob_fixture as BF
from tests import goldens


def same_bits(a, b) -> bool:
    a, b = np.asarray(a), np.asarray(b)
    if a.dtype == np.float32:
        a, b = a.view(np.uint32), np.asarray(b, np.float32).view(np.uint32)
    return a.shape == b.shape and bool(np.array_equal(a, b))


def rne_quantize_rows(x, ties_away=False, reciprocal=False):
    """quantize_rows with one rule changed: ties away from zero, or a multiply
    by the reciprocal of the scale instead of reef's IEEE division."""
    x = np.asarray(x, np.float32)
    amax = np.abs(x).max(axis=1)
    scale = np.where(amax > 0, (amax / np.float32(127)).astype(np.float32), np.float32(1))
    if reciprocal:
        v = x * (np.float32(1) / scale)[:, None]
    else:
        v = x / scale[:, None]
    v = v.astype(np.float32)
    r = np.sign(v) * np.floor(np.abs(v) + 0.5) if ties_away else np.rint(v)
    return np.clip(r, -127, 127).astype(np.int8), scale


# ---- W8A8 linear --------------------------------------------------------------

def test_w8a8_epilogue_association_is_caught():
    """float(acc) * x_scale * w_scale associated left to right instead of
    reef's float(acc) * (x_scale * w_scale)."""
    caught = False
    for table in ("kW8a8", "kW8a8Bias"):
        for c in goldens.cases("linear", table):
            x = c["x"].reshape(c["rows"], c["in"])
            w = c["qt"].reshape(c["in"], c["out"]).T
            xq, xs = ro.quantize_rows(x)
            acc = ro.gemm_i8(xq, w).astype(np.float32)
            y = (acc * xs[:, None]).astype(np.float32) * c["qs"][None, :]
            if c.get("bias") is not None:
                y = y + c["bias"]
            caught |= not same_bits(y.astype(np.float32).ravel(), c["y"])
    assert caught


def test_quantize_ties_away_from_zero_is_caught():
    """reef rounds ties to even (test_quant.cpp:46-53: 2.5 -> 2, -2.5 -> -2)."""
    x = np.array([[2.5, 3.5, -2.5, 2.4, 127.0]], np.float32)
    want, _ = ro.quantize_rows(x)
    got, _ = rne_quantize_rows(x, ties_away=True)
    assert same_bits(rne_quantize_rows(x)[0], want)
    assert not same_bits(got, want)


def test_quantize_by_reciprocal_is_caught():
    """v * (1 / scale) instead of reef's IEEE v / scale.  On Gaussian rows the
    two almost never differ (a one-ulp quotient error rarely crosses a
    rounding boundary), so like reef's tie-forcing cases this uses a crafted
    row: amax 128 gives scale 128/127, and these values land on the other side
    of .5 under the reciprocal.  The GPU quantiser tests run the same rows."""
    x = np.array([[128.0, 5.543306827545166, 7.559054851531982, 88.18897247314453]],
                 np.float32)
    want, _ = ro.quantize_rows(x)
    got, _ = rne_quantize_rows(x, reciprocal=True)
    assert same_bits(rne_quantize_rows(x)[0], want)
    assert list(want[0]) == [127, 6, 8, 88]
    assert not same_bits(got, want)
    # on Gaussian rows the mutant goes unseen: such rows cannot stand in for it
    g = ro.normal(11, (64, 4096))
    assert same_bits(rne_quantize_rows(g, reciprocal=True)[0], ro.quantize_rows(g)[0])


# ---- int8 linear / softmax / head -----------------------------------------------

def test_int8_truncating_shift_is_caught():
    """v >> shift instead of reef's round-half-up shift (the shift-1 cases
    force ties, gen_golden.cpp:526-528)."""
    caught = False
    for c in goldens.cases("int8", "kInt8Linear"):
        x = c["x"].reshape(c["rows"], c["in"]).astype(np.int32)
        wt = c["wt"].reshape(c["in"], c["out"]).astype(np.int32)
        y = np.clip((x @ wt) >> c["shift"], -128, 127).astype(np.int8)
        caught |= not same_bits(y.ravel(), c["y"])
    assert caught


def test_softmax_int8_table_offset_is_caught():
    """Weights looked up one step too far from the row maximum."""
    caught = False
    for c in goldens.cases("int8", "kInt8Softmax"):
        table = np.concatenate([c["table"][1:], c["table"][-1:]])
        s = c["scores"].reshape(c["rows"], c["n"])
        p = ro.softmax_int8(s, c["shift"], table)
        caught |= not same_bits(p.ravel(), c["probs"])
    assert caught


# ---- float operators --------------------------------------------------------------

def naive_head(q, k, v, query_start, window):
    """A plausible float head: BLAS dot products, numpy exp, pairwise sums."""
    out = np.empty((q.shape[0], v.shape[1]), np.float32)
    for i in range(q.shape[0]):
        pos = query_start + i
        lo = 0 if window == 0 else max(0, pos - window + 1)
        s = (k[lo:pos + 1] @ q[i]).astype(np.float32)
        e = np.exp(s - s.max()).astype(np.float32)
        p = (e / e.sum(dtype=np.float32)).astype(np.float32)
        out[i] = p @ v[lo:pos + 1]
    return out


def test_float_head_other_order_is_caught():
    caught = False
    for c in goldens.cases("attention", "kAttention"):
        d = c["head_dim"]
        y = naive_head(c["q"].reshape(-1, d), c["k"].reshape(-1, d), c["v"].reshape(-1, d),
                       c["query_start"], c["window"])
        caught |= not same_bits(y.ravel(), c["y"])
    assert caught


def test_layernorm_one_pass_variance_is_caught():
    """var = E[x^2] - mean^2 instead of reef's second pass over (x - mean)^2."""
    caught = False
    for c in goldens.cases("layernorm", "kLayerNorm"):
        x = c["x"].reshape(c["rows"], c["width"]).astype(np.float32)
        w = np.float32(c["width"])
        y = np.empty_like(x)
        for r in range(x.shape[0]):
            mean, sq = np.float32(0), np.float32(0)
            for v in x[r]:
                mean = np.float32(mean + v)
                sq = np.float32(sq + np.float32(v * v))
            mean = np.float32(mean / w)
            var = np.float32(np.float32(sq / w) - np.float32(mean * mean))
            inv = np.float32(np.float32(1) / np.sqrt(np.float32(var + np.float32(c["eps"]))))
            y[r] = ((x[r] - mean) * inv).astype(np.float32) * c["gain"] + c["shift"]
        caught |= not same_bits(y.astype(np.float32).ravel(), c["y"])
    assert caught


def test_library_exp_tanh_are_caught():
    """numpy's exp and tanh in place of reef's exp_nonpositive / tanh_float."""
    (e,) = goldens.cases("math", "kExp")
    assert not same_bits(np.exp(e["x"]).astype(np.float32), e["y"])
    (t,) = goldens.cases("math", "kTanh")
    assert not same_bits(np.tanh(t["x"]).astype(np.float32), t["y"])


def test_matvec_blas_order_is_caught():
    caught = False
    for c in goldens.cases("linear", "kMatvec"):
        w = c["w"].reshape(c["out"], c["in"])
        caught |= not same_bits((w @ c["x"]).astype(np.float32), c["y"])
    assert caught


def test_argmax_last_maximum_is_caught():
    caught = False
    for c in goldens.cases("elementwise", "kArgmax"):
        x = c["x"]
        last = int(x.size - 1 - np.argmax(x[::-1]))
        caught |= last != c["index"]
    assert caught


# ---- int8 element-wise ---------------------------------------------------------------

def test_layernorm_int8_truncating_mean_is_caught():
    """mean = sum / width truncated toward zero instead of reef's floor_div,
    on the goldens and on the oracle's seeded rows (the GPU test's inputs)."""
    def mutant(x, gain, shift):
        x = np.asarray(x, np.int64)
        width = x.shape[1]
        s = x.sum(axis=1)
        mean = np.where(s < 0, -((-s) // width), s // width)
        c = x - mean[:, None]
        import math
        dev = np.array([math.isqrt(int(v) // width) for v in (c * c).sum(axis=1)], np.int64)
        inv = (1 << 20) // np.maximum(dev, 1)
        scaled = ((c * inv[:, None]) >> 16) * np.asarray(gain, np.int64) + \
            np.asarray(shift, np.int64) * 32
        return np.clip((scaled >> 5) + ((scaled >> 4) & 1), -128, 127).astype(np.int8)

    rng = np.random.default_rng(300 * 768)
    x = rng.integers(-128, 128, (300, 768), dtype=np.int8)
    g = rng.integers(-128, 128, 768, dtype=np.int8)
    s = rng.integers(-128, 128, 768, dtype=np.int8)
    assert not same_bits(mutant(x, g, s), ro.layernorm_int8(x, g, s))


# ---- whole model ---------------------------------------------------------------------

def test_gptneo_window_off_by_one_is_caught():
    """Local layers seeing one key too many: reef's kGptNeo logits reject it."""
    blob, prompt, tokens, logits = BF.golden_model("w8a8")
    h = BF.header(blob)
    m = BF.model_arrays(blob)
    seq = np.concatenate([prompt, tokens[:-1]]).astype(np.int64)
    x = (m["wte"][seq] + m["wpe"][np.arange(seq.size)]).astype(np.float32)
    for i in range(h["layers"]):
        p, local = BF.layer(blob, i)
        x = ro.gptneo_block_w8a8(x, p, h["heads"], window=h["window"] + 1 if local else 0,
                                 eps=h["eps"])
    normed = ro.layernorm(x, m["ln_f_g"], m["ln_f_b"], h["eps"])
    got = np.stack([ro.matvec_rows_f32(m["wte"], normed[t])[0]
                    for t in range(prompt.size - 1, seq.size)])
    assert not same_bits(got, logits)


# ---- the Llama layer's own definitions (parity unpinned by reef) ----------------------

def test_rmsnorm_sequential_sum_is_caught():
    """The RMSNorm's sum of squares in plain left-to-right order instead of the
    fixed 8-chunk tree that makes TP shards reproduce TP=1: the GPU test's
    restatement of the tree tells the scales apart."""
    from tests.test_rmsnorm_gpu import rmsnorm_quant_ref
    f32 = np.float32
    x = ro.normal(3, (4, 4096))
    gain = (1.0 + 0.1 * ro.normal(4, (4096,))).astype(f32)
    eps = f32(1e-5)
    _, want = rmsnorm_quant_ref(x, gain, eps)
    got = np.empty(4, f32)
    for r in range(4):
        total = f32(0)
        for v in x[r]:
            total = f32(total + f32(v * v))
        rr = f32(f32(1) / np.sqrt(f32(f32(total / f32(4096)) + eps)))
        mx = f32(np.abs((x[r] * gain).astype(f32)).max() * rr)
        got[r] = f32(mx / f32(127))
    assert not same_bits(got, want)
