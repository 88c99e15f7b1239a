"""Parity of reef's two attention heads on the GPU (bit for bit).

* integer softmax / integer head against reef's golden vectors
  (gen_golden.cpp write_int8: 3 softmax cases incl. equal scores and a wide
  spread at shift 0; 7 heads incl. windows and query offsets);
* float head against reef's golden vectors (write_attention, 7 heads);
* both heads against the oracle on larger seeded shapes, and the multi-head
  launch (Attention::context) at the config-1 shape.
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


@pytest.fixture(autouse=True)
def _no_device_errors(cuda_lib):
    yield
    K.check_device_error()


def test_softmax_int8_goldens():
    for c in goldens.cases("int8", "kInt8Softmax"):
        p = K.softmax_int8(dev(c["scores"].reshape(c["rows"], c["n"])), c["shift"],
                           K.exp_table_device(c["table"]))
        np.testing.assert_array_equal(host(p).ravel(), c["probs"])


def test_attention_int8_goldens():
    for c in goldens.cases("int8", "kInt8Attention"):
        d = c["head_dim"]
        y = K.attention_head_int8(dev(c["q"].reshape(-1, d)), dev(c["k"].reshape(-1, d)),
                                  dev(c["v"].reshape(-1, d)), c["query_start"], c["window"],
                                  c["score_shift"], K.exp_table_device(c["table"]),
                                  c["out_shift"])
        np.testing.assert_array_equal(host(y).ravel(), c["y"])


def test_attention_f32_goldens():
    for c in goldens.cases("attention", "kAttention"):
        d = c["head_dim"]
        y = K.attention_head_f32(dev(c["q"].reshape(-1, d)), dev(c["k"].reshape(-1, d)),
                                 dev(c["v"].reshape(-1, d)), c["query_start"], c["window"])
        np.testing.assert_array_equal(bits(host(y).ravel()), bits(c["y"]))


HEADS = [  # query_len, key_len, head_dim, query_start, window, score_shift
    (64, 64, 64, 0, 0, 10), (16, 300, 128, 284, 100, 9), (128, 128, 64, 0, 0, 8),
    (3, 5000, 64, 4997, 0, 11), (33, 1030, 128, 997, 256, 12), (1, 4096, 128, 4095, 0, 12),
]


@pytest.mark.parametrize("ql,kl,d,qs,win,sh", HEADS)
def test_attention_int8_matches_oracle(ql, kl, d, qs, win, sh):
    seed = ql + kl + d
    q = ro.int8_uniform(seed, (ql, d))
    k = ro.int8_uniform(seed + 1, (kl, d))
    v = ro.int8_uniform(seed + 2, (kl, d))
    want = ro.attention_head_int8(q, k, v, qs, win, sh, 8)
    got = K.attention_head_int8(dev(q), dev(k), dev(v), qs, win, sh,
                                K.exp_table_device(ro.exp_table()), 8)
    np.testing.assert_array_equal(host(got), want)


@pytest.mark.parametrize("ql,kl,d,qs,win,sh", HEADS)
def test_attention_f32_matches_oracle(ql, kl, d, qs, win, sh):
    seed = 3 * ql + kl + d
    q = ro.normal(seed, (ql, d), 0.0, 0.3)
    k = ro.normal(seed + 1, (kl, d), 0.0, 0.3)
    v = ro.normal(seed + 2, (kl, d))
    want = ro.attention_head_f32(q, k, v, qs, win)
    got = K.attention_head_f32(dev(q), dev(k), dev(v), qs, win)
    np.testing.assert_array_equal(bits(host(got)), bits(want))


def test_random_heads_match_oracle():
    """80 seeded random heads, int8 and float (query lengths 1-40, key
    lengths 1-600, head dims 1-128, offsets past the last key, windows from 1
    to wider than the keys, shifts): bit for bit against the oracle, and the
    GPU entry points refuse exactly the configurations the oracle refuses
    (a query row that sees no key)."""
    from reef_b200._lib import ReefError
    rng = np.random.default_rng(2718)
    table = K.exp_table_device(ro.exp_table())
    refused = 0
    for case in range(80):
        ql, kl = int(rng.integers(1, 41)), int(rng.integers(1, 601))
        d = int(rng.choice([1, 8, 32, 64, 128, int(rng.integers(1, 129))]))
        qs = int(rng.integers(0, kl + 3))
        win = int(rng.choice([0, 0, 1, 2, int(rng.integers(1, kl + 4))]))
        if case % 2 == 0:
            q = rng.integers(-128, 128, (ql, d)).astype(np.int8)
            k = rng.integers(-128, 128, (kl, d)).astype(np.int8)
            v = rng.integers(-128, 128, (kl, d)).astype(np.int8)
            sh, osh = int(rng.integers(0, 17)), int(rng.integers(4, 13))
            oracle = lambda: ro.attention_head_int8(q, k, v, qs, win, sh, osh)
            gpu = lambda: host(K.attention_head_int8(dev(q), dev(k), dev(v), qs, win, sh,
                                                     table, osh))
        else:
            scale = float(10.0 ** rng.uniform(-2, 0.5))
            q = (rng.standard_normal((ql, d)) * scale).astype(np.float32)
            k = (rng.standard_normal((kl, d)) * scale).astype(np.float32)
            v = rng.standard_normal((kl, d)).astype(np.float32)
            oracle = lambda: ro.attention_head_f32(q, k, v, qs, win)
            gpu = lambda: host(K.attention_head_f32(dev(q), dev(k), dev(v), qs, win))
        try:
            want = oracle()
        except ValueError:
            refused += 1
            with pytest.raises(ReefError):
                gpu()
            continue
        np.testing.assert_array_equal(bits(gpu()), bits(want),
                                      err_msg=f"case {case}: {ql}x{kl}x{d} at {qs}, window {win}")
    assert 0 < refused < 40


def test_context_all_heads_config1_shape():
    """Attention::context at config 1: seq 128, 4 heads x 64, causal."""
    seq, dm, heads = 128, 256, 4
    hd = dm // heads
    q, k, v = (ro.normal(s, (seq, dm)) for s in (41, 42, 43))
    got = host(K.attention_heads_f32(dev(q), dev(k), dev(v), heads))
    for h in range(heads):
        sl = slice(h * hd, (h + 1) * hd)
        want = ro.attention_head_f32(q[:, sl].copy(), k[:, sl].copy(), v[:, sl].copy(), 0, 0)
        np.testing.assert_array_equal(bits(got[:, sl].copy()), bits(want))
